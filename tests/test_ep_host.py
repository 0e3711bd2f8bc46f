"""Expert-parallel host logic on CPU: the shard plan, the partial-sum
decomposition the kernels implement, and the two-rank reduction path over
gloo (the device call replaced by the oracle).

Rank r's partial = sum over its local selected experts of score * expert
output + shared gate * (the shared expert restricted to rank r's 128-channel
intermediate quarters); the partials of all ranks add up to the block.
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import _lib, ep, inputs, ops

BITS, SEED, T = 4, 1, 3


def _weights(blk):
    return oracle.BlockWeights(bits=blk.bits, group=64, **blk.weight_fields())


def shared_quarters(blk, x_bits, mask):
    """Shared expert output over the intermediate quarters in `mask` (oracle arithmetic)."""
    xf = oracle.bf16_to_f32(x_bits)
    I, H = blk.I, blk.H
    out = np.zeros((x_bits.shape[0], H), np.float32)
    if not mask:
        return out
    for t in range(xf.shape[0]):
        gu = oracle.affine_matvec(blk.sgu_w, blk.sgu_s, blk.sgu_b, xf[t], blk.bits, 64)
        up, gate = gu[:I], gu[I:]
        h = (gate / (1.0 + np.exp(-gate.astype(np.float64)))).astype(np.float32) * up
        for q in range(I // 128):
            if not (mask >> q) & 1:
                continue
            wq = 128 * blk.bits // 32
            cols = slice(q * wq, (q + 1) * wq)
            sc = slice(q * 2, q * 2 + 2)
            out[t] += oracle.affine_matvec(np.ascontiguousarray(blk.sdn_w[:, cols]),
                                           np.ascontiguousarray(blk.sdn_s[:, sc]),
                                           np.ascontiguousarray(blk.sdn_b[:, sc]),
                                           np.ascontiguousarray(h[q * 128:(q + 1) * 128]), blk.bits, 64)
    return out


def partial_block(blk, x_bits, lo, hi, mask, full_shared=False):
    w = _weights(blk)
    _, inds, scores, sg = oracle.router(w, x_bits, k=8)
    y = oracle.switchglu(w, x_bits, inds)
    local = (inds >= lo) & (inds < hi)
    out = np.einsum("tk,tkh->th", np.where(local, scores, 0.0).astype(np.float32), y)
    if full_shared:
        out += sg[:, None] * oracle.shared_expert(w, x_bits)
    else:
        out += sg[:, None] * shared_quarters(blk, x_bits, mask)
    return out.astype(np.float32)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_partitions_experts_and_shared_quarters(world):
    covered, masks = [], 0
    for r in range(world):
        lo, hi, mask = ep.plan(r, world)
        covered.extend(range(lo, hi))
        assert masks & mask == 0
        masks |= mask
    assert covered == list(range(256))
    assert masks == 0xF


def test_plan_rejects_bad_worlds():
    with pytest.raises(ValueError):
        ep.plan(2, 2)
    with pytest.raises(ValueError):
        ep.plan(0, 3)  # 256 experts do not split over 3 ranks


@pytest.mark.parametrize("world", [2, 8])
def test_rank_partials_sum_to_block(world):
    blk = inputs.make_block(BITS, seed=SEED, T=T)
    ref, _, _ = oracle.moe_block(_weights(blk), blk.x, k=8)
    total = np.zeros_like(ref)
    for r in range(world):
        lo, hi, mask = ep.plan(r, world)
        total += partial_block(blk, blk.x, lo, hi, mask)
    err = np.linalg.norm(total - ref) / np.linalg.norm(ref)
    assert err < 1e-5, err


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # handle exchange keeps rank order
        got = ep.gather_handles(bytes([rank]) * _lib.EP_HANDLE_BYTES)
        assert got == [bytes([q]) * _lib.EP_HANDLE_BYTES for q in range(world)]
        blk = inputs.make_block(BITS, seed=SEED, T=T)
        lo, hi, _ = ep.plan(rank, world)
        shard = ops.BlockTensors.from_numpy(blk, "cpu", E_range=(lo, hi))

        def partial_fn(bt, x):
            assert bt.flags & _lib.FLAG_Y_F32
            assert bool(bt.flags & _lib.FLAG_NO_SHARED) == (rank != 0)
            p = partial_block(blk, blk.x, bt.expert_offset, bt.expert_offset + bt.E, 0,
                              full_shared=not (bt.flags & _lib.FLAG_NO_SHARED))
            return torch.from_numpy(p)

        x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16)
        out = ep.moe_block_nccl(shard, x, rank, partial_fn=partial_fn)
        ref, _, _ = oracle.moe_block(_weights(blk), blk.x, k=8)
        err = np.abs(out.float().numpy() - ref).max() / np.abs(ref).max()
        assert err < 1e-2, err
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_reduction_over_gloo():
    import torch.multiprocessing as mp

    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)


def _a2a_rank_main(rank, world, port):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blk = inputs.make_block(BITS, seed=SEED, T=2 * world)
        w = _weights(blk)
        mine = blk.x[rank * 2:(rank + 1) * 2]  # every rank has its own tokens
        if rank == world - 1:
            mine = mine[:1]  # ragged
        lo, hi, _ = ep.plan(rank, world)
        shard = ops.BlockTensors.from_numpy(blk, "cpu", E_range=(lo, hi))
        seen = {}

        def block_fn(bt, x):
            assert bt.flags & _lib.FLAG_Y_F32 and (bt.expert_offset, bt.E) == (lo, hi - lo)
            xb = x.view(torch.int16).numpy().view(np.uint16)
            _, inds, scores, _ = oracle.router(w, xb, k=8)
            p = partial_block(blk, xb, lo, hi, 0, full_shared=True)
            return torch.from_numpy(p), torch.from_numpy(inds.astype(np.int32)), torch.from_numpy(scores)

        def experts_fn(bt, x, inds, scores):
            seen["rows"] = x.shape[0]
            if x.shape[0] == 0:
                return torch.zeros((0, bt.H), dtype=torch.float32)
            xb = x.view(torch.int16).numpy().view(np.uint16)
            ind = inds.numpy()
            seen["all_local"] = bool((((ind >= lo) & (ind < hi)).any(axis=1)).all())
            y = oracle.switchglu(w, xb, ind.astype(np.uint32))
            local = (ind >= lo) & (ind < hi)
            return torch.from_numpy(np.einsum("tk,tkh->th", np.where(local, scores.numpy(), 0.0)
                                              .astype(np.float32), y).astype(np.float32))

        x = torch.from_numpy(mine).view(torch.int16).view(torch.bfloat16)
        stats = {}
        out = ep.moe_block_a2a(shard, x, rank, world, block_fn=block_fn, experts_fn=experts_fn, stats=stats)
        ref, _, _ = oracle.moe_block(w, mine, k=8)
        err = np.abs(out.float().numpy() - ref).max() / np.abs(ref).max()
        assert err < 1e-2, err
        assert stats["received"] == seen["rows"]
        assert seen.get("all_local", True)  # the all-to-all sends only rows with an expert here
        tot = torch.tensor([stats["sent"], stats["received"]])
        dist.all_reduce(tot)
        assert tot[0] == tot[1]  # every row sent is received once
        # gather / reduce-scatter form (equal token counts on every rank)
        eq = blk.x[rank * 2:(rank + 1) * 2]
        xe = torch.from_numpy(eq).view(torch.int16).view(torch.bfloat16)

        def gather(outb, inp):
            parts = list(outb.unbind(0))
            dist.all_gather(parts, inp)

        def reduce_scatter(outb, inp):
            full = inp.clone()
            dist.all_reduce(full)
            outb.copy_(full.view(world, -1, full.shape[-1])[rank])

        out = ep.moe_block_gather(shard, xe, rank, world, block_fn=block_fn, experts_fn=experts_fn,
                                  gather_fn=gather, reduce_scatter_fn=reduce_scatter)
        ref, _, _ = oracle.moe_block(w, eq, k=8)
        err = np.abs(out.float().numpy() - ref).max() / np.abs(ref).max()
        assert err < 1e-2, err
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_all_to_all_dispatch_combine_over_gloo(world):
    import torch.multiprocessing as mp

    mp.spawn(_a2a_rank_main, args=(world, _free_port()), nprocs=world, join=True)
