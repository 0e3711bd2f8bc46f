"""Expert-parallel decode on GPUs: the in-kernel NVLink exchange
(rnb_moe_block_ep_fwd) and the NCCL baseline against the oracle.

The two-rank test needs two GPUs (one process each) and is skipped on a
single-GPU box; the single-rank test runs the same entry point with world 1.
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import _lib, ep, inputs, ops
from tests._parity import assert_close, assert_close_gpu_pair, oracle_block

pytestmark = pytest.mark.gpu

BITS, SEED = 4, 1


def _ref(blk, T):
    """(ref, inds, scores, bound) of the oracle on the first T tokens."""
    w = oracle.BlockWeights(bits=BITS, group=64, **blk.weight_fields())
    return oracle_block(w, blk.x[:T])


def test_single_rank_context_matches_block():
    blk = inputs.make_block(BITS, seed=SEED, T=8)
    dev = torch.device("cuda", 0)
    bt = ep.shard_tensors(blk, 0, 1, dev)
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).to(dev)
    ctx = ep.ExpertParallel(0, 1, handles_fn=lambda h: [h])
    try:
        for T in (1, 8, 5):
            out, inds, _ = ctx.moe_block(bt, x[:T], return_routing=True)
            ref, oinds, _, bound = _ref(blk, T)
            np.testing.assert_array_equal(inds.cpu().numpy(), oinds)
            assert_close(out.float().cpu().numpy(), ref, f"ep world 1 T={T}", bound=bound)
        f32 = ops.BlockTensors(**{**bt.__dict__, "flags": _lib.FLAG_Y_F32})
        out = ctx.moe_block(f32, x[:2])
        assert out.dtype == torch.float32
        r2 = _ref(blk, 2)
        assert_close(out.cpu().numpy(), r2[0], "ep world 1 fp32", bound=r2[3])
    finally:
        ctx.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    gloo = dist.new_group(backend="gloo")
    ctx = None
    try:
        blk = inputs.make_block(BITS, seed=SEED, T=8)
        shard = ep.shard_tensors(blk, rank, world, dev)
        x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).to(dev)
        ws = ops.Workspace(dev)
        ctx = ep.ExpertParallel(rank, world, handles_fn=lambda h: ep.gather_handles(h, group=gloo))
        for T in (1, 8, 3, 1, 8, 2):  # repeated calls alternate the exchange parity
            dist.barrier(group=gloo)  # ranks enter each exchange together
            out, inds, _ = ctx.moe_block(shard, x[:T], ws=ws, return_routing=True)
            ref, oinds, _, bound = _ref(blk, T)
            np.testing.assert_array_equal(inds.cpu().numpy(), oinds)
            assert_close(out.float().cpu().numpy(), ref, f"ep p2p rank {rank} T={T}", bound=bound)
            # every rank holds the same bits (the sum runs in rank order everywhere)
            allv = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(allv, out)
            for v in allv:
                assert torch.equal(v, out)
        assert ws.status() == 0
        out_n = ep.moe_block_nccl(shard, x[:8], rank, ws=ws)
        r8 = _ref(blk, 8)
        assert_close(out_n.float().cpu().numpy(), r8[0], f"ep nccl rank {rank}", bound=r8[3])
        # a two-layer stack, expert parallel, against the same stack on one GPU
        from runnel_b200 import stack
        lo, hi, _ = ep.plan(rank, world)
        full_l, norms = stack.synthetic_layers(2, BITS, seed=3, device=dev)
        shard_l, _ = stack.synthetic_layers(2, BITS, seed=3, device=dev, E_range=(lo, hi))
        one = stack.LayerStack(full_l, norms, ws=ops.Workspace(dev)).forward(x[:1])
        dist.barrier(group=gloo)
        par = stack.LayerStack(shard_l, norms, ep=ctx, ws=ws).forward(x[:1])
        assert_close_gpu_pair(par.float().cpu().numpy(), one.float().cpu().numpy(), f"ep stack rank {rank}")
        assert ws.status() == 0
        # all-to-all dispatch/combine over each rank's own tokens against the
        # whole bank on one GPU (prefill-size, decode-size, ragged and empty)
        full = ops.BlockTensors.from_numpy(blk, dev)
        g = torch.Generator(device=dev)
        for i, (t0, t1) in enumerate(((300, 77), (5, 64), (0, 130))):
            g.manual_seed(100 * i + rank)
            xr = torch.randn(((t0, t1)[rank % 2], blk.H), device=dev, generator=g).to(torch.bfloat16)
            dist.barrier(group=gloo)
            stats = {}
            got = ep.moe_block_a2a(shard, xr, rank, world, ws=ws, stats=stats)
            want, winds, _ = ops.moe_block(full, xr, ws=ws, return_routing=True)
            if xr.shape[0]:
                assert_close_gpu_pair(got.float().cpu().numpy(), want.float().cpu().numpy(),
                                      f"ep a2a rank {rank} case {i}")
            assert stats["sent"] <= xr.shape[0] * (world - 1)
            if t0 == t1:  # the gather / reduce-scatter form needs equal token counts
                got = ep.moe_block_gather(shard, xr, rank, world, ws=ws)
                if xr.shape[0]:
                    assert_close_gpu_pair(got.float().cpu().numpy(), want.float().cpu().numpy(),
                                          f"ep gather rank {rank} case {i}")
        g.manual_seed(7 + rank)
        xr = torch.randn((200, blk.H), device=dev, generator=g).to(torch.bfloat16)
        dist.barrier(group=gloo)
        got = ep.moe_block_gather(shard, xr, rank, world, ws=ws)
        want = ops.moe_block(full, xr, ws=ws)
        assert_close_gpu_pair(got.float().cpu().numpy(), want.float().cpu().numpy(), f"ep gather rank {rank} T=200")
        assert ws.status() == 0
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        if ctx is not None:
            ctx.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_expert_parallel_decode():
    import torch.multiprocessing as mp

    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_every_gpu_expert_parallel_decode():
    """The expert-parallel decode paths on every GPU of the box (4 or 8 ranks)."""
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    mp.spawn(_rank_main, args=(world, _free_port()), nprocs=world, join=True)


def _idle_rank(conn):
    """Rank 1 of a two-rank context that never makes a block call: it makes
    its receive buffer, hands over its handle and waits to be told to exit
    (no kernel of its own ever runs)."""
    import ctypes

    import torch

    from runnel_b200 import _lib

    torch.cuda.set_device(0)
    ep = ctypes.c_void_p()
    buf = (ctypes.c_char * _lib.EP_HANDLE_BYTES)()
    _lib.call("rnb_ep_create", 1, 2, 2048, ctypes.byref(ep), buf)
    conn.send(bytes(buf))
    conn.recv()
    _lib.load().rnb_ep_destroy(ep)


def test_peer_that_never_calls_times_out_then_a_fresh_context_is_correct():
    """A two-rank expert-parallel call whose second rank never calls: the
    bounded wait for its words (lowered to 50 ms) runs out, the call returns
    with RNB_STATUS_TIMEOUT, and a fresh context computes correctly again.
    The missing rank is a host process that never launches (no GPU fault)."""
    import multiprocessing

    ctx = multiprocessing.get_context("spawn")
    parent, child = ctx.Pipe()
    proc = ctx.Process(target=_idle_rank, args=(child,))
    proc.start()
    dev = torch.device("cuda", 0)
    blk = inputs.make_block(BITS, seed=SEED, T=2)
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).to(dev)
    try:
        assert parent.poll(180), "the idle rank did not start"
        h1 = parent.recv()
        ctx2 = ep.ExpertParallel(0, 2, handles_fn=lambda h: [h, h1])
        try:
            ctx2.set_wait_limit_ms(50)
            shard = ep.shard_tensors(blk, 0, 2, dev)
            ws = ops.Workspace(dev)
            for T in (1, 2):  # the persistent kernel (T <= 2) and again on the same context
                ctx2.moe_block(shard, x[:T], ws=ws)
                torch.cuda.synchronize()
                assert ws.status() & _lib.STATUS_TIMEOUT
        finally:
            ctx2.close()
    finally:
        parent.send(1)
        proc.join(60)
    one = ep.ExpertParallel(0, 1, handles_fn=lambda h: [h])
    try:
        bt = ep.shard_tensors(blk, 0, 1, dev)
        ws = ops.Workspace(dev)
        out = one.moe_block(bt, x, ws=ws)
        torch.cuda.synchronize()
        assert ws.status() == 0
        ref, _, _, bound = _ref(blk, 2)
        assert_close(out.float().cpu().numpy(), ref, "fresh context after a timeout", bound=bound)
    finally:
        one.close()


def _idle_rank_a2a(conn):
    """Rank 1 of a two-rank device all-to-all that never makes a call: it
    makes its areas, hands over its handle and waits to be told to exit."""
    import ctypes

    import torch

    from runnel_b200 import _lib

    torch.cuda.set_device(0)
    a = ctypes.c_void_p()
    buf = (ctypes.c_char * _lib.A2A_HANDLE_BYTES)()
    _lib.call("rnb_a2a_create", 1, 2, 2048, 8, 64, ctypes.byref(a), buf)
    conn.send(bytes(buf))
    conn.recv()
    _lib.load().rnb_a2a_destroy(a)


def test_all_to_all_peer_that_never_calls_times_out_then_a_fresh_context_is_correct():
    """A device all-to-all call whose second rank never calls: both bounded
    waits (rows in, sums back; lowered to 50 ms) run out, the call returns
    with RNB_STATUS_TIMEOUT in its workspace, and a fresh context computes
    correctly.  The missing rank is a host process that never launches."""
    import multiprocessing

    mpc = multiprocessing.get_context("spawn")
    parent, child = mpc.Pipe()
    proc = mpc.Process(target=_idle_rank_a2a, args=(child,))
    proc.start()
    dev = torch.device("cuda", 0)
    blk = inputs.make_block(BITS, seed=SEED, T=40)
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).to(dev)
    try:
        assert parent.poll(180), "the idle rank did not start"
        h1 = parent.recv()
        a2a = ep.DeviceAllToAll(0, 2, max_tokens=64, handles_fn=lambda h: [h, h1])
        try:
            a2a.set_wait_limit_ms(50)
            shard = ep.shard_tensors(blk, 0, 2, dev)
            for T in (40, 3):
                a2a.moe_block(shard, x[:T])
                torch.cuda.synchronize()
                assert a2a.status() & _lib.STATUS_TIMEOUT
        finally:
            a2a.close()
    finally:
        parent.send(1)
        proc.join(60)
    one = ep.DeviceAllToAll(0, 1, max_tokens=64, handles_fn=lambda h: [h])
    try:
        bt = ep.shard_tensors(blk, 0, 1, dev)
        out = one.moe_block(bt, x)
        torch.cuda.synchronize()
        assert one.status() == 0
        want = ops.moe_block(ops.BlockTensors.from_numpy(blk, dev), x)
        assert torch.equal(out, want)
    finally:
        one.close()


def test_single_rank_device_all_to_all_is_the_block():
    blk = inputs.make_block(BITS, seed=SEED, T=130)
    dev = torch.device("cuda", 0)
    bt = ep.shard_tensors(blk, 0, 1, dev)
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).to(dev)
    a2a = ep.DeviceAllToAll(0, 1, max_tokens=256, handles_fn=lambda h: [h])
    try:
        got = a2a.moe_block(bt, x)
        want = ops.moe_block(ops.BlockTensors.from_numpy(blk, dev), x)
        assert torch.equal(got, want)
    finally:
        a2a.close()


def _rank_main_a2a(rank, world, port):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    a2a = None
    try:
        blk = inputs.make_block(8, seed=5, T=1)
        shard = ep.shard_tensors(blk, rank, world, dev)
        full = ops.BlockTensors.from_numpy(blk, dev)
        w = oracle.BlockWeights(bits=8, group=64, **blk.weight_fields())
        a2a = ep.DeviceAllToAll(rank, world, max_tokens=512, handles_fn=lambda h: ep.gather_handles(h))
        a2a.set_wait_limit_ms(20000)
        g = torch.Generator(device=dev)
        # prefill- and decode-size calls; repeated calls alternate the areas' parity
        for i, T in enumerate((300, 5, 512, 300, 64)):
            g.manual_seed(1000 * i + rank)
            xr = torch.randn((T, blk.H), device=dev, generator=g).to(torch.bfloat16)
            dist.barrier()
            got, inds, scores = a2a.moe_block(shard, xr, return_routing=True)
            want, winds, wscores = ops.moe_block(full, xr, return_routing=True)
            assert torch.equal(inds, winds) and torch.equal(scores, wscores)
            assert_close_gpu_pair(got.float().cpu().numpy(), want.float().cpu().numpy(),
                                  f"device all-to-all rank {rank} T={T}")
            rows = np.linspace(0, T - 1, min(T, 16)).astype(int)
            xb = xr[rows].view(torch.int16).cpu().numpy().view(np.uint16)
            ref, oinds, _, bound = oracle_block(w, np.ascontiguousarray(xb))
            np.testing.assert_array_equal(inds.cpu().numpy()[rows], oinds)
            assert_close(got.float().cpu().numpy()[rows], ref, f"device all-to-all rank {rank} T={T} (oracle)",
                         bound=bound)
        # back-to-back calls, no host barrier between them: each call's
        # exchange stream forks from and joins the caller's stream
        xs = []
        for i in range(4):
            g.manual_seed(7000 + 10 * i + rank)
            xs.append(torch.randn((384, blk.H), device=dev, generator=g).to(torch.bfloat16))
        wants = [ops.moe_block(full, xi) for xi in xs]
        dist.barrier()
        gots = [a2a.moe_block(shard, xi) for xi in xs]
        for i, (gt, wt) in enumerate(zip(gots, wants)):
            assert_close_gpu_pair(gt.float().cpu().numpy(), wt.float().cpu().numpy(),
                                  f"device all-to-all rank {rank} back-to-back call {i}")
        st = a2a.status()
        assert st == 0, f"rank {rank}: status bits {st:#x}"
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        if a2a is not None:
            a2a.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_device_all_to_all():
    import torch.multiprocessing as mp

    mp.spawn(_rank_main_a2a, args=(2, _free_port()), nprocs=2, join=True)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_every_gpu_device_all_to_all():
    """The same on every GPU of the box (4 or 8 ranks): the slot mapping and
    the flag arrays at more than two ranks."""
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    mp.spawn(_rank_main_a2a, args=(world, _free_port()), nprocs=world, join=True)
