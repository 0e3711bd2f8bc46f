"""GPU parity of the prefill path (T > 64: sorted grouped tcgen05 GEMMs).

Checked against the CPU oracle on whole small batches and on sampled tokens
of large ones (the block is per-token, so a token's output depends only on
its own row), and against the decode kernels (RNB_FLAG_CHAIN) on the same
input.  Routing must match exactly; outputs use the bounds of tests/_parity.py.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import _lib, inputs, ops
from tests._parity import assert_close, assert_close_gpu_pair, oracle_block

pytestmark = pytest.mark.gpu


def _run(bits, seed, T, skew=None, sample=None):
    blk = inputs.make_block(bits, seed=seed, T=T, skew=skew)
    bt = ops.BlockTensors.from_numpy(blk, "cuda")
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
    out, inds, scores = ops.moe_block(bt, x, return_routing=True)
    w = oracle.BlockWeights(bits=bits, group=64, **blk.weight_fields())
    rows = np.arange(T) if sample is None else np.sort(np.random.default_rng(seed).choice(T, sample, replace=False))
    ref, oinds, oscores, bound = oracle_block(w, np.ascontiguousarray(blk.x[rows]))
    np.testing.assert_array_equal(inds.cpu().numpy()[rows], oinds)
    np.testing.assert_allclose(scores.cpu().numpy()[rows], oscores, rtol=2e-5, atol=1e-7)
    s = assert_close(out.float().cpu().numpy()[rows], ref, f"prefill q{bits} T={T} skew={skew}", bound=bound)
    return blk, bt, x, out, s


@pytest.mark.parametrize("bits", [8, 4])
def test_prefill_matches_oracle_small_batch(bits):
    _run(bits, seed={8: 0, 4: 1}[bits], T=128)


@pytest.mark.parametrize("bits,T", [(8, 200), (4, 65)])
def test_prefill_ragged_token_counts(bits, T):
    _run(bits, seed=5, T=T)


def test_prefill_zipf_skew_config3_sampled():
    """Configuration 3 of the benchmark set: q8, 2048 tokens, log-Zipf routing skew."""
    blk, bt, x, out, _ = _run(8, seed=2, T=2048, skew="zipf", sample=48)
    chain = ops.BlockTensors(**{**bt.__dict__, "flags": bt.flags | _lib.FLAG_CHAIN})
    out_c = ops.moe_block(chain, x)
    assert_close_gpu_pair(out.float().cpu().numpy(), out_c.float().cpu().numpy(), "prefill vs decode chain")


@pytest.mark.parametrize("T", [4096, 8194])
def test_host_entry_point_chunked_copies(T):
    """From 4096 tokens rnb_moe_block_fwd_host splits the call into chunks of
    whole tokens (2 here; 4 uneven ones at 8194) whose copies overlap compute.
    The host buffer must hold exactly one block call per chunk, and the same
    bits as the whole-batch device call: every prefill stage (routing, row
    scales, the slot-order sum) is per token, so the split changes nothing."""
    blk = inputs.make_block(4, seed=1, T=64)
    bt = ops.BlockTensors.from_numpy(blk, "cuda")
    x = torch.from_numpy(inputs.make_tokens(11, T)).view(torch.int16).view(torch.bfloat16).cuda()
    n = min(4, T // 2048)
    bounds = [T * j // n for j in range(n + 1)]
    per_chunk = torch.cat([ops.moe_block(bt, x[a:b]) for a, b in zip(bounds[:-1], bounds[1:])]).cpu()
    whole = ops.moe_block(bt, x).cpu()
    bc = ops.BlockCall(bt, T)
    xh = x.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    for _ in range(2):
        oh.zero_()
        bc.host(xh, oh)
        torch.cuda.current_stream().synchronize()
        assert torch.equal(oh, per_chunk)
    assert torch.equal(oh, whole), f"chunked host call T={T} differs from the whole-batch call"
    assert bc.ws.status() == 0


@pytest.mark.parametrize("skew", [None, "adversarial"])
def test_config5_T16384_sampled(skew):
    """Benchmark configuration 5 at its size: q8, 16384 tokens, seed 4, the
    uniform and the adversarial step (a quarter of the tokens forced onto one
    expert); 64 tokens sampled for the oracle."""
    _run(8, seed=4, T=16384, skew=skew, sample=64)


def test_prefill_adversarial_routing_sampled():
    """A quarter of the tokens all route to one expert (many 128-row tiles of one expert)."""
    blk, bt, x, out, _ = _run(8, seed=4, T=1024, skew="adversarial", sample=32)
    hot = blk.meta["hot_expert"]
    inds = ops.router_topk(bt, x)[0].cpu().numpy()
    assert (inds == hot).any(axis=1).sum() >= 200


def test_prefill_workspace_and_status():
    blk = inputs.make_block(4, seed=1, T=256)
    bt = ops.BlockTensors.from_numpy(blk, "cuda")
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
    ws = ops.Workspace("cuda")
    a = ops.moe_block(bt, x, ws=ws)
    b = ops.moe_block(bt, x, ws=ws)
    assert ws.status() == 0
    # the per-token sum runs in slot order: repeated calls give the same bits
    assert torch.equal(a, b)


def test_decode_after_prefill_on_one_workspace():
    """Prefill, chained decode and the persistent decode kernel alternate on
    one workspace; each call still matches a call on a fresh workspace."""
    blk = inputs.make_block(8, seed=6, T=200)
    bt = ops.BlockTensors.from_numpy(blk, "cuda")
    chain = ops.BlockTensors(**{**bt.__dict__, "flags": bt.flags | _lib.FLAG_CHAIN})
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
    shared = ops.Workspace("cuda")
    for tensors, xs in ((bt, x), (chain, x), (bt, x[:3]), (bt, x), (chain, x[:64]), (bt, x[:1])):
        got = ops.moe_block(tensors, xs, ws=shared)
        fresh = ops.moe_block(tensors, xs, ws=ops.Workspace("cuda"))
        assert shared.status() == 0
        assert torch.equal(got, fresh), "a shared workspace changed a result"


def test_experts_fwd_given_routing_matches_oracle():
    """rnb_moe_experts_fwd (the receive side of all-to-all expert parallelism):
    given ids and weights, the shard's experts only, no router or shared expert."""
    blk = inputs.make_block(4, seed=1, T=70)
    w = oracle.BlockWeights(bits=4, group=64, **blk.weight_fields())
    _, inds, scores, _ = oracle.router(w, blk.x, k=8)
    y = oracle.switchglu(w, blk.x, inds)
    ybound = oracle.block_bound(w, blk.x, inds)
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
    ti = torch.from_numpy(inds.astype(np.int32)).cuda()
    ts = torch.from_numpy(scores).cuda()
    for lo, hi in ((0, 256), (64, 128)):
        bt = ops.BlockTensors.from_numpy(blk, "cuda", E_range=(lo, hi))
        local = (inds >= lo) & (inds < hi)
        wk = np.where(local, scores, 0.0).astype(np.float32)
        ref = np.einsum("tk,tkh->th", wk, y)
        bound = np.einsum("tk,tkh->th", wk, ybound)
        for T in (70, 3):
            out = ops.experts_fwd(bt, x[:T], ti[:T], ts[:T])
            assert out.dtype == torch.float32
            assert_close(out.cpu().numpy(), ref[:T], f"experts_fwd [{lo},{hi}) T={T}", bound=bound[:T])
    out16 = ops.experts_fwd(bt, x, ti, ts, out_f32=False)
    assert out16.dtype == torch.bfloat16
    assert_close(out16.float().cpu().numpy(), ref, "experts_fwd bf16", bound=bound)
    # an id outside [0, E_total) is skipped and flagged
    bad = ti.clone()
    bad[0, 0] = 999
    import ctypes
    need = ctypes.c_size_t()
    d = ops.BlockTensors(**{**bt.__dict__, "flags": _lib.FLAG_Y_F32}).desc(2, 8)
    _lib.call("rnb_moe_experts_workspace_size", ctypes.byref(d), ctypes.byref(need))
    ws = torch.zeros(need.value, dtype=torch.uint8, device="cuda")
    out = ops.experts_fwd(bt, x[:2], bad[:2], ts[:2], ws=ws)
    st = int(ws[:4].view(torch.int32).item())
    assert st & _lib.STATUS_BAD_INDEX
    keep = np.where(local[:2], scores[:2], 0.0)
    keep[0, 0] = 0.0
    assert_close(out.cpu().numpy(), np.einsum("tk,tkh->th", keep.astype(np.float32), y[:2]), "experts_fwd bad id",
                 bound=np.einsum("tk,tkh->th", keep.astype(np.float32), ybound[:2]))
