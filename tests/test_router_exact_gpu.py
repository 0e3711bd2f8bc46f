"""Exact router selection on inputs built to defeat fp32 accumulation.

A router logit is the correctly rounded bf16 of the exact dot product.  Here
every logit is a bf16 rounding midpoint plus a term far below fp32
resolution, so an fp32 sum lands exactly on the midpoint while the exact sum
lies above it, below it, or on it (ties to even).  Rounded bases collide
with their neighbours, so the lower-index tie rule decides slots too.  All
three kernels that route (the chain router, the persistent decode kernel and
the prefill router) must agree with the oracle bit for bit.
"""
import dataclasses

import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import inputs, ops
from runnel_b200.quant import bf16_bits_to_f32, f32_to_bf16_bits
from tests._parity import assert_close, oracle_block

H, E = 2048, 256


def _midpoint_block(bits, seed, T):
    e = np.arange(E)
    base = (1.0 + (e % 128) / 128.0) * np.where(e < 128, 1.0, 0.5)
    half_ulp = np.where(e < 128, 2.0 ** -8, 2.0 ** -9)
    sign = np.array([1.0, -1.0, 0.0])[e % 3]
    w = np.zeros((E, H), np.float32)
    w[:, 0] = base
    w[:, 1] = half_ulp
    w[:, 2] = sign * base * 2.0 ** -30
    w *= 2.0 ** -4  # exact scaling into a router-like range
    s_t = np.array([1.0, -1.0, 0.0, 1.0, -1.0, 0.0, 2.0, -2.0])
    x = np.zeros((T, H), np.float32)
    x[:, 0] = 1.0
    x[:, 1] = 1.0
    x[:, 2] = s_t[np.arange(T) % 8]
    blk = inputs.make_block(bits, seed=seed, T=T)
    return dataclasses.replace(blk, x=f32_to_bf16_bits(x), router_w=f32_to_bf16_bits(w))


def _oracle(blk, bits):
    return oracle.BlockWeights(bits=bits, group=64, **blk.weight_fields())


def test_midpoint_logits_need_exact_rounding():
    """CPU: the construction really separates fp32 from exact rounding."""
    blk = _midpoint_block(8, 0, 8)
    w = _oracle(blk, 8)
    logits, _, _, _ = oracle.router(w, blk.x, k=8)
    x = bf16_bits_to_f32(blk.x)
    rw = bf16_bits_to_f32(blk.router_w)
    f32 = (x @ rw.T).astype(np.float32)  # lands on the midpoints
    naive = bf16_bits_to_f32(f32_to_bf16_bits(f32))
    assert (naive != logits).mean() > 0.2


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [8, 4])
def test_router_midpoints_chain(bits):
    blk = _midpoint_block(bits, 0, 8)
    bt = ops.BlockTensors.from_numpy(blk, "cuda")
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
    inds, scores, logits = ops.router_topk(bt, x, return_logits=True)
    ologits, oinds, oscores, _ = oracle.router(_oracle(blk, bits), blk.x, k=8)
    np.testing.assert_array_equal(logits.cpu().numpy(), ologits)
    np.testing.assert_array_equal(inds.cpu().numpy(), oinds)
    np.testing.assert_allclose(scores.cpu().numpy(), oscores, rtol=2e-5, atol=1e-7)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 8, 128])
def test_block_midpoints(T):
    """T <= 8: persistent decode kernel; T = 128: prefill router."""
    bits = 4
    blk = _midpoint_block(bits, 1, T)
    bt = ops.BlockTensors.from_numpy(blk, "cuda")
    x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
    out, inds, scores = ops.moe_block(bt, x, return_routing=True)
    ref, oinds, oscores, bound = oracle_block(_oracle(blk, bits), blk.x)
    np.testing.assert_array_equal(inds.cpu().numpy(), oinds)
    np.testing.assert_allclose(scores.cpu().numpy(), oscores, rtol=2e-5, atol=1e-7)
    assert_close(out.float().cpu().numpy(), ref, f"midpoint block T={T}", bound=bound)


@pytest.mark.gpu
def test_zero_tokens_route_to_lowest_indices():
    """An all-zero token has all-zero logits: a full tie, lowest indices win."""
    blk = inputs.make_block(8, seed=3, T=130)
    x = blk.x.copy()
    x[[0, 5, 129]] = 0
    blk = dataclasses.replace(blk, x=x)
    bt = ops.BlockTensors.from_numpy(blk, "cuda")
    xt = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
    for xs in (xt[:1], xt):  # decode kernel, prefill router
        inds, scores = ops.moe_block(bt, xs, return_routing=True)[1:]
        np.testing.assert_array_equal(inds[0].cpu().numpy(), np.arange(8))
        np.testing.assert_allclose(scores[0].cpu().numpy(), np.full(8, 0.125), rtol=1e-6)
    _, oinds, oscores, _ = oracle.router(_oracle(blk, 8), blk.x, k=8)
    np.testing.assert_array_equal(inds.cpu().numpy(), oinds)
    np.testing.assert_allclose(scores.cpu().numpy(), oscores, rtol=2e-5, atol=1e-7)


# ---------------------------------------------------------- 8-bit router
# Real Ornith checkpoints store mlp.gate and mlp.shared_expert_gate as 8-bit
# MLX affine (codes, bf16 scale and bias per 64 inputs).  A logit is then the
# bf16 rounding of the exact dot product with the dequantised rows.

def _q8_midpoint_block(bits, seed, T):
    """The midpoint construction with an 8-bit router: the three active
    inputs 0, 64 and 128 sit in three groups whose codes there are 0, so
    each weight is its group's bias; every other code is random and meets a
    zero activation."""
    blk = inputs.make_block(bits, seed=seed, T=T, router_bits=8)
    e = np.arange(E)
    base = (1.0 + (e % 128) / 128.0) * np.where(e < 128, 1.0, 0.5) * 2.0 ** -4
    half_ulp = np.where(e < 128, 2.0 ** -8, 2.0 ** -9) * 2.0 ** -4
    sign = np.array([1.0, -1.0, 0.0])[e % 3]
    q = blk.router_q.copy()
    for pos in (0, 64, 128):  # code 0 at the active inputs (byte pos % 4 of word pos / 4)
        q[:, pos // 4] &= np.uint32(~(0xFF << (8 * (pos % 4))) & 0xFFFFFFFF)
    b = np.zeros((E, H // 64), np.float32)
    b[:, 0], b[:, 1], b[:, 2] = base, half_ulp, sign * base * 2.0 ** -30
    s_t = np.array([1.0, -1.0, 0.0, 1.0, -1.0, 0.0, 2.0, -2.0])
    x = np.zeros((T, H), np.float32)
    x[:, 0] = 1.0
    x[:, 64] = 1.0
    x[:, 128] = s_t[np.arange(T) % 8]
    return dataclasses.replace(blk, x=f32_to_bf16_bits(x), router_q=q, router_b=f32_to_bf16_bits(b))


def test_q8_midpoint_logits_need_exact_rounding():
    """CPU: the 8-bit construction is exact in bf16 biases and still lands
    fp32 sums on the midpoints."""
    blk = _q8_midpoint_block(4, 0, 8)
    assert np.array_equal(bf16_bits_to_f32(blk.router_b)[:, 2],
                          (np.array([1.0, -1.0, 0.0])[np.arange(E) % 3]
                           * (1.0 + (np.arange(E) % 128) / 128.0) * np.where(np.arange(E) < 128, 1.0, 0.5)
                           * 2.0 ** -34).astype(np.float32))
    logits, _, _, _ = oracle.router(_oracle(blk, 4), blk.x, k=8)
    b = bf16_bits_to_f32(blk.router_b)
    f32 = (b[:, 0][None] + b[:, 1][None]).astype(np.float32) + np.zeros((8, 1), np.float32)
    naive = bf16_bits_to_f32(f32_to_bf16_bits(f32))
    assert (naive != logits).mean() > 0.2


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 8, 128])
def test_q8_router_logits_chain(T):
    """The chain router's logits (hi + lo bf16 MMAs, certified intervals,
    exact recompute from the codes) equal the oracle's bit for bit."""
    for blk in (inputs.make_block(4, seed=11, T=T, router_bits=8), _q8_midpoint_block(4, 2, T)):
        bt = ops.BlockTensors.from_numpy(blk, "cuda")
        assert bt.router_bits == 8 and bt.router_w.dtype == torch.uint32
        x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
        inds, scores, logits = ops.router_topk(bt, x, return_logits=True)
        ologits, oinds, oscores, _ = oracle.router(_oracle(blk, 4), blk.x, k=8)
        np.testing.assert_array_equal(logits.cpu().numpy(), ologits)
        np.testing.assert_array_equal(inds.cpu().numpy(), oinds)
        np.testing.assert_allclose(scores.cpu().numpy(), oscores, rtol=2e-5, atol=1e-7)


@pytest.mark.gpu
@pytest.mark.parametrize("bits,T", [(4, 1), (8, 1), (4, 2), (8, 2), (4, 8), (4, 128), (8, 300)])
def test_q8_router_block(bits, T):
    """The whole block with an 8-bit router and shared gate: T = 1, 2 the
    persistent decode kernel (T = 2 at 8 bits the chain), 8 the chain, 128
    and 300 the prefill path (split rows, two-pass router GEMM)."""
    for blk in (inputs.make_block(bits, seed=12 + T, T=T, router_bits=8), _q8_midpoint_block(bits, 3, T)):
        bt = ops.BlockTensors.from_numpy(blk, "cuda")
        x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).cuda()
        out, inds, scores = ops.moe_block(bt, x, return_routing=True)
        rows = np.arange(T) if T <= 16 else np.linspace(0, T - 1, 16).astype(int)
        ref, oinds, oscores, bound = oracle_block(_oracle(blk, bits), np.ascontiguousarray(blk.x[rows]))
        np.testing.assert_array_equal(inds.cpu().numpy()[rows], oinds)
        np.testing.assert_allclose(scores.cpu().numpy()[rows], oscores, rtol=2e-5, atol=1e-7)
        assert_close(out.float().cpu().numpy()[rows], ref, f"q8 router block q{bits} T={T}", bound=bound)
