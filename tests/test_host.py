"""Host-side logic: MLX affine packing, synthetic inputs, module transforms."""
import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import inputs, quant
from runnel_b200 import mlx as rmlx
from runnel_b200 import switch_layers as sl


@pytest.mark.parametrize("bits", [4, 8])
def test_pack_unpack_round_trip(bits):
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 1 << bits, size=(3, 128), dtype=np.uint32)
    words = quant.pack_codes(codes, bits)
    assert words.shape == (3, 128 * bits // 32)
    np.testing.assert_array_equal(quant.unpack_codes(words, bits), codes)
    # LSB-first: code 0 in the low bits of word 0
    assert (words[0, 0] & ((1 << bits) - 1)) == codes[0, 0]


def test_bf16_rounding_matches_oracle_and_torch():
    v = np.random.default_rng(1).standard_normal(10000).astype(np.float32) * 100
    v[:4] = [np.inf, -np.inf, 0.0, -0.0]
    a = quant.f32_to_bf16_bits(v)
    np.testing.assert_array_equal(a, oracle.f32_to_bf16(v))
    t = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(a, t)


@pytest.mark.parametrize("bits", [4, 8])
def test_dequant_matches_oracle_matvec(bits):
    rng = np.random.default_rng(2)
    w = rng.standard_normal((16, 256)).astype(np.float32)
    words, s, b = quant.quantize(w, bits)
    deq = quant.dequantize(words, s, b, bits)
    assert np.max(np.abs(deq - w)) < (np.max(w) - np.min(w)) / ((1 << bits) - 1)
    x = rng.standard_normal(256).astype(np.float32)
    y = oracle.affine_matvec(words, s, b, x, bits, 64)
    np.testing.assert_allclose(y, deq @ x, rtol=1e-4, atol=1e-4)


def test_synthetic_block_is_deterministic_and_all_nibbles_random():
    a = inputs.make_block(4, seed=7, T=2, H=512, I=256, E=8)
    b = inputs.make_block(4, seed=7, T=2, H=512, I=256, E=8)
    for name, arr in a.weight_fields().items():
        np.testing.assert_array_equal(arr, getattr(b, name), err_msg=name)
    codes = quant.unpack_codes(a.gu_w, 4)
    odd = codes.reshape(-1)[1::2]
    assert odd.max() == 15 and odd.mean() > 6  # odd nibbles are populated (unlike the reference KATs)
    s = quant.bf16_bits_to_f32(a.gu_s)
    assert 0.00099 <= s.min() and s.max() <= 0.0101  # U(0.001, 0.01) after bf16 rounding


def test_skews_are_data_only():
    z = inputs.make_block(8, seed=2, T=64, H=512, I=256, E=16, skew="zipf")
    plain = inputs.make_block(8, seed=2, T=64, H=512, I=256, E=16)
    np.testing.assert_array_equal(z.gu_w, plain.gu_w)
    assert np.all(quant.bf16_bits_to_f32(z.x[:, -1]) == 1.0)
    adv = inputs.make_block(8, seed=4, T=256, H=512, I=256, E=16, skew="adversarial")
    _, inds, _, _ = oracle.router(oracle.BlockWeights(bits=8, group=64, **_routed(adv)), adv.x, k=4)
    hot = adv.meta["hot_expert"]
    frac = np.mean(np.any(inds == hot, axis=1))
    assert frac >= 0.2


def _routed(blk):
    return {k: v for k, v in blk.weight_fields().items()}


def _switch_modules(E=4, I=256, H=512, bits=4, bias_mismatch=False):
    rng = np.random.default_rng(3)
    def lin(rows, K):
        w = torch.from_numpy(rng.integers(0, 1 << 32, size=(E, rows, K * bits // 32), dtype=np.uint32))
        s = torch.ones(E, rows, K // 64, dtype=torch.bfloat16)
        return sl.QuantizedSwitchLinear(w, s, s.clone(), bits=bits)
    up, gate, down = lin(I, H), lin(I, H), lin(H, I)
    if bias_mismatch:
        gate.biases = None
    return sl.SwitchGLU(gate, up, down)


def test_fused_switchglu_packs_up_then_gate():
    old = _switch_modules()
    fused = sl.FusedQuantizedSwitchGLU(old)
    I = old.up_proj.weight.shape[1]
    assert torch.equal(fused.weight[:, :I], old.up_proj.weight)
    assert torch.equal(fused.weight[:, I:], old.gate_proj.weight)
    assert fused.bits == 4 and fused.group_size == 64 and fused.mode == "affine"
    assert fused.down_proj is old.down_proj
    assert "bias" not in fused and fused.get("biases") is not None


def test_fuse_rejects_mismatched_formats():
    old = _switch_modules()
    old.gate_proj.bits = 8
    with pytest.raises(ValueError, match="routed gate/up quantization formats differ"):
        sl.FusedQuantizedSwitchGLU(old)
    with pytest.raises(ValueError, match="affine-bias formats differ"):
        sl.FusedQuantizedSwitchGLU(_switch_modules(bias_mismatch=True))


def test_fuse_routed_gate_up_walks_layers():
    class Obj:
        pass

    model = Obj()
    model.language_model = Obj()
    model.language_model.layers = []
    for _ in range(3):
        layer = Obj()
        layer.mlp = Obj()
        layer.mlp.switch_mlp = _switch_modules()
        model.language_model.layers.append(layer)
    assert rmlx.fuse_routed_gate_up(model) == 3
    assert all(isinstance(l.mlp.switch_mlp, sl.FusedQuantizedSwitchGLU) for l in model.language_model.layers)
    bad = Obj()
    bad.language_model = Obj()
    layer = Obj()
    layer.mlp = Obj()
    layer.mlp.switch_mlp = Obj()
    layer.mlp.switch_mlp.gate_proj = torch.nn.Linear(2, 2)
    bad.language_model.layers = [layer]
    with pytest.raises(ValueError, match="not quantized as expected"):
        rmlx.fuse_routed_gate_up(bad)


def test_oracle_block_routing_semantics():
    blk = inputs.make_block(8, seed=5, T=4, H=512, I=256, E=16)
    w = oracle.BlockWeights(bits=8, group=64, **_routed(blk))
    logits, inds, scores, sg = oracle.router(w, blk.x, k=4)
    for t in range(4):
        order = sorted(range(16), key=lambda e: (-logits[t, e], e))
        assert list(inds[t]) == order[:4]
        p = np.exp(logits[t] - logits[t].max())
        p /= p.sum()
        np.testing.assert_allclose(scores[t], p[inds[t]] / p[inds[t]].sum(), rtol=1e-5)
    out, i2, s2 = oracle.moe_block(w, blk.x, k=4)
    y = oracle.switchglu(w, blk.x, inds)
    ys = oracle.shared_expert(w, blk.x)
    ref = np.einsum("tk,tkh->th", scores, y) + sg[:, None] * ys
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-4)


def test_oracle_eight_bit_router_is_the_exact_dot_with_dequantised_rows():
    # an 8-bit router's logit is the bf16 rounding of the exact dot product
    # of the token with the dequantised row s * code + b (every term exact in
    # fp64 here); the shared gate is fp32 with the same weights
    blk = inputs.make_block(4, seed=7, T=5, H=512, I=256, E=16, router_bits=8)
    assert blk.router_q.shape == (16, 128) and blk.sgate_q.reshape(-1).shape == (128,)
    w = oracle.BlockWeights(bits=4, group=64, **_routed(blk))
    logits, inds, scores, sg = oracle.router(w, blk.x, k=4)
    def exact_rows(q, s_, b_):
        codes = quant.unpack_codes(q, 8).astype(np.float64)
        sc = np.repeat(quant.bf16_bits_to_f32(s_).astype(np.float64), 64, axis=-1)
        bi = np.repeat(quant.bf16_bits_to_f32(b_).astype(np.float64), 64, axis=-1)
        return codes * sc + bi
    wq = exact_rows(blk.router_q, blk.router_s, blk.router_b)
    x = quant.bf16_bits_to_f32(blk.x).astype(np.float64)
    exact = x @ wq.T
    # one rounding, fp64 -> bf16 (8 significant bits, nearest, ties to even)
    m, e = np.frexp(exact)
    np.testing.assert_array_equal(logits, np.ldexp(np.round(m * 256.0), e - 8).astype(np.float32))
    gq = exact_rows(blk.sgate_q.reshape(1, -1), blk.sgate_s.reshape(1, -1), blk.sgate_b.reshape(1, -1))
    np.testing.assert_allclose(sg, 1.0 / (1.0 + np.exp(-(x @ gq.T)[:, 0])), rtol=1e-5)
    # the quantized rows differ from the bf16 ones: the two routers are not the same
    l16, _, _, _ = oracle.router(oracle.BlockWeights(bits=4, group=64, **{
        k: v for k, v in _routed(blk).items() if k not in ("router_bits", "router_q", "router_s", "router_b",
                                                          "sgate_q", "sgate_s", "sgate_b")}), blk.x, k=4)
    assert not np.array_equal(l16, logits)


def test_prepared_block_call_refuses_host_tensors():
    # the prepared call builds the same descriptor as every other entry point:
    # a bank held in host memory fails loudly instead of running anywhere else
    from runnel_b200 import ops

    blk = inputs.make_block(4, seed=3, T=1, H=512, I=256, E=16)
    bt = ops.BlockTensors(bits=4, **{f: torch.from_numpy(np.ascontiguousarray(getattr(blk, f)))
                                    for f in ("gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b")})
    with pytest.raises(ValueError, match="must be CUDA tensors"):
        ops.BlockCall(bt, 1)
    with pytest.raises(ValueError, match="T must be positive"):
        ops.BlockCall(bt, 0)
