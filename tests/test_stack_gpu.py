"""Decoder stack of MoE blocks (configuration 4): the fused residual-add +
RMSNorm glue against numpy, and a short stack checked layer by layer against
the oracle (each block on the GPU's own input, so routing must match exactly
at every layer; each glue step on the GPU's own previous values)."""
import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import inputs, ops, stack
from runnel_b200.quant import bf16_bits_to_f32, f32_to_bf16_bits
from tests._parity import assert_close, oracle_block

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits)).view(torch.int16).view(torch.bfloat16).to(DEV)


def _ulp_steps(a_bits, b_bits):
    """bf16 steps between two bf16 arrays of the same sign (ordered integers)."""
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    a = np.where(a & 0x8000, 0x8000 - (a & 0x7FFF), a + 0x8000)
    b = np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), b + 0x8000)
    return np.abs(a - b)


def test_add_rmsnorm_matches_numpy():
    rng = np.random.default_rng(7)
    T, H = 5, 2048
    x = f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    y = f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32) * 0.3)
    w = f32_to_bf16_bits((1 + 0.02 * rng.standard_normal(H)).astype(np.float32))
    for yy in (None, y):
        xo = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
        xn = torch.empty_like(xo)
        stack.add_rmsnorm(_dev(x), None if yy is None else _dev(yy), _dev(w), xo, xn)
        rxo, rxn = stack.reference_add_rmsnorm(x, yy, w)
        np.testing.assert_array_equal(_bits(xo), rxo)
        steps = _ulp_steps(_bits(xn), rxn)
        assert steps.max() <= 1 and (steps > 0).mean() < 0.01


def test_stack_layer_by_layer_matches_oracle():
    L, bits = 3, 4
    blks = [inputs.make_block(bits, seed=3000 + l, T=1) for l in range(L)]
    layers = [ops.BlockTensors.from_numpy(b, DEV) for b in blks]
    norms_bits = [f32_to_bf16_bits(b.norm_w) for b in blks]
    st = stack.LayerStack(layers, [_dev(n) for n in norms_bits], ws=ops.Workspace(DEV))
    ws = [oracle.BlockWeights(bits=bits, group=64, **b.weight_fields()) for b in blks]
    x = _dev(blks[0].x)
    for tok in range(2):  # two sequential tokens: the second starts from the first's output
        rec = []
        out = st.forward(x, record=rec)
        xa_prev = _bits(x)
        for l, (xa, xn, y) in enumerate(rec):
            # glue into layer l: residual stream and its norm
            if l == 0:
                rxa, rxn = stack.reference_add_rmsnorm(xa_prev, None, norms_bits[0])
            else:
                rxa, rxn = stack.reference_add_rmsnorm(_bits(rec[l - 1][0]), _bits(rec[l - 1][2]), norms_bits[l])
            np.testing.assert_array_equal(_bits(xa), rxa)
            assert _ulp_steps(_bits(xn), rxn).max() <= 1
            # block l on the GPU's own input
            ref, oinds, _, bound = oracle_block(ws[l], _bits(xn))
            assert_close(y.float().cpu().numpy(), ref, f"token {tok} layer {l}", bound=bound)
        last = stack.reference_add_rmsnorm(_bits(rec[-1][0]), _bits(rec[-1][2]), norms_bits[-1])[0]
        np.testing.assert_array_equal(_bits(out), last)
        x = out


def test_stack_graph_replay_chains_tokens():
    """The benchmark's form: one token's layers captured once, replayed per token."""
    layers, norms = stack.synthetic_layers(2, 4, seed=3, device=DEV)
    st = stack.LayerStack(layers, norms, ws=ops.Workspace(DEV))
    x0 = torch.from_numpy(inputs.make_tokens(3, 1)).view(torch.int16).view(torch.bfloat16).to(DEV)
    # eager chain
    xs = x0.clone()
    eager = []
    for _ in range(3):
        xs = st.forward(xs).clone()
        eager.append(xs)
    # graph chain
    xin = x0.clone()
    xout = torch.empty_like(xin)
    st.forward(xin, out=xout)  # allocate the workspace outside the capture
    xin.copy_(x0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            st.forward(xin, out=xout)
            xin.copy_(xout)
    for i in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(xout, eager[i])


@pytest.mark.parametrize("T", [1, 2, 3])
def test_fused_layer_glue_is_bit_identical(T):
    """rnb_moe_block_norm_fwd (glue inside the persistent launch for T <= 2, the
    glue kernel then the block otherwise) equals rnb_add_rmsnorm + the block."""
    L, bits = 3, 4
    blks = [inputs.make_block(bits, seed=4000 + l, T=T) for l in range(L)]
    layers = [ops.BlockTensors.from_numpy(b, DEV) for b in blks]
    norms = [_dev(f32_to_bf16_bits(b.norm_w)) for b in blks]
    x = _dev(blks[0].x)
    fused = stack.LayerStack(layers, norms, ws=ops.Workspace(DEV)).forward(x)
    xa = torch.empty_like(x)
    xn = torch.empty_like(x)
    y = torch.empty_like(x)
    ws = ops.Workspace(DEV)
    stack.add_rmsnorm(x, None, norms[0], xa, xn)
    for l in range(L):
        ops.moe_block(layers[l], xn, ws=ws, out=y)
        stack.add_rmsnorm(xa, y, norms[l + 1] if l + 1 < L else norms[l], xa, xn)
    assert torch.equal(_dev(_bits(fused)), _dev(_bits(xa)))


def test_config4_forty_layers_eight_tokens_against_oracle():
    """Benchmark configuration 4 as benchmarked: the 40 canonical q4 layers
    (inputs.make_block(4, seed=3000 + l)) and 8 sequential batch-1 tokens,
    each token's input the previous token's output.  Every layer's block is
    checked against the oracle on the GPU's own input, and every glue step
    against numpy, so error growth over the 40 residual layers is covered."""
    L, bits, seed, ntok = 40, 4, 3, 8
    layers, norms = stack.canonical_layers(L, bits, seed, DEV)
    st = stack.LayerStack(layers, norms, ws=ops.Workspace(DEV))
    norms_bits = [_bits(n) for n in norms]
    x = _dev(inputs.make_tokens(seed, 1))
    xn_in = np.zeros((L, ntok, 2048), np.uint16)
    y_out = np.zeros((L, ntok, 2048), np.float32)
    for tok in range(ntok):
        rec = []
        out = st.forward(x, record=rec)
        prev = _bits(x)
        for l, (xa, xn, y) in enumerate(rec):
            if l == 0:
                rxa, rxn = stack.reference_add_rmsnorm(prev, None, norms_bits[0])
            else:
                rxa, rxn = stack.reference_add_rmsnorm(_bits(rec[l - 1][0]), _bits(rec[l - 1][2]), norms_bits[l])
            np.testing.assert_array_equal(_bits(xa), rxa)
            assert _ulp_steps(_bits(xn), rxn).max() <= 1
            xn_in[l, tok] = _bits(xn)[0]
            y_out[l, tok] = y.float().cpu().numpy()[0]
        last = stack.reference_add_rmsnorm(_bits(rec[-1][0]), _bits(rec[-1][2]), norms_bits[-1])[0]
        np.testing.assert_array_equal(_bits(out), last)
        x = out
    del layers, st
    torch.cuda.empty_cache()
    worst = 0.0
    for l0 in range(0, L, 8):
        seeds = [inputs.stack_layer_seed(seed, l) for l in range(l0, min(L, l0 + 8))]
        for i, b in enumerate(inputs.make_blocks(bits, seeds, T=1)):
            l = l0 + i
            w = oracle.BlockWeights(bits=bits, group=64, **b.weight_fields())
            ref, _, _, bound = oracle_block(w, xn_in[l])
            s = assert_close(y_out[l], ref, f"config 4 layer {l}, {ntok} tokens", bound=bound)
            worst = max(worst, s["max_tol_ratio"])
    print(f"config 4: worst max_tol_ratio over 40 layers x {ntok} tokens = {worst:.3f}")
