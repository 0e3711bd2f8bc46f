"""The vectorised CPU baseline (oracle/rnb_cpu_fast.c) against the
exact-order oracle.

bench.py times this restatement as its CPU baseline and reference arm, so it
must compute the same block: the same expert indices and routing weights
(bit for bit: its fp64 router gives the oracle's bf16 logits), and outputs
within the parity tolerance of tests/_parity.py (fp32 in another summation
order).  Both its AVX2/FMA kernels and its plain C loops are checked."""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle
from runnel_b200 import inputs

from tests._parity import assert_close, oracle_block

CASES = [(8, 1, 16), (4, 1, 16), (4, 5, 16), (8, 40, 8), (4, 67, 16)]


@pytest.mark.parametrize("bits,T,router_bits", CASES)
def test_fast_block_matches_oracle(bits, T, router_bits):
    blk = inputs.make_block(bits, seed=11 + T, T=T, router_bits=router_bits)
    w = oracle.BlockWeights(bits=bits, group=64, **blk.weight_fields())
    ref, oinds, oscores, bound = oracle_block(w, blk.x)
    out, inds, scores = oracle.moe_block_fast(w, blk.x)
    np.testing.assert_array_equal(inds, oinds)
    np.testing.assert_array_equal(scores, oscores)
    assert_close(out, ref, f"CPU baseline q{bits} T={T} router {router_bits}", bound=bound)


def test_fast_block_adversarial_routing():
    """A quarter of the tokens on one expert: a many-token expert next to
    single-token ones (both of the restatement's expert paths)."""
    blk = inputs.make_block(8, seed=21, T=48, adversarial_frac=0.25)
    w = oracle.BlockWeights(bits=8, group=64, **blk.weight_fields())
    ref, oinds, _, bound = oracle_block(w, blk.x)
    out, inds, _ = oracle.moe_block_fast(w, blk.x)
    np.testing.assert_array_equal(inds, oinds)
    assert_close(out, ref, "CPU baseline adversarial", bound=bound)


def test_fast_block_small_bank():
    """A 16-expert bank of other sizes (H 512, I 256): most experts hold many
    tokens, so the panel tiles carry the block."""
    blk = inputs.make_block(4, seed=8, T=37, H=512, I=256, E=16)
    w = oracle.BlockWeights(bits=4, group=64, **blk.weight_fields())
    ref, oinds, oscores, bound = oracle_block(w, blk.x)
    out, inds, scores = oracle.moe_block_fast(w, blk.x)
    np.testing.assert_array_equal(inds, oinds)
    np.testing.assert_array_equal(scores, oscores)
    assert_close(out, ref, "CPU baseline, 16-expert bank", bound=bound)


def test_fast_block_empty_and_threads():
    blk = inputs.make_block(4, seed=2, T=3)
    w = oracle.BlockWeights(bits=4, group=64, **blk.weight_fields())
    out, inds, _ = oracle.moe_block_fast(w, blk.x[:0])
    assert out.shape == (0, blk.H) and inds.shape == (0, 8)
    a = oracle.moe_block_fast(w, blk.x, nthreads=1)[0]
    b = oracle.moe_block_fast(w, blk.x, nthreads=4)[0]
    np.testing.assert_array_equal(a, b)  # the partition never changes a sum's order


def test_fast_block_plain_c_loops():
    """The same checks with the AVX2 kernels switched off (a fresh process:
    the choice is made once per process)."""
    code = (
        "import numpy as np\n"
        "from oracle import oracle\n"
        "from runnel_b200 import inputs\n"
        "from tests._parity import assert_close, oracle_block\n"
        "assert not oracle.fast_simd()\n"
        "for bits, T in ((8, 2), (4, 7)):\n"
        "    blk = inputs.make_block(bits, seed=5, T=T)\n"
        "    w = oracle.BlockWeights(bits=bits, group=64, **blk.weight_fields())\n"
        "    ref, oinds, oscores, bound = oracle_block(w, blk.x)\n"
        "    out, inds, scores = oracle.moe_block_fast(w, blk.x)\n"
        "    np.testing.assert_array_equal(inds, oinds)\n"
        "    np.testing.assert_array_equal(scores, oscores)\n"
        "    assert_close(out, ref, f'plain C q{bits} T={T}', bound=bound)\n"
    )
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, RNB_CPU_NO_SIMD="1", PYTHONPATH=root)
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
