"""The allocation-free block entry point, rnb_moe_block_fwd_noalloc.

Some callers cannot call cudaMalloc -- a host capturing a CUDA graph, where
allocation is not allowed, or an engine plugin that owns no allocator -- so
they cannot provide the workspace rnb_moe_block_fwd needs.  The no-alloc
variant keeps its scratch in a static device array of the library instead.
Here it is called through the C ABI and must agree with the workspace entry
point on the same inputs, on two calls in a row (the second with other
tokens, so nothing left in the shared scratch by the first can leak in).
The status bits of these calls are read back with rnb_moe_noalloc_status,
since the caller has no workspace to pass to rnb_moe_status.
This file sorts last so a run that stops at the first failure has run every
other test before it.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import _lib, inputs, ops
from tests._parity import assert_close, oracle_block


def test_noalloc_rejects_shapes_beyond_its_scratch():
    # E=512, k=16, I=1024 need more scratch than the static array holds; the
    # call is refused before any device work (the pointers are never used)
    fake = 256
    d = _lib.RnbMoeDesc(T=1, H=2048, I=1024, E=512, E_total=512, k=16, bits=8, group=64,
                        gu_w=fake, gu_s=fake, gu_b=fake, dn_w=fake, dn_s=fake, dn_b=fake,
                        router_w=fake)
    rc = _lib.load().rnb_moe_block_fwd_noalloc(ctypes.byref(d), fake, fake, None, None, None)
    assert rc == -3  # RNB_ERR_WORKSPACE
    assert "static scratch" in _lib.load().rnb_last_error().decode()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice():
    blk = inputs.make_block(4, seed=1, T=5)
    bt = ops.BlockTensors.from_numpy(blk, "cuda")
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    xs = [blk.x, inputs.make_tokens(1, 3)]
    for x_np in xs:
        x = torch.from_numpy(x_np).view(torch.int16).view(torch.bfloat16).cuda()
        T = x.shape[0]
        ref, rinds, rscores = ops.moe_block(bt, x, return_routing=True)
        out = torch.empty_like(x)
        inds = torch.empty((T, 8), dtype=torch.int32, device="cuda")
        scores = torch.empty((T, 8), dtype=torch.float32, device="cuda")
        d = bt.desc(T, 8)
        rc = lib.rnb_moe_block_fwd_noalloc(ctypes.byref(d), x.data_ptr(), out.data_ptr(),
                                           inds.data_ptr(), scores.data_ptr(), stream)
        assert rc == 0, lib.rnb_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(inds, rinds)
        np.testing.assert_allclose(scores.cpu().numpy(), rscores.cpu().numpy(), rtol=2e-5, atol=1e-7)
        assert torch.equal(out, ref), "the no-alloc call differs from the workspace call"
        # and on its own against the CPU oracle
        w = oracle.BlockWeights(bits=4, group=64, **blk.weight_fields())
        oref, oinds, _, bound = oracle_block(w, x_np)
        np.testing.assert_array_equal(inds.cpu().numpy(), oinds)
        assert_close(out.float().cpu().numpy(), oref, "noalloc vs oracle", bound=bound)
    # the two calls set no status bit (no timeout, no bad index), and reading
    # the status clears it
    status = ctypes.c_uint32(0xFFFFFFFF)
    rc = lib.rnb_moe_noalloc_status(ctypes.byref(status), stream)
    assert rc == 0, lib.rnb_last_error().decode()
    assert status.value == 0
    rc = lib.rnb_moe_noalloc_status(ctypes.byref(status), stream)
    assert rc == 0 and status.value == 0
