"""Tolerance checks shared by the parity tests.

Block and SwitchGLU outputs are bf16 (or fp32); they are compared with the
oracle's fp32-accumulated result, element by element, by the bound the
reference's correctness criterion states:

* relative L2 error ``||out - ref|| / ||ref|| <= 5e-3``;
* every element ``|out - ref| <= max(2 ulp_bf16(|ref|), bound)``: two bf16
  units in the last place at the element's OWN magnitude, with one floor,
  ``bound``, the element's fp32 accumulation error bound from the oracle
  (``oracle.block_bound``): every dot product of the block (gate/up over H,
  down over I, the combine over the slots) may err by the classical
  any-order fp32 summation bound gamma_n * sum|terms| (u = 2^-24), and that
  error is propagated through SwiGLU, the down projection and the weighted
  combine.  An element is held to the floor only where its exact value
  cancels to less than its fp32 evaluation can resolve.

``strict_ulp_max`` (the largest error in ulps of the element's own value,
no floor) and ``floor_elements`` (how many elements needed the floor) are
printed with every comparison.

Routing must match exactly: the same expert indices in the same slot order.
"""
from __future__ import annotations

import numpy as np

REL_L2 = 5e-3
ULPS = 2.0


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """One bf16 unit in the last place at |v| (normal range)."""
    v = np.maximum(np.abs(np.asarray(v, np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(v)) - 7)


def compare(out, ref, bound=None, rel_l2: float = REL_L2, ulps: float = ULPS) -> dict:
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(out - ref)
    own = ulps * bf16_ulp(ref)
    tol = own if bound is None else np.maximum(own, np.asarray(bound, np.float64))
    ratio = err / tol
    stats = {
        "rel_l2": float(np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30)),
        "max_abs": float(np.max(err)) if err.size else 0.0,
        "strict_ulp_max": float(np.max(err / bf16_ulp(ref))) if err.size else 0.0,
        "max_tol_ratio": float(np.max(ratio)) if err.size else 0.0,
        "floor_elements": int(np.count_nonzero(err > own)),
        "elements": int(err.size),
    }
    stats["ok"] = bool(stats["rel_l2"] <= rel_l2 and stats["max_tol_ratio"] <= 1.0)
    return stats


def assert_close(out, ref, what: str = "output", bound=None, **kw):
    s = compare(out, ref, bound=bound, **kw)
    print(f"{what}: strict_ulp_max={s['strict_ulp_max']:.3f} rel_l2={s['rel_l2']:.2e} "
          f"floor_elements={s['floor_elements']}/{s['elements']} max_tol_ratio={s['max_tol_ratio']:.3f}")
    assert s["ok"], f"{what}: {s}"
    return s


def assert_close_gpu_pair(a, b, what: str = "output"):
    """Cross-check of two GPU paths of the same block (no oracle in the
    loop), e.g. expert-parallel against single-GPU.  Each side is already
    held to the oracle bound in its own test; here elements below the
    tensor's RMS are measured at the RMS (two correct results can differ by
    both errors, and without the oracle's magnitudes there is no per-element
    floor).  Never used for an oracle comparison."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    rms = float(np.sqrt(np.mean(b * b))) if b.size else 0.0
    err = np.abs(a - b)
    tol = 2 * ULPS * bf16_ulp(np.maximum(np.abs(b), rms))
    rel = float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
    ratio = float(np.max(err / tol)) if err.size else 0.0
    print(f"{what} (GPU pair): rel_l2={rel:.2e} max_ratio={ratio:.3f}")
    assert rel <= REL_L2 and ratio <= 1.0, f"{what}: rel_l2={rel} max_ratio={ratio}"


def oracle_block(w, x, k: int = 8):
    """The oracle's block output, routing and per-element fp32 error bound
    for x: (ref [T,H], inds [T,k], scores [T,k], bound [T,H])."""
    from oracle import oracle

    _, inds, scores, sg = oracle.router(w, x, k=k)
    ref, oinds, oscores = oracle.moe_block(w, x, k=k)
    bound = oracle.block_bound(w, x, inds, scores, sg if w.sgu_w is not None else None)
    return ref, oinds, oscores, bound
