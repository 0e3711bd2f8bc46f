"""Tolerance checks shared by the parity tests.

Block and SwitchGLU outputs are bf16; they are compared with the oracle's
fp32-accumulated result by two bounds (stated once here, used everywhere):

* relative L2 error ``||out - ref|| / ||ref|| <= 5e-3``;
* element-wise ``|out - ref| <= 2 ulp_bf16(max(|ref|, rms(ref)))`` -- two
  bf16 units in the last place at the element's own magnitude, with
  magnitudes below the tensor's RMS measured at the RMS (an element far
  below the typical output magnitude is a cancellation, and its absolute
  error is that of the typical terms that cancelled).

Routing must match exactly: the same expert indices in the same slot order.
"""
from __future__ import annotations

import numpy as np

REL_L2 = 5e-3
ULPS = 2.0


def bf16_ulp(mag: np.ndarray) -> np.ndarray:
    mag = np.maximum(np.abs(np.asarray(mag, np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(mag)) - 7)


def compare(out, ref, rel_l2: float = REL_L2, ulps: float = ULPS) -> dict:
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    err = out - ref
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    mag = np.maximum(np.abs(ref), rms)
    tol = ulps * bf16_ulp(mag)
    ratio = np.abs(err) / tol
    stats = {
        "rel_l2": float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30)),
        "max_abs": float(np.max(np.abs(err))) if err.size else 0.0,
        "max_ulp_ratio": float(np.max(ratio)) if err.size else 0.0,
        "strict_ulp_max": float(np.max(np.abs(err) / bf16_ulp(ref))) if err.size else 0.0,
        "rms_ref": rms,
    }
    stats["ok"] = bool(stats["rel_l2"] <= rel_l2 and stats["max_ulp_ratio"] <= 1.0)
    return stats


def assert_close(out, ref, what: str = "output", **kw):
    s = compare(out, ref, **kw)
    assert s["ok"], f"{what}: {s}"
    return s
