"""ctypes front end of the CPU oracle (``librnb_oracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU legs of ``bench.py`` as the checker.  The product package
``runnel_b200`` never imports it.

The arithmetic lives in ``rnb_oracle.c``; this module only marshals numpy
arrays.  Weight layout is MLX affine: uint32 words with ``32 // bits`` codes
packed LSB-first, bf16 scales and biases per 64-element group (stored here as
raw ``uint16`` bit patterns).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "librnb_oracle.so")
_lib = None

_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)


class _Block(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("T", "H", "I", "E", "k", "bits", "group")] + [
        ("x", _u16p),
        ("router_w", _u16p),
        ("shared_gate_w", _u16p),
        ("gu_w", _u32p), ("gu_s", _u16p), ("gu_b", _u16p),
        ("dn_w", _u32p), ("dn_s", _u16p), ("dn_b", _u16p),
        ("sgu_w", _u32p), ("sgu_s", _u16p), ("sgu_b", _u16p),
        ("sdn_w", _u32p), ("sdn_s", _u16p), ("sdn_b", _u16p),
        ("router_bits", ctypes.c_int),
        ("router_q", _u32p), ("router_s", _u16p), ("router_b", _u16p),
        ("sgate_q", _u32p), ("sgate_s", _u16p), ("sgate_b", _u16p),
    ]


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    srcs = ("rnb_oracle.c", "rnb_cpu_fast.c", "rnb_oracle.h", "Makefile")
    if force or not os.path.exists(_LIB_PATH) or any(
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, f)) for f in srcs
    ):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.rnbo_f32_to_bf16.restype = ctypes.c_uint16
        _lib.rnbo_f32_to_bf16.argtypes = [ctypes.c_float]
        _lib.rnbo_bf16_to_f32.restype = ctypes.c_float
        _lib.rnbo_bf16_to_f32.argtypes = [ctypes.c_uint16]
    return _lib


def _p(a: np.ndarray | None, t):
    if a is None:
        return ctypes.cast(None, t)
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(t)


def nthreads_default() -> int:
    return os.cpu_count() or 1


# ------------------------------------------------------------ bf16 helpers


def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().rnbo_f32_to_bf16_array(_p(a, _f32p), _p(out, _u16p), ctypes.c_size_t(a.size))
    return out


def bf16_to_f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    out = np.empty(a.shape, dtype=np.float32)
    lib().rnbo_bf16_to_f32_array(_p(a, _u16p), _p(out, _f32p), ctypes.c_size_t(a.size))
    return out


# ------------------------------------------------------------ MoE block


@dataclass
class BlockWeights:
    """Numpy view of one sparse-MoE block in MLX layout (bf16 as uint16)."""

    bits: int
    group: int
    router_w: np.ndarray  # [E,H] u16
    gu_w: np.ndarray  # [E,2I,H*bits/32] u32  (rows 0..I-1 up, I..2I-1 gate)
    gu_s: np.ndarray  # [E,2I,H/group] u16
    gu_b: np.ndarray
    dn_w: np.ndarray  # [E,H,I*bits/32] u32
    dn_s: np.ndarray  # [E,H,I/group] u16
    dn_b: np.ndarray
    shared_gate_w: np.ndarray | None = None  # [H] u16
    sgu_w: np.ndarray | None = None  # [2I,H*bits/32]
    sgu_s: np.ndarray | None = None
    sgu_b: np.ndarray | None = None
    sdn_w: np.ndarray | None = None  # [H,I*bits/32]
    sdn_s: np.ndarray | None = None
    sdn_b: np.ndarray | None = None
    # 8-bit affine router and shared gate (router_bits=8): codes [E,H/4] /
    # [H/4], bf16 scales and biases [E,H/64] / [H/64]; router_w and
    # shared_gate_w are then unused
    router_bits: int = 16
    router_q: np.ndarray | None = None
    router_s: np.ndarray | None = None
    router_b: np.ndarray | None = None
    sgate_q: np.ndarray | None = None
    sgate_s: np.ndarray | None = None
    sgate_b: np.ndarray | None = None

    @property
    def E(self) -> int:
        return self.gu_w.shape[0]

    @property
    def H(self) -> int:
        return self.dn_w.shape[1]

    @property
    def I(self) -> int:  # noqa: E743 - matches the model's name for the size
        return self.gu_w.shape[1] // 2


def _block_struct(w: BlockWeights, x: np.ndarray, k: int, keep: list) -> _Block:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    keep.append(x)
    T = x.shape[0]
    arrays = {}
    for name in ("router_w", "gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b", "shared_gate_w",
                 "sgu_w", "sgu_s", "sgu_b", "sdn_w", "sdn_s", "sdn_b",
                 "router_q", "router_s", "router_b", "sgate_q", "sgate_s", "sgate_b"):
        a = getattr(w, name)
        if a is not None:
            a = np.ascontiguousarray(a)
            keep.append(a)
        arrays[name] = a
    u32 = {"gu_w", "dn_w", "sgu_w", "sdn_w", "router_q", "sgate_q"}
    kw = {n: _p(a, _u32p if n in u32 else _u16p) for n, a in arrays.items()}
    return _Block(T=T, H=w.H, I=w.I, E=w.E, k=k, bits=w.bits, group=w.group, x=_p(x, _u16p),
                  router_bits=w.router_bits, **kw)


def router(w: BlockWeights, x: np.ndarray, k: int = 8, nthreads: int | None = None):
    """Returns (logits_bf16_as_f32 [T,E], inds [T,k] int32, scores [T,k], shared_gate [T])."""
    keep: list = []
    d = _block_struct(w, x, k, keep)
    T = d.T
    logits = np.empty((T, w.E), np.float32)
    inds = np.empty((T, k), np.int32)
    scores = np.empty((T, k), np.float32)
    sg = np.empty((T,), np.float32)
    rc = lib().rnbo_router(ctypes.byref(d), _p(logits, _f32p), _p(inds, _i32p), _p(scores, _f32p),
                           _p(sg, _f32p), nthreads or nthreads_default())
    if rc:
        raise ValueError(f"oracle router rejected the block (rc={rc})")
    return logits, inds, scores, sg


def switchglu(w: BlockWeights, x: np.ndarray, inds: np.ndarray, nthreads: int | None = None):
    """Per-slot unweighted expert outputs [T,k,H] fp32."""
    inds = np.ascontiguousarray(inds, dtype=np.int32)
    keep: list = []
    d = _block_struct(w, x, inds.shape[1], keep)
    y = np.empty((d.T, inds.shape[1], w.H), np.float32)
    rc = lib().rnbo_switchglu(ctypes.byref(d), _p(inds, _i32p), _p(y, _f32p),
                              nthreads or nthreads_default())
    if rc:
        raise ValueError(f"oracle switchglu rejected the call (rc={rc})")
    return y


def shared_expert(w: BlockWeights, x: np.ndarray, nthreads: int | None = None):
    keep: list = []
    d = _block_struct(w, x, 8, keep)
    y = np.empty((d.T, w.H), np.float32)
    rc = lib().rnbo_shared_expert(ctypes.byref(d), _p(y, _f32p), nthreads or nthreads_default())
    if rc:
        raise ValueError(f"oracle shared expert rejected the call (rc={rc})")
    return y


def moe_block(w: BlockWeights, x: np.ndarray, k: int = 8, nthreads: int | None = None):
    """Whole block. Returns (out fp32 [T,H], inds [T,k], scores [T,k])."""
    keep: list = []
    d = _block_struct(w, x, k, keep)
    T = d.T
    out = np.empty((T, w.H), np.float32)
    inds = np.empty((T, k), np.int32)
    scores = np.empty((T, k), np.float32)
    rc = lib().rnbo_moe_block(ctypes.byref(d), _p(out, _f32p), _p(inds, _i32p), _p(scores, _f32p),
                              _p(None, _f32p), nthreads or nthreads_default())
    if rc:
        raise ValueError(f"oracle block rejected the call (rc={rc})")
    return out, inds, scores


def moe_block_fast(w: BlockWeights, x: np.ndarray, k: int = 8, nthreads: int | None = None):
    """The vectorised CPU baseline of the whole block (rnb_cpu_fast.c): the
    oracle's routing, experts grouped with each weight panel dequantised once
    for all of its tokens, AVX2/FMA fp32 tiles.  Same return as
    :func:`moe_block`; outputs agree with it within the parity tolerance."""
    keep: list = []
    d = _block_struct(w, x, k, keep)
    T = d.T
    out = np.empty((T, w.H), np.float32)
    inds = np.empty((T, k), np.int32)
    scores = np.empty((T, k), np.float32)
    rc = lib().rnbc_moe_block(ctypes.byref(d), _p(out, _f32p), _p(inds, _i32p), _p(scores, _f32p),
                              nthreads or nthreads_default())
    if rc:
        raise ValueError(f"CPU baseline rejected the call (rc={rc})")
    return out, inds, scores


def fast_simd() -> bool:
    """True when the CPU baseline's AVX2/FMA kernels run on this host."""
    return bool(lib().rnbc_simd())


def block_bound(w: BlockWeights, x: np.ndarray, inds: np.ndarray, scores: np.ndarray | None = None,
                sg: np.ndarray | None = None, nthreads: int | None = None) -> np.ndarray:
    """First-order forward error bound of an fp32 evaluation of every output.

    With ``scores`` (and the shared gate ``sg`` of :func:`router`) it bounds
    the block output ``[T, H]``; without, each slot's unweighted SwitchGLU
    output ``[T, k, H]``.  Every dot product is allowed the classical
    any-order fp32 summation error gamma_n * sum|terms| (n its length, u =
    2^-24), propagated through SwiGLU, the down projection and the combine
    (rnb_oracle.c, rnbo_block_bound).  The parity tolerance uses it as the
    floor for outputs that cancel (tests/_parity.py)."""
    inds = np.ascontiguousarray(inds, dtype=np.int32)
    keep: list = []
    d = _block_struct(w, x, inds.shape[1], keep)
    T, K = d.T, inds.shape[1]
    if scores is not None:
        scores = np.ascontiguousarray(scores, dtype=np.float32)
        keep.append(scores)
        out = np.empty((T, w.H), np.float32)
    else:
        out = np.empty((T, K, w.H), np.float32)
    if sg is not None:
        sg = np.ascontiguousarray(sg, dtype=np.float32)
        keep.append(sg)
    rc = lib().rnbo_block_bound(ctypes.byref(d), _p(inds, _i32p), _p(scores, _f32p), _p(sg, _f32p),
                                _p(out, _f32p), nthreads or nthreads_default())
    if rc:
        raise ValueError(f"oracle block_bound rejected the call (rc={rc})")
    return out


def affine_matvec(w, s, b, x_f32, bits: int, group: int, nthreads: int | None = None):
    w = np.ascontiguousarray(w, np.uint32)
    s = np.ascontiguousarray(s, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    x_f32 = np.ascontiguousarray(x_f32, np.float32)
    rows = w.shape[0]
    K = x_f32.shape[0]
    y = np.empty((rows,), np.float32)
    rc = lib().rnbo_affine_matvec(_p(w, _u32p), _p(s, _u16p), _p(b, _u16p), _p(x_f32, _f32p), rows,
                                  K, bits, group, _p(y, _f32p), nthreads or nthreads_default())
    if rc:
        raise ValueError("oracle matvec rejected the call")
    return y


# ------------------------------------------------- reference KAT generators


def kat_qmv(bits: int, out_rows: int, K: int = 2048, group: int = 64, bank_rows: int = 0,
            rows_per_expert: int = 0, selected=()):
    """Regenerates a quantized_qmv_probe dataset; returns (data dict, y, checksum)."""
    bank_rows = bank_rows or out_rows
    rows_per_expert = rows_per_expert or out_rows
    sel = np.asarray(selected, np.uint32)
    w = np.empty((bank_rows, K * bits // 32), np.uint32)
    s = np.empty((bank_rows, K // group), np.uint16)
    b = np.empty_like(s)
    x = np.empty((K,), np.uint16)
    L = lib()
    sz = ctypes.c_size_t
    rc = L.rnbo_kat_qmv_data(bits, sz(K), sz(group), sz(bank_rows), _p(w, _u32p), _p(s, _u16p),
                             _p(b, _u16p), _p(x, _u16p))
    assert rc == 0
    y = np.empty((out_rows,), np.float32)
    cs = ctypes.c_double()
    L.rnbo_kat_qmv_expected(bits, sz(K), sz(group), sz(out_rows), sz(rows_per_expert),
                            _p(sel if sel.size else None, _u32p), sz(sel.size), _p(w, _u32p),
                            _p(s, _u16p), _p(b, _u16p), _p(x, _u16p), _p(y, _f32p), ctypes.byref(cs))
    return {"w": w, "s": s, "b": b, "x": x, "selected": sel}, y, cs.value


def kat_qmm(bits: int, tokens: int = 64, outputs: int = 4096, K: int = 2048, group: int = 64,
            nthreads: int | None = None):
    w = np.empty((outputs, K * bits // 32), np.uint32)
    s = np.empty((outputs, K // group), np.uint16)
    b = np.empty_like(s)
    x = np.empty((tokens, K), np.uint16)
    L = lib()
    sz = ctypes.c_size_t
    rc = L.rnbo_kat_qmm_data(bits, sz(tokens), sz(outputs), sz(K), sz(group), _p(w, _u32p),
                             _p(s, _u16p), _p(b, _u16p), _p(x, _u16p))
    assert rc == 0
    y = np.empty((tokens, outputs), np.float32)
    cs = ctypes.c_double()
    L.rnbo_kat_qmm_expected(bits, sz(tokens), sz(outputs), sz(K), sz(group), _p(w, _u32p),
                            _p(s, _u16p), _p(b, _u16p), _p(x, _u16p), _p(y, _f32p), ctypes.byref(cs),
                            nthreads or nthreads_default())
    return {"w": w, "s": s, "b": b, "x": x}, y, cs.value


def kat_two_stage(bits: int, experts: int = 64, selected=(3, 17, 29, 42, 50, 61, 7, 55),
                  H: int = 2048, I: int = 512, group: int = 64):
    k = len(selected)
    sel = np.asarray(selected, np.uint32)
    x = np.empty((H,), np.uint16)
    guw = np.empty((experts, 2 * I, H * bits // 32), np.uint32)
    gus = np.empty((experts, 2 * I, H // group), np.uint16)
    gub = np.empty_like(gus)
    dnw = np.empty((experts, H, I * bits // 32), np.uint32)
    dns = np.empty((experts, H, I // group), np.uint16)
    dnb = np.empty_like(dns)
    rw = np.empty((k,), np.float32)
    L = lib()
    sz = ctypes.c_size_t
    rc = L.rnbo_kat_two_stage_data(bits, sz(experts), sz(H), sz(I), sz(group), sz(k), _p(x, _u16p),
                                   _p(guw, _u32p), _p(gus, _u16p), _p(gub, _u16p), _p(dnw, _u32p),
                                   _p(dns, _u16p), _p(dnb, _u16p), _p(rw, _f32p))
    assert rc == 0
    out = np.empty((H,), np.float32)
    cs = ctypes.c_double()
    L.rnbo_kat_two_stage_expected(bits, sz(H), sz(I), sz(group), sz(k), _p(sel, _u32p), _p(x, _u16p),
                                  _p(guw, _u32p), _p(gus, _u16p), _p(gub, _u16p), _p(dnw, _u32p),
                                  _p(dns, _u16p), _p(dnb, _u16p), _p(rw, _f32p), _p(out, _f32p),
                                  ctypes.byref(cs))
    data = {"x": x, "gu_w": guw, "gu_s": gus, "gu_b": gub, "dn_w": dnw, "dn_s": dns, "dn_b": dnb,
            "route_w": rw, "selected": sel}
    return data, out, cs.value
