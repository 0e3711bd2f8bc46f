"""ctypes binding of ``librnb_moe.so`` (the C ABI declared in include/rnb_moe.h).

The shared library is built in-tree (``runnel_b200/csrc/Makefile`` ->
``runnel_b200/librnb_moe.so``).  There is no fallback: if the library is
missing or the device is not an sm_100 GPU, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librnb_moe.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "rnb_moe.h")

RNB_OK = 0
ERRORS = {
    -1: "RNB_ERR_INVALID",
    -2: "RNB_ERR_ALIGN",
    -3: "RNB_ERR_WORKSPACE",
    -4: "RNB_ERR_CUDA",
    -5: "RNB_ERR_DEVICE",
    -6: "RNB_ERR_TIMEOUT",
}
STATUS_BAD_INDEX = 0x1
STATUS_TIMEOUT = 0x2
FLAG_SHARED_ON_THIS_RANK = 0x1
FLAG_NO_SHARED = 0x2
FLAG_Y_F32 = 0x4
FLAG_CHAIN = 0x8
EP_HANDLE_BYTES = 64
A2A_HANDLE_BYTES = 64

# Every function include/rnb_moe.h declares, with its ctypes signature.
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t


class RnbMoeDesc(ctypes.Structure):
    _fields_ = [
        ("T", ctypes.c_int32), ("H", ctypes.c_int32), ("I", ctypes.c_int32),
        ("E", ctypes.c_int32), ("E_total", ctypes.c_int32), ("expert_offset", ctypes.c_int32),
        ("k", ctypes.c_int32), ("bits", ctypes.c_int32), ("group", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("gu_w", _vp), ("gu_s", _vp), ("gu_b", _vp),
        ("dn_w", _vp), ("dn_s", _vp), ("dn_b", _vp),
        ("router_w", _vp), ("shared_gate_w", _vp),
        ("sgu_w", _vp), ("sgu_s", _vp), ("sgu_b", _vp),
        ("sdn_w", _vp), ("sdn_s", _vp), ("sdn_b", _vp),
        ("router_bits", ctypes.c_int32), ("reserved0", ctypes.c_int32),
        ("router_s", _vp), ("router_b", _vp), ("sgate_s", _vp), ("sgate_b", _vp),
    ]


_DescP = ctypes.POINTER(RnbMoeDesc)
SIGNATURES = {
    "rnb_version": (ctypes.c_int, []),
    "rnb_last_error": (ctypes.c_char_p, []),
    "rnb_moe_workspace_size": (ctypes.c_int, [_DescP, ctypes.POINTER(_sz)]),
    "rnb_moe_workspace_init": (ctypes.c_int, [_vp, _sz, _vp]),
    "rnb_router_topk": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "rnb_switchglu_fwd": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, _sz, _vp]),
    "rnb_moe_block_fwd": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "rnb_moe_status": (ctypes.c_int, [_vp, _sz, ctypes.POINTER(ctypes.c_uint32), _vp]),
    "rnb_moe_block_fwd_noalloc": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, _vp]),
    "rnb_moe_noalloc_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), _vp]),
    "rnb_moe_block_fwd_host": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "rnb_moe_experts_workspace_size": (ctypes.c_int, [_DescP, ctypes.POINTER(_sz)]),
    "rnb_moe_experts_fwd": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "rnb_qmv": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, _vp, _vp, _vp, _vp,
                               ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, ctypes.c_int64, ctypes.c_int64, _vp,
                               _vp]),
    "rnb_qmm_workspace_size": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.POINTER(_sz)]),
    "rnb_qmm": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp,
                               _vp, _vp, ctypes.c_int, _vp, _sz, _vp]),
    "rnb_ep_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp), _vp]),
    "rnb_ep_connect": (ctypes.c_int, [_vp, _vp]),
    "rnb_ep_destroy": (ctypes.c_int, [_vp]),
    "rnb_ep_set_wait_limit_ms": (ctypes.c_int, [_vp, ctypes.c_int]),
    "rnb_moe_block_ep_fwd": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "rnb_a2a_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.POINTER(_vp), _vp]),
    "rnb_a2a_connect": (ctypes.c_int, [_vp, _vp]),
    "rnb_a2a_destroy": (ctypes.c_int, [_vp]),
    "rnb_a2a_set_wait_limit_ms": (ctypes.c_int, [_vp, ctypes.c_int]),
    "rnb_moe_block_a2a_workspace_size": (ctypes.c_int, [_DescP, _vp, ctypes.POINTER(_sz)]),
    "rnb_moe_block_a2a_fwd": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "rnb_moe_block_norm_fwd": (ctypes.c_int, [_DescP, _vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _sz,
                                              _vp]),
    "rnb_add_rmsnorm": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp]),
    "rnb_stage_timing": (ctypes.c_int, [ctypes.c_int]),
    "rnb_stage_times": (ctypes.c_int, [ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
}

STAGES = ("decode", "route", "sort", "scatter", "gateup", "down", "final")  # RNB_STAGE_* ids


def stage_timing(enable: bool) -> None:
    """Turn per-stage device timing of block calls on or off."""
    load().rnb_stage_timing(1 if enable else 0)


def stage_times() -> tuple[dict, int]:
    """({stage: summed ms} over the timed calls since the last read, calls)."""
    ms = (ctypes.c_float * len(STAGES))()
    n = ctypes.c_int(0)
    rc = load().rnb_stage_times(ms, len(STAGES), ctypes.byref(n))
    if rc < 0:
        raise RnbError("rnb_stage_times", rc, load().rnb_last_error().decode())
    return {name: float(ms[i]) for i, name in enumerate(STAGES) if ms[i] > 0}, int(n.value)

_lib = None
_lock = threading.Lock()


class RnbError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with {ERRORS.get(code, code)}: {msg}")
        self.code = code


def build() -> str:
    """Compile the CUDA library in-tree with nvcc (sm_100a)."""
    subprocess.run(["make", "-s", "-C", os.path.join(_HERE, "csrc")], check=True)
    return LIB_PATH


def load(path: str | None = None):
    """Load (once) and return the CDLL with typed entry points."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"{p} is missing: build the CUDA extension first (python -c 'import "
                "__graft_entry__ as g; g.build()' or make -C runnel_b200/csrc)")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(fn: str, rc: int) -> None:
    if rc != RNB_OK:
        msg = load().rnb_last_error()
        raise RnbError(fn, rc, msg.decode() if msg else "")


def call(fn: str, *args) -> None:
    check(fn, getattr(load(), fn)(*args))
