"""The C-ABI library loads and exports exactly what include/rnb_moe.h declares;
host-side validation errors surface with their codes (no GPU needed)."""
import ctypes
import os
import re

import pytest

from runnel_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "rnb_moe.h")).read()
    return set(re.findall(r"RNB_API\s+[\w\s\*]+?\b(rnb_\w+)\s*\(", text))


def test_header_declares_entry_points():
    names = _declared()
    assert {"rnb_switchglu_fwd", "rnb_moe_block_fwd", "rnb_router_topk",
            "rnb_moe_workspace_size", "rnb_last_error"} <= names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_lib.SIGNATURES) == _declared()
    assert lib.rnb_version() >= 100


def test_desc_struct_matches_header_field_order():
    text = open(os.path.join(ROOT, "include", "rnb_moe.h")).read()
    body = text[text.index("typedef struct rnb_moe_desc"):text.index("} rnb_moe_desc;")]
    fields = re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(\w+);", body, re.M)
    assert fields == [f for f, _ in _lib.RnbMoeDesc._fields_]


def _desc(**kw):
    d = _lib.RnbMoeDesc(T=1, H=2048, I=512, E=256, E_total=256, k=8, bits=8, group=64)
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("field,value,msg", [
    ("group", 32, "group size"),
    ("bits", 3, "bits"),
    ("H", 1000, "H must"),
    ("H", 4096, "H must"),
    ("I", 100, "I must"),
    ("k", 0, "k must"),
    ("E_total", 600, "E_total"),
    ("E", 300, "expert shard"),
    ("expert_offset", 10, "expert shard"),
])
def test_workspace_size_rejects_bad_shapes(field, value, msg):
    n = ctypes.c_size_t()
    with pytest.raises(_lib.RnbError) as ei:
        _lib.call("rnb_moe_workspace_size", ctypes.byref(_desc(**{field: value})), ctypes.byref(n))
    assert ei.value.code == -1 and msg in str(ei.value)


def test_workspace_size_positive():
    n = ctypes.c_size_t()
    _lib.call("rnb_moe_workspace_size", ctypes.byref(_desc()), ctypes.byref(n))
    assert n.value > 0 and n.value % 256 == 0


def test_calls_without_device_fail_loudly():
    # no CUDA device here (or a wrong one): the call must fail, never fall back
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    n = ctypes.c_size_t()
    d = _desc()
    _lib.call("rnb_moe_workspace_size", ctypes.byref(d), ctypes.byref(n))
    rc = _lib.load().rnb_switchglu_fwd(ctypes.byref(d), 16, 16, 16, 16, n.value, None)
    assert rc != 0
    # the host-buffer entry point checks the device before it queues a copy
    rc = _lib.load().rnb_moe_block_fwd_host(ctypes.byref(d), 16, 16, 16, 16, 16, n.value, None)
    assert rc != 0


@pytest.mark.parametrize("kw,msg", [
    (dict(K=100), "K must"),
    (dict(bits=3), "bits"),
    (dict(rows=20), "rows must"),
    (dict(sel=[5], rpe=16, rows=16, bank=64), "outside the bank"),
    (dict(sel=[0, 1], rpe=16, rows=16, bank=64), "expert mode"),
])
def test_qmv_rejects_bad_shapes(kw, msg):
    sel = kw.get("sel")
    arr = (ctypes.c_uint32 * len(sel))(*sel) if sel else None
    fake = ctypes.c_void_p(1 << 20)  # never dereferenced: validation fails first
    rc = _lib.load().rnb_qmv(kw.get("bits", 4), 64, kw.get("rows", 16), kw.get("K", 512), fake, fake, fake, fake,
                             arr, len(sel) if sel else 0, kw.get("rpe", 0), kw.get("bank", 0), fake, None)
    assert rc == -1  # RNB_ERR_INVALID
    assert msg in _lib.load().rnb_last_error().decode()


def test_qmm_workspace_size_rejects_bad_shapes():
    n = ctypes.c_size_t()
    assert _lib.load().rnb_qmm_workspace_size(4, 64, 64, 100, 2048, ctypes.byref(n)) == -1
    assert _lib.load().rnb_qmm_workspace_size(4, 64, 64, 4096, 2048, ctypes.byref(n)) == 0
    assert n.value > 64 * 2048 * 2
