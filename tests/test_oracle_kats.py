"""The CPU oracle reproduces every known-answer value the reference recorded.

The reference's native probes validated their Metal kernels against a CPU
reference over synthetic data from an xorshift64 generator; their result
files (bench/results/m0/native-m1-*.json in the reference tree) record the
CPU checksum to three decimals and, for the QMV probes, the first eight
CPU outputs.  tests/golden/kats.json holds those values (extracted by
tests/golden/make_golden.py); here the oracle regenerates the same data and
must print the same numbers.
"""
import functools
import json
import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "kats.json")))["records"]


def _bits(proto):
    return 4 if proto["bits"] == "q4" else 8


@functools.lru_cache(maxsize=None)
def _run(kind, key):
    proto = dict(key)
    bits = _bits(proto)
    if kind == "qmv":
        sel = tuple(proto.get("selected_experts", ()))
        _, y, cs = oracle.kat_qmv(
            bits, proto["output_size"], K=proto["reduction_size"], group=proto["quant_group_size"],
            bank_rows=proto.get("weight_bank_output_size", 0),
            rows_per_expert=proto.get("rows_per_expert", 0), selected=sel)
        return y[:8].copy(), cs
    if kind == "qmm":
        _, y, cs = oracle.kat_qmm(bits, proto["tokens"], proto["outputs"], proto["reduction_size"])
        return y.reshape(-1)[:8].copy(), cs
    _, y, cs = oracle.kat_two_stage(bits, proto["total_experts"], tuple(proto["selected_experts"]))
    return y[:8].copy(), cs


def _key(proto):
    return tuple(sorted((k, tuple(v) if isinstance(v, list) else v) for k, v in proto.items()
                        if k not in ("threadgroups", "warmups", "trials", "groups", "schedule",
                                     "token_tile", "output_tile", "reduction_tile")))


@pytest.mark.parametrize("rec", GOLDEN, ids=[r["source"].split("/")[-1] for r in GOLDEN])
def test_reference_kat(rec):
    first, checksum = _run(rec["kind"], _key(rec["protocol"]))
    assert round(checksum, 3) == pytest.approx(rec["reference_checksum"], abs=1e-9), rec["source"]
    if "first_reference" in rec:
        np.testing.assert_array_equal(np.round(first.astype(np.float64), 3), rec["first_reference"])


def test_golden_covers_all_probe_kinds():
    kinds = {r["kind"] for r in GOLDEN}
    assert kinds == {"qmv", "qmm", "two_stage"}
    assert len(GOLDEN) >= 18


def test_bf16_round_trip_rne():
    vals = np.array([1.0, 1.00390625, 1.01171875, -3.14159, 65504.0, 1e-30, np.inf, -np.inf],
                    np.float32)
    b = oracle.f32_to_bf16(vals)
    back = oracle.bf16_to_f32(b)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: RNE keeps the even mantissa (1.0)
    assert back[1] == 1.0
    assert back[2] == np.float32(1.015625)
    assert np.isinf(back[6]) and np.isinf(back[7])
    torch = pytest.importorskip("torch")
    ref = torch.tensor(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(b, ref)
