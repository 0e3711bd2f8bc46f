"""Extracts the reference's recorded known-answer values into kats.json.

Pass the root of a waylake/runnel checkout as argv[1] (or set RUNNEL_REF).  Every record comes from the reference's own result
files under bench/results/m0/: the protocol the native probe ran with, the
checksum its CPU reference produced and, where recorded, the first eight
CPU-reference outputs.  Only the reference's CPU-side numbers are kept (the
Metal outputs of its two-stage kernel are loosely gated and not an oracle),
and records measured on real checkpoint layers (dataset_loaded) are skipped
because their inputs are not regenerable from a seed.

    python tests/golden/make_golden.py /path/to/runnel
"""
from __future__ import annotations

import glob
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(root: str) -> None:
    records = []
    pattern = os.path.join(root, "bench", "results", "m0", "native-m1-*.json")
    for path in sorted(glob.glob(pattern)):
        name = os.path.basename(path)
        if "stream" in name:
            continue
        data = json.load(open(path))
        proto = data["protocol"]
        if proto.get("dataset_loaded"):
            continue  # real Ornith checkpoint weights, not regenerable from a seed
        meas = data.get("measurements") or [data["measurement"]]
        m = meas[0]
        if "reference_checksum" not in m:
            continue
        if "qmm" in name:
            kind = "qmm"
        elif "two-stage" in name:
            kind = "two_stage"
        elif "fused-moe" in name:
            kind = "two_stage"  # the megakernel record shares the same CPU reference
        else:
            kind = "qmv"
        rec = {
            "source": f"bench/results/m0/{name}",
            "kind": kind,
            "protocol": proto,
            "reference_checksum": m["reference_checksum"],
        }
        if "first_reference" in m:
            rec["first_reference"] = m["first_reference"]
        records.append(rec)
    out = os.path.join(HERE, "kats.json")
    with open(out, "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "records": records}, f, indent=1)
    print(f"wrote {len(records)} records to {out}")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RUNNEL_REF")
    if not ref:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/runnel  (or set RUNNEL_REF)")
    main(ref)
