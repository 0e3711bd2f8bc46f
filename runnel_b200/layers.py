"""Per-layer sweep of a real checkpoint through the two-stage MoE probe.

The B200 form of the reference's bench/run_native_ornith_layers.py:19-114:
for each requested layer, export its routed bank to a temporary RNLMOE01
dataset (:func:`runnel_b200.checkpoint.export_layer`), run the two-stage
probe on it (:func:`runnel_b200.probes.measure_two_stage`) and collect one
record per layer (manifest + measurement) in a JSON document.  Weights never
leave the temporary directory; only hashes and measurements are written.

    python -m runnel_b200.layers --model DIR --bits q4 --layers 0,1,2,10,20,30,39 --output out.json
"""
from __future__ import annotations

import argparse
import datetime as dt
import json
import os
import sys
import tempfile

from . import checkpoint, probes


def sweep(model: str, bits: str, layers: list[int], experts: str = "3,17,29,42,50,61,7,55", warmups: int = 2,
          trials: int = 5, device="cuda") -> dict:
    store = checkpoint.TensorStore(model)
    sel = [int(e) for e in experts.split(",")]
    nbits = 4 if bits == "q4" else 8
    records = []
    with tempfile.TemporaryDirectory(prefix="runnel-b200-layers-") as tmp:
        for layer in layers:
            path = os.path.join(tmp, f"layer-{layer}.bin")
            man = checkpoint.export_layer(store, layer, sel, path, os.path.join(tmp, f"layer-{layer}.manifest.json"))
            ds = checkpoint.read_layer_dataset(path, bits=nbits)
            meas = probes.measure_two_stage(ds, warmups, trials, device)
            records.append({"layer": layer, "manifest": man,
                            "native": {"protocol": {"bits": bits, "total_experts": ds.E, "selected_experts": sel,
                                                    "schedule": "two-stage", "dataset_loaded": True,
                                                    "warmups": warmups, "trials": trials},
                                       "measurements": [meas]}})
    return {"schema_version": 1, "created_at_utc": dt.datetime.now(dt.timezone.utc).isoformat(),
            "protocol": {"engine": "runnel-b200 two-stage MoE (rnb_moe_experts_fwd)",
                         "model_name": os.path.basename(os.path.normpath(model)), "bits": bits, "layers": layers,
                         "experts": experts, "warmups": warmups, "trials": trials, "weights_included": False},
            "records": records}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m runnel_b200.layers")
    ap.add_argument("--model", required=True)
    ap.add_argument("--layers", default="0,1,2,10,20,30,39")
    ap.add_argument("--experts", default="3,17,29,42,50,61,7,55")
    ap.add_argument("--bits", choices=["q4", "q8"], required=True)
    ap.add_argument("--warmups", type=int, default=2)
    ap.add_argument("--trials", type=int, default=5)
    ap.add_argument("--output", required=True)
    args = ap.parse_args(argv)
    doc = sweep(args.model, args.bits, [int(v) for v in args.layers.split(",")], args.experts, args.warmups,
                args.trials)
    os.makedirs(os.path.dirname(os.path.abspath(args.output)), exist_ok=True)
    with open(args.output, "w") as f:
        f.write(json.dumps(doc, indent=2, sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
