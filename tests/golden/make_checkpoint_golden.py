"""Golden values for the checkpoint exporter (runnel_b200.checkpoint.export_layer).

Builds a small synthetic MLX checkpoint directory (one layer, 8 experts of
the Ornith shapes, 4-bit routed and shared experts, 8-bit router and shared
gate) with :func:`synthetic_checkpoint`, runs the REFERENCE exporter
(bench/export_ornith_moe_layer.py of the reference tree) on it and records the
hashes of the RNLMOE01 file it writes in tests/golden/rnlmoe_export.json.
tests/test_checkpoint.py rebuilds the same directory and requires the B200
exporter to write byte-identical output.

    python tests/golden/make_checkpoint_golden.py /path/to/reference
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
EXPERTS = "3,1,7,0,5,2,6,4"
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from runnel_b200.checkpoint import write_safetensors  # noqa: E402
from runnel_b200.quant import f32_to_bf16_bits  # noqa: E402


def synthetic_checkpoint(root: str, bits: int = 4, E: int = 8, I: int = 512, H: int = 2048, seed: int = 7) -> None:
    """One layer of MLX-named tensors in ``root/model.safetensors``."""
    rng = np.random.default_rng(seed)
    p = "language_model.model.layers.0"

    def quant(rows_shape, K, b):
        w = rng.integers(0, 2 ** 32, size=(*rows_shape, K * b // 32), dtype=np.uint64).astype(np.uint32)
        s = f32_to_bf16_bits(rng.uniform(0.001, 0.01, size=(*rows_shape, K // 64)).astype(np.float32))
        bb = f32_to_bf16_bits(rng.normal(0, 0.01, size=(*rows_shape, K // 64)).astype(np.float32))
        return w, s, bb

    t = {}
    for proj, rows, K in (("gate", I, H), ("up", I, H), ("down", H, I)):
        w, s, b = quant((E, rows), K, bits)
        t[f"{p}.mlp.switch_mlp.{proj}_proj.weight"] = (w, "U32")
        t[f"{p}.mlp.switch_mlp.{proj}_proj.scales"] = (s, "BF16")
        t[f"{p}.mlp.switch_mlp.{proj}_proj.biases"] = (b, "BF16")
    for proj, rows, K in (("gate", I, H), ("up", I, H), ("down", H, I)):
        w, s, b = quant((rows,), K, bits)
        t[f"{p}.mlp.shared_expert.{proj}_proj.weight"] = (w, "U32")
        t[f"{p}.mlp.shared_expert.{proj}_proj.scales"] = (s, "BF16")
        t[f"{p}.mlp.shared_expert.{proj}_proj.biases"] = (b, "BF16")
    for name, rows in (("gate", E), ("shared_expert_gate", 1)):
        w, s, b = quant((rows,), H, 8)
        t[f"{p}.mlp.{name}.weight"] = (w, "U32")
        t[f"{p}.mlp.{name}.scales"] = (s, "BF16")
        t[f"{p}.mlp.{name}.biases"] = (b, "BF16")
    t[f"{p}.post_attention_layernorm.weight"] = (
        f32_to_bf16_bits((1.0 + rng.normal(0, 0.02, size=H)).astype(np.float32)), "BF16")
    os.makedirs(root, exist_ok=True)
    write_safetensors(os.path.join(root, "model.safetensors"), t, {"format": "mlx"})


def main() -> int:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RUNNEL_REFERENCE", "")
    exporter = os.path.join(ref, "bench", "export_ornith_moe_layer.py")
    if not os.path.exists(exporter):
        print("usage: make_checkpoint_golden.py REFERENCE_TREE", file=sys.stderr)
        return 2
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        model = os.path.join(tmp, "ornith-synthetic")
        synthetic_checkpoint(model)
        dst = os.path.join(tmp, "layer0.bin")
        subprocess.run([sys.executable, exporter, "--model", model, "--layer", "0", "--experts", EXPERTS,
                        "--output", dst], check=True, stdout=subprocess.DEVNULL)
        man = json.load(open(os.path.join(tmp, "layer0.manifest.json")))
        out = {"generator": "tests/golden/make_checkpoint_golden.py:synthetic_checkpoint(bits=4, E=8, seed=7)",
               "exporter": f"bench/export_ornith_moe_layer.py (reference), --layer 0 --experts {EXPERTS}",
               "output_sha256": man["output_sha256"], "output_bytes": man["output_bytes"],
               "tensor_sha256": man["tensor_sha256"], "bits": man["bits"], "total_experts": man["total_experts"],
               "selected_experts": man["selected_experts"]}
    with open(os.path.join(HERE, "rnlmoe_export.json"), "w") as f:
        f.write(json.dumps(out, indent=2, sort_keys=True) + "\n")
    print(json.dumps(out, indent=2, sort_keys=True))
    return 0


if __name__ == "__main__":
    sys.exit(main())
