"""Real-weight loading on the host: safetensors indexing, the routed-bank
packing, the RNLMOE01 layer dataset (byte-identical to the reference
exporter's output on the same checkpoint, tests/golden/rnlmoe_export.json),
its reader's checks, and whole-block assembly with the 8-bit router and
shared gate dequantised."""
import importlib.util
import json
import os

import numpy as np
import pytest

from runnel_b200 import checkpoint
from runnel_b200.quant import bf16_bits_to_f32, dequantize

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "rnlmoe_export.json")))
_spec = importlib.util.spec_from_file_location("mkgold", os.path.join(HERE, "golden", "make_checkpoint_golden.py"))
mkgold = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mkgold)
P = "language_model.model.layers.0.mlp"


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    root = str(tmp_path_factory.mktemp("ckpt") / "ornith-synthetic")
    mkgold.synthetic_checkpoint(root)
    return root


def test_store_indexes_and_hashes(model):
    st = checkpoint.TensorStore(model)
    w, h = st.read(f"{P}.switch_mlp.gate_proj.weight")
    assert w.shape == (8, 512, 256) and w.dtype == np.uint32
    assert h == GOLDEN["tensor_sha256"][f"{P}.switch_mlp.gate_proj.weight"]
    with pytest.raises(KeyError, match="tensor is missing"):
        st.read(f"{P}.switch_mlp.nope.weight")


def test_routed_bank_packs_up_then_gate(model):
    st = checkpoint.TensorStore(model)
    r, hashes = checkpoint.read_routed(st, 0)
    assert r["bits"] == 4 and r["gu_w"].shape == (8, 1024, 256)
    np.testing.assert_array_equal(r["gu_w"][:, :512], st.read(f"{P}.switch_mlp.up_proj.weight")[0])
    np.testing.assert_array_equal(r["gu_s"][:, 512:], st.read(f"{P}.switch_mlp.gate_proj.scales")[0])
    assert hashes == GOLDEN["tensor_sha256"]


def test_export_matches_reference_exporter_bytes(model, tmp_path):
    out = str(tmp_path / "layer0.bin")
    man = checkpoint.export_layer(checkpoint.TensorStore(model), 0, GOLDEN["selected_experts"], out)
    assert man["output_sha256"] == GOLDEN["output_sha256"]
    assert man["output_bytes"] == GOLDEN["output_bytes"] == os.path.getsize(out)
    assert json.load(open(str(tmp_path / "layer0.manifest.json")))["tensor_sha256"] == GOLDEN["tensor_sha256"]
    ds = checkpoint.read_layer_dataset(out, bits=4, total_experts=8)
    assert ds.selected.tolist() == GOLDEN["selected_experts"]
    assert abs(float(ds.route_w.sum()) - 1.0) < 1e-6 and ds.x.shape == (2048,)
    back = str(tmp_path / "again.bin")
    checkpoint.write_layer_dataset(back, ds)
    assert open(back, "rb").read() == open(out, "rb").read()


def test_dataset_reader_checks(model, tmp_path):
    out = str(tmp_path / "l.bin")
    checkpoint.export_layer(checkpoint.TensorStore(model), 0, GOLDEN["selected_experts"], out)
    with pytest.raises(ValueError, match="does not match"):
        checkpoint.read_layer_dataset(out, bits=8)
    with pytest.raises(ValueError, match="does not match"):
        checkpoint.read_layer_dataset(out, total_experts=256)
    data = open(out, "rb").read()
    cut = str(tmp_path / "cut.bin")
    open(cut, "wb").write(data[:-4])
    with pytest.raises(ValueError, match="truncated"):
        checkpoint.read_layer_dataset(cut)
    bad = str(tmp_path / "bad.bin")
    open(bad, "wb").write(b"XXLMOE01" + data[8:])
    with pytest.raises(ValueError, match="does not match"):
        checkpoint.read_layer_dataset(bad)


def test_export_rejects_bad_expert_lists(model, tmp_path):
    st = checkpoint.TensorStore(model)
    with pytest.raises(ValueError, match="eight unique"):
        checkpoint.export_layer(st, 0, [0, 1, 2], str(tmp_path / "a.bin"))
    with pytest.raises(ValueError, match="outside the checkpoint"):
        checkpoint.export_layer(st, 0, [0, 1, 2, 3, 4, 5, 6, 9], str(tmp_path / "a.bin"))


def test_whole_block_arrays_dequantise_router(model):
    st = checkpoint.TensorStore(model)
    a = checkpoint.load_block_arrays(st, 0)
    assert a["router_w"].shape == (8, 2048) and a["router_w"].dtype == np.uint16
    w, s, b = (st.read(f"{P}.gate.{n}")[0] for n in ("weight", "scales", "biases"))
    ref = dequantize(w, s, b, 8)
    got = bf16_bits_to_f32(a["router_w"])
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 2.0 ** -8  # one bf16 rounding
    assert a["shared_gate_w"].shape == (2048,)
    # the 8-bit router and shared gate also come as stored, for the block
    assert a["router_bits"] == 8
    np.testing.assert_array_equal(a["router_q"], w)
    np.testing.assert_array_equal(a["router_s"], s)
    np.testing.assert_array_equal(a["router_b"], b)
    assert a["sgate_q"].shape == (512,) and a["sgate_s"].shape == (32,) and a["sgate_b"].shape == (32,)
    assert a["sgu_w"].shape == (1024, 256)
    np.testing.assert_array_equal(a["sgu_w"][512:], st.read(f"{P}.shared_expert.gate_proj.weight")[0])
    assert a["norm_w"].shape == (2048,)


def test_safetensors_round_trip(tmp_path):
    arrs = {"a": (np.arange(12, dtype=np.uint32).reshape(3, 4), "U32"),
            "b": (np.arange(6, dtype=np.uint16), "BF16"), "c": (np.ones((2, 2), np.float32), "F32")}
    checkpoint.write_safetensors(str(tmp_path / "m.safetensors"), arrs)
    st = checkpoint.TensorStore(str(tmp_path))
    for k, (v, _) in arrs.items():
        np.testing.assert_array_equal(st.read(k)[0], v)
