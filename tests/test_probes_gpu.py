"""GPU parity of the standalone QMV / QMM probes (rnb_qmv, rnb_qmm) against
the reference's recorded known-answer values.

The data of every QMV and QMM record in tests/golden/kats.json is regenerated
by the oracle's restatement of the reference generators; the GPU result must
pass the reference CLI's own validation bars (native/bench/quantized_qmv.cpp:
rmse <= 1e-4 and |checksum - reference| <= 1e-3; quantized_qmm.cpp: max abs
<= 0.2 and rmse <= 0.05) against the oracle's outputs, and its checksum must
match the checksum the reference recorded.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import _lib, probes

pytestmark = pytest.mark.gpu

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "kats.json")))["records"]
QMV = [r for r in GOLDEN if r["kind"] == "qmv"]
QMM = [r for r in GOLDEN if r["kind"] == "qmm"]


def _dev(a):
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda().view(torch.uint32)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.uint16)
    return torch.from_numpy(a).cuda()


@pytest.mark.parametrize("rec", QMV, ids=[r["source"].split("/")[-1] for r in QMV])
def test_qmv_reference_kat(rec):
    pr = rec["protocol"]
    bits = 4 if pr["bits"] == "q4" else 8
    sel = tuple(pr.get("selected_experts", ()))
    data, y_ref, cs_ref = oracle.kat_qmv(bits, pr["output_size"], K=pr["reduction_size"],
                                         bank_rows=pr.get("weight_bank_output_size", 0),
                                         rows_per_expert=pr.get("rows_per_expert", 0), selected=sel)
    x = _dev(data["x"]).view(torch.bfloat16)
    y = probes.qmv(bits, _dev(data["w"]), _dev(data["s"]), _dev(data["b"]), x, selected=sel or None,
                   rows_per_expert=pr.get("rows_per_expert", 0), rows=pr["output_size"])
    yh = y.cpu().numpy().astype(np.float64)
    rmse = float(np.sqrt(np.mean((yh - y_ref) ** 2)))
    cs = float(yh.sum())
    assert rmse <= 1e-4, rmse
    assert abs(cs - cs_ref) <= 1e-3, (cs, cs_ref)
    assert abs(cs - rec["reference_checksum"]) <= 1.5e-3, (cs, rec["reference_checksum"])


@pytest.mark.parametrize("rec", QMM[::2], ids=[r["source"].split("/")[-1] for r in QMM[::2]])
def test_qmm_reference_kat(rec):
    pr = rec["protocol"]
    bits = 4 if pr["bits"] == "q4" else 8
    data, y_ref, cs_ref = oracle.kat_qmm(bits, pr["tokens"], pr["outputs"], pr["reduction_size"])
    x = _dev(data["x"]).view(torch.bfloat16)
    for f32 in (True, False):
        y = probes.qmm(bits, _dev(data["w"]), _dev(data["s"]), _dev(data["b"]), x, out_f32=f32)
        yh = y.float().cpu().numpy().astype(np.float64)
        err = np.abs(yh - y_ref)
        assert err.max() <= 0.2 and np.sqrt(np.mean(err ** 2)) <= 0.05, (err.max(), np.sqrt(np.mean(err ** 2)))
    # fp32 output: the checksum agrees with the recorded one to the fp16-weight rounding
    y = probes.qmm(bits, _dev(data["w"]), _dev(data["s"]), _dev(data["b"]), x).cpu().numpy().astype(np.float64)
    rel = abs(y.sum() - rec["reference_checksum"]) / np.abs(y_ref).sum()
    assert rel < 1e-4, rel


@pytest.mark.parametrize("bits", [4, 8])
def test_qmv_dense_and_gather_match_float64(bits):
    w, s, b, x = probes.synthetic(bits, 4096, 4096 if bits == 4 else 2560, seed=bits)
    x = x[0]
    y = probes.qmv(bits, w, s, b, x)
    ref = probes.dequant_reference(bits, w, s, b) @ x.to(torch.float64)
    err = (y.double() - ref).abs()
    assert float(err.max()) <= 2e-5 * float(ref.abs().max()) + 1e-5
    sel = [31, 0, 7, 7]
    y = probes.qmv(bits, w, s, b, x, selected=sel, rows_per_expert=128)
    rows = torch.tensor(sel, device=w.device).repeat_interleave(128) * 128 + torch.arange(512, device=w.device) % 128
    torch.testing.assert_close(y.double(), ref[rows], rtol=0, atol=2e-5 * float(ref.abs().max()) + 1e-5)
    assert probes.qmv(bits, w, s, b, x, rows=0).numel() == 0


def test_qmm_ragged_tokens_match_float64():
    w, s, b, x = probes.synthetic(8, 1024, 1536, tokens=300, seed=3)
    y = probes.qmm(8, w, s, b, x)
    ref = x.to(torch.float64) @ probes.dequant_reference(8, w, s, b).T
    err = (y.double() - ref).abs()
    assert float(err.max()) <= 1e-3 * float(ref.abs().max())


@pytest.mark.parametrize("bits,expected", [(8, 6.836), (4, 170.073)])
def test_two_stage_dataset_probe_reference_kat(bits, expected, tmp_path):
    """The two-stage KAT bank written as an RNLMOE01 dataset, read back and run
    by the dataset probe (rnb_moe_experts_fwd): the reference's recorded checksum."""
    from runnel_b200 import checkpoint
    data, ref_out, ref_cs = oracle.kat_two_stage(bits)
    ds = checkpoint.LayerDataset(bits=bits, selected=data["selected"], x=data["x"], route_w=data["route_w"],
                                 **{k: data[k] for k in ("gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b")})
    path = str(tmp_path / "kat.bin")
    checkpoint.write_layer_dataset(path, ds)
    back = checkpoint.read_layer_dataset(path, bits=bits, total_experts=64)
    y = probes.two_stage(back).cpu().numpy().astype(np.float64)
    from tests._parity import assert_close
    kw = oracle.BlockWeights(bits=bits, group=64, router_w=np.zeros((64, 2048), np.uint16),
                             **{n: data[n] for n in ("gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b")})
    bound = oracle.block_bound(kw, data["x"].reshape(1, -1), data["selected"].astype(np.int32).reshape(1, 8),
                           data["route_w"].reshape(1, 8))[0]
    assert_close(y, ref_out, f"two-stage dataset q{bits}", bound=bound)
    # The grouped GEMM feeds the SwiGLU rows to the down projection as fp16
    # (11-bit significand); every output shares those rows, so their rounding
    # reaches the checksum coherently: within 1e-3 of it, not the 5e-3
    # absolute of the decode kernels' split-fp16 activations.
    assert abs(y.sum() - expected) < 1e-3 * abs(expected) + 5e-4, (y.sum(), expected)
    meas = probes.measure_two_stage(back, warmups=1, trials=2)
    assert meas["rmse"] < 1e-3 and abs(meas["output_checksum"] - meas["reference_checksum"]) < 1e-3 * abs(expected)


def test_checkpoint_block_and_layer_sweep(tmp_path):
    """A synthetic MLX checkpoint: the whole block loaded by name (its 8-bit
    router and shared gate as stored) runs and matches the oracle on the same
    arrays; the layer sweep writes one record per layer."""
    import importlib.util
    from runnel_b200 import checkpoint, layers, ops
    spec = importlib.util.spec_from_file_location(
        "mkgold", os.path.join(os.path.dirname(__file__), "golden", "make_checkpoint_golden.py"))
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    root = str(tmp_path / "ornith-synthetic")
    mk.synthetic_checkpoint(root)
    st = checkpoint.TensorStore(root)
    bt = checkpoint.load_block(st, 0)
    a = checkpoint.load_block_arrays(st, 0)
    x_bits = np.random.default_rng(5).standard_normal((3, 2048)).astype(np.float32)
    from runnel_b200.quant import f32_to_bf16_bits
    x_bits = f32_to_bf16_bits(x_bits)
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16).cuda()
    out, inds, _ = ops.moe_block(bt, x, return_routing=True)
    fields = {k: a[k] for k in ("router_w", "shared_gate_w", "gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b",
                                "sgu_w", "sgu_s", "sgu_b", "sdn_w", "sdn_s", "sdn_b", "router_bits",
                                "router_q", "router_s", "router_b", "sgate_q", "sgate_s", "sgate_b")}
    assert bt.router_bits == 8 and fields["router_bits"] == 8  # the checkpoint's router is 8-bit
    from tests._parity import assert_close, oracle_block
    ref, oinds, _, bound = oracle_block(oracle.BlockWeights(bits=4, group=64, **fields), x_bits)
    np.testing.assert_array_equal(np.sort(inds.cpu().numpy(), 1), np.sort(oinds, 1))
    assert_close(out.float().cpu().numpy(), ref, "checkpoint block", bound=bound)
    doc = layers.sweep(root, "q4", [0], experts="3,1,7,0,5,2,6,4", warmups=1, trials=2)
    rec = doc["records"][0]
    assert rec["layer"] == 0 and rec["manifest"]["total_experts"] == 8
    m = rec["native"]["measurements"][0]
    assert m["rmse"] < 1e-3 and abs(m["output_checksum"] - m["reference_checksum"]) < 1e-3 * abs(m["reference_checksum"]) + 5e-3
