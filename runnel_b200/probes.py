"""Standalone quantized matvec / matmul probes (``rnb_qmv`` / ``rnb_qmm``).

The B200 form of the reference's probe CLIs ``runnel-metal-qmv`` and
``runnel-metal-qmm`` (native/bench/quantized_qmv.cpp,
native/bench/quantized_qmm.cpp).  :func:`qmv` and :func:`qmm` take torch CUDA
tensors in MLX affine layout; ``python -m runnel_b200.probes qmv|qmm ...``
accepts the reference CLIs' options and prints their JSON shape (protocol,
then the measurement: weight bytes, GiB/s, median GPU microseconds,
checksums and errors).  The CLI's data is seeded synthetic (torch), and its
check is a float64 dequantised matmul of the same tensors on the GPU.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import sys

import torch

from . import _lib
from .ops import _ptr, _stream

MAX_EXPERTS = 64


def _check(w, s, b, x, bits):
    for name, t in (("w", w), ("scales", s), ("biases", b), ("x", x)):
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous CUDA tensor")
    K = w.shape[-1] * 32 // bits
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} columns, the weights {K}")
    return K


def qmv(bits: int, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, x: torch.Tensor,
        selected=None, rows_per_expert: int = 0, rows: int | None = None) -> torch.Tensor:
    """fp32 ``W[row(r)] . x``.  Dense: every row of ``w`` (or the first
    ``rows``).  Expert mode: the ``rows_per_expert`` rows of each expert in
    ``selected`` (host ids) out of the bank ``w``."""
    K = _check(w, scales, biases, x, bits)
    bank = w.shape[0]
    sel_arr, nsel = None, 0
    if selected is not None and len(selected):
        nsel = len(selected)
        sel_arr = (ctypes.c_uint32 * nsel)(*[int(e) for e in selected])
        rows = nsel * rows_per_expert
    elif rows is None:
        rows = bank
    y = torch.empty(rows, dtype=torch.float32, device=w.device)
    if rows == 0:
        return y
    _lib.call("rnb_qmv", bits, 64, rows, K, _ptr(w), _ptr(scales), _ptr(biases), _ptr(x), sel_arr, nsel,
              rows_per_expert, bank, _ptr(y), _stream())
    return y


def qmm(bits: int, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, x: torch.Tensor,
        out_f32: bool = True, ws: torch.Tensor | None = None) -> torch.Tensor:
    """``x[T, K] . W[N, K]^T`` -> [T, N] (fp32, or bf16 with out_f32=False)."""
    K = _check(w, scales, biases, x, bits)
    N, T = w.shape[0], x.shape[0]
    need = ctypes.c_size_t()
    _lib.call("rnb_qmm_workspace_size", bits, 64, T, N, K, ctypes.byref(need))
    if ws is None or ws.numel() < need.value:
        ws = torch.empty(need.value, dtype=torch.uint8, device=w.device)
    y = torch.empty((T, N), dtype=torch.float32 if out_f32 else torch.bfloat16, device=w.device)
    _lib.call("rnb_qmm", bits, 64, T, N, K, _ptr(w), _ptr(scales), _ptr(biases), _ptr(x), _ptr(y),
              1 if out_f32 else 0, ws.data_ptr(), ws.numel(), _stream())
    return y


def dequant_reference(bits: int, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                      rows: torch.Tensor | None = None) -> torch.Tensor:
    """float64 W = s*q + b, optionally of the given rows only (for the CLI's
    check and the tests)."""
    per = 32 // bits
    wi = w.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    s = scales.view(torch.int16)
    b = biases.view(torch.int16)
    if rows is not None:
        wi, s, b = wi[rows], s[rows], b[rows]
    shifts = torch.arange(per, device=w.device, dtype=torch.int64) * bits
    q = ((wi.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)).reshape(wi.shape[0], -1).to(torch.float64)
    s = s.view(torch.bfloat16).to(torch.float64).repeat_interleave(64, dim=1)
    b = b.view(torch.bfloat16).to(torch.float64).repeat_interleave(64, dim=1)
    return s * q + b


def synthetic(bits: int, rows: int, K: int, tokens: int = 1, seed: int = 0, device="cuda"):
    """Seeded uniform codes, scales U(0.001, 0.01), biases N(0, 0.01), x N(0, 1)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = torch.randint(-2 ** 31, 2 ** 31, (rows, K * bits // 32), dtype=torch.int64, device=device,
                      generator=g).to(torch.int32).view(torch.uint32)
    s = (torch.rand((rows, K // 64), device=device, generator=g) * 0.009 + 0.001).to(torch.bfloat16)
    b = (torch.randn((rows, K // 64), device=device, generator=g) * 0.01).to(torch.bfloat16)
    x = torch.randn((tokens, K), device=device, generator=g).to(torch.bfloat16)
    return w, s.view(torch.uint16), b.view(torch.uint16), x


def dataset_tensors(ds, device="cuda"):
    """A :class:`runnel_b200.checkpoint.LayerDataset` on the device:
    (BlockTensors of the whole bank, x [1, H] bf16, ids [1, k], weights [1, k])."""
    import numpy as np

    from .ops import BlockTensors

    def up(a):
        if a.dtype == np.uint32:
            return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(device).view(torch.uint32)
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device).view(torch.bfloat16)

    bt = BlockTensors(bits=ds.bits, gu_w=up(ds.gu_w), gu_s=up(ds.gu_s), gu_b=up(ds.gu_b), dn_w=up(ds.dn_w),
                      dn_s=up(ds.dn_s), dn_b=up(ds.dn_b))
    x = up(ds.x).reshape(1, -1)
    inds = torch.from_numpy(ds.selected.astype(np.int32)).reshape(1, -1).to(device)
    w = torch.from_numpy(ds.route_w.astype(np.float32)).reshape(1, -1).to(device)
    return bt, x, inds, w


def two_stage(ds, device="cuda", tensors=None) -> torch.Tensor:
    """The reference's two-stage MoE probe on one dataset: fp32 [H] =
    sum_j w_j * down_e(silu(gate_e x) * up_e x) over the dataset's experts,
    through ``rnb_moe_experts_fwd``."""
    from .ops import experts_fwd

    bt, x, inds, w = tensors or dataset_tensors(ds, device)
    return experts_fwd(bt, x, inds, w)[0]


def two_stage_reference(ds, device="cuda") -> torch.Tensor:
    """float64 form of :func:`two_stage` (dequantised weights, exact SwiGLU)."""
    bt, x, inds, w = dataset_tensors(ds, device)
    xf = x[0].to(torch.float64)
    out = torch.zeros(bt.H, dtype=torch.float64, device=x.device)
    for j, e in enumerate(ds.selected.tolist()):
        gu = dequant_reference(ds.bits, bt.gu_w[e], bt.gu_s[e].view(torch.uint16), bt.gu_b[e].view(torch.uint16)) @ xf
        up_, gate = gu[:bt.I], gu[bt.I:]
        h = gate / (1.0 + torch.exp(-gate)) * up_
        out += float(ds.route_w[j]) * (dequant_reference(ds.bits, bt.dn_w[e], bt.dn_s[e].view(torch.uint16),
                                                         bt.dn_b[e].view(torch.uint16)) @ h)
    return out


def measure_two_stage(ds, warmups: int = 2, trials: int = 5, device="cuda") -> dict:
    """One measurement record in the reference fused-MoE CLI's shape."""
    tensors = dataset_tensors(ds, device)
    y = two_stage(ds, tensors=tensors)
    ref = two_stage_reference(ds, device)
    err = y.to(torch.float64) - ref
    gpu = _time(lambda: two_stage(ds, tensors=tensors), warmups, trials)
    bt = tensors[0]
    per_expert = (bt.gu_w[0].numel() + bt.dn_w[0].numel()) * 4 + (bt.gu_s[0].numel() + bt.dn_s[0].numel()) * 4
    nbytes = per_expert * len(ds.selected)
    med = _median(gpu)
    return {"weight_bytes": nbytes, "two_stage": True, "weight_gib_per_second": nbytes / (med * 1e3),
            "median_gpu_micros": med, "output_checksum": float(y.to(torch.float64).sum()),
            "reference_checksum": float(ref.sum()), "max_absolute_error": float(err.abs().max()),
            "rmse": float(err.pow(2).mean().sqrt()), "trials": [{"gpu_micros": t} for t in gpu]}


def _time(fn, warmups: int, trials: int) -> list[float]:
    for _ in range(warmups):
        fn()
    out = []
    for _ in range(trials):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        out.append(e0.elapsed_time(e1) * 1e3)
    return out


def _median(v):
    v = sorted(v)
    n = len(v)
    return v[n // 2] if n % 2 else 0.5 * (v[n // 2 - 1] + v[n // 2])


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m runnel_b200.probes")
    sub = ap.add_subparsers(dest="probe", required=True)
    a = sub.add_parser("qmv")
    a.add_argument("--bits", default="q4", choices=["q4", "q8"])
    a.add_argument("--output-size", type=int, default=65536)
    a.add_argument("--reduction-size", type=int, default=2048)
    a.add_argument("--quant-group-size", type=int, default=64)
    a.add_argument("--weight-bank-output-size", type=int, default=0)
    a.add_argument("--rows-per-expert", type=int, default=0)
    a.add_argument("--experts", default="")
    a.add_argument("--warmups", type=int, default=2)
    a.add_argument("--trials", type=int, default=7)
    m = sub.add_parser("qmm")
    m.add_argument("--bits", default="q4", choices=["q4", "q8"])
    m.add_argument("--tokens", type=int, default=64)
    m.add_argument("--outputs", type=int, default=4096)
    m.add_argument("--reduction-size", type=int, default=2048)
    m.add_argument("--quant-group-size", type=int, default=64)
    m.add_argument("--warmups", type=int, default=2)
    m.add_argument("--trials", type=int, default=7)
    t = sub.add_parser("two-stage")
    t.add_argument("--bits", default="q4", choices=["q4", "q8"])
    t.add_argument("--total-experts", type=int, default=256)
    t.add_argument("--experts", default="3,17,29,42,50,61,7,55")
    t.add_argument("--dataset", required=True)
    t.add_argument("--warmups", type=int, default=2)
    t.add_argument("--trials", type=int, default=5)
    t.set_defaults(quant_group_size=64)
    args = ap.parse_args(argv)
    if args.probe == "two-stage":
        from .checkpoint import read_layer_dataset

        bits = 4 if args.bits == "q4" else 8
        ds = read_layer_dataset(args.dataset, bits=bits, total_experts=args.total_experts)
        if [int(e) for e in args.experts.split(",")] != ds.selected.tolist():
            print("runnel_b200.probes: fused MoE dataset expert selection does not match the probe",
                  file=sys.stderr)
            return 1
        meas = measure_two_stage(ds, args.warmups, args.trials)
        limit = max(5.0, abs(meas["reference_checksum"]) * 0.25)
        if meas["max_absolute_error"] > 1.0 or meas["rmse"] > 0.2 or \
                abs(meas["output_checksum"] - meas["reference_checksum"]) > limit:
            print("runnel_b200.probes: fused MoE failed reference validation", file=sys.stderr)
            return 1
        proto = {"bits": args.bits, "total_experts": args.total_experts, "selected_experts": ds.selected.tolist(),
                 "schedule": "two-stage", "dataset_loaded": True, "warmups": args.warmups, "trials": args.trials}
        print(json.dumps({"protocol": proto, "measurements": [meas]}, indent=2))
        return 0
    if args.quant_group_size != 64:
        print("runnel_b200.probes: only group size 64 is supported", file=sys.stderr)
        return 1
    bits = 4 if args.bits == "q4" else 8
    K = args.reduction_size
    if args.probe == "qmv":
        sel = [int(e) for e in args.experts.split(",") if e != ""]
        expert_mode = bool(sel or args.weight_bank_output_size or args.rows_per_expert)
        if expert_mode and not (sel and args.weight_bank_output_size and args.rows_per_expert):
            print("runnel_b200.probes: expert mode requires bank size, rows per expert, and expert list",
                  file=sys.stderr)
            return 1
        bank = args.weight_bank_output_size or args.output_size
        w, s, b, x = synthetic(bits, bank, K)
        x = x[0]
        fn = lambda: qmv(bits, w, s, b, x, selected=sel or None, rows_per_expert=args.rows_per_expert,
                         rows=args.output_size)
        y = fn()
        rows = torch.arange(y.numel(), device=w.device)
        if sel:
            rpe = args.rows_per_expert
            rows = torch.tensor(sel, device=w.device).repeat_interleave(rpe) * rpe + rows % rpe
        wd = dequant_reference(bits, w, s, b, rows)
        ref = wd @ x.to(torch.float64)
        nbytes = int(rows.numel()) * (K * bits // 8 + 2 * (K // 64) * 2)
        proto = {"bits": args.bits, "output_size": y.numel(), "reduction_size": K,
                 "quant_group_size": 64, "weight_bank_output_size": bank,
                 "rows_per_expert": args.rows_per_expert or y.numel(), "selected_experts": sel,
                 "warmups": args.warmups, "trials": args.trials}
    else:
        w, s, b, x = synthetic(bits, args.outputs, K, tokens=args.tokens)
        ws = torch.empty(1, dtype=torch.uint8, device=w.device)
        need = ctypes.c_size_t()
        _lib.call("rnb_qmm_workspace_size", bits, 64, args.tokens, args.outputs, K, ctypes.byref(need))
        ws = torch.empty(need.value, dtype=torch.uint8, device=w.device)
        fn = lambda: qmm(bits, w, s, b, x, ws=ws)
        y = fn()
        ref = x.to(torch.float64) @ dequant_reference(bits, w, s, b).T
        nbytes = args.outputs * (K * bits // 8 + 2 * (K // 64) * 2)
        proto = {"bits": args.bits, "tokens": args.tokens, "outputs": args.outputs, "reduction_size": K,
                 "warmups": args.warmups, "trials": args.trials}
    gpu = _time(fn, args.warmups, args.trials)
    err = (y.to(torch.float64) - ref)
    med = _median(gpu)
    meas = {"weight_bytes": nbytes, "weight_gib_per_second": nbytes / (med * 1e3),
            "median_gpu_micros": med, "output_checksum": float(y.to(torch.float64).sum()),
            "reference_checksum": float(ref.sum()), "max_absolute_error": float(err.abs().max()),
            "rmse": float(err.pow(2).mean().sqrt()), "trials": [{"gpu_micros": t} for t in gpu]}
    print(json.dumps({"protocol": proto, "measurement": meas}, indent=2))
    return 0


if __name__ == "__main__":
    sys.exit(main())
