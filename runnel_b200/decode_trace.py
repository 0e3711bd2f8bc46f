"""Phase timeline of the persistent decode kernel (k_decode).

Loads the trace build of the library (``make -C runnel_b200/csrc trace`` ->
runnel_b200/librnb_moe_trace.so, compiled with RNB_TRACE), in which thread 0
of every CTA writes ``%globaltimer`` at each phase mark into the
workspace's scratch area.  Prints, per mark, the time from the earliest CTA
start (min / median / max over the CTAs that reach it), for the last call of
a CUDA-graph replay of back-to-back calls and for an isolated call.  The
marks cost a few tens of ns each, so the trace build runs slightly slower
than the product library.

    python -m runnel_b200.decode_trace [--bits 4 8] [--tokens 1]
"""
from __future__ import annotations

import argparse
import ctypes
import os

import numpy as np
import torch

from . import _lib

TRACE_LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "librnb_moe_trace.so")

NAMES = {0: "start", 1: "prologue", 2: "griddep", 3: "router", 4: "xprep", 5: "sh-gateup", 6: "logits",
         7: "routed", 8: "tasks", 9: "gu-wait0", 10: "gu-mma0", 11: "gu-done", 12: "gu-epi", 13: "dn-start",
         14: "h-conv", 15: "dn-done", 16: "dn-sync", 17: "end", 18: "route-body", 19: "combine",
         20: "task-list", 21: "pre-issue", 22: "issued", 23: "h-polled"}
VALUES = {30: "h-word poll rounds of the down phase (thread 0)", 31: "exact router recomputes (CTA 0)"}


def summarise(tr: np.ndarray) -> list[str]:
    """Lines of the timeline table from the raw [CTAs][64] int64 trace."""
    ck, ts = tr[:, 32:], tr[:, :32]
    lines = []
    ok = (ts[:, 0] > 1e12) & (ts[:, 17] > 1e12)
    mhz = (ck[ok, 17] - ck[ok, 0]) / (ts[ok, 17] - ts[ok, 0]) * 1e3
    lines.append(f"   SM clock over start..end (clock64 / globaltimer): median {np.median(mhz):.0f} MHz")
    for i, what in VALUES.items():
        v = ts[:, i][(ts[:, i] > 0) & (ts[:, i] < 1e9)]
        if len(v):
            lines.append(f"   {what}: median {int(np.median(v))}, max {int(v.max())}")
    t0 = ts[:, 0][ts[:, 0] > 1e12].min()

    def med(m):
        v = ts[:, m][ts[:, m] > 1e12]
        return np.median(v) if len(v) else 1e30
    lines.append("   mark             CTAs      min   median      max   (ns from the earliest CTA start)")
    for m in sorted(NAMES, key=med):
        v = ts[:, m][ts[:, m] > 1e12] - t0
        if len(v):
            lines.append(f"   {m:2d} {NAMES[m]:10s}  n={len(v):3d}  {v.min():7d}  {int(np.median(v)):7d}  {v.max():7d}")
    return lines


def run(bits: int, T: int, reps: int = 24, device: int = 0) -> list[str]:
    from . import inputs, ops
    dev = torch.device("cuda", device)
    torch.cuda.set_device(dev)
    lib = _lib.load(TRACE_LIB)
    if lib._name != TRACE_LIB:
        raise RuntimeError("the product library was loaded first: run the trace in a fresh process")
    lib.rnb_trace_offset.restype = ctypes.c_size_t
    lib.rnb_trace_offset.argtypes = [ctypes.POINTER(_lib.RnbMoeDesc)]
    nc = torch.cuda.get_device_properties(dev).multi_processor_count
    blk = inputs.make_block(bits, seed=1, T=T)
    base = ops.BlockTensors.from_numpy(blk, dev)
    # distinct weight copies so that back-to-back calls do not hit in L2
    copies = [base] + [ops.BlockTensors(**{f: (v.clone() if isinstance(v, torch.Tensor) else v)
                                          for f, v in base.__dict__.items()}) for _ in range(reps - 1)]
    xs = torch.from_numpy(inputs.make_tokens(1, T * reps)).view(torch.int16).view(torch.bfloat16).to(dev)
    xs = xs.reshape(reps, T, -1)
    ws = ops.Workspace(dev)
    outs = torch.empty_like(xs)
    st = torch.cuda.Stream(dev)
    with torch.cuda.stream(st):
        for i in range(2 * reps):
            ops.moe_block(copies[i % reps], xs[i % reps], ws=ws, out=outs[i % reps])
    torch.cuda.synchronize()
    off = lib.rnb_trace_offset(ctypes.byref(copies[0].desc(T)))
    span = nc * 64 * 8

    def grab():
        return ws.buf[off:off + span].cpu().view(torch.int64).numpy().reshape(nc, 64).astype(np.int64)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(reps):
            ops.moe_block(copies[i], xs[i], ws=ws, out=outs[i])
    for _ in range(20):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(200):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    out = [f"q{bits} T={T}: trace build, graph of {reps} calls: {e0.elapsed_time(e1) * 1e3 / (200 * reps):.2f} us/call"]
    ws.buf[off:off + span].zero_()
    g.replay()
    torch.cuda.synchronize()
    out.append(f"-- q{bits} T={T}, last call of a graph replay")
    out += summarise(grab())
    for rep in range(3):
        ws.buf[off:off + span].zero_()
        torch.cuda.synchronize()
        with torch.cuda.stream(st):
            ops.moe_block(copies[rep], xs[rep], ws=ws, out=outs[0])
        torch.cuda.synchronize()
    out.append(f"-- q{bits} T={T}, isolated call")
    out += summarise(grab())
    if ws.status():
        raise RuntimeError("the traced calls reported a status bit")
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--bits", type=int, nargs="+", default=[4, 8])
    ap.add_argument("--tokens", type=int, default=1)
    a = ap.parse_args()
    for bits in a.bits:
        print("\n".join(run(bits, a.tokens)))


if __name__ == "__main__":
    main()
