"""Benchmark of the sparse-MoE block on B200.

Default workload (N=1): configuration 2 of the reference's hot-path benchmark
set -- one Ornith MoE block, 4-bit MLX affine (group 64), batch-1 decode --
measured as microseconds per token.  A step is one block call on one batch of
T tokens (router, top-8, routed experts, shared expert, combine).
``--config 3`` (q8, 2048 tokens, log-Zipf routing skew) and ``--config 5``
(q8, 16384 tokens, uniform and adversarial routing on alternate steps) time
the prefill path in tokens per second instead; their roofline is the tensor
pipe (the two grouped GEMM launches, timed with CUDA events on the launching
stream through the library's stage timing).

Timing: W warm-up steps, then K steps bracketed by barrier + synchronize,
device-timed with CUDA events.  Every step uses a different token and one of
R device copies of the block's weights, R chosen so that the copies exceed the
L2 cache several times over (no step can hit weights left in L2 by the
previous ones); the K steps are replayed from one CUDA graph.

Also reported:
  e2e           the same metric through the public API with the token in pinned
                host memory: per step H2D copy of the token, block, and the
                output written back to pinned host memory, launched from Python,
                device-timed over the K steps.  On one GPU this is one C-ABI
                call (ops.BlockCall.host -> rnb_moe_block_fwd_host, whose kernels
                store the output straight into the mapped pinned buffer); under
                expert parallelism it is two torch copies around the
                expert-parallel block call.
  roofline      algorithmic HBM bytes per step (distinct experts' weights +
                shared expert + router + activations) / step time, against
                MEASURED_PEAKS.json hbm_gbs.
  cpu_baseline  the vectorised CPU restatement of the block (oracle/rnb_cpu_fast.c:
                -O3, AVX2/FMA, OpenMP over every host thread, experts grouped;
                routing identical to the exact-order oracle) on a bounded
                sample of the same workload.
  --impl reference  times that CPU path alone (the reference's own MLX path
                cannot run here: no Apple GPU, no MLX).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
HBM_NOMINAL_GBS = 8000.0


def expert_bytes(bits, H=2048, I=512, group=64):
    gu = 2 * I * H * bits // 8 + 2 * I * (H // group) * 4
    dn = H * I * bits // 8 + H * (I // group) * 4
    return gu, dn


def step_bytes(bits, distinct_experts, T, H=2048, I=512, E=256, shared=True):
    gu, dn = expert_bytes(bits, H, I)
    b = distinct_experts * (gu + dn)
    if shared:
        b += gu + dn + H * 2  # shared expert + its gate row
    b += E * H * 2  # router
    b += T * H * 2 * 2  # x in, out
    return b


# DRAM bytes (read + write) per step of the dominant kernel, from one ncu
# capture of the same workload (profiles/ holds the summary and the command).
MEASURED_TRAFFIC = {
    "config1 q8 decode T=1": (31_422_720, "profiles/k_decode_q8_T1.md"),
    "config2 q4 decode T=1": (17_211_648, "profiles/k_decode_q4_T1.md"),
    "config3 q8 prefill T=2048": (577_900_000, "profiles/k_pre_gemm_q8_T2048.md"),
    "config5 q8 prefill T=16384": (2_400_000_000, "profiles/k_pre_gemm_q8_T16384.md"),
}


def prefill_flops(T, H=2048, I=512, E=256, k=8, shared=True):
    """Algorithmic FLOPs of one block call on T tokens: (routed GEMMs, all)."""
    gemm = 2.0 * T * (k + (1 if shared else 0)) * 3 * I * H
    return gemm, gemm + 2.0 * T * E * H + (2.0 * T * H if shared else 0.0)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            self.path = f"/tmp/rnb_clocks_{os.getpid()}.csv"
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def timed_trials(run_k, stream, dist, dev, min_s):
    """Times run_k() -- exactly K steps queued on `stream` -- in repeated
    trials, each bracketed by a barrier (under torchrun) and a device
    synchronize and timed with CUDA events on `stream`, until at least min_s
    seconds of trials have run; every rank runs the same number of trials.
    Returns the per-trial milliseconds, each the maximum over ranks."""
    import torch

    def one():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            run_k()
            e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    first = one()
    n = int(min(10000, max(3, np.ceil(min_s * 1e3 / max(first, 1e-3)))))
    if dist:
        t = torch.tensor([n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        n = int(t.item())
    return [first] + [one() for _ in range(n - 1)]


def cpu_port_desc():
    """How the timed CPU path computes (the vectorised restatement)."""
    from oracle import oracle

    return ("the vectorised CPU restatement, oracle/rnb_cpu_fast.c: C -O3, "
            + ("AVX2/FMA" if oracle.fast_simd() else "plain C (no AVX2/FMA on this host)")
            + " kernels, OpenMP over every host thread, experts grouped so each weight panel is dequantised "
              "once per call; routing identical to the exact-order oracle, outputs within the parity tolerance")


def cpu_baseline(bits, T, budget_s=10.0, seed=1):
    from oracle import oracle
    from runnel_b200 import inputs

    blk = inputs.make_block(bits, seed=seed, T=T)
    w = oracle.BlockWeights(bits=bits, group=64, **blk.weight_fields())
    n = 0
    t0 = time.perf_counter()
    while True:
        oracle.moe_block_fast(w, blk.x, k=8)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 10000:
            break
    cores = os.cpu_count() or 1
    return {"value": el / (n * T) * 1e6, "unit": "us/token", "cores": cores, "kind": "port",
            "sample": f"{n} block calls of T={T} tokens, q{bits} ({cpu_port_desc()})"}


def run_reference(args, cfg=None):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if cfg is not None:
        return run_reference_prefill(args, cfg)
    bits, T = args.bits, args.tokens
    from oracle import oracle
    from runnel_b200 import inputs

    blk = inputs.make_block(bits, seed=args.seed, T=T)
    w = oracle.BlockWeights(bits=bits, group=64, **blk.weight_fields())
    for _ in range(args.warmup):
        oracle.moe_block_fast(w, blk.x, k=8)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.moe_block_fast(w, blk.x, k=8)
    el = time.perf_counter() - t0
    us_tok = el / (args.steps * T) * 1e6
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": "moe_block_decode_us_per_token", "value": us_tok,
        "unit": "us/token", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config{args.config} q{bits} decode T={T}", "bits": bits, "tokens_per_step": T},
        "cpu_baseline": {"value": us_tok, "unit": "us/token", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} block calls of T={T} ({cpu_port_desc()})"},
        "e2e": {"value": us_tok, "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_stack(args, cfg, n_layers=4):
    """The CPU path (oracle) on the stack workload: each step is one token
    through n_layers seeded q4 layers, scaled to the configuration's layers."""
    from oracle import oracle
    from runnel_b200 import inputs, stack
    from runnel_b200.quant import f32_to_bf16_bits

    bits, L = args.bits, args.layers or cfg["layers"]
    blks = [inputs.make_block(bits, seed=args.seed * 1000 + l, T=1) for l in range(n_layers)]
    ws = [oracle.BlockWeights(bits=bits, group=64, **b.weight_fields()) for b in blks]
    nw = [f32_to_bf16_bits(b.norm_w) for b in blks] + [f32_to_bf16_bits(blks[-1].norm_w)]
    x = blks[0].x

    def token(x):
        xa, xn = stack.reference_add_rmsnorm(x, None, nw[0])
        for l in range(n_layers):
            y, _, _ = oracle.moe_block_fast(ws[l], xn, k=8)
            xa, xn = stack.reference_add_rmsnorm(xa, f32_to_bf16_bits(y), nw[l + 1])
        return xa

    for _ in range(args.warmup):
        x = token(x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        x = token(x)
    el = time.perf_counter() - t0
    us_tok = el / args.steps * 1e6 * L / n_layers
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": "moe_stack_decode_us_per_token", "value": us_tok, "unit": "us/token",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": us_tok * 1e-3,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config4 {L} q{bits} layers, batch-1 sequential decode", "bits": bits, "layers": L},
        "cpu_baseline": {"value": us_tok, "unit": "us/token", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} tokens through {n_layers} layers, scaled by {L}/{n_layers} "
                                   f"({cpu_port_desc()})"},
        "e2e": {"value": us_tok, "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_prefill(args, cfg, sample_T=2048):
    """The CPU path (oracle) on the prefill workload: each step is the first
    sample_T tokens of that step's batch, alternating over the step kinds."""
    from oracle import oracle

    bits = args.bits
    blocks, routing = prefill_blocks(cfg, bits, args.seed)
    ws = [(oracle.BlockWeights(bits=bits, group=64, **b.weight_fields()), np.ascontiguousarray(b.x[:sample_T]))
          for b in blocks]
    for i in range(args.warmup):
        w, x = ws[i % len(ws)]
        oracle.moe_block_fast(w, x, k=8)
    t0 = time.perf_counter()
    for i in range(args.steps):
        w, x = ws[i % len(ws)]
        oracle.moe_block_fast(w, x, k=8)
    el = time.perf_counter() - t0
    tok_s = args.steps * sample_T / el
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": "moe_block_prefill_tokens_per_s", "value": tok_s, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config{args.config} q{bits} prefill T={cfg['T']}", "bits": bits,
                   "tokens_per_step": sample_T, "routing": routing},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} calls of the first {sample_T} tokens of each batch ({cpu_port_desc()})"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_profile(args, cfg=None):
    """Small fixed case for ncu captures: two block copies (~1 GB for q4),
    W + K plain (non-graph) block calls, no timing, no CPU baseline."""
    import torch

    from runnel_b200 import inputs, ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if cfg is not None:
        # prefill: the configuration's first step kind, plain calls
        blk = prefill_blocks(cfg, args.bits, args.seed)[0][0]
        bt = ops.BlockTensors.from_numpy(blk, dev)
        x = torch.from_numpy(blk.x).view(torch.int16).view(torch.bfloat16).to(dev)
        ws = ops.Workspace(dev)
        for _ in range(args.warmup + args.steps):
            ops.moe_block(bt, x, ws=ws)
        torch.cuda.synchronize()
        print(json.dumps({"profile": True, "bits": args.bits, "tokens": cfg["T"],
                          "calls": args.warmup + args.steps}))
        return
    blk = inputs.make_block(args.bits, seed=args.seed, T=1)
    copies = [ops.BlockTensors.from_numpy(blk, dev)]
    copies.append(ops.BlockTensors(**{f: (v.clone() if isinstance(v, torch.Tensor) else v)
                                      for f, v in copies[0].__dict__.items()}))
    xs = torch.from_numpy(inputs.make_tokens(args.seed, 64 * args.tokens)).view(torch.int16)
    xs = xs.view(torch.bfloat16).to(dev).reshape(64, args.tokens, -1)
    ws = ops.Workspace(dev)
    for i in range(args.warmup + args.steps):
        ops.moe_block(copies[i % 2], xs[i % 64], ws=ws)
    torch.cuda.synchronize()
    print(json.dumps({"profile": True, "bits": args.bits, "tokens": args.tokens,
                      "calls": args.warmup + args.steps}))


def cpu_baseline_prefill(blocks, bits, sample_T=2048, budget_s=10.0):
    """CPU tokens/s on a bounded sample: the first sample_T tokens of each
    step's batch, alternating over the step kinds of the workload."""
    from oracle import oracle

    ws = [(oracle.BlockWeights(bits=bits, group=64, **b.weight_fields()), np.ascontiguousarray(b.x[:sample_T]))
          for b in blocks]
    n = 0
    t0 = time.perf_counter()
    while True:
        w, x = ws[n % len(ws)]
        oracle.moe_block_fast(w, x, k=8)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"value": n * sample_T / el, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{n} block calls of {sample_T} tokens (first tokens of the workload's batches), "
                      f"q{bits} ({cpu_port_desc()})"}


def prefill_blocks(cfg, bits, seed):
    """Synthetic blocks of one prefill configuration: one per step kind."""
    from runnel_b200 import inputs

    T = cfg["T"]
    if cfg.get("skew") == "zipf":
        return [inputs.make_block(bits, seed=seed, T=T, skew="zipf")], "log-Zipf(s=1.1) expert skew"
    return ([inputs.make_block(bits, seed=seed, T=T), inputs.make_block(bits, seed=seed, T=T, skew="adversarial")],
            "uniform / adversarial (25% of tokens on one expert) on alternate steps")


def run_prefill_bench(args, cfg):
    import torch

    from runnel_b200 import _lib, ops

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    bits, T = args.bits, cfg["T"]
    blocks, routing = prefill_blocks(cfg, bits, args.seed)
    a2a = world > 1 and args.prefill_par in ("device", "a2a", "gather")
    E_range = None
    dctx = None
    if a2a:
        from runnel_b200 import ep as epm
        E_range = epm.plan(rank, world)[:2]
        if args.prefill_par == "device":
            dctx = epm.DeviceAllToAll(rank, world, max_tokens=T)
    base = ops.BlockTensors.from_numpy(blocks[0], dev, E_range=E_range)
    kinds = [base]
    for b in blocks[1:]:  # same expert weights, the step kind's router
        rw = torch.from_numpy(b.router_w).view(torch.int16).view(torch.bfloat16).to(dev)
        kinds.append(ops.BlockTensors(**{**base.__dict__, "router_w": rw}))
    # every rank has its own tokens (the batch rotated by a rank-dependent offset)
    xs = [torch.roll(torch.from_numpy(b.x).view(torch.int16).view(torch.bfloat16).to(dev), 997 * rank, 0)
          for b in blocks]
    out = torch.empty_like(xs[0])
    ws = ops.Workspace(dev)
    stream = torch.cuda.Stream(dev)
    nk = len(kinds)
    moved = {"sent": 0, "received": 0}

    def block(i, x, o):
        if dctx is not None:
            dctx.moe_block(kinds[i % nk], x, out=o)
        elif a2a and args.prefill_par == "gather":
            o.copy_(epm.moe_block_gather(kinds[i % nk], x, rank, world, ws=ws))
            moved["sent"] += x.shape[0] * (world - 1)
            moved["received"] += x.shape[0] * (world - 1)
        elif a2a:
            st = {}
            o.copy_(epm.moe_block_a2a(kinds[i % nk], x, rank, world, ws=ws, stats=st))
            moved["sent"] += st["sent"]
            moved["received"] += st["received"]
        else:
            ops.moe_block(kinds[i % nk], x, ws=ws, out=o)

    def step(i):
        block(i, xs[i % nk], out)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    stream.synchronize()
    assert ws.status() == 0
    dev_rows = None
    if dctx is not None:
        # rows each step sends: (token, other rank owning one of its experts)
        assert dctx.status() == 0
        rows = []
        for i in range(nk):
            _, inds, _ = dctx.moe_block(kinds[i], xs[i], out=out, return_routing=True)
            own = inds.long() // (256 // world)
            hit = torch.zeros((inds.shape[0], world), dtype=torch.bool, device=dev).scatter_(1, own, True)
            hit[:, rank] = False
            rows.append(int(hit.sum()))
        dev_rows = sum(rows) / len(rows)
    K = args.steps
    moved.update(sent=0, received=0)
    sampler = ClockSampler(local)
    sampler.start()
    _lib.stage_timing(True)

    def run_k():
        for i in range(K):
            step(i)

    trials = timed_trials(run_k, stream, dist, dev, args.min_time)
    _lib.stage_timing(False)
    stages, ncalls = _lib.stage_times()
    clocks = sampler.stop()
    moved_timed = {k: v / len(trials) for k, v in moved.items()}
    ms = statistics.median(trials)
    ms_step = ms / K
    tok_s = T * K * world / (ms * 1e-3)
    assert ws.status() == 0
    if dctx is not None:
        assert dctx.status() == 0

    # end to end through the public API: pinned host tokens in, host output back
    xh = [x.cpu().pin_memory() for x in xs]
    oh = torch.empty_like(xh[0]).pin_memory()
    xd = torch.empty_like(xs[0])
    od = torch.empty_like(xd)
    if not a2a:
        # one C call per step (rnb_moe_block_fwd_host): the batch is split into
        # chunks whose copies in and out overlap the other chunks' compute
        calls = [ops.BlockCall(kd, T, ws=ws) for kd in kinds]

        def host_step(i):
            calls[i % nk].host(xh[i % nk], oh)
    else:
        def host_step(i):
            xd.copy_(xh[i % nk], non_blocking=True)
            block(i, xd, od)
            oh.copy_(od, non_blocking=True)
    with torch.cuda.stream(stream):
        for i in range(3):
            host_step(i)
    stream.synchronize()

    def e2e_k():  # K steps through the public API, each from and to pinned host memory
        for i in range(K):
            host_step(i)

    e2e_ms = statistics.median(timed_trials(e2e_k, stream, dist, dev, args.min_time / 2))
    e2e_tok_s = T * K * world / (e2e_ms * 1e-3)

    gemm_flops, all_flops = prefill_flops(T)
    _, bf16_burst, src = peaks()
    sustained = None
    pth = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pth):
        sustained = json.load(open(pth)).get("bf16_tflops_sustained")
    peak = sustained or bf16_burst
    # stage times are summed over every timed call (all trials); per step:
    calls_per_step = max(ncalls, 1) / (K * len(trials))
    gemm_ms = (stages.get("gateup", 0.0) + stages.get("down", 0.0)) / max(ncalls, 1) * calls_per_step
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
    line = {
        "metric": "moe_block_prefill_tokens_per_s", "value": tok_s, "unit": "tokens/s",
        "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": ms_step,
        "trials": len(trials), "trial_ms": {"median": ms, "min": min(trials), "max": max(trials)},
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "mma_operands": "fp16 (tcgen05 kind::f16: weights dequantised to fp16, tokens scaled by exact powers "
                        "of two), fp32 accumulation in TMEM",
        "data": "synthetic (seeded MLX-affine block, N(0,1) bf16 tokens)",
        "config": {"workload": f"config{args.config} q{bits} prefill T={T}", "bits": bits,
                   "tokens_per_step": T, "routing": routing, "H": 2048, "I": 512, "E": 256, "top_k": 8,
                   "l2": "inputs larger than L2: every step reads the whole expert bank (>= 0.8 GB)",
                   "tokens_per_step_per_gpu": T,
                   "parallelism": ((f"ep{world} device all-to-all ({256 // world} experts/GPU; rows and fp32 "
                                    "sums by NVLink stores inside the kernels, no host synchronisation; shared "
                                    "expert on every rank for its own tokens)" if args.prefill_par == "device" else
                                    f"ep{world} ({256 // world} experts/GPU; dispatch NCCL all_gather, combine "
                                    "NCCL reduce_scatter of fp32 partials; shared expert on every rank for its "
                                    "own tokens)" if args.prefill_par == "gather" else
                                    f"ep{world} all-to-all ({256 // world} experts/GPU, NCCL all_to_all_single "
                                    "dispatch/combine, shared expert on every rank for its own tokens)")
                                   if a2a else "replica") if world > 1 else "single"},
        "e2e": {"value": e2e_tok_s, "unit": "tokens/s", "h2d_bytes_per_step": T * 2048 * 2,
                "d2h_bytes_per_step": T * 2048 * 2},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": (achieved / peak) if achieved else None,
                     "peak_source": f"{src} bf16 {'sustained' if sustained else 'burst'}",
                     "frac_of_burst": (achieved / bf16_burst) if achieved and bf16_burst else None,
                     "traffic": MEASURED_TRAFFIC.get(f"config{args.config} q{bits} prefill T={T}", (None,))[0],
                     "traffic_source": MEASURED_TRAFFIC.get(f"config{args.config} q{bits} prefill T={T}", (None, None))[1],
                     "algorithmic_flops_per_step": gemm_flops,
                     "kernel": "k_pre_gemm (gate/up + down launches)", "gemm_ms_per_step": gemm_ms,
                     "block_tflops": all_flops / (ms_step * 1e-3) / 1e12,
                     **({"note": "the home and the remote experts' GEMMs run at the same time on two streams; "
                                 "their event-timed durations overlap, so achieved is a lower bound"}
                        if a2a and args.prefill_par == "device" and world > 1 else {})},
        "stages_ms_per_step": {k: v / max(ncalls, 1) * calls_per_step for k, v in stages.items()},
        # route, sort, scatter, gather, gate/up, row scale, down, final (twice per step with all-to-all)
        "gpu_launches": K * (21 if dctx is not None else 8 * (2 if a2a else 1)),
        "clocks": clocks,
    }
    if dctx is not None:
        line["ep_rows_per_step"] = {"sent": dev_rows, "bytes_out": dev_rows * (2048 * 2 + 64),
                                    "bytes_back": dev_rows * 2048 * 4, "rank": rank, "exchange": "device"}
    elif a2a:
        mv = moved_timed
        line["ep_rows_per_step"] = {"sent": mv["sent"] / K, "received": mv["received"] / K,
                                    "bytes_out": mv["sent"] / K * (2048 * 2 + 64),
                                    "bytes_back": mv["sent"] / K * 2048 * 4, "rank": rank,
                                    "exchange": args.prefill_par}
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline_prefill(blocks, bits, budget_s=args.cpu_budget)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        if dctx is not None:
            torch.cuda.synchronize()
            dctx.close()  # every rank past the barrier: no peer reads its areas any more
            dist.barrier()
        dist.destroy_process_group()


def run_stack_bench(args, cfg):
    """Configuration 4: a stack of L distinct q4 MoE blocks with residual adds
    and RMSNorms, batch-1 decode of sequential tokens (each token's input is
    the previous token's output).  One token's layers are one CUDA graph that
    also copies its output back to its input; a step is one replay (one token
    through all layers).  N > 1: expert parallel, every layer sharded."""
    import torch

    from runnel_b200 import ops, stack

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    from runnel_b200 import ep as epm
    from runnel_b200.inputs import make_tokens

    bits, L = args.bits, args.layers or cfg["layers"]
    E_range = epm.plan(rank, world)[:2] if world > 1 else None
    # layer l = inputs.make_block(bits, seed=1000 * seed + l): the canonical generator
    layers, norms = stack.canonical_layers(L, bits, args.seed, dev, E_range=E_range)
    ctx = epm.ExpertParallel(rank, world) if world > 1 else None
    ws = ops.Workspace(dev)
    st = stack.LayerStack(layers, norms, ep=ctx, ws=ws)
    x0 = torch.from_numpy(make_tokens(args.seed, 1)).view(torch.int16).view(torch.bfloat16).to(dev)
    xin, xout = x0.clone(), torch.empty_like(x0)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        st.forward(xin, out=xout)  # workspace allocation outside the capture
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            st.forward(xin, out=xout)
            xin.copy_(xout)
    # routing of every layer for the roofline's bytes (one eager pass on token 0)
    rec = []
    with torch.cuda.stream(stream):
        xin.copy_(x0)
        st.forward(xin, out=xout, record=rec)
    stream.synchronize()
    rws = ops.Workspace(dev)
    distinct = []
    for l, (_, xn, _) in enumerate(rec):
        inds = ops.router_topk(layers[l], xn, ws=rws)[0]
        distinct.append(len(np.unique(inds.cpu().numpy())))
    per_tok = sum(step_bytes(bits, d, 1) for d in distinct)
    K, W = args.steps, args.warmup
    with torch.cuda.stream(stream):
        xin.copy_(x0)
        for _ in range(W):
            g.replay()
    stream.synchronize()
    sampler = ClockSampler(local)
    sampler.start()

    def run_k():  # K sequential tokens: each replay is one token through every layer
        for _ in range(K):
            g.replay()

    trials = timed_trials(run_k, stream, dist, dev, args.min_time)
    clocks = sampler.stop()
    ms = statistics.median(trials)
    us_tok = ms * 1e3 / K
    # end to end: each token's input copied in from pinned host memory and its
    # output read back, every step
    xh = x0.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    hb = [xh, oh]

    def e2e_k():
        for _ in range(K):
            xin.copy_(hb[0], non_blocking=True)
            g.replay()
            hb[1].copy_(xout, non_blocking=True)
            hb.reverse()

    e2e_ms = statistics.median(timed_trials(e2e_k, stream, dist, dev, args.min_time / 2))
    assert ws.status() == 0, "device status reported a timeout or a bad index"
    hbm, _, src = peaks()
    achieved = per_tok / (us_tok * 1e-6) / 1e9
    line = {
        "metric": "moe_stack_decode_us_per_token", "value": us_tok, "unit": "us/token",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": us_tok * 1e-3,
        "trials": len(trials), "trial_ms": {"median": ms, "min": min(trials), "max": max(trials)},
        "higher_is_better": False, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "bf16",
        "mma_operands": "fp16 (codes exact, activations scaled by exact powers of two), fp32 accumulation",
        "data": "synthetic (runnel_b200.inputs: layer l = make_block(4, seed=1000*seed + l), numpy PCG64)",
        "config": {"workload": f"config4 {L} q{bits} layers, batch-1 sequential decode", "bits": bits,
                   "layers": L, "tokens_per_step": 1, "H": 2048, "I": 512, "E": 256, "top_k": 8,
                   "l2": f"inputs larger than L2: {L} layers of weights per step",
                   "parallelism": f"ep{world}" if world > 1 else "single"},
        "e2e": {"value": e2e_ms * 1e3 / K, "unit": "us/token", "h2d_bytes_per_step": 2048 * 2,
                "d2h_bytes_per_step": 2048 * 2},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm * world, "unit": "GB/s",
                     "frac": achieved / (hbm * world), "peak_source": f"{src} x {world} GPU",
                     "traffic": None, "algorithmic_bytes_per_step": per_tok,
                     "kernel": "k_decode per layer (residual add + RMSNorm fused into its prologue), "
                               "one k_add_rmsnorm per token (the last residual add)"},
        "gpu_launches": K * (L + 1),
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline_stack(layers, norms, bits, x0, budget_s=args.cpu_budget)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        del g
        dist.barrier()
        if ctx is not None:
            ctx.close()
        dist.destroy_process_group()


def cpu_baseline_stack(layers, norms, bits, x0, n_layers=4, budget_s=10.0):
    """CPU oracle on a bounded sample: one token through the first n_layers
    layers (same weights, copied to the host), repeated; scaled to all layers."""
    import torch

    from oracle import oracle
    from runnel_b200 import stack
    from runnel_b200.quant import f32_to_bf16_bits

    def u16(t):
        return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)

    def u32(t):
        return t.cpu().contiguous().view(torch.int32).numpy().view(np.uint32)

    ws = []
    for bt in layers[:n_layers]:
        ws.append(oracle.BlockWeights(bits=bits, group=64, router_w=u16(bt.router_w), shared_gate_w=u16(bt.shared_gate_w),
                                      gu_w=u32(bt.gu_w), gu_s=u16(bt.gu_s), gu_b=u16(bt.gu_b), dn_w=u32(bt.dn_w),
                                      dn_s=u16(bt.dn_s), dn_b=u16(bt.dn_b), sgu_w=u32(bt.sgu_w), sgu_s=u16(bt.sgu_s),
                                      sgu_b=u16(bt.sgu_b), sdn_w=u32(bt.sdn_w), sdn_s=u16(bt.sdn_s),
                                      sdn_b=u16(bt.sdn_b)))
    nw = [u16(w) for w in norms[:n_layers + 1]]
    x = u16(x0)
    n = 0
    t0 = time.perf_counter()
    while True:
        xa, xn = stack.reference_add_rmsnorm(x, None, nw[0])
        for l in range(n_layers):
            y, _, _ = oracle.moe_block_fast(ws[l], xn, k=8)
            xa, xn = stack.reference_add_rmsnorm(xa, f32_to_bf16_bits(y), nw[l + 1])
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    L = len(layers)
    return {"value": el / n * 1e6 * L / n_layers, "unit": "us/token", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{n} tokens through the first {n_layers} of {L} layers ({cpu_port_desc()}), "
                      f"scaled by {L}/{n_layers}"}


def run_ours(args):
    import torch

    from runnel_b200 import inputs, ops

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    bits, T = args.bits, args.tokens
    blk = inputs.make_block(bits, seed=args.seed, T=1)
    ctx = None
    ws = ops.Workspace(dev)
    if world > 1:
        # expert parallel: this rank's expert shard and shared-expert quarters,
        # partial outputs exchanged over NVLink inside the decode kernel
        from runnel_b200 import ep as epm

        lo, hi, _ = epm.plan(rank, world, blk.E, blk.I)
        base = ops.BlockTensors.from_numpy(blk, dev, E_range=(lo, hi))
        ctx = epm.ExpertParallel(rank, world, blk.H)

        def block_call(bt, x, out):
            return ctx.moe_block(bt, x, ws=ws, out=out)
    else:
        base = ops.BlockTensors.from_numpy(blk, dev)

        def block_call(bt, x, out):
            return ops.moe_block(bt, x, ws=ws, out=out)
    gu, dn = expert_bytes(bits)
    # bytes one rank streams per step: its share of the selected experts and
    # of the shared expert, plus the whole router
    per_step = step_bytes(bits, min(8 * T, 256), T) / world + 256 * 2048 * 2 * (1 - 1 / world)
    R = max(4, int(np.ceil(4 * L2_BYTES / per_step)))
    R = min(R, 48 if world == 1 else 160)
    copies = [base]
    for _ in range(R - 1):
        c = ops.BlockTensors(**{f: (v.clone() if isinstance(v, torch.Tensor) else v)
                                for f, v in base.__dict__.items()})
        copies.append(c)
    ntok = R * T
    xs_np = inputs.make_tokens(args.seed, ntok)
    xs = torch.from_numpy(xs_np).view(torch.int16).view(torch.bfloat16).to(dev).reshape(R, T, -1)
    outs = torch.empty_like(xs)
    stream = torch.cuda.Stream(dev)

    def one(i):
        block_call(copies[i], xs[i], outs[i])

    with torch.cuda.stream(stream):
        for i in range(R):
            one(i)
    stream.synchronize()
    # distinct experts actually touched per step (for the roofline's bytes)
    inds_all = []
    rws = ops.Workspace(dev)
    with torch.cuda.stream(stream):
        for i in range(R):
            inds_all.append(ops.router_topk(copies[i], xs[i], ws=rws)[0])
    stream.synchronize()
    distinct = float(np.mean([len(np.unique(ii.cpu().numpy())) for ii in inds_all]))
    per_step = step_bytes(bits, distinct, T)  # whole block, all ranks

    # The K timed steps and the W warm-up steps are each one CUDA graph; step
    # i uses weight copy i % R and token block i % R.
    K, W = args.steps, args.warmup

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                one(i % R)
        return g

    g_warm, g_time = capture(W), capture(K)
    with torch.cuda.stream(stream):
        g_warm.replay()
    stream.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    trials = timed_trials(g_time.replay, stream, dist, dev, args.min_time)
    clocks = sampler.stop()
    ms = statistics.median(trials)
    ms_step = ms / K
    us_tok = ms_step * 1e3 / T

    # end to end through the public API with host buffers
    xh = torch.from_numpy(xs_np).view(torch.int16).view(torch.bfloat16).reshape(R, T, -1).pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    xd = torch.empty((T, xs.shape[-1]), dtype=torch.bfloat16, device=dev)
    od = torch.empty_like(xd)
    if world == 1:
        # one prepared call per bank copy: copy-in, block and copy-out are one
        # C call (rnb_moe_block_fwd_host) from pinned host memory
        calls = [ops.BlockCall(copies[i], T, ws=ws) for i in range(R)]

        def host_step(i):
            calls[i].host(xh[i], oh[i])
    else:
        def host_step(i):
            xd.copy_(xh[i], non_blocking=True)
            block_call(copies[i], xd, od)
            oh[i].copy_(od, non_blocking=True)
    with torch.cuda.stream(stream):
        for i in range(W):
            host_step(i % R)
    stream.synchronize()

    def e2e_k():  # K steps through the public API, each from and to pinned host memory
        for s_ in range(K):
            host_step(s_ % R)

    e2e_trials = timed_trials(e2e_k, stream, dist, dev, args.min_time / 2)
    e2e_us = statistics.median(e2e_trials) * 1e3 / (K * T)
    assert ws.status() == 0, "device status reported a timeout or a bad index"

    hbm, _, src = peaks()
    achieved = per_step / (ms_step * 1e-3) / 1e9  # all ranks together
    persistent = T == 1 or (T == 2 and bits == 4)
    line = {
        "metric": "moe_block_decode_us_per_token", "value": us_tok, "unit": "us/token",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms_step,
        "trials": len(trials), "trial_ms": {"median": ms, "min": min(trials), "max": max(trials)},
        "higher_is_better": False, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "bf16",
        "mma_operands": "fp16 (codes exact, activations scaled by exact powers of two), fp32 accumulation",
        "data": "synthetic (seeded MLX-affine block, N(0,1) bf16 tokens)",
        "config": {"workload": f"config{args.config} q{bits} decode T={T}", "bits": bits,
                   "tokens_per_step": T, "H": 2048, "I": 512, "E": 256, "top_k": 8,
                   "weight_copies_rotated": R, "l2": "inputs rotate over R block copies (>= 4x L2 where memory allows)",
                   "parallelism": f"ep{world} (experts {256 // world}/GPU, NVLink exchange in-kernel)"
                   if world > 1 else "single"},
        "e2e": {"value": e2e_us, "unit": "us/token", "h2d_bytes_per_step": T * 2048 * 2,
                "d2h_bytes_per_step": T * 2048 * 2},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm * world, "unit": "GB/s",
                     "frac": achieved / (hbm * world), "peak_source": f"{src} x {world} GPU",
                     "frac_of_nominal_8tbs": achieved / (HBM_NOMINAL_GBS * world),
                     "traffic": MEASURED_TRAFFIC.get(f"config{args.config} q{bits} decode T={T}", (None,))[0]
                     if world == 1 else None,
                     "traffic_source": MEASURED_TRAFFIC.get(f"config{args.config} q{bits} decode T={T}", (None, None))[1]
                     if world == 1 else None,
                     "algorithmic_bytes_per_step": per_step,
                     "distinct_experts_per_step": distinct,
                     "kernel": "k_decode (persistent, one launch per step)" if persistent
                     else "k_route+k_gateup+k_down chain" + (" + k_ep_reduce" if world > 1 else "")},
        "gpu_launches": K if persistent else (3 + (1 if world > 1 else 0)) * K * ((T + 63) // 64),
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(bits, T, budget_s=args.cpu_budget, seed=args.seed)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        del g_time, g_warm
        dist.barrier()
        if ctx is not None:
            ctx.close()
        dist.destroy_process_group()


def run_probe(args):
    """The reference's QMV / QMM probe CLIs on their default shapes
    (quantized_qmv.cpp: 65536 x 2048; quantized_qmm.cpp: 64 tokens x 4096 x
    2048), K-step timed with CUDA events over weight copies rotated so that
    every step reads from HBM (4 copies > L2).  --impl reference times the
    oracle's restatement of the probes' CPU reference on the host cores."""
    import torch

    from runnel_b200 import probes

    bits = args.bits or 4
    qmv = args.probe == "qmv"
    rows, K, T = (65536, 2048, 1) if qmv else (4096, 2048, 64)
    wbytes = rows * (K * bits // 8 + 2 * (K // 64) * 2)
    workload = f"{args.probe} q{bits} " + (f"{rows}x{K}" if qmv else f"T={T} N={rows} K={K}")
    if args.impl == "reference":
        from oracle import oracle
        data = (oracle.kat_qmv(bits, 4096, K=K) if qmv else oracle.kat_qmm(bits, T, 512, K))[0]
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min(args.cpu_budget, 10.0):
            if qmv:
                oracle.kat_qmv(bits, 4096, K=K)
            else:
                oracle.kat_qmm(bits, T, 512, K)
            n += 1
        el = (time.perf_counter() - t0) / n
        # the sample regenerates its data each call: the rate is a bound from below
        frac = 4096 / rows if qmv else 512 / rows
        value = wbytes * frac / el / 1e9
        print(json.dumps({"metric": f"{args.probe}_weight_GBps", "value": value, "unit": "GB/s", "impl": "reference",
                          "n_gpus": 1, "steps": n, "warmup": 0, "higher_is_better": True, "dtype": f"u{bits}",
                          "config": {"workload": workload},
                          "cpu_baseline": {"value": value, "unit": "GB/s", "cores": os.cpu_count() or 1,
                                           "kind": "port", "sample": f"{n} oracle calls on {frac:.4f} of the rows "
                                                                     "(data generation included)"},
                          "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    copies = [probes.synthetic(bits, rows, K, tokens=T, seed=i) for i in range(4)]
    ws = None
    if not qmv:
        import ctypes
        from runnel_b200 import _lib
        need = ctypes.c_size_t()
        _lib.call("rnb_qmm_workspace_size", bits, 64, T, rows, K, ctypes.byref(need))
        ws = torch.empty(need.value, dtype=torch.uint8, device=dev)

    def step(i):
        w, s_, b_, x = copies[i % 4]
        return probes.qmv(bits, w, s_, b_, x[0]) if qmv else probes.qmm(bits, w, s_, b_, x, ws=ws)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    sampler.start()
    K_ = args.steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_end = time.time() + args.soak  # clock samples under load
    while time.time() < t_end:
        for i in range(64):
            step(i)
        torch.cuda.synchronize()
    ev0.record()
    for i in range(K_):
        step(i)
    ev1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1) / K_
    gbs = wbytes / (ms * 1e-3) / 1e9
    hbm, bf16_burst, src = peaks()
    flops = 2.0 * T * rows * K
    line = {"metric": f"{args.probe}_weight_GBps", "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": K_,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": f"u{bits}", "data": "synthetic (seeded uniform codes, N(0,1) bf16 x)",
            "config": {"workload": workload, "l2": "4 rotated weight copies (> L2)"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_source": src, "traffic": None, "kernel": "k_qmv" if qmv else "k_pre_gemm<1>",
                         "tflops": flops / (ms * 1e-3) / 1e12},
            "gpu_launches": K_ * (1 if qmv else 3), "clocks": clocks}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=480)
    ap.add_argument("--warmup", type=int, default=48)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--bits", type=int, default=None)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--layers", type=int, default=None, help="configuration 4: number of layers (default 40)")
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--soak", type=float, default=1.5, help="probe mode: seconds of load before timing")
    ap.add_argument("--min-time", type=float, default=1.0,
                    help="seconds of timed trials (each trial is exactly --steps steps; the median is reported)")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--prefill-par", default="device", choices=["device", "gather", "a2a", "replica"],
                    help="prefill at N > 1: expert parallel with gather/reduce-scatter or all-to-all exchange, "
                         "or whole-bank replicas")
    ap.add_argument("--profile", action="store_true",
                    help="small case for ncu captures (2 weight copies, plain launches)")
    ap.add_argument("--probe", default=None, choices=["qmv", "qmm"],
                    help="time the standalone QMV / QMM probe instead of a configuration")
    args = ap.parse_args()
    if args.probe:
        args.steps = args.steps if "--steps" in sys.argv else 200
        return run_probe(args) if int(os.environ.get("RANK", "0")) == 0 else None
    from runnel_b200.inputs import CONFIGS
    cfg = CONFIGS[args.config]
    args.bits = args.bits or cfg["bits"]
    args.seed = cfg["seed"] if args.seed is None else args.seed
    args.warmup = max(args.warmup, 3)
    prefill = cfg.get("T", 1) > 64
    if "layers" in cfg and not args.profile:
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                run_reference_stack(args, cfg)
            return
        if "--steps" not in sys.argv:
            args.steps = cfg.get("steps", 64)
        return run_stack_bench(args, cfg)
    if args.impl == "reference":
        run_reference(args, cfg) if prefill else run_reference(args)
    elif args.profile:
        run_profile(args, cfg if prefill else None)
    elif prefill:
        run_prefill_bench(args, cfg)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
