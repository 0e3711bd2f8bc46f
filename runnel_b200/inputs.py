"""Seeded synthetic sparse-MoE blocks in MLX affine layout.

One generator for the GPU path, the CPU oracle checks and the benchmarks, so
every consumer sees identical bytes for a given (seed, shape).  Distributions
follow the benchmark configurations of the reference's hot path (Ornith-1.5
MoE block: H=2048, E=256 experts of I=512, top-8, group 64):

* codes uniform on ``[0, 2^bits)`` -- every nibble of a 4-bit word random --
  which makes every packed uint32 word uniform, so words are drawn directly;
* scales ``U(0.001, 0.01)`` and biases ``N(0, 0.01)``, rounded to bf16 (RNE);
* router and shared-expert-gate weights ``N(0, 0.02)`` in bf16;
* activations ``x ~ N(0, 1)`` in bf16;
* RMSNorm weights ``1 + N(0, 0.02)`` (eps 1e-6) for layer stacks.

Draw order from ``numpy.random.default_rng(seed)``: x, router W, shared-gate
W, routed gate/up (words, scales, biases), routed down (words, scales,
biases), shared gate/up, shared down, RMSNorm weight.  Routing skews draw from
an independent stream ``default_rng([seed, 1])`` so the weights do not change
with the skew.

Skews (data-only; the block's arithmetic is untouched):

* ``"zipf"``: per-expert logit offset ``-s * log(rank_e)`` for a seeded random
  rank permutation (s = 1.1), carried by feature ``H-1``: ``x[:, H-1] = 1`` and
  ``router_w[:, H-1] = offset``.
* ``"adversarial"``: a fraction (default 25%) of tokens get ``x[t, H-2] = 1``
  and one expert gets ``router_w[e_hot, H-2] = +30`` so those tokens all route
  to it.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .quant import f32_to_bf16_bits


@dataclass
class SyntheticBlock:
    bits: int
    group: int
    x: np.ndarray  # [T,H] u16 (bf16 bits)
    router_w: np.ndarray  # [E,H] u16
    shared_gate_w: np.ndarray  # [H] u16
    gu_w: np.ndarray  # [E,2I,H*bits/32] u32 (up rows, then gate rows)
    gu_s: np.ndarray  # [E,2I,H/64] u16
    gu_b: np.ndarray
    dn_w: np.ndarray  # [E,H,I*bits/32] u32
    dn_s: np.ndarray  # [E,H,I/64] u16
    dn_b: np.ndarray
    sgu_w: np.ndarray  # [2I,H*bits/32]
    sgu_s: np.ndarray
    sgu_b: np.ndarray
    sdn_w: np.ndarray  # [H,I*bits/32]
    sdn_s: np.ndarray
    sdn_b: np.ndarray
    norm_w: np.ndarray  # [H] fp32 RMSNorm weight
    meta: dict = field(default_factory=dict)
    # 8-bit affine router and shared gate (router_bits=8, as real Ornith
    # checkpoints store mlp.gate / mlp.shared_expert_gate): the same fp32
    # draws quantized per 64 inputs (quant.quantize); router_w and
    # shared_gate_w then hold their plain bf16 roundings, unused by the block
    router_bits: int = 16
    router_q: np.ndarray | None = None  # [E,H/4] u32
    router_s: np.ndarray | None = None  # [E,H/64] u16
    router_b: np.ndarray | None = None
    sgate_q: np.ndarray | None = None  # [H/4] u32
    sgate_s: np.ndarray | None = None  # [H/64] u16
    sgate_b: np.ndarray | None = None

    @property
    def E(self) -> int:
        return self.gu_w.shape[0]

    @property
    def H(self) -> int:
        return self.dn_w.shape[1]

    @property
    def I(self) -> int:  # noqa: E743
        return self.gu_w.shape[1] // 2

    def weight_fields(self) -> dict:
        names = ("router_w", "shared_gate_w", "gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b",
                 "sgu_w", "sgu_s", "sgu_b", "sdn_w", "sdn_s", "sdn_b")
        out = {n: getattr(self, n) for n in names}
        if self.router_bits == 8:
            out["router_bits"] = 8
            for n in ("router_q", "router_s", "router_b", "sgate_q", "sgate_s", "sgate_b"):
                out[n] = getattr(self, n)
        return out


def _words(rng, shape) -> np.ndarray:
    return rng.integers(0, 1 << 32, size=shape, dtype=np.uint32)


def _scales(rng, shape) -> np.ndarray:
    return f32_to_bf16_bits(rng.uniform(0.001, 0.01, size=shape).astype(np.float32))


def _biases(rng, shape) -> np.ndarray:
    return f32_to_bf16_bits(rng.normal(0.0, 0.01, size=shape).astype(np.float32))


def _bank(rng, lead, rows, K, bits, group):
    w = _words(rng, (*lead, rows, K * bits // 32))
    s = _scales(rng, (*lead, rows, K // group))
    b = _biases(rng, (*lead, rows, K // group))
    return w, s, b


def make_block(bits: int, seed: int, T: int = 1, H: int = 2048, I: int = 512, E: int = 256,
               group: int = 64, skew: str | None = None, zipf_s: float = 1.1,
               adversarial_frac: float = 0.25, router_bits: int = 16) -> SyntheticBlock:
    if bits not in (4, 8):
        raise ValueError("bits must be 4 or 8")
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32)
    router = rng.normal(0.0, 0.02, size=(E, H)).astype(np.float32)
    sgate = rng.normal(0.0, 0.02, size=(H,)).astype(np.float32)
    gu = _bank(rng, (E,), 2 * I, H, bits, group)
    dn = _bank(rng, (E,), H, I, bits, group)
    sgu = _bank(rng, (), 2 * I, H, bits, group)
    sdn = _bank(rng, (), H, I, bits, group)
    norm_w = (1.0 + rng.normal(0.0, 0.02, size=(H,))).astype(np.float32)
    meta = {"bits": bits, "seed": seed, "T": T, "H": H, "I": I, "E": E, "skew": skew}
    if skew is not None:
        srng = np.random.default_rng([seed, 1])
        if skew == "zipf":
            rank = srng.permutation(E) + 1
            offset = (-zipf_s * np.log(rank)).astype(np.float32)
            x[:, H - 1] = 1.0
            router[:, H - 1] = offset
            meta["zipf_rank"] = rank
        elif skew == "adversarial":
            hot = int(srng.integers(0, E))
            chosen = srng.random(T) < adversarial_frac
            x[:, H - 2] = chosen.astype(np.float32)
            router[:, H - 2] = 0.0
            router[hot, H - 2] = 30.0
            meta["hot_expert"] = hot
            meta["hot_tokens"] = int(chosen.sum())
        else:
            raise ValueError(f"unknown skew {skew!r}")
    blk = SyntheticBlock(
        bits=bits, group=group, x=f32_to_bf16_bits(x), router_w=f32_to_bf16_bits(router),
        shared_gate_w=f32_to_bf16_bits(sgate), gu_w=gu[0], gu_s=gu[1], gu_b=gu[2], dn_w=dn[0],
        dn_s=dn[1], dn_b=dn[2], sgu_w=sgu[0], sgu_s=sgu[1], sgu_b=sgu[2], sdn_w=sdn[0],
        sdn_s=sdn[1], sdn_b=sdn[2], norm_w=norm_w, meta=meta)
    if router_bits == 8:
        from .quant import quantize
        blk.router_bits = 8
        blk.router_q, blk.router_s, blk.router_b = quantize(router, 8, group)
        blk.sgate_q, blk.sgate_s, blk.sgate_b = quantize(sgate, 8, group)
        meta["router_bits"] = 8
    elif router_bits != 16:
        raise ValueError("router_bits must be 16 or 8")
    return blk


def _make_block_args(args):
    bits, seed, kw = args
    return make_block(bits, seed=seed, **kw)


def make_blocks(bits: int, seeds, workers: int | None = None, **kw) -> list[SyntheticBlock]:
    """:func:`make_block` for several seeds, in spawned worker processes (so
    it may run after CUDA is initialised); identical to calling it in turn."""
    import concurrent.futures
    import multiprocessing
    import os

    seeds = list(seeds)
    if len(seeds) <= 1:
        return [make_block(bits, seed=s, **kw) for s in seeds]
    n = workers or min(len(seeds), max(1, (os.cpu_count() or 1) // 2), 16)
    ctx = multiprocessing.get_context("spawn")
    with concurrent.futures.ProcessPoolExecutor(max_workers=n, mp_context=ctx) as pool:
        return list(pool.map(_make_block_args, [(bits, s, kw) for s in seeds]))


def stack_layer_seed(seed: int, layer: int) -> int:
    """Seed of layer ``layer`` of configuration 4's stack (``seed`` = 3)."""
    return seed * 1000 + layer


def make_tokens(seed: int, T: int, H: int = 2048) -> np.ndarray:
    """Extra bf16 activations ``[T,H]`` from an independent stream."""
    rng = np.random.default_rng([seed, 2])
    return f32_to_bf16_bits(rng.standard_normal((T, H), dtype=np.float32))


# Benchmark configurations of the reference's hot path (seeded as listed).
CONFIGS = {
    1: {"bits": 8, "seed": 0, "T": 1, "name": "q8 decode T=1"},
    2: {"bits": 4, "seed": 1, "T": 1, "name": "q4 decode T=1 and T=8", "T_alt": 8},
    3: {"bits": 8, "seed": 2, "T": 2048, "skew": "zipf", "name": "q8 prefill T=2048 Zipf skew"},
    4: {"bits": 4, "seed": 3, "T": 1, "layers": 40, "steps": 64,
        "name": "40 q4 layers, 64 sequential batch-1 tokens"},
    5: {"bits": 8, "seed": 4, "T": 16384, "name": "q8 T=16384, uniform / adversarial"},
}
