"""A decoder stack of MoE blocks only (benchmark configuration 4).

    x <- x + block_l(rms_norm_l(x))   for l = 0 .. L-1

with bf16 activations between layers (mlx-lm's Qwen3.5 decoder layer without
attention: ``h = x + mlp(post_attention_layernorm(x))``).  Each layer is one
:class:`runnel_b200.ops.BlockTensors` (or this rank's expert shard of it) and a
bf16 RMSNorm weight.  A layer is one call, ``rnb_moe_block_norm_fwd``: the
residual add of the previous block's output and this layer's norm, then the
block; for one or two tokens the glue runs inside the block's persistent
launch (bit-identical to ``rnb_add_rmsnorm`` + block).  With an
:class:`runnel_b200.ep.ExpertParallel` context every block call is expert
parallel: each rank holds its shard of every layer and all ranks end with
the same activations.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .ops import BlockTensors, Workspace, _ptr, _stream

RMS_EPS = 1e-6


def add_rmsnorm(x: torch.Tensor, y: torch.Tensor | None, w: torch.Tensor, x_out: torch.Tensor,
                xn_out: torch.Tensor, eps: float = RMS_EPS) -> None:
    """x_out = bf16(x + y) (y may be None), xn_out = bf16(rms_norm(x_out) * w); [T, H] bf16."""
    T, H = x.shape
    _lib.call("rnb_add_rmsnorm", _ptr(x), _ptr(y), _ptr(w), _ptr(x_out), _ptr(xn_out), T, H,
              ctypes.c_float(eps), _stream())


class LayerStack:
    """L MoE blocks with residual adds and RMSNorms between them."""

    def __init__(self, layers: list[BlockTensors], norm_w: list[torch.Tensor], eps: float = RMS_EPS,
                 ep=None, ws: Workspace | None = None):
        if len(layers) != len(norm_w) or not layers:
            raise ValueError("need one RMSNorm weight per layer")
        self.layers, self.norm_w, self.eps, self.ep = layers, norm_w, eps, ep
        self.ws = ws

    def _layer(self, bt: BlockTensors, resid, y_prev, w, resid_out, xn, y) -> None:
        """resid_out = resid + y_prev, xn = norm(resid_out) * w, y = block(xn)."""
        from .ops import default_workspace
        T = resid.shape[0]
        d = bt.desc(T, 8)
        ws = self.ws or default_workspace(resid.device)
        wp, wn = ws.get(d)
        ep = self.ep._ep if self.ep is not None else None
        if self.ep is not None and not ep:
            raise RuntimeError("ExpertParallel context is closed")
        _lib.call("rnb_moe_block_norm_fwd", ctypes.byref(d), ep, _ptr(resid), _ptr(y_prev), _ptr(w),
                  ctypes.c_float(self.eps), _ptr(resid_out), _ptr(xn), _ptr(y), wp, wn, _stream())

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, record: list | None = None) -> torch.Tensor:
        """[T, H] bf16 -> [T, H] bf16.  ``record`` (a list) receives per layer
        (norm input x, block input xn, block output y) copies, for checking."""
        T, H = x.shape
        if out is None:
            out = torch.empty_like(x)
        resid_bufs = (torch.empty_like(x), torch.empty_like(x))  # the residual stream, alternating
        xn = torch.empty_like(x)
        y = torch.empty_like(x)
        resid, y_prev = x, None
        for l, bt in enumerate(self.layers):
            r_out = resid_bufs[l % 2]
            self._layer(bt, resid, y_prev, self.norm_w[l], r_out, xn, y)
            if record is not None:
                record.append([r_out.clone(), xn.clone(), y.clone()])
            resid, y_prev = r_out, y
        # the last block's residual add (its norm output is not used)
        add_rmsnorm(resid, y, self.norm_w[-1], out, xn, self.eps)
        return out


def reference_add_rmsnorm(x_bits: np.ndarray, y_bits: np.ndarray | None, w_bits: np.ndarray,
                          eps: float = RMS_EPS) -> tuple[np.ndarray, np.ndarray]:
    """numpy form of rnb_add_rmsnorm on bf16 bit patterns (for tests)."""
    from .quant import bf16_bits_to_f32, f32_to_bf16_bits

    x = bf16_bits_to_f32(x_bits)
    if y_bits is not None:
        x = bf16_bits_to_f32(f32_to_bf16_bits(x + bf16_bits_to_f32(y_bits)))
    xo = f32_to_bf16_bits(x)
    ss = (x.astype(np.float32) ** 2).sum(axis=-1, dtype=np.float32)
    r = (1.0 / np.sqrt(ss / np.float32(x.shape[-1]) + np.float32(eps))).astype(np.float32)
    xn = f32_to_bf16_bits((x * r[..., None]).astype(np.float32) * bf16_bits_to_f32(w_bits))
    return xo, xn


def canonical_layers(L: int, bits: int, seed: int, device, E_range: tuple[int, int] | None = None,
                     on_block=None) -> tuple[list[BlockTensors], list[torch.Tensor]]:
    """The stack of benchmark configuration 4 from the canonical generator:
    layer l is ``inputs.make_block(bits, seed=inputs.stack_layer_seed(seed, l))``
    (numpy PCG64, the distributions of runnel_b200.inputs) with its RMSNorm
    weight ``norm_w`` rounded to bf16.  Layers are generated eight at a time
    in worker processes and uploaded; ``on_block(l, block)`` sees each host
    block before it is dropped.  With E_range only that expert shard of each
    layer is uploaded."""
    from . import inputs
    from .quant import f32_to_bf16_bits

    layers, norms = [], []
    for l0 in range(0, L, 8):
        seeds = [inputs.stack_layer_seed(seed, l) for l in range(l0, min(L, l0 + 8))]
        for i, b in enumerate(inputs.make_blocks(bits, seeds, T=1)):
            layers.append(BlockTensors.from_numpy(b, device, E_range=E_range))
            norms.append(torch.from_numpy(f32_to_bf16_bits(b.norm_w).view(np.int16)).view(torch.bfloat16).to(device))
            if on_block is not None:
                on_block(l0 + i, b)
    return layers, norms


def synthetic_layers(L: int, bits: int, seed: int, device, E_range: tuple[int, int] | None = None,
                     H: int = 2048, I: int = 512, E: int = 256) -> tuple[list[BlockTensors], list[torch.Tensor]]:
    """L distinct blocks generated on the device from a seeded torch generator
    with the distributions of runnel_b200.inputs (uniform codes, scales
    U(0.001, 0.01), biases N(0, 0.01), router and shared gate N(0, 0.02), RMSNorm
    weights 1 + N(0, 0.02)); fast enough for 40-layer stacks.  With E_range only
    that expert shard of each layer is kept (the full bank is drawn, so every
    rank sees the same weights)."""
    g = torch.Generator(device=device)
    lo, hi = E_range if E_range else (0, E)
    layers, norms = [], []

    def words(shape):
        return torch.randint(-2 ** 31, 2 ** 31, shape, dtype=torch.int64, device=device,
                             generator=g).to(torch.int32).view(torch.uint32)

    def scales(shape):
        return (torch.rand(shape, device=device, generator=g) * 0.009 + 0.001).to(torch.bfloat16)

    def biases(shape):
        return (torch.randn(shape, device=device, generator=g) * 0.01).to(torch.bfloat16)

    for l in range(L):
        g.manual_seed(seed * 1000 + l)
        router = (torch.randn((E, H), device=device, generator=g) * 0.02).to(torch.bfloat16)
        sgate = (torch.randn((H,), device=device, generator=g) * 0.02).to(torch.bfloat16)
        gu_w = words((E, 2 * I, H * bits // 32))[lo:hi].contiguous()
        gu_s = scales((E, 2 * I, H // 64))[lo:hi].contiguous()
        gu_b = biases((E, 2 * I, H // 64))[lo:hi].contiguous()
        dn_w = words((E, H, I * bits // 32))[lo:hi].contiguous()
        dn_s = scales((E, H, I // 64))[lo:hi].contiguous()
        dn_b = biases((E, H, I // 64))[lo:hi].contiguous()
        bt = BlockTensors(bits=bits, gu_w=gu_w, gu_s=gu_s, gu_b=gu_b, dn_w=dn_w, dn_s=dn_s, dn_b=dn_b,
                          router_w=router, shared_gate_w=sgate,
                          sgu_w=words((2 * I, H * bits // 32)), sgu_s=scales((2 * I, H // 64)),
                          sgu_b=biases((2 * I, H // 64)), sdn_w=words((H, I * bits // 32)),
                          sdn_s=scales((H, I // 64)), sdn_b=biases((H, I // 64)),
                          E_total=E, expert_offset=lo)
        layers.append(bt)
        norms.append((1.0 + torch.randn((H,), device=device, generator=g) * 0.02).to(torch.bfloat16))
        if E_range:
            torch.cuda.empty_cache()
    return layers, norms
