"""Torch modules with the names, attributes and call signatures of the MLX /
mlx-lm modules on Runnel's hot path, backed by the B200 kernels.

* :class:`QuantizedSwitchLinear`, :class:`SwitchGLU` -- mlx-lm
  ``switch_layers`` (per-expert quantized projections, ``__call__(x, indices)``).
* :class:`FusedQuantizedSwitchGLU` -- Runnel's packed routed gate/up module
  (src/runnel/mlx.py:23-82): one packed ``[E, 2I, ...]`` tensor, up rows then
  gate rows, ``__call__(x, indices) -> [..., k, H]``.
* :class:`QuantizedLinear`, :class:`SharedExpertMLP`,
  :class:`FusedQuantizedSharedMLP` -- the shared expert, stock and packed
  (bench/mlx_lm_adapter.py:49-94, packed on axis 0).
* :class:`SparseMoeBlock` -- the Qwen3.5 sparse-MoE block ``mlp(x)``: router
  ``gate``, ``switch_mlp``, ``shared_expert``, ``shared_expert_gate``.

Modules are dict-like the way MLX modules are (``m["weight"]``,
``m.get("biases")``, ``"bias" in m``) so Runnel's transform code reads the
same.  Tensors live on a CUDA device; quantized codes are ``torch.uint32``.
"""
from __future__ import annotations

import torch
from torch import nn

from . import ops

_PARAM_NAMES = ("weight", "scales", "biases", "bias")


def _cat(tensors, dim):
    """torch.cat that also works for uint32 (concatenated through int32 views)."""
    if tensors[0].dtype == torch.uint32:
        return torch.cat([t.view(torch.int32) for t in tensors], dim=dim).view(torch.uint32)
    return torch.cat(tensors, dim=dim)


class _DictLike(nn.Module):
    def _names(self):
        return [n for n in _PARAM_NAMES if getattr(self, n, None) is not None]

    def __getitem__(self, name):
        if name not in self:
            raise KeyError(name)
        return getattr(self, name)

    def get(self, name, default=None):
        return getattr(self, name) if name in self else default

    def __contains__(self, name):
        return name in self._names()


class QuantizedSwitchLinear(_DictLike):
    """Per-expert affine-quantized projection: weight [E, out, in*bits/32]."""

    def __init__(self, weight, scales, biases=None, group_size: int = 64, bits: int = 4,
                 mode: str = "affine"):
        super().__init__()
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.group_size = group_size
        self.bits = bits
        self.mode = mode

    @property
    def num_experts(self):
        return self.weight.shape[0]


class QuantizedLinear(_DictLike):
    """Affine-quantized dense projection: weight [out, in*bits/32]."""

    def __init__(self, weight, scales, biases=None, group_size: int = 64, bits: int = 4,
                 mode: str = "affine"):
        super().__init__()
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.group_size = group_size
        self.bits = bits
        self.mode = mode


class SwiGLU(nn.Module):
    """``activation(x, gate) = silu(gate) * x`` (mlx-lm argument order)."""

    def forward(self, x, gate):
        return torch.nn.functional.silu(gate) * x


def _check_pair(gate, up, what: str):
    if not (isinstance(gate, type(up)) and gate.bits == up.bits
            and gate.group_size == up.group_size and gate.mode == up.mode):
        raise ValueError(f"{what} gate/up quantization formats differ")
    if ("bias" in gate) or ("bias" in up):
        raise ValueError("module biases are not expected for this checkpoint"
                         if what == "routed" else "shared module biases are not expected")
    if gate.mode != "affine":
        raise ValueError(f"{what} gate/up must use affine quantization")
    if (up.get("biases") is None) != (gate.get("biases") is None):
        raise ValueError(f"{what} gate/up affine-bias formats differ")
    if up.get("biases") is None:
        raise ValueError(f"{what} gate/up without affine biases are not supported")


class FusedQuantizedSwitchGLU(_DictLike):
    """Packed routed gate/up: one quantized tensor [E, 2I, ...], rows [0, I)
    from ``up_proj`` and [I, 2I) from ``gate_proj`` (src/runnel/mlx.py:23-82)."""

    def __init__(self, old: "SwitchGLU"):
        super().__init__()
        gate, up = old.gate_proj, old.up_proj
        _check_pair(gate, up, "routed")
        self.register_buffer("weight", _cat([up["weight"], gate["weight"]], 1))
        self.register_buffer("scales", _cat([up["scales"], gate["scales"]], 1))
        self.register_buffer("biases", _cat([up["biases"], gate["biases"]], 1))
        self.group_size = gate.group_size
        self.bits = gate.bits
        self.mode = gate.mode
        self.down_proj = old.down_proj
        self.activation = old.activation
        if self.group_size != 64:
            raise ValueError("the B200 kernels support group_size 64")
        self._ws = None

    def block_tensors(self, E_total=None, expert_offset=0) -> ops.BlockTensors:
        return ops.BlockTensors(
            bits=self.bits, gu_w=self.weight, gu_s=self.scales, gu_b=self.biases,
            dn_w=self.down_proj.weight, dn_s=self.down_proj.scales, dn_b=self.down_proj.biases,
            group=self.group_size, E_total=E_total, expert_offset=expert_offset)

    def forward(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """x [..., H] bf16, indices [..., k] -> per-slot outputs [..., k, H] bf16."""
        return ops.switchglu(self.block_tensors(), x, indices)


class SwitchGLU(nn.Module):
    """Stock mlx-lm SwitchGLU (separate gate/up/down expert banks).  Its
    forward runs the packed kernel on a gate/up pack built on first use."""

    def __init__(self, gate_proj: QuantizedSwitchLinear, up_proj: QuantizedSwitchLinear,
                 down_proj: QuantizedSwitchLinear):
        super().__init__()
        self.gate_proj = gate_proj
        self.up_proj = up_proj
        self.down_proj = down_proj
        self.activation = SwiGLU()
        self._packed = None

    def forward(self, x, indices):
        if self._packed is None:
            self._packed = FusedQuantizedSwitchGLU(self)
        return self._packed(x, indices)


class SharedExpertMLP(nn.Module):
    """Stock shared expert: gate_proj, up_proj, down_proj (QuantizedLinear)."""

    def __init__(self, gate_proj: QuantizedLinear, up_proj: QuantizedLinear,
                 down_proj: QuantizedLinear):
        super().__init__()
        self.gate_proj = gate_proj
        self.up_proj = up_proj
        self.down_proj = down_proj


class FusedQuantizedSharedMLP(_DictLike):
    """Shared expert with up||gate packed on axis 0 (bench/mlx_lm_adapter.py:49-94)."""

    def __init__(self, old: SharedExpertMLP):
        super().__init__()
        gate, up = old.gate_proj, old.up_proj
        _check_pair(gate, up, "shared")
        self.register_buffer("weight", _cat([up["weight"], gate["weight"]], 0))
        self.register_buffer("scales", _cat([up["scales"], gate["scales"]], 0))
        self.register_buffer("biases", _cat([up["biases"], gate["biases"]], 0))
        self.group_size = gate.group_size
        self.bits = gate.bits
        self.mode = gate.mode
        self.down_proj = old.down_proj


class SparseMoeBlock(nn.Module):
    """Qwen3.5 sparse-MoE block: ``forward(x [B,L,H]) -> [B,L,H]``.

    out = sum_k score_k * switch_mlp(x, inds)_k + sigmoid(shared_expert_gate(x)) * shared_expert(x)
    with scores the top-k of softmax(gate(x)) renormalised to sum 1.
    """

    def __init__(self, gate: nn.Linear, switch_mlp, shared_expert=None,
                 shared_expert_gate: nn.Linear | None = None, top_k: int = 8,
                 norm_topk_prob: bool = True):
        super().__init__()
        if not norm_topk_prob:
            raise ValueError("the B200 block renormalises the top-k weights (norm_topk_prob=True)")
        self.gate = gate
        self.switch_mlp = switch_mlp
        self.shared_expert = shared_expert
        self.shared_expert_gate = shared_expert_gate
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.ws = None

    @property
    def num_experts(self):
        return self.gate.weight.shape[0]

    def _packed(self):
        sw = self.switch_mlp
        if isinstance(sw, SwitchGLU):
            if sw._packed is None:
                sw._packed = FusedQuantizedSwitchGLU(sw)
            sw = sw._packed
        sh = self.shared_expert
        if isinstance(sh, SharedExpertMLP):
            sh = FusedQuantizedSharedMLP(sh)
            self.shared_expert = sh
        return sw, sh

    def block_tensors(self) -> ops.BlockTensors:
        sw, sh = self._packed()
        bt = sw.block_tensors(E_total=self.num_experts)
        bt.router_w = self.gate.weight.contiguous()
        if sh is not None:
            if sh.bits != sw.bits or sh.group_size != sw.group_size:
                raise ValueError("shared and routed experts must share one quantization format")
            bt.shared_gate_w = self.shared_expert_gate.weight.reshape(-1).contiguous()
            bt.sgu_w, bt.sgu_s, bt.sgu_b = sh.weight, sh.scales, sh.biases
            bt.sdn_w, bt.sdn_s, bt.sdn_b = sh.down_proj.weight, sh.down_proj.scales, sh.down_proj.biases
        return bt

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.moe_block(self.block_tensors(), x, k=self.top_k, ws=self.ws)

    def route(self, x: torch.Tensor):
        """(indices [.., k] int32, scores [.., k] fp32) of the router alone."""
        inds, scores = ops.router_topk(self.block_tensors(), x, k=self.top_k, ws=self.ws)
        return inds.reshape(*x.shape[:-1], self.top_k), scores.reshape(*x.shape[:-1], self.top_k)


def block_from_tensors(bt: ops.BlockTensors, top_k: int = 8, fused: bool = True) -> SparseMoeBlock:
    """Build a :class:`SparseMoeBlock` from device tensors in packed layout."""
    I = bt.I
    down = QuantizedSwitchLinear(bt.dn_w, bt.dn_s, bt.dn_b, bits=bt.bits)
    gate_p = QuantizedSwitchLinear(bt.gu_w[:, I:].contiguous(), bt.gu_s[:, I:].contiguous(),
                                   bt.gu_b[:, I:].contiguous(), bits=bt.bits)
    up_p = QuantizedSwitchLinear(bt.gu_w[:, :I].contiguous(), bt.gu_s[:, :I].contiguous(),
                                 bt.gu_b[:, :I].contiguous(), bits=bt.bits)
    sw = SwitchGLU(gate_p, up_p, down)
    if fused:
        sw = FusedQuantizedSwitchGLU(sw)
    H = bt.H
    gate = nn.Linear(H, bt.E_total or bt.E, bias=False, device=bt.gu_w.device, dtype=torch.bfloat16)
    with torch.no_grad():
        gate.weight.copy_(bt.router_w)
    shared = sgate = None
    if bt.sgu_w is not None:
        shared = SharedExpertMLP(
            QuantizedLinear(bt.sgu_w[I:].contiguous(), bt.sgu_s[I:].contiguous(), bt.sgu_b[I:].contiguous(), bits=bt.bits),
            QuantizedLinear(bt.sgu_w[:I].contiguous(), bt.sgu_s[:I].contiguous(), bt.sgu_b[:I].contiguous(), bits=bt.bits),
            QuantizedLinear(bt.sdn_w, bt.sdn_s, bt.sdn_b, bits=bt.bits))
        sgate = nn.Linear(H, 1, bias=False, device=bt.gu_w.device, dtype=torch.bfloat16)
        with torch.no_grad():
            sgate.weight.copy_(bt.shared_gate_w.reshape(1, H))
    return SparseMoeBlock(gate, sw, shared, sgate, top_k=top_k)
