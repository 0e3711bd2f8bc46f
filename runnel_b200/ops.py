"""Functional layer over the C ABI: descriptors, workspaces, calls on torch tensors.

All tensors are CUDA tensors in MLX layout: quantized codes ``torch.uint32``
(or int32 with the same bits), scales/biases/activations ``torch.bfloat16``.
Calls are asynchronous on the current torch stream; nothing here falls back
to another implementation.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

GROUP_SIZE = 64


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("tensors passed to the MoE kernels must be CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("tensors passed to the MoE kernels must be contiguous")
    return t.data_ptr()


# the descriptor's tensor fields, in rnb_moe_desc order
_BANK_FIELDS = ("gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b", "router_w", "shared_gate_w",
                "sgu_w", "sgu_s", "sgu_b", "sdn_w", "sdn_s", "sdn_b",
                "router_s", "router_b", "sgate_s", "sgate_b")


@dataclass
class BlockTensors:
    """Device tensors of one sparse-MoE block (MLX layout)."""

    bits: int
    gu_w: torch.Tensor  # [E, 2I, H*bits/32]  up rows then gate rows
    gu_s: torch.Tensor  # [E, 2I, H/64] bf16
    gu_b: torch.Tensor
    dn_w: torch.Tensor  # [E, H, I*bits/32]
    dn_s: torch.Tensor
    dn_b: torch.Tensor
    router_w: torch.Tensor | None = None  # [E_total, H] bf16 (router_bits 8: [E_total, H/4] uint32)
    shared_gate_w: torch.Tensor | None = None  # [H] or [1, H] bf16 (router_bits 8: [H/4] uint32)
    sgu_w: torch.Tensor | None = None  # [2I, H*bits/32]
    sgu_s: torch.Tensor | None = None
    sgu_b: torch.Tensor | None = None
    sdn_w: torch.Tensor | None = None  # [H, I*bits/32]
    sdn_s: torch.Tensor | None = None
    sdn_b: torch.Tensor | None = None
    group: int = GROUP_SIZE
    E_total: int | None = None
    expert_offset: int = 0
    flags: int = 0
    # 8-bit affine router and shared gate (mlp.gate / mlp.shared_expert_gate
    # stored 8-bit): bf16 scales and biases per 64 inputs
    router_bits: int = 16
    router_s: torch.Tensor | None = None  # [E_total, H/64] bf16
    router_b: torch.Tensor | None = None
    sgate_s: torch.Tensor | None = None  # [H/64] bf16
    sgate_b: torch.Tensor | None = None

    @property
    def E(self) -> int:
        return self.gu_w.shape[0]

    @property
    def H(self) -> int:
        return self.dn_w.shape[1]

    @property
    def I(self) -> int:  # noqa: E743
        return self.gu_w.shape[1] // 2

    @classmethod
    def from_numpy(cls, blk, device="cuda", E_range: tuple[int, int] | None = None,
                   with_shared: bool = True) -> "BlockTensors":
        """Upload a :class:`runnel_b200.inputs.SyntheticBlock` (optionally an expert shard)."""
        def up(a, dtype):
            t = torch.from_numpy(a)
            if dtype == torch.bfloat16:
                t = t.view(torch.int16).view(torch.bfloat16)
            return t.to(device)

        lo, hi = E_range if E_range else (0, blk.E)
        q8 = getattr(blk, "router_bits", 16) == 8
        bt = cls(
            bits=blk.bits, group=blk.group,
            gu_w=up(blk.gu_w[lo:hi], torch.uint32), gu_s=up(blk.gu_s[lo:hi], torch.bfloat16),
            gu_b=up(blk.gu_b[lo:hi], torch.bfloat16), dn_w=up(blk.dn_w[lo:hi], torch.uint32),
            dn_s=up(blk.dn_s[lo:hi], torch.bfloat16), dn_b=up(blk.dn_b[lo:hi], torch.bfloat16),
            router_w=up(blk.router_q, torch.uint32) if q8 else up(blk.router_w, torch.bfloat16),
            E_total=blk.E, expert_offset=lo)
        if q8:
            bt.router_bits = 8
            bt.router_s = up(blk.router_s, torch.bfloat16)
            bt.router_b = up(blk.router_b, torch.bfloat16)
        if with_shared:
            if q8:
                bt.shared_gate_w = up(np.ascontiguousarray(blk.sgate_q.reshape(-1)), torch.uint32)
                bt.sgate_s = up(np.ascontiguousarray(blk.sgate_s.reshape(-1)), torch.bfloat16)
                bt.sgate_b = up(np.ascontiguousarray(blk.sgate_b.reshape(-1)), torch.bfloat16)
            else:
                bt.shared_gate_w = up(blk.shared_gate_w, torch.bfloat16)
            bt.sgu_w = up(blk.sgu_w, torch.uint32)
            bt.sgu_s = up(blk.sgu_s, torch.bfloat16)
            bt.sgu_b = up(blk.sgu_b, torch.bfloat16)
            bt.sdn_w = up(blk.sdn_w, torch.uint32)
            bt.sdn_s = up(blk.sdn_s, torch.bfloat16)
            bt.sdn_b = up(blk.sdn_b, torch.bfloat16)
        return bt

    def desc(self, T: int, k: int = 8) -> _lib.RnbMoeDesc:
        d = _lib.RnbMoeDesc()
        d.T, d.H, d.I, d.E = T, self.H, self.I, self.E
        d.E_total = self.E_total if self.E_total is not None else self.E
        d.expert_offset = self.expert_offset
        d.k, d.bits, d.group, d.flags = k, self.bits, self.group, self.flags
        d.router_bits = self.router_bits
        for name in _BANK_FIELDS:
            setattr(d, name, _ptr(getattr(self, name)))
        return d


class Workspace:
    """Caller-owned device workspace, grown on demand and zeroed when allocated."""

    def __init__(self, device=None):
        self.device = torch.device(device or "cuda")
        self.buf: torch.Tensor | None = None

    def get(self, desc: _lib.RnbMoeDesc) -> tuple[int, int]:
        need = ctypes.c_size_t()
        _lib.call("rnb_moe_workspace_size", ctypes.byref(desc), ctypes.byref(need))
        if self.buf is None or self.buf.numel() < need.value:
            # torch.zeros gives the required zero-filled initial state
            self.buf = torch.zeros(need.value, dtype=torch.uint8, device=self.device)
        return self.buf.data_ptr(), self.buf.numel()

    def status(self) -> int:
        """Reads and clears the device status bits (synchronises the stream)."""
        if self.buf is None:
            return 0
        out = ctypes.c_uint32()
        _lib.call("rnb_moe_status", self.buf.data_ptr(), self.buf.numel(), ctypes.byref(out),
                  _stream())
        return out.value


_workspaces: dict[int, Workspace] = {}


def default_workspace(device: torch.device) -> Workspace:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None:
        ws = _workspaces[idx] = Workspace(torch.device("cuda", idx))
    return ws


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _tokens(x: torch.Tensor, H: int) -> torch.Tensor:
    if x.dtype != torch.bfloat16:
        raise ValueError("x must be bfloat16")
    if x.shape[-1] != H:
        raise ValueError(f"x must have last dimension {H}")
    return x.reshape(-1, H).contiguous()


def _indices(ind: torch.Tensor, T: int, k: int) -> torch.Tensor:
    ind = ind.reshape(T, k)
    if ind.dtype in (torch.int64, torch.int16, torch.uint8):
        ind = ind.to(torch.int32)
    if ind.dtype not in (torch.int32, torch.uint32):
        raise ValueError("indices must be an integer tensor")
    return ind.contiguous()


def switchglu(bt: BlockTensors, x: torch.Tensor, indices: torch.Tensor,
              ws: Workspace | None = None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Per-slot expert outputs ``[..., k, H]`` (unweighted), bf16 or fp32."""
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be bfloat16 or float32")
    k = indices.shape[-1]
    xt = _tokens(x, bt.H)
    T = xt.shape[0]
    ind = _indices(indices, T, k)
    y = torch.empty((T, k, bt.H), dtype=out_dtype, device=xt.device)
    if T:
        d = bt.desc(T, k)
        if out_dtype == torch.float32:
            d.flags |= _lib.FLAG_Y_F32
        ws = ws or default_workspace(xt.device)
        wp, wn = ws.get(d)
        _lib.call("rnb_switchglu_fwd", ctypes.byref(d), _ptr(xt), _ptr(ind), _ptr(y), wp, wn, _stream())
    return y.reshape(*x.shape[:-1], k, bt.H)


def moe_block(bt: BlockTensors, x: torch.Tensor, k: int = 8, ws: Workspace | None = None,
              return_routing: bool = False, out: torch.Tensor | None = None, out_dtype=None):
    """Whole block ``[..., H] -> [..., H]`` bf16; optionally (out, inds, scores).

    ``out`` (contiguous, x's shape) receives the result in place.  With
    ``bt.flags & FLAG_Y_F32`` the result is fp32 (``out_dtype=torch.float32``)."""
    xt = _tokens(x, bt.H)
    T = xt.shape[0]
    dt = torch.float32 if bt.flags & _lib.FLAG_Y_F32 else torch.bfloat16
    if out_dtype is not None and out_dtype != dt:
        raise ValueError(f"out_dtype {out_dtype} does not match the descriptor's output ({dt})")
    if out is None:
        out = torch.empty(xt.shape, dtype=dt, device=xt.device)
    elif out.dtype != dt or out.numel() != xt.numel() or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {dt} tensor with x's number of elements")
    inds = scores = None
    if return_routing:
        inds = torch.empty((T, k), dtype=torch.int32, device=xt.device)
        scores = torch.empty((T, k), dtype=torch.float32, device=xt.device)
    if T:
        d = bt.desc(T, k)
        ws = ws or default_workspace(xt.device)
        wp, wn = ws.get(d)
        _lib.call("rnb_moe_block_fwd", ctypes.byref(d), _ptr(xt), _ptr(out), _ptr(inds), _ptr(scores),
                  wp, wn, _stream())
    out = out.reshape(x.shape)
    if return_routing:
        return out, inds, scores
    return out


class BlockCall:
    """``moe_block`` prepared once for a fixed token count ``T``, for callers
    that repeat one call shape (decode loops, serving steps).

    The descriptor and the device staging buffers are built here, so a call is
    one C call with no per-call descriptor or workspace-size query.  The bank's
    tensors are captured at construction: in-place updates of them are seen,
    but assigning a new tensor to a ``BlockTensors`` field is not.  Calls are
    asynchronous on the current stream and reuse the staging buffers, so calls
    on one object must share a stream.

    ``host(x_host, out_host)`` takes CPU tensors and queues copy-in, block and
    copy-out as one C call (``rnb_moe_block_fwd_host``).  Pin both tensors so
    the copies are asynchronous; ``out_host`` holds the result once the stream
    is synchronised.  ``__call__(x, out)`` runs on CUDA tensors."""

    def __init__(self, bt: BlockTensors, T: int, k: int = 8, ws: Workspace | None = None):
        if T <= 0:
            raise ValueError("T must be positive")
        self.T, self.H, self.k = T, bt.H, k
        self._bank = tuple(getattr(bt, f) for f in _BANK_FIELDS)  # keeps the pointed-to tensors alive
        self.desc = bt.desc(T, k)
        self._dref = ctypes.byref(self.desc)
        self.device = bt.gu_w.device
        self.ws = ws or Workspace(self.device)
        self.ws.get(self.desc)  # sized (and zeroed) for this call once
        self.out_dtype = torch.float32 if bt.flags & _lib.FLAG_Y_F32 else torch.bfloat16
        self.x_dev = torch.empty((T, bt.H), dtype=torch.bfloat16, device=self.device)
        self.out_dev = torch.empty((T, bt.H), dtype=self.out_dtype, device=self.device)
        lib = _lib.load()
        self._fwd, self._fwd_host = lib.rnb_moe_block_fwd, lib.rnb_moe_block_fwd_host

    def _check(self, x: torch.Tensor, out: torch.Tensor, cuda: bool) -> None:
        n = self.T * self.H
        if (x.is_cuda != cuda or out.is_cuda != cuda or x.dtype != torch.bfloat16 or out.dtype != self.out_dtype
                or x.numel() != n or out.numel() != n or not x.is_contiguous() or not out.is_contiguous()):
            where = "CUDA" if cuda else "CPU"
            raise ValueError(f"x must be a contiguous {where} bfloat16 tensor of {self.T}x{self.H} elements and "
                             f"out a contiguous {where} {self.out_dtype} tensor of as many")

    def host(self, x_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        self._check(x_host, out_host, cuda=False)
        buf = self.ws.buf
        _lib.check("rnb_moe_block_fwd_host",
                   self._fwd_host(self._dref, x_host.data_ptr(), out_host.data_ptr(), self.x_dev.data_ptr(),
                                  self.out_dev.data_ptr(), buf.data_ptr(), buf.numel(), _stream()))
        return out_host

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if out is None:
            out = torch.empty(x.shape, dtype=self.out_dtype, device=x.device)
        self._check(x, out, cuda=True)
        buf = self.ws.buf
        _lib.check("rnb_moe_block_fwd", self._fwd(self._dref, x.data_ptr(), out.data_ptr(), None, None,
                                                  buf.data_ptr(), buf.numel(), _stream()))
        return out


def experts_fwd(bt: BlockTensors, x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor,
                out_f32: bool = True, ws: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed experts of this shard with given routing: [T, H] bf16 rows,
    [T, k] int32 global expert ids and fp32 weights -> [T, H] weighted sum over
    the ids this shard holds (fp32 by default; ``out``, contiguous, receives
    it in place).  No router, no shared expert."""
    xt = _tokens(x, bt.H)
    T, k = inds.shape
    flags = (bt.flags | _lib.FLAG_Y_F32) if out_f32 else (bt.flags & ~_lib.FLAG_Y_F32)
    d = BlockTensors(**{**bt.__dict__, "flags": flags}).desc(T, k)
    dt = torch.float32 if out_f32 else torch.bfloat16
    if out is None:
        out = torch.empty(xt.shape, dtype=dt, device=xt.device)
    elif out.dtype != dt or out.numel() != xt.numel() or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {dt} tensor with x's number of elements")
    if T == 0:
        return out
    need = ctypes.c_size_t()
    _lib.call("rnb_moe_experts_workspace_size", ctypes.byref(d), ctypes.byref(need))
    if ws is None or ws.numel() < need.value:
        ws = torch.zeros(need.value, dtype=torch.uint8, device=xt.device)
    inds = inds.to(torch.int32).contiguous()
    scores = scores.to(torch.float32).contiguous()
    _lib.call("rnb_moe_experts_fwd", ctypes.byref(d), _ptr(xt), _ptr(inds), _ptr(scores), _ptr(out),
              ws.data_ptr(), ws.numel(), _stream())
    return out


def router_topk(bt: BlockTensors, x: torch.Tensor, k: int = 8, ws: Workspace | None = None,
                return_logits: bool = False):
    """(inds int32 [T,k], scores fp32 [T,k][, bf16-rounded logits fp32 [T,E_total]])."""
    xt = _tokens(x, bt.H)
    T = xt.shape[0]
    Et = bt.E_total if bt.E_total is not None else bt.E
    inds = torch.empty((T, k), dtype=torch.int32, device=xt.device)
    scores = torch.empty((T, k), dtype=torch.float32, device=xt.device)
    logits = torch.empty((T, Et), dtype=torch.float32, device=xt.device) if return_logits else None
    if T:
        d = bt.desc(T, k)
        ws = ws or default_workspace(xt.device)
        wp, wn = ws.get(d)
        _lib.call("rnb_router_topk", ctypes.byref(d), _ptr(xt), _ptr(inds), _ptr(scores),
                  _ptr(logits), wp, wn, _stream())
    if return_logits:
        return inds, scores, logits
    return inds, scores
