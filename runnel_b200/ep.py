"""Expert parallelism over the GPUs of one node (one process per GPU).

The reference runs one Apple GPU and has no expert parallelism; this is the
B200 build's multi-GPU form of the same block.  With N ranks:

* rank r holds experts ``[r*E/N, (r+1)*E/N)`` (:func:`plan`), the router and
  the shared expert, whose four 128-channel intermediate quarters are split
  round-robin (quarter q on rank q % N) -- the down projection is linear in
  the intermediate activations, so the per-rank partial outputs simply add;
* every rank routes the (replicated) tokens itself, computes its partial sum
  over its local selected experts and shared quarters, and the partials are
  all-reduced.

Two reductions are offered:

* ``"p2p"`` (default, decode T <= 8): :class:`ExpertParallel` -- the
  persistent decode kernel stores its fp32 partial tiles into every peer's
  receive buffer over NVLink (CUDA IPC mappings, no multicast) and sums the
  ranks' tiles in rank order, all in one launch (``rnb_moe_block_ep_fwd``);
* ``"nccl"``: the block with ``RNB_FLAG_Y_F32`` (fp32 partial, shared expert
  on rank 0 only) followed by ``torch.distributed.all_reduce`` -- the
  library-collective baseline, any T.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import BlockTensors, Workspace, _ptr, _stream, _tokens, default_workspace


def plan(rank: int, world: int, E_total: int = 256, I: int = 512) -> tuple[int, int, int]:
    """(first expert, end expert, shared-quarter bitmask) of one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if E_total % world:
        raise ValueError(f"{E_total} experts do not split evenly over {world} ranks")
    per = E_total // world
    mask = 0
    for q in range(rank, I // 128, world):
        mask |= 1 << q
    return rank * per, (rank + 1) * per, mask


def gather_handles(handle: bytes, group=None) -> list[bytes]:
    """Every rank's IPC handle, in rank order (host collective)."""
    import torch.distributed as dist

    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


class ExpertParallel:
    """This rank's NVLink exchange context for expert-parallel decode."""

    def __init__(self, rank: int, world: int, H: int = 2048, handles_fn=gather_handles):
        self.rank, self.world, self.H = rank, world, H
        self._ep = ctypes.c_void_p()
        buf = (ctypes.c_char * _lib.EP_HANDLE_BYTES)()
        _lib.call("rnb_ep_create", rank, world, H, ctypes.byref(self._ep), buf)
        try:
            handles = handles_fn(bytes(buf))
            if len(handles) != world or any(len(h) != _lib.EP_HANDLE_BYTES for h in handles):
                raise ValueError("handle exchange returned a malformed list")
            joined = b"".join(handles)
            _lib.call("rnb_ep_connect", self._ep, ctypes.c_char_p(joined))
        except BaseException:
            _lib.load().rnb_ep_destroy(self._ep)
            self._ep = None
            raise

    def close(self) -> None:
        """Release the buffers (after a host barrier on every rank)."""
        if self._ep:
            _lib.load().rnb_ep_destroy(self._ep)
            self._ep = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may be gone
            pass

    def moe_block(self, bt: BlockTensors, x: torch.Tensor, k: int = 8, ws: Workspace | None = None,
                  out: torch.Tensor | None = None, return_routing: bool = False):
        """Full block output on every rank from this rank's shard ``bt``."""
        if not self._ep:
            raise RuntimeError("ExpertParallel context is closed")
        xt = _tokens(x, bt.H)
        T = xt.shape[0]
        f32 = bool(bt.flags & _lib.FLAG_Y_F32)
        dt = torch.float32 if f32 else torch.bfloat16
        if out is None:
            out = torch.empty(xt.shape, dtype=dt, device=xt.device)
        elif out.dtype != dt or out.numel() != xt.numel() or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous {dt} tensor with x's number of elements")
        inds = scores = None
        if return_routing:
            inds = torch.empty((T, k), dtype=torch.int32, device=xt.device)
            scores = torch.empty((T, k), dtype=torch.float32, device=xt.device)
        d = bt.desc(T, k)
        ws = ws or default_workspace(xt.device)
        wp, wn = ws.get(d)
        _lib.call("rnb_moe_block_ep_fwd", ctypes.byref(d), self._ep, _ptr(xt), _ptr(out), _ptr(inds),
                  _ptr(scores), wp, wn, _stream())
        out = out.reshape(x.shape)
        return (out, inds, scores) if return_routing else out


def shard_tensors(blk, rank: int, world: int, device) -> BlockTensors:
    """Upload rank's expert shard of a synthetic block (router, shared expert replicated)."""
    lo, hi, _ = plan(rank, world, blk.E, blk.I)
    return BlockTensors.from_numpy(blk, device, E_range=(lo, hi))


def moe_block_nccl(bt: BlockTensors, x: torch.Tensor, rank: int, group=None, k: int = 8,
                   ws: Workspace | None = None, partial_fn=None):
    """Library-collective baseline: fp32 partial block (shared expert on rank 0
    only) then all_reduce(SUM) and a bf16 cast.  ``partial_fn(bt, x) -> fp32``
    replaces the device call (host tests)."""
    import torch.distributed as dist

    flags = bt.flags | _lib.FLAG_Y_F32 | (0 if rank == 0 else _lib.FLAG_NO_SHARED)
    shard = BlockTensors(**{**bt.__dict__, "flags": flags})
    if partial_fn is None:
        from .ops import moe_block
        part = moe_block(shard, x, k=k, ws=ws, out_dtype=torch.float32)
    else:
        part = partial_fn(shard, x)
    dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    return part.to(torch.bfloat16)
