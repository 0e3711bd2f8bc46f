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

For throughput (every rank with its own tokens, e.g. a 16384-token prefill
chunk per GPU) two exchanges are offered.  :func:`moe_block_gather` needs no
host synchronisation: every rank gathers all ranks' tokens with their routing
(``all_gather``), runs its experts on the other ranks' rows, and the fp32
partials are summed onto their home ranks (``reduce_scatter``).
:func:`moe_block_a2a` sends only the rows each rank needs: each
rank routes its tokens, runs its local experts and the whole shared expert on
them, sends every token once to each other rank that holds one of its
selected experts (with its full routing row), and the owners send back fp32
partial sums (``rnb_moe_experts_fwd`` on the received rows), which are added
to the home partial.
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

    def set_wait_limit_ms(self, ms: int) -> None:
        """How long a call waits for the other ranks before it gives up and
        sets RNB_STATUS_TIMEOUT (default 2000 ms)."""
        if not self._ep:
            raise RuntimeError("ExpertParallel context is closed")
        _lib.call("rnb_ep_set_wait_limit_ms", self._ep, int(ms))

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


class DeviceAllToAll:
    """This rank's device-side all-to-all context for expert-parallel blocks
    over many tokens (``rnb_a2a_*``): every rank holds its own ``T`` tokens
    (the same ``T`` everywhere, at most ``max_tokens``) and its expert shard.
    A call routes the rank's tokens, sends each row by NVLink stores to the
    ranks that own one of its experts, runs this shard's experts on the rows
    it received, returns the fp32 sums the same way and adds them up -- all
    on the stream, with no host synchronisation."""

    def __init__(self, rank: int, world: int, H: int = 2048, k: int = 8, max_tokens: int = 16384,
                 handles_fn=gather_handles):
        self.rank, self.world, self.H, self.k, self.max_tokens = rank, world, H, k, max_tokens
        self._a = ctypes.c_void_p()
        buf = (ctypes.c_char * _lib.A2A_HANDLE_BYTES)()
        _lib.call("rnb_a2a_create", rank, world, H, k, max_tokens, ctypes.byref(self._a), buf)
        try:
            handles = handles_fn(bytes(buf))
            if len(handles) != world or any(len(h) != _lib.A2A_HANDLE_BYTES for h in handles):
                raise ValueError("handle exchange returned a malformed list")
            _lib.call("rnb_a2a_connect", self._a, ctypes.c_char_p(b"".join(handles)))
        except BaseException:
            _lib.load().rnb_a2a_destroy(self._a)
            self._a = None
            raise
        self._ws: torch.Tensor | None = None

    def set_wait_limit_ms(self, ms: int) -> None:
        """How long a call waits for the other ranks before it gives up and
        sets RNB_STATUS_TIMEOUT (default 2000 ms)."""
        if not self._a:
            raise RuntimeError("DeviceAllToAll context is closed")
        _lib.call("rnb_a2a_set_wait_limit_ms", self._a, int(ms))

    def close(self) -> None:
        """Release the buffers (after a host barrier on every rank)."""
        if self._a:
            _lib.load().rnb_a2a_destroy(self._a)
            self._a = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may be gone
            pass

    def status(self) -> int:
        """Reads and clears the status bits of this context's workspace (synchronises)."""
        if self._ws is None:
            return 0
        out = ctypes.c_uint32()
        _lib.call("rnb_moe_status", self._ws.data_ptr(), self._ws.numel(), ctypes.byref(out), _stream())
        return out.value

    def moe_block(self, bt: BlockTensors, x: torch.Tensor, out: torch.Tensor | None = None,
                  return_routing: bool = False):
        """The block on this rank's tokens ``x`` from its shard ``bt``."""
        if not self._a:
            raise RuntimeError("DeviceAllToAll context is closed")
        xt = _tokens(x, bt.H)
        T = xt.shape[0]
        f32 = bool(bt.flags & _lib.FLAG_Y_F32)
        dt = torch.float32 if f32 else torch.bfloat16
        if out is None:
            out = torch.empty(xt.shape, dtype=dt, device=xt.device)
        inds = scores = None
        if return_routing:
            inds = torch.empty((T, self.k), dtype=torch.int32, device=xt.device)
            scores = torch.empty((T, self.k), dtype=torch.float32, device=xt.device)
        d = bt.desc(T, self.k)
        need = ctypes.c_size_t()
        _lib.call("rnb_moe_block_a2a_workspace_size", ctypes.byref(d), self._a, ctypes.byref(need))
        if self._ws is None or self._ws.numel() < need.value:
            self._ws = torch.zeros(need.value, dtype=torch.uint8, device=xt.device)
        _lib.call("rnb_moe_block_a2a_fwd", ctypes.byref(d), self._a, _ptr(xt), _ptr(out), _ptr(inds),
                  _ptr(scores), self._ws.data_ptr(), self._ws.numel(), _stream())
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


def _a2a_rows(t: torch.Tensor, send: list[int], recv: list[int], group) -> torch.Tensor:
    import torch.distributed as dist

    out = t.new_empty((sum(recv),) + tuple(t.shape[1:]))
    dist.all_to_all_single(out, t.contiguous(), output_split_sizes=recv, input_split_sizes=send, group=group)
    return out


def moe_block_a2a(bt: BlockTensors, x: torch.Tensor, rank: int, world: int, group=None, k: int = 8,
                  ws: Workspace | None = None, block_fn=None, experts_fn=None, stats: dict | None = None):
    """Expert-parallel block over this rank's own tokens with all-to-all
    dispatch and combine.  ``bt`` is this rank's expert shard (experts
    ``[rank*E, (rank+1)*E)`` of ``E_total``, router and shared expert whole).

    1. home: ``moe_block`` with fp32 output -> router, this rank's selected
       experts and the whole shared expert for every local token;
    2. dispatch: token t goes once to each other rank owning one of its k
       experts, as one int32 row (bf16 x, k ids, k fp32 weights);
    3. remote: ``rnb_moe_experts_fwd`` sums the receiving shard's experts
       of each row (fp32);
    4. combine: the fp32 rows go back and are added to the home partial,
       which is rounded to bf16 once.

    ``block_fn(bt, x) -> (fp32 out, inds, scores)`` and
    ``experts_fn(bt, x, inds, scores) -> fp32`` replace the device calls
    (host tests).  ``stats`` (a dict) receives the rows sent and received."""
    import torch.distributed as dist

    from .ops import experts_fwd, moe_block

    xt = _tokens(x, bt.H)
    T, H = xt.shape
    Et = bt.E_total if bt.E_total is not None else bt.E
    per = bt.E
    if per * world != Et or bt.expert_offset != rank * per:
        raise ValueError(f"shard [{bt.expert_offset}, +{per}) is not rank {rank}'s of {Et} experts over {world}")
    f32 = BlockTensors(**{**bt.__dict__, "flags": bt.flags | _lib.FLAG_Y_F32})
    if block_fn is None:
        part, inds, scores = moe_block(f32, xt, k=k, ws=ws, return_routing=True)
    else:
        part, inds, scores = block_fn(f32, xt)
    # (destination rank, token) pairs, sorted by rank then token; home excluded
    dest = torch.zeros((T, world), dtype=torch.bool, device=xt.device)
    dest.scatter_(1, (inds.long() // per).clamp_(0, world - 1), True)
    dest[:, rank] = False
    d_idx, t_idx = dest.t().nonzero(as_tuple=True)
    send_n = torch.bincount(d_idx, minlength=world)
    recv_n = torch.empty_like(send_n)
    dist.all_to_all_single(recv_n, send_n, group=group)
    send, recv = send_n.tolist(), recv_n.tolist()
    if stats is not None:
        stats.update(sent=sum(send), received=sum(recv))
    hw = H // 2
    rows = torch.cat([xt.view(torch.int32)[t_idx], inds.to(torch.int32)[t_idx],
                      scores.view(torch.int32)[t_idx]], dim=1)
    got = _a2a_rows(rows, send, recv, group)
    rx = got[:, :hw].contiguous().view(torch.bfloat16)
    ri = got[:, hw:hw + k].contiguous()
    rs = got[:, hw + k:].contiguous().view(torch.float32)
    if experts_fn is None:
        y = experts_fwd(bt, rx, ri, rs) if rx.shape[0] else rx.new_zeros((0, H), dtype=torch.float32)
    else:
        y = experts_fn(bt, rx, ri, rs)
    back = _a2a_rows(y, recv, send, group)
    part.index_add_(0, t_idx, back)
    return part.to(torch.bfloat16).reshape(x.shape)


def moe_block_gather(bt: BlockTensors, x: torch.Tensor, rank: int, world: int, group=None, k: int = 8,
                     ws: Workspace | None = None, block_fn=None, experts_fn=None,
                     gather_fn=None, reduce_scatter_fn=None):
    """Expert-parallel block over this rank's own tokens (every rank the same
    token count) with gather dispatch and reduce-scatter combine:

    1. home: ``moe_block`` with fp32 output -> routing, this rank's selected
       experts and the whole shared expert for its tokens, written into its
       slot of a [world, T, H] fp32 partial;
    2. dispatch: ``all_gather`` of every rank's rows (bf16 x, k ids, k fp32
       weights as one int32 row);
    3. remote: ``rnb_moe_experts_fwd`` on each other rank's rows (experts of
       other shards are skipped, so a row none of whose experts is here costs
       no tensor-core work) into that rank's slot;
    4. combine: ``reduce_scatter`` (sum) of the partial: each rank gets the
       sum for its own tokens, rounded to bf16 once.

    ``block_fn``/``experts_fn`` replace the device calls and
    ``gather_fn(out, inp)`` / ``reduce_scatter_fn(out, inp)`` the collectives
    (host tests)."""
    import torch.distributed as dist

    from .ops import experts_fwd, moe_block

    xt = _tokens(x, bt.H)
    T, H = xt.shape
    Et = bt.E_total if bt.E_total is not None else bt.E
    if bt.E * world != Et or bt.expert_offset != rank * bt.E:
        raise ValueError(f"shard [{bt.expert_offset}, +{bt.E}) is not rank {rank}'s of {Et} experts over {world}")
    gather_fn = gather_fn or (lambda out, inp: dist.all_gather_into_tensor(out, inp, group=group))
    reduce_scatter_fn = reduce_scatter_fn or (
        lambda out, inp: dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM, group=group))
    f32 = BlockTensors(**{**bt.__dict__, "flags": bt.flags | _lib.FLAG_Y_F32})
    part = torch.empty((world, T, H), dtype=torch.float32, device=xt.device)
    if block_fn is None:
        _, inds, scores = moe_block(f32, xt, k=k, ws=ws, return_routing=True, out=part[rank])
    else:
        home, inds, scores = block_fn(f32, xt)
        part[rank].copy_(home)
    hw = H // 2
    rows = torch.cat([xt.view(torch.int32), inds.to(torch.int32), scores.view(torch.int32)], dim=1).contiguous()
    allrows = torch.empty((world,) + tuple(rows.shape), dtype=torch.int32, device=xt.device)
    gather_fn(allrows, rows)
    for q in range(world):
        if q == rank:
            continue
        rq = allrows[q]
        xq = rq[:, :hw].contiguous().view(torch.bfloat16)
        iq = rq[:, hw:hw + k].contiguous()
        sq = rq[:, hw + k:].contiguous().view(torch.float32)
        if experts_fn is None:
            experts_fwd(bt, xq, iq, sq, out=part[q])
        else:
            part[q].copy_(experts_fn(bt, xq, iq, sq))
    out = torch.empty((T, H), dtype=torch.float32, device=xt.device)
    reduce_scatter_fn(out, part.view(world * T, H))
    return out.to(torch.bfloat16).reshape(x.shape)
