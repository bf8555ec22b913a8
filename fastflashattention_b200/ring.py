"""Context-parallel ring attention over NCCL for very long causal sequences.

The reference has no sequence parallelism (it scales S only by tiling inside one GPU); this
module builds it on the reference's base-2 log-sum-exp (``_kernel.py:274-279``), which
lets partial results over disjoint key ranges be merged exactly.

Layout (zig-zag, balanced for causal masking): the sequence of length S is cut into 2P
chunks of C = S / (2P) tokens; rank r holds chunks r and 2P-1-r, concatenated, as its
local ``[B, H, 2C, D]`` tensors (``shard_sequence`` / ``unshard_sequence`` convert).

Forward, P steps: at step t rank r holds the K/V chunks of rank (r - t) mod P.  For each
local query chunk x and held key chunk y: y < x -> full attention, y == x -> causal
attention, y > x -> nothing.  Partial outputs are merged in fp32 with their base-2 LSE
(``ffa_lse_merge``).  K/V for step t+1 travel (send to r+1, receive from r-1) while step t
computes.

Backward, P steps plus one hand-back: delta = rowsum(O*dO) is local (per query row); dQ
accumulates locally; dK/dV accumulators (fp32) travel with their K/V around the ring and
every rank adds its contribution in the same fixed order, so the result is deterministic;
after the last step the accumulators are handed back to the owning rank.

The per-block arithmetic goes through a ``BlockOps`` object.  ``CudaBlockOps`` (the
default) calls the sm_100a kernels through the C ABI; tests on CPU ranks (gloo) pass
their own fp32 implementation to check the schedule, masking, merge and accumulation
order without a GPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib
from ._kernel import _default_scale


# ------------------------------------------------------------------------------ layout
def chunk_ids(rank: int, world: int) -> tuple[int, int]:
    """The two global chunk indices a rank holds (zig-zag)."""
    return rank, 2 * world - 1 - rank


def shard_sequence(x: torch.Tensor, rank: int, world: int, dim: int = 2) -> torch.Tensor:
    """Slice a full-sequence tensor into this rank's zig-zag pair of chunks."""
    S = x.shape[dim]
    if S % (2 * world):
        raise ValueError(f"sequence length {S} must be a multiple of 2*world_size={2 * world}")
    parts = x.chunk(2 * world, dim=dim)
    a, b = chunk_ids(rank, world)
    return torch.cat([parts[a], parts[b]], dim=dim).contiguous()


def unshard_sequence(shards: list[torch.Tensor], dim: int = 2) -> torch.Tensor:
    """Inverse of ``shard_sequence`` given every rank's shard (rank order)."""
    world = len(shards)
    parts = [None] * (2 * world)
    for r, sh in enumerate(shards):
        a, b = chunk_ids(r, world)
        pa, pb = sh.chunk(2, dim=dim)
        parts[a], parts[b] = pa, pb
    return torch.cat(parts, dim=dim)


def block_kind(x: int, y: int) -> str | None:
    """Attention between query chunk x and key chunk y under causal masking."""
    if y < x:
        return "full"
    if y == x:
        return "causal"
    return None


# ------------------------------------------------------------------------ block ops
class CudaBlockOps:
    """Per-block kernels on the sm_100a library (tensors [BH, C, D] contiguous; bf16 inputs,
    fp32 accumulators).  Partial results never round to bf16: the forward folds each block
    into an fp32 running result in its epilogue (``ffa_fwd_merge``) and the backward adds
    each block's gradients into fp32 accumulators (``ffa_bwd_dkdv_acc`` / ``ffa_bwd_dq_acc``),
    dQ on a side stream beside dK/dV."""

    def __init__(self):
        self._side = {}

    def _stream(self, t):
        return torch.cuda.current_stream(t.device).cuda_stream

    def fwd_merge(self, q, k, v, causal: bool, scale: float, acc, acc_lse, first: bool):
        BH, C, D = q.shape
        lib = _lib.load()
        _lib.check(lib.ffa_fwd_merge(q.data_ptr(), k.data_ptr(), v.data_ptr(), acc.data_ptr(), acc_lse.data_ptr(),
                                     BH, C, D, C * D, D, scale, int(causal), int(first), self._stream(q)),
                   "ffa_fwd_merge")

    def delta(self, o, do):
        BH, C, D = o.shape
        d = torch.empty(BH, C, device=o.device, dtype=torch.float32)
        lib = _lib.load()
        _lib.check(lib.ffa_bwd_preprocess(o.data_ptr(), do.data_ptr(), d.data_ptr(), BH, C, D, C * D, D,
                                          self._stream(o)), "ffa_bwd_preprocess")
        return d

    def bwd_acc(self, q, k, v, do, lse, delta, causal: bool, scale: float, dq_acc, dk_acc, dv_acc):
        BH, C, D = q.shape
        lib = _lib.load()
        cur = torch.cuda.current_stream(q.device)
        side = self._side.get(q.device)
        if side is None:
            side = self._side[q.device] = torch.cuda.Stream(device=q.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            _lib.check(lib.ffa_bwd_dq_acc(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                          delta.data_ptr(), dq_acc.data_ptr(), BH, C, D, C * D, D, scale,
                                          int(causal), side.cuda_stream), "ffa_bwd_dq_acc")
        _lib.check(lib.ffa_bwd_dkdv_acc(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                        delta.data_ptr(), dk_acc.data_ptr(), dv_acc.data_ptr(), BH, C, D, C * D, D,
                                        scale, int(causal), cur.cuda_stream), "ffa_bwd_dkdv_acc")
        cur.wait_stream(side)


# --------------------------------------------------------------------------- comm
class P2PExchange:
    """Ring neighbour exchange over torch.distributed point-to-point (NCCL or gloo)."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def post(self, tensors: list[torch.Tensor]):
        """Start sending `tensors` to rank+1 and receiving the same shapes from rank-1.
        Returns a callable that waits and returns the received tensors."""
        g = self.group
        nxt = (self.rank + 1) % self.world
        prv = (self.rank - 1) % self.world
        if g is not None:
            nxt, prv = dist.get_global_rank(g, nxt), dist.get_global_rank(g, prv)
        bufs = [torch.empty_like(t) for t in tensors]
        ops = [dist.P2POp(dist.isend, t, nxt, g) for t in tensors]
        ops += [dist.P2POp(dist.irecv, b, prv, g) for b in bufs]
        works = dist.batch_isend_irecv(ops)

        def wait():
            for w in works:
                w.wait()
            return bufs

        return wait


def _chunks(x):
    """[B, H, 2C, D] -> two contiguous [B*H, C, D] chunks."""
    B, H, S2, D = x.shape
    a, b = x.chunk(2, dim=2)
    return a.reshape(B * H, S2 // 2, D).contiguous(), b.reshape(B * H, S2 // 2, D).contiguous()


def _unchunks(a, b, B, H):
    BH, C, D = a.shape
    return torch.cat([a.reshape(B, H, C, D), b.reshape(B, H, C, D)], dim=2)


@dataclass
class RingState:
    rank: int
    world: int
    exchange: object  # .post(tensors) -> wait(); wait() returns the previous rank's tensors


def ring_forward(q, k, v, state: RingState, scale: float, ops) -> tuple[torch.Tensor, torch.Tensor]:
    """Causal ring attention forward on this rank's zig-zag shard.

    q, k, v: [B, H, 2C, D] bf16.  Returns (o [B, H, 2C, D] bf16, lse [B*H, 2C] fp32 base 2).
    Each block's result is folded into an fp32 running output in a fixed order (step t,
    then key chunk), so the output is rounded to bf16 once, at the end."""
    B, H, S2, D = q.shape
    r, P = state.rank, state.world
    qc = _chunks(q)
    my_ids = chunk_ids(r, P)
    kv = list(_chunks(k)) + list(_chunks(v))  # k_a, k_b, v_a, v_b
    acc = [torch.empty(qc[0].shape, device=q.device, dtype=torch.float32) for _ in range(2)]
    acc_lse = [torch.empty(qc[0].shape[:2], device=q.device, dtype=torch.float32) for _ in range(2)]
    started = [False, False]
    for t in range(P):
        src = (r - t) % P
        kv_ids = chunk_ids(src, P)
        pending = state.exchange.post(kv) if t + 1 < P else None  # next step's K/V, overlapping this step
        for xi in range(2):
            for yi in range(2):
                kind = block_kind(my_ids[xi], kv_ids[yi])
                if kind is None:
                    continue
                ops.fwd_merge(qc[xi], kv[yi], kv[2 + yi], kind == "causal", scale, acc[xi], acc_lse[xi],
                              not started[xi])
                started[xi] = True
        if pending is not None:
            kv = pending()
    out = _unchunks(acc[0].to(q.dtype), acc[1].to(q.dtype), B, H)
    return out, torch.cat(acc_lse, dim=1)


def ring_backward(q, k, v, o, lse, do, state: RingState, scale: float, ops):
    """Deterministic ring backward; returns dq, dk, dv ([B, H, 2C, D], dtype of q).

    Every block adds its gradients in fp32 into accumulators: dQ locally, dK/dV into the
    accumulators that travel with their K/V chunk.  A chunk's accumulators leave for the
    next rank as soon as this rank's blocks of the step are done, and their transfer
    overlaps the next step's blocks (they are needed again only one step later, by the
    next rank).  The order of the additions is fixed by the ring, so the result is
    bitwise reproducible."""
    B, H, S2, D = q.shape
    r, P = state.rank, state.world
    qc, oc, doc = _chunks(q), _chunks(o), _chunks(do)
    C = S2 // 2
    lse_c = (lse[:, :C].contiguous(), lse[:, C:].contiguous())
    delta = [ops.delta(oc[i], doc[i]) for i in range(2)]
    my_ids = chunk_ids(r, P)
    kv = list(_chunks(k)) + list(_chunks(v))
    dq = [torch.zeros(qc[0].shape, device=q.device, dtype=torch.float32) for _ in range(2)]
    dkv = [torch.zeros(qc[0].shape, device=q.device, dtype=torch.float32) for _ in range(4)]  # dk_a, dk_b, dv_a, dv_b
    pending_dkv = None
    for t in range(P):
        src = (r - t) % P
        kv_ids = chunk_ids(src, P)
        # next step's K/V do not depend on this step: their transfer overlaps the blocks
        pending_kv = state.exchange.post(kv) if t + 1 < P else None
        if pending_dkv is not None:
            dkv = pending_dkv()  # the accumulators of the chunk this step's K/V belong to
        for xi in range(2):
            for yi in range(2):
                kind = block_kind(my_ids[xi], kv_ids[yi])
                if kind is None:
                    continue
                ops.bwd_acc(qc[xi], kv[yi], kv[2 + yi], doc[xi], lse_c[xi], delta[xi], kind == "causal", scale,
                            dq[xi], dkv[yi], dkv[2 + yi])
        if P == 1:
            break
        # the dK/dV accumulators go to rank + 1 after every step; after the last step
        # they arrive back at the rank that owns them
        pending_dkv = state.exchange.post(dkv)
        if pending_kv is not None:
            kv = pending_kv()
    if pending_dkv is not None:
        dkv = pending_dkv()
    dtype = q.dtype
    return (_unchunks(dq[0].to(dtype), dq[1].to(dtype), B, H), _unchunks(dkv[0].to(dtype), dkv[1].to(dtype), B, H),
            _unchunks(dkv[2].to(dtype), dkv[3].to(dtype), B, H))


class RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, state: RingState, scale, ops):
        o, lse = ring_forward(q, k, v, state, scale, ops)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.state, ctx.scale, ctx.ops = state, scale, ops
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = ring_backward(q, k, v, o, lse, do.contiguous(), ctx.state, ctx.scale, ctx.ops)
        return dq, dk, dv, None, None, None


def ring_attention(q, k, v, group=None, scale=None, ops=None, exchange=None, rank=None, world=None):
    """Causal attention over a sequence sharded zig-zag across the ranks of `group`.

    q, k, v: this rank's ``[B, H, 2C, D]`` shard (see ``shard_sequence``).  Differentiable;
    the backward is deterministic.  ``ops`` defaults to the sm_100a kernels (CUDA tensors) and
    ``exchange`` to NCCL/gloo point-to-point on `group`; a custom ``exchange`` (an object whose
    ``post(tensors)`` starts sending to the next rank and returns a callable yielding the
    previous rank's tensors) needs explicit ``rank`` and ``world``."""
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k and v must have the same shape")
    D = q.shape[-1]
    if D not in (64, 128):
        raise ValueError("ring_attention supports head_dim 64 or 128")
    if ops is None:
        if not q.is_cuda:
            raise RuntimeError("ring_attention runs on CUDA tensors (sm_100a kernels); there is no CPU path")
        ops = CudaBlockOps()
    if exchange is None:
        exchange = P2PExchange(group)
        rank, world = exchange.rank, exchange.world
    elif rank is None or world is None:
        raise ValueError("a custom exchange needs rank and world")
    sm = _default_scale(D) if scale is None else float(scale)
    return RingAttention.apply(q, k, v, RingState(rank, world, exchange), sm, ops)
