"""Sequence-sharded causal screening attention for long contexts.

A sequence of length T is cut into `world` contiguous blocks of T/world
tokens, one per rank (global offset rank * L).  Because the softmask is
exactly zero for keys at distance >= w (multiscreen/attention.py:117-118),
the only keys a rank needs from other ranks are the `halo` = ceil(max w) - 1
rows before its block.  They arrive by NCCL point-to-point (one grouped
send/recv per peer; several peers when halo > L), and only K and V cross
the link -- queries, outputs and everything else stay local.

Per layer, per rank:
  1. post the halo exchange (the send buffers are the last rows of k, v);
  2. attend the interior query rows i >= halo on the local keys alone
     (q_offset = halo), while the exchange is in flight;
  3. wait for the halo, attend the boundary rows i < halo over
     [halo keys ; local keys 0 .. halo-1] (q_offset = halo length).
Both calls are the fused kernels with their q_offset argument, so the row
results are the same as one call over the whole sequence.  Under autograd
the exchange runs in reverse in the backward: the gradient rows of the halo
keys/values go back to the ranks that own them and are added there.

Use:

    with sequence_parallel(local_len=T // world, group=pg):
        out = model(ids[:, rank * L:(rank + 1) * L])     # MultiscreenLM
"""
from __future__ import annotations

import contextlib
import contextvars
import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

_ACTIVE: contextvars.ContextVar = contextvars.ContextVar("screening_sequence_shard",
                                                          default=None)


@dataclass(frozen=True)
class SequenceShard:
    """This rank's contiguous block of a sequence sharded over a process group."""
    group: object
    rank: int
    world: int
    local_len: int

    @property
    def start(self) -> int:
        return self.rank * self.local_len

    def global_rank(self, r: int) -> int:
        return r if self.group is None else dist.get_global_rank(self.group, r)


@contextlib.contextmanager
def sequence_parallel(local_len: int, group=None):
    """Within this context, causal self-attention of ScreeningAttention and
    MultiscreenLM.forward/prefill treat their (B, local_len, ...) inputs as
    block `rank` of a sequence sharded over `group` (default: WORLD)."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    tok = _ACTIVE.set(SequenceShard(group, rank, world, int(local_len)))
    try:
        yield _ACTIVE.get()
    finally:
        _ACTIVE.reset(tok)


def current_shard() -> SequenceShard | None:
    return _ACTIVE.get()


_TIMELINE: contextvars.ContextVar = contextvars.ContextVar("screening_shard_timeline",
                                                            default=None)


@contextlib.contextmanager
def shard_timeline():
    """Record CUDA events around the three phases of every sharded attention
    call made inside the context: [start, interior done, halo ready,
    boundary done] per call.  Yields the list; read it after a synchronize
    with shard_timeline_summary()."""
    events: list = []
    tok = _TIMELINE.set(events)
    try:
        yield events
    finally:
        _TIMELINE.reset(tok)


def _mark(events, slot):
    if events is not None:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        slot.append(e)


def shard_timeline_summary(events) -> dict:
    """Mean per call (ms): interior attention, the stream's stall for the
    halo once the interior rows are done (0 when the exchange is hidden),
    boundary attention."""
    rows = [c for c in events if len(c) == 4]
    if not rows:
        return {}
    n = len(rows)
    return {"calls": n,
            "interior_ms": sum(c[0].elapsed_time(c[1]) for c in rows) / n,
            "halo_stall_ms": sum(c[1].elapsed_time(c[2]) for c in rows) / n,
            "boundary_ms": sum(c[2].elapsed_time(c[3]) for c in rows) / n}


def halo_plan(rank: int, world: int, local_len: int, halo: int):
    """Rows exchanged for a halo of `halo` keys with equal blocks of `local_len`.

    Returns (sends, recvs): sends = [(dst_rank, lo, hi)] local rows [lo, hi)
    that rank dst needs; recvs = [(src_rank, lo, hi)] rows [lo, hi) of rank
    src's block that this rank needs, oldest first, so their concatenation is
    the halo in sequence order (length min(halo, rank * local_len))."""
    sends, recvs = [], []
    if halo <= 0 or local_len <= 0:
        return sends, recvs
    m = 1
    while True:
        lo = m * local_len - halo       # rows of a block m ranks back that are still needed
        if lo >= local_len:
            break
        lo = max(0, lo)
        if rank + m < world:
            sends.append((rank + m, lo, local_len))
        if rank - m >= 0:
            recvs.append((rank - m, lo, local_len))
        m += 1
    recvs.reverse()
    return sends, recvs


def _post(ops):
    if not ops:
        return []
    return dist.batch_isend_irecv(ops)


def _wait(works):
    for wk in works:
        wk.wait()


class _HaloStart:
    """Posted forward exchange: send buffers must live until the wait."""

    def __init__(self, shard: SequenceShard, k: torch.Tensor, v: torch.Tensor, halo: int,
                 extra: torch.Tensor | None = None):
        B, L, H, D = k.shape
        self.shard, self.halo = shard, halo
        self.sends, self.recvs = halo_plan(shard.rank, shard.world, L, halo)
        ops, self.keep, self.bufs = [], [], []
        for dst, lo, hi in self.sends:
            buf = torch.stack([k[:, lo:hi], v[:, lo:hi]]).contiguous()
            self.keep.append(buf)
            ops.append(dist.P2POp(dist.isend, buf, shard.global_rank(dst), shard.group))
            if extra is not None:
                mb = extra[:, lo:hi].contiguous()
                self.keep.append(mb)
                ops.append(dist.P2POp(dist.isend, mb, shard.global_rank(dst), shard.group))
        for src, lo, hi in self.recvs:
            buf = torch.empty(2, B, hi - lo, H, D, dtype=k.dtype, device=k.device)
            ops.append(dist.P2POp(dist.irecv, buf, shard.global_rank(src), shard.group))
            mb = None
            if extra is not None:
                mb = torch.empty(B, hi - lo, dtype=extra.dtype, device=extra.device)
                ops.append(dist.P2POp(dist.irecv, mb, shard.global_rank(src), shard.group))
            self.bufs.append((buf, mb))
        self.works = _post(ops)

    def finish(self):
        _wait(self.works)
        self.keep = []
        if not self.bufs:
            return None, None, None
        kh = torch.cat([b[0] for b, _ in self.bufs], dim=1)
        vh = torch.cat([b[1] for b, _ in self.bufs], dim=1)
        mh = None
        if self.bufs[0][1] is not None:
            mh = torch.cat([m for _, m in self.bufs], dim=1)
        return kh, vh, mh


class HaloExchange(torch.autograd.Function):
    """(k, v) local (B, L, H, D) -> (k_halo, v_halo) (B, n, H, D): the n =
    min(halo, start) key/value rows before this rank's block.  The backward
    returns the halo gradients to their owners and adds them to the local
    rows they were sent from."""

    @staticmethod
    def forward(ctx, k, v, shard, halo, pending):
        ctx.shard, ctx.halo, ctx.shape = shard, halo, k.shape
        ctx.dtype, ctx.device = k.dtype, k.device
        if pending is None:
            pending = _HaloStart(shard, k, v, halo)
        kh, vh, _ = pending.finish()
        ctx.sends, ctx.recvs = pending.sends, pending.recvs
        B, _, H, D = k.shape
        if kh is None:
            kh = k.new_zeros(B, 0, H, D)
            vh = v.new_zeros(B, 0, H, D)
        return kh, vh

    @staticmethod
    def backward(ctx, gk, gv):
        shard = ctx.shard
        B, L, H, D = ctx.shape
        dk = torch.zeros(ctx.shape, dtype=ctx.dtype, device=ctx.device)
        dv = torch.zeros_like(dk)
        ops, keep, bufs = [], [], []
        off = 0
        for src, lo, hi in ctx.recvs:          # halo rows go back to their owners
            n = hi - lo
            g = torch.stack([gk[:, off:off + n], gv[:, off:off + n]]).to(ctx.dtype).contiguous()
            keep.append(g)
            ops.append(dist.P2POp(dist.isend, g, shard.global_rank(src), shard.group))
            off += n
        for dst, lo, hi in ctx.sends:          # gradients of rows this rank sent
            g = torch.empty(2, B, hi - lo, H, D, dtype=ctx.dtype, device=ctx.device)
            ops.append(dist.P2POp(dist.irecv, g, shard.global_rank(dst), shard.group))
            bufs.append((g, lo, hi))
        _wait(_post(ops))
        for g, lo, hi in bufs:
            dk[:, lo:hi] += g[0]
            dv[:, lo:hi] += g[1]
        return dk, dv, None, None, None


def _default_attention():
    from .functional import screening_attention
    return screening_attention


def window_halo(w: torch.Tensor) -> int:
    """Keys before a query that can still carry weight: ceil(max w) - 1."""
    if w.numel() == 0:
        return 0
    return max(0, int(math.ceil(float(w.detach().max()))) - 1)


def screening_attention_sharded(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                r: torch.Tensor, w: torch.Tensor,
                                key_padding_mask: torch.Tensor | None = None,
                                eps: float = 1e-8, shard: SequenceShard | None = None,
                                attn_fn=None) -> torch.Tensor:
    """Causal screening attention of this rank's block of a sharded sequence.

    q, k, v: (B, L, H, D) raw projections of the local block; r, w (H,);
    key_padding_mask (B, L) of the local keys (True = ignore) or None.
    Returns (B, L, H, D), the rows one unsharded call would give for these
    positions.  `attn_fn` is the single-device attention with the signature
    of functional.screening_attention (default: the CUDA kernels)."""
    shard = shard or current_shard()
    if shard is None:
        raise RuntimeError("screening_attention_sharded needs a sequence_parallel() context")
    attn = attn_fn or _default_attention()
    B, L, H, D = q.shape
    if L != shard.local_len or k.shape[1] != L:
        raise ValueError(f"local block length {L} != shard length {shard.local_len}")
    halo = window_halo(w)
    tl = _TIMELINE.get()
    marks: list = []
    if tl is not None:
        tl.append(marks)
    _mark(tl, marks)
    pending = None
    if shard.world > 1 and halo > 0:
        pending = _HaloStart(shard, k.detach(), v.detach(), halo,
                             None if key_padding_mask is None else
                             key_padding_mask.to(torch.uint8))
    nb = min(halo, L)                      # boundary rows: their window leaves the block
    parts = []
    if nb < L:
        # interior rows, overlapped with the exchange
        parts.append((nb, attn(q[:, nb:], k, v, r, w, True, key_padding_mask, eps, nb)))
    _mark(tl, marks)
    if nb > 0:
        mh = None
        if pending is not None:
            # the mask rows come with the exchange; K/V go through the
            # autograd function so their gradients return to the owners
            mh_bufs = [m for _, m in pending.bufs]
            kh, vh = HaloExchange.apply(k, v, shard, halo, pending)
            if key_padding_mask is not None and mh_bufs:
                mh = torch.cat(mh_bufs, dim=1).bool()
        else:
            kh = k.new_zeros(B, 0, H, D)
            vh = v.new_zeros(B, 0, H, D)
        _mark(tl, marks)
        n = kh.shape[1]
        ke = torch.cat([kh.to(k.dtype), k[:, :nb]], dim=1)
        ve = torch.cat([vh.to(v.dtype), v[:, :nb]], dim=1)
        kpm = None
        if key_padding_mask is not None:
            kpm = key_padding_mask[:, :nb]
            if n > 0:
                kpm = torch.cat([mh if mh is not None else kpm.new_zeros(B, n), kpm], dim=1)
        parts.append((0, attn(q[:, :nb], ke, ve, r, w, True, kpm, eps, n)))
        _mark(tl, marks)
    parts.sort(key=lambda p: p[0])
    ys = [p[1] for p in parts]
    return ys[0] if len(ys) == 1 else torch.cat(ys, dim=1)
