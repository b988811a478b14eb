"""Sequence split of one long sequence over the ranks of a process group, with a K/V halo.

The (batch, KV head) split (``sharding.py``) needs no communication, but it cannot use more
ranks than there are units.  For very long sequences the query rows can be split instead:
rank r owns rows [start_r, end_r) of q, k, v (contiguous, in rank order).  With the mask
``j <= i and (i - j < W or j < S)`` its queries need, besides its own keys, only the
W' = W - 1 keys before ``start_r`` (the halo, owned by rank r - 1) and the S sink keys (owned
by rank 0).  So:

forward   rank 0 broadcasts its S sink rows of K and V; every rank sends its last W' rows of
          K and V to the next rank.  Rank r > 0 then runs the ordinary kernels on a local
          problem whose key rows are [sinks | zero gap | halo | own] and whose query rows are
          [zero rows | own]; the prefix length ``pre`` (a multiple of 128) makes local
          distances equal absolute ones: i_loc - j_loc = i - j for every halo / own key, the
          sink keys sit at local positions < S, and the gap keys are out of every own
          query's window.
backward  the same local problem with zero dO rows in the prefix (they add nothing to dK or
          dV).  dQ is complete locally.  The local dK / dV of the halo rows go back to the
          previous rank, which adds them to its last W' rows, and the sink rows' partials
          are summed onto rank 0 (fp32).

This is the only data-path communication in the library (NCCL point-to-point and a reduce
when the group's backend is NCCL).  It replaces nothing in the reference, whose entry point
runs on one device (flash_attention_gpt_oss.py:437-438).

The local compute is injectable (``fwd_fn``, ``bwd_fn``) so that the exchange protocol can be
tested on CPU ranks; by default it is this library's CUDA path.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist

TILE = 128


def split_bounds(seq_len: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous [start, end) row ranges, one per rank, in multiples of 128 rows (the last
    range takes the remainder; trailing ranks may be empty only if seq_len is tiny)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    per = -(-seq_len // world)
    per = -(-per // TILE) * TILE
    return [(min(r * per, seq_len), min((r + 1) * per, seq_len)) for r in range(world)]


def _window(w: int, seq_len: int) -> int:
    return 0 if w <= 0 else min(w, max(seq_len, 1))


def layout(seq_len: int, world: int, rank: int, window_size: int, sink_size: int):
    """(start, end, halo, pre) of `rank`: its rows, the halo length W' it receives and the
    local prefix length.  Raises ValueError when a halo would reach past the previous rank
    or into the sink rows (use the (batch, KV head) split for such shapes)."""
    bounds = split_bounds(seq_len, world)
    start, end = bounds[rank]
    if rank == 0:
        return start, end, 0, 0
    w = _window(window_size, seq_len)
    s = max(0, min(sink_size, seq_len))
    halo = min(max(w - 1, 0), start)
    prev_n = bounds[rank - 1][1] - bounds[rank - 1][0]
    if halo > prev_n:
        raise ValueError(f"window {window_size} is longer than a rank's {prev_n} rows")
    if start - halo < s:
        raise ValueError("the halo of a rank would overlap the sink rows")
    pre = -(-(s + halo) // TILE) * TILE
    return start, end, halo, pre


def _default_fwd(q, k, v, w, s, scale):
    from .flash_attention_gpt_oss import swa_forward
    return swa_forward(q, k, v, w, s, scale)


def _default_bwd(q, k, v, o, lse, do, w, s, scale):
    from .flash_attention_gpt_oss import swa_backward
    return swa_backward(q, k, v, o, lse, do, w, s, scale)


def _prefixed(x: torch.Tensor, pre: int, head: Optional[torch.Tensor] = None,
              tail: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[B, H, pre + n, D]: `head` at rows [0, head_n), zeros, `tail` ending at row pre, then x
    (one concatenation: x is read once and the result written once)."""
    b, h, n, d = x.shape
    hn = head.shape[2] if head is not None else 0
    tn = tail.shape[2] if tail is not None else 0
    parts = [head] if hn else []
    if pre - hn - tn > 0:
        parts.append(x.new_zeros((b, h, pre - hn - tn, d)))
    if tn:
        parts.append(tail)
    parts.append(x)
    return torch.cat(parts, dim=2) if len(parts) > 1 else x


def _staged(group, device) -> bool:
    """True when CUDA tensors must go through host memory (a gloo group: CPU transport)."""
    return device.type == "cuda" and dist.get_backend(group) == dist.Backend.GLOO


def _global(group, r: int) -> int:
    return dist.get_global_rank(group, r) if group is not None else r


def _exchange(send_next: Optional[torch.Tensor], recv_prev_shape, rank, world, group,
              reverse=False):
    """Point-to-point: send to rank+1 and receive from rank-1 (or the other way round)."""
    dst = rank - 1 if reverse else rank + 1
    src = rank + 1 if reverse else rank - 1
    ops, got, out = [], None, None
    if send_next is not None and 0 <= dst < world:
        t = send_next.contiguous()
        if _staged(group, t.device):
            t = t.cpu()
        ops.append(dist.P2POp(dist.isend, t, _global(group, dst), group))
    if recv_prev_shape is not None and 0 <= src < world:
        shape, dtype, dev = recv_prev_shape
        out = torch.empty(shape, dtype=dtype, device=dev)
        got = out.cpu() if _staged(group, dev) else out
        ops.append(dist.P2POp(dist.irecv, got, _global(group, src), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    if got is not None and got is not out:
        out.copy_(got)
    return out


def _broadcast0(t: torch.Tensor, group):
    if _staged(group, t.device):
        h = t.cpu()
        dist.broadcast(h, src=_global(group, 0), group=group)
        t.copy_(h)
    else:
        dist.broadcast(t, src=_global(group, 0), group=group)


def _reduce0(t: torch.Tensor, group):
    if _staged(group, t.device):
        h = t.cpu()
        dist.reduce(h, dst=_global(group, 0), group=group)
        t.copy_(h)
    else:
        dist.reduce(t, dst=_global(group, 0), group=group)


_SIDE = {}


def _side_stream(device):
    """One side stream per device for the exchanges (created once)."""
    if device not in _SIDE:
        _SIDE[device] = torch.cuda.Stream(device)
    return _SIDE[device]


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class SeqShardState:
    """What the backward needs from the forward of one rank."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def seq_sharded_forward(q, k, v, seq_len: int, window_size: int, sink_size: int = 0,
                        softmax_scale: Optional[float] = None, group=None,
                        fwd_fn: Callable = _default_fwd):
    """This rank's o ([B, Hq, n, D]) and the state for :func:`seq_sharded_backward`.  q, k, v
    are this rank's rows (``split_bounds(seq_len, world)[rank]``)."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    start, end, halo, pre = layout(seq_len, world, rank, window_size, sink_size)
    if q.shape[2] != end - start or k.shape[2] != end - start:
        raise ValueError(f"rank {rank} holds rows [{start}, {end}) but got {q.shape[2]}")
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    s = max(0, min(sink_size, seq_len))
    b, hkv, _, d = k.shape
    # the exchanges run on a side stream, beside the query prefix copy or rank 0's forward
    main = torch.cuda.current_stream(q.device) if q.is_cuda else None
    side = _side_stream(q.device) if q.is_cuda else None
    if side is not None:
        side.wait_stream(main)
    with torch.cuda.stream(side) if side is not None else _nullctx():
        # sink rows from rank 0
        kvs = torch.cat([k[:, :, :s], v[:, :, :s]], 1).contiguous() if rank == 0 else \
            k.new_empty((b, 2 * hkv, s, d))
        if world > 1 and s > 0:
            _broadcast0(kvs, group)
        # halo rows from the previous rank: it sends its last W'(rank + 1) rows
        nxt_halo = layout(seq_len, world, rank + 1, window_size, sink_size)[2] \
            if rank + 1 < world else 0
        send = torch.cat([k[:, :, k.shape[2] - nxt_halo:], v[:, :, v.shape[2] - nxt_halo:]], 1) \
            if nxt_halo > 0 else None
        recv_shape = ((b, 2 * hkv, halo, d), k.dtype, k.device) if halo > 0 else None
        got = _exchange(send, recv_shape, rank, world, group)
    ql = _prefixed(q, pre) if rank > 0 else q
    if side is not None and rank > 0:   # rank 0's own forward needs nothing it receives
        main.wait_stream(side)
        for t in (kvs, got, send):
            if t is not None:
                t.record_stream(main)
    if rank == 0:
        o, lse = fwd_fn(q, k, v, window_size, sink_size, softmax_scale)
        return o, SeqShardState(rank=rank, world=world, pre=0, halo=0, s=s, q=q, k=k, v=v, o=o,
                                lse=lse, w=window_size, sink=sink_size, scale=softmax_scale,
                                seq_len=seq_len, group=group)
    kh = got[:, :hkv] if got is not None else None
    vh = got[:, hkv:] if got is not None else None
    kl = _prefixed(k, pre, kvs[:, :hkv], kh)
    vl = _prefixed(v, pre, kvs[:, hkv:], vh)
    ol, lse = fwd_fn(ql, kl, vl, window_size, sink_size, softmax_scale)
    return ol[:, :, pre:], SeqShardState(rank=rank, world=world, pre=pre, halo=halo, s=s, q=ql,
                                         k=kl, v=vl, o=ol, lse=lse, w=window_size,
                                         sink=sink_size, scale=softmax_scale, seq_len=seq_len,
                                         group=group)


def seq_sharded_backward(st: SeqShardState, do, bwd_fn: Callable = _default_bwd):
    """This rank's (dq, dk, dv) for its rows, after the halo and sink exchanges."""
    rank, world, pre, group = st.rank, st.world, st.pre, st.group
    dol = do if rank == 0 else _prefixed(do.to(st.q.dtype), pre)
    dql, dkl, dvl = bwd_fn(st.q, st.k, st.v, st.o, st.lse, dol, st.w, st.sink, st.scale)
    n = dql.shape[2] - pre
    dq, dk, dv = dql[:, :, pre:], dkl[:, :, pre:], dvl[:, :, pre:]
    acc = torch.promote_types(dkl.dtype, torch.float32)  # the added rows sum in fp32 (or wider)
    hkv = dkl.shape[1]

    def add_rows(rows: slice, extra: torch.Tensor):
        for t, e in ((dk, extra[:, :hkv]), (dv, extra[:, hkv:])):
            t[:, :, rows] = (t[:, :, rows].to(acc) + e).to(t.dtype)

    # halo gradients go back to the previous rank, which owns those keys
    send = torch.cat([dkl[:, :, pre - st.halo:pre], dvl[:, :, pre - st.halo:pre]], 1).to(acc) \
        if st.halo > 0 else None
    nxt_halo = layout(st.seq_len, world, rank + 1, st.w, st.sink)[2] if rank + 1 < world else 0
    shape = ((dk.shape[0], 2 * hkv, nxt_halo, dk.shape[3]), acc, dk.device) \
        if nxt_halo > 0 else None
    got = _exchange(send, shape, rank, world, group, reverse=True)
    if got is not None:
        add_rows(slice(n - nxt_halo, n), got)
    # sink rows: every rank's partial summed onto rank 0
    if world > 1 and st.s > 0:
        part = torch.cat([dkl[:, :, :st.s], dvl[:, :, :st.s]], 1).to(acc) if rank > 0 else \
            torch.zeros((dk.shape[0], 2 * hkv, st.s, dk.shape[3]), dtype=acc, device=dk.device)
        _reduce0(part, group)
        if rank == 0:
            add_rows(slice(0, st.s), part)
    return dq, dk, dv


class SeqShardedSWDA(torch.autograd.Function):
    """Autograd form: ``o = SeqShardedSWDA.apply(q, k, v, seq_len, window_size, sink_size,
    softmax_scale, group)`` with this rank's rows of q, k, v; backward returns this rank's
    dq, dk, dv (the exchanges run inside)."""

    @staticmethod
    def forward(ctx, q, k, v, seq_len, window_size, sink_size=0, softmax_scale=None, group=None):
        o, st = seq_sharded_forward(q, k, v, seq_len, window_size, sink_size, softmax_scale, group)
        ctx.st = st
        return o

    @staticmethod
    def backward(ctx, do):
        dq, dk, dv = seq_sharded_backward(ctx.st, do)
        ctx.st = None
        return dq, dk, dv, None, None, None, None, None
