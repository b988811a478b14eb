"""Multi-GPU partitioning of the attention by independent (batch, KV head) units.

A unit is one batch entry and one KV head together with the G = Hq / Hkv query heads that read
it.  Units share nothing in the forward or the backward, so ranks process disjoint unit sets
with no collective on the data path (one process per GPU).  A rank's units are repacked as an
independent batch of single-KV-head problems ([n_units, G, L, D] queries, [n_units, 1, L, D]
keys / values), which the kernels take unchanged.
"""
from __future__ import annotations

from typing import Callable, List, Sequence, Tuple

import torch

Unit = Tuple[int, int]  # (batch index, KV head)


def all_units(batch: int, n_kv_heads: int) -> List[Unit]:
    return [(b, h) for b in range(batch) for h in range(n_kv_heads)]


def plan_units(batch: int, n_kv_heads: int, world: int) -> List[List[Unit]]:
    """Contiguous, balanced split of the units over `world` ranks (sizes differ by <= 1)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    units = all_units(batch, n_kv_heads)
    n = len(units)
    out, start = [], 0
    for r in range(world):
        cnt = n // world + (1 if r < n % world else 0)
        out.append(units[start:start + cnt])
        start += cnt
    return out


def _flat_index(units: Sequence[Unit], n_kv_heads: int) -> torch.Tensor:
    return torch.tensor([b * n_kv_heads + h for b, h in units], dtype=torch.long)


def to_unit_batch(q, k, v, units: Sequence[Unit], *extra_q):
    """Gather `units` of [B, Hq, L, D] / [B, Hkv, L, D] tensors into unit batches.

    Returns (q_u [n, G, L, D], k_u [n, 1, L, D], v_u [n, 1, L, D], *extra_u) where `extra_q`
    are further tensors shaped like q (e.g. dO).
    """
    b, hq, l, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    idx = _flat_index(units, hkv).to(q.device)
    def qsel(t):
        return t.reshape(b * hkv, g, l, d).index_select(0, idx)
    def ksel(t):
        return t.reshape(b * hkv, 1, l, d).index_select(0, idx)
    return (qsel(q), ksel(k), ksel(v)) + tuple(qsel(t) for t in extra_q)


def from_unit_batch(x_u, units: Sequence[Unit], batch: int, n_kv_heads: int, out=None):
    """Scatter unit results ([n, H, L, D], H = G or 1) back into [B, Hkv*H, L, D]."""
    n, hh, l, d = x_u.shape
    if out is None:
        out = torch.zeros(batch, n_kv_heads * hh, l, d, dtype=x_u.dtype, device=x_u.device)
    idx = _flat_index(units, n_kv_heads).to(x_u.device)
    out.view(batch * n_kv_heads, hh, l, d).index_copy_(0, idx, x_u)
    return out


def sharded_backward(q, k, v, do, window_size: int, sink_size: int,
                     compute: Callable, group=None):
    """Run `compute(q_u, k_u, v_u, do_u, W, S) -> (o, dq, dk, dv)` on this rank's units and
    all-gather the full results (a utility for checks and small jobs; the benchmark keeps
    each rank's results local)."""
    import torch.distributed as dist
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    b, hq, l, d = q.shape
    hkv = k.shape[1]
    plans = plan_units(b, hkv, world)
    mine = plans[rank]
    outs = [None, None, None, None]
    if mine:
        qu, ku, vu, dou = to_unit_batch(q, k, v, mine, do)
        outs = list(compute(qu, ku, vu, dou, window_size, sink_size))
    full = [torch.zeros_like(q), torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)]
    for r, units in enumerate(plans):
        if not units:
            continue
        shapes = [(len(units), hq // hkv, l, d)] * 2 + [(len(units), 1, l, d)] * 2
        for i in range(4):
            buf = outs[i] if r == rank else torch.empty(shapes[i], dtype=q.dtype, device=q.device)
            buf = buf.contiguous()
            if world > 1:
                dist.broadcast(buf, src=r, group=group)
            from_unit_batch(buf, units, b, hkv, out=full[i])
    return tuple(full)
