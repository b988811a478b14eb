"""CPU oracle for causal sliding-window + sink-token + GQA attention (forward and backward).

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA kernels are compared
against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product path (the package's
``flash_swda_with_sink``) never calls into this file and has no CPU fallback.

It restates, in plain PyTorch-on-CPU arithmetic, the reference project's naive attention
(junhown3/FlashAttention-GPT-OSS-finetuning):

* mask            -- ``create_mask_bool``        benchmark_backward_speed.py:40-46
* GQA expansion   -- ``repeat_kv``               benchmark_backward_speed.py:49-54
* forward         -- ``pytorch_naive_attention`` benchmark_backward_speed.py:68-85
* backward        -- the gradient autograd derives for that forward, written out
                     explicitly (dV = P^T dO, dP = dO V^T, dS = P (dP - rowsum(dO*O)),
                     dQ = scale dS K, dK = scale dS^T Q), the same algebra as the
                     reference kernel's pass 2 (flash_attention_gpt_oss.py:273-332).
* softmax scale   -- ``1/sqrt(D)`` when ``None`` (flash_attention_gpt_oss.py:345-346);
                     the naive function always uses ``1/sqrt(D)``; here it is a parameter.

Empty rows.  With ``window_size <= 0`` and ``sink_size == 0`` a query row sees no key.  The
naive reference then yields NaN; the reference's fused kernel writes O = 0 for such rows
(``l_i == 0 -> 1``, flash_attention_gpt_oss.py:170).  The product follows the fused kernel,
so ``empty_rows="zero"`` (the default here) returns 0 for O and for the gradients of such
rows; ``empty_rows="nan"`` reproduces the naive function.

Parity pin.  ``tests/golden/make_golden.py`` runs the reference's own
``pytorch_naive_attention`` + autograd and the reference's Triton entry point
``FlashSWDAWithSink`` (under the Triton CPU interpreter) on seeded inputs and stores the
results under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this file against them.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np
import torch

LOG2E = 1.4426950408889634


def visible_mask(seq_len: int, window_size: int, sink_size: int) -> torch.Tensor:
    """Boolean [L, L] mask: key j visible to query i iff j <= i and (i - j < W or j < S).

    Follows benchmark_backward_speed.py:40-46 (``create_mask_bool``).
    """
    idx = torch.arange(seq_len)
    row = idx[:, None]
    col = idx[None, :]
    sliding = (col <= row) & (col >= row - (window_size - 1))
    sink = (col < sink_size) & (col <= row)
    return sliding | sink


def _expand_kv(x: torch.Tensor, n_q_heads: int) -> torch.Tensor:
    """GQA: query head h reads KV head h // (Hq // Hkv) (benchmark_backward_speed.py:49-54)."""
    group = n_q_heads // x.shape[1]
    if group == 1:
        return x
    b, hkv, l, d = x.shape
    return x[:, :, None].expand(b, hkv, group, l, d).reshape(b, hkv * group, l, d)


def _scale(d: int, scale: Optional[float]) -> float:
    return 1.0 / math.sqrt(d) if scale is None else float(scale)


def _probs(q, k, mask, scale, empty_rows):
    s = (q @ k.transpose(-1, -2)) * scale
    s = s.masked_fill(~mask, float("-inf"))
    m = s.amax(dim=-1, keepdim=True)
    empty = torch.isneginf(m)
    if empty_rows == "zero":
        m = torch.where(empty, torch.zeros_like(m), m)
    e = torch.exp(s - m)
    l = e.sum(dim=-1, keepdim=True)
    if empty_rows == "zero":
        l_safe = torch.where(l == 0, torch.ones_like(l), l)
        p = e / l_safe
        lse = torch.where(empty, torch.full_like(m, float("-inf")), m + torch.log(l_safe))
    else:
        p = e / l
        lse = m + torch.log(l)
    return p, lse.squeeze(-1)


def forward(q, k, v, window_size: int, sink_size: int = 0, scale: Optional[float] = None,
            empty_rows: str = "zero", compute_dtype=torch.float64) -> Tuple[torch.Tensor, torch.Tensor]:
    """O = softmax(mask(scale QK^T)) V on CPU in ``compute_dtype``.

    Returns ``(o, lse)`` with ``lse`` the natural-log logsumexp of the masked scaled scores
    ([B, Hq, L]; -inf for an empty row).  Follows benchmark_backward_speed.py:68-85.
    """
    q, k, v = (t.detach().to("cpu", compute_dtype) for t in (q, k, v))
    hq, l = q.shape[1], q.shape[2]
    k, v = _expand_kv(k, hq), _expand_kv(v, hq)
    mask = visible_mask(l, window_size, sink_size)
    p, lse = _probs(q, k, mask, _scale(q.shape[-1], scale), empty_rows)
    return p @ v, lse


def backward(q, k, v, do, window_size: int, sink_size: int = 0, scale: Optional[float] = None,
             empty_rows: str = "zero", compute_dtype=torch.float64):
    """(o, dq, dk, dv) for loss = <O, dO>; dk/dv are summed over each KV head's query group.

    Explicit form of the gradient of benchmark_backward_speed.py:68-85, the same algebra as
    flash_attention_gpt_oss.py:273-332 (without that kernel's ``+1e-6`` on the row sum).
    """
    q, k, v, do = (t.detach().to("cpu", compute_dtype) for t in (q, k, v, do))
    b, hq, l, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    sc = _scale(d, scale)
    ke, ve = _expand_kv(k, hq), _expand_kv(v, hq)
    mask = visible_mask(l, window_size, sink_size)
    p, _ = _probs(q, ke, mask, sc, empty_rows)
    o = p @ ve
    delta = (do * o).sum(-1, keepdim=True)                  # rowsum(dO * O)
    dp = do @ ve.transpose(-1, -2)
    ds = p * (dp - delta)
    dq = (ds @ ke) * sc
    dk_e = (ds.transpose(-1, -2) @ q) * sc
    dv_e = p.transpose(-1, -2) @ do
    dk = dk_e.reshape(b, hkv, g, l, d).sum(2)
    dv = dv_e.reshape(b, hkv, g, l, d).sum(2)
    return o, dq, dk, dv


def backward_chunked(q, k, v, do, window_size: int, sink_size: int = 0, scale=None,
                     compute_dtype=torch.float32, heads=None):
    """Same as :func:`backward`, one (batch, KV head) unit at a time to bound memory.

    ``heads``: optional iterable of (b, kv_head) units to compute; the others stay zero.
    Used for the CPU baseline and for large parity cases.
    """
    b, hq, l, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    o = torch.zeros(q.shape, dtype=compute_dtype)
    dq = torch.zeros(q.shape, dtype=compute_dtype)
    dk = torch.zeros(k.shape, dtype=compute_dtype)
    dv = torch.zeros(v.shape, dtype=compute_dtype)
    units = heads if heads is not None else [(bi, h) for bi in range(b) for h in range(hkv)]
    for bi, h in units:
        sl = slice(h * g, (h + 1) * g)
        r = backward(q[bi:bi + 1, sl], k[bi:bi + 1, h:h + 1], v[bi:bi + 1, h:h + 1],
                     do[bi:bi + 1, sl], window_size, sink_size, scale,
                     compute_dtype=compute_dtype)
        o[bi, sl], dq[bi, sl], dk[bi, h], dv[bi, h] = r[0][0], r[1][0], r[2][0, 0], r[3][0, 0]
    return o, dq, dk, dv


# --------------------------------------------------------------------------------------
# Work accounting (useful window + sink pairs only)
# --------------------------------------------------------------------------------------

def visible_pairs_per_head(seq_len: int, window_size: int, sink_size: int) -> int:
    """sum_i [min(i+1, W) + max(0, min(S, i-W+1))] in closed form (W clamped to >= 0)."""
    w = max(0, int(window_size))
    s = max(0, int(sink_size))
    i = np.arange(seq_len, dtype=np.int64)
    win = np.minimum(i + 1, w)
    sink = np.maximum(0, np.minimum(s, i - w + 1))
    return int((win + sink).sum())


def useful_flops(b, hq, seq_len, d, window_size, sink_size, which="fwd+bwd") -> float:
    pairs = b * hq * visible_pairs_per_head(seq_len, window_size, sink_size)
    per = {"fwd": 4, "bwd": 10, "fwd+bwd": 14}[which]
    return float(per * d * pairs)


# --------------------------------------------------------------------------------------
# Windowed oracle for very long sequences (one query head / KV head pair, [L, D] tensors)
# --------------------------------------------------------------------------------------

def rows_backward(qh, kh, vh, doh, r0: int, r1: int, window_size: int, sink_size: int,
                  scale: Optional[float] = None, compute_dtype=torch.float64):
    """Exact O, dQ for query rows [r0, r1) using only the keys they can see, plus the dense
    P and dS over those keys (for dK / dV contributions).

    The same algebra as :func:`backward` (benchmark_backward_speed.py:68-85 and its autograd
    gradient), restricted to the key set sinks [0, S) U window [r0 - W + 1, r1).  Returns
    (o [R, D], dq [R, D], keys [K] (absolute indices), p [R, K], ds [R, K]); ds excludes the
    softmax scale (dK_j = scale * sum_i ds_ij q_i).
    """
    L, d = qh.shape
    sc = _scale(d, scale)
    w = max(0, int(window_size))
    lo = max(0, r0 - w + 1)
    keys = sorted(set(range(min(sink_size, r1))) | set(range(lo, r1)))
    keys_t = torch.tensor(keys, dtype=torch.long)
    q = qh[r0:r1].to(compute_dtype)
    do = doh[r0:r1].to(compute_dtype)
    k = kh[keys_t].to(compute_dtype)
    v = vh[keys_t].to(compute_dtype)
    i = torch.arange(r0, r1)[:, None]
    j = keys_t[None, :]
    mask = (j <= i) & ((i - j < w) | (j < sink_size))
    p, _ = _probs(q, k, mask, sc, "zero")
    o = p @ v
    delta = (do * o).sum(-1, keepdim=True)
    ds = p * (do @ v.transpose(-1, -2) - delta)
    dq = (ds @ k) * sc
    return o, dq, keys_t, p, ds


# ---------------------------------------------------------------------------------------
# Learned per-head sink logits (an additional mode; not part of the reference).
#
# The form GPT-OSS uses: each query head h has a learned logit sink_h that joins every row's
# softmax as one more column with value 0 -- P = softmax([scale q k^T (masked), sink_h]),
# O = P[:, :-1] V.  Restated here from that published formula; the gradients come from
# autograd on this float64 restatement, including d loss / d sink_h = -sum_i P_i,sink Delta_i.
# It combines with the token sinks (sink_size) of the reference's mask.
# ---------------------------------------------------------------------------------------

def _sink_logit_attention(q, k, v, window_size, sink_size, sinks, scale):
    b, hq, l, d = q.shape
    ke, ve = _expand_kv(k, hq), _expand_kv(v, hq)
    mask = visible_mask(l, window_size, sink_size)
    s = (q @ ke.transpose(-1, -2)) * _scale(d, scale)
    s = s.masked_fill(~mask, float("-inf"))
    col = sinks.reshape(1, hq, 1, 1).expand(b, hq, l, 1)
    p = torch.softmax(torch.cat([s, col], dim=-1), dim=-1)
    lse = torch.logsumexp(torch.cat([s, col], dim=-1), dim=-1)
    return p[..., :l] @ ve, lse


def forward_sink_logits(q, k, v, window_size: int, sink_size: int, sinks, scale: Optional[float] = None,
                        compute_dtype=torch.float64):
    """(o, lse) with the learned sink logits ``sinks`` ([Hq], natural-log units)."""
    q, k, v = (t.detach().to("cpu", compute_dtype) for t in (q, k, v))
    sinks = torch.as_tensor(sinks).detach().to("cpu", compute_dtype)
    with torch.no_grad():
        return _sink_logit_attention(q, k, v, window_size, sink_size, sinks, scale)


def backward_sink_logits(q, k, v, do, window_size: int, sink_size: int, sinks,
                         scale: Optional[float] = None, compute_dtype=torch.float64):
    """(o, dq, dk, dv, dsinks) for loss = <O, dO> with learned sink logits."""
    q, k, v, do = (t.detach().to("cpu", compute_dtype).requires_grad_(r)
                   for t, r in zip((q, k, v, do), (True, True, True, False)))
    sinks = torch.as_tensor(sinks).detach().to("cpu", compute_dtype).requires_grad_(True)
    with torch.enable_grad():
        o, _ = _sink_logit_attention(q, k, v, window_size, sink_size, sinks, scale)
        (o * do).sum().backward()
    return o.detach(), q.grad, k.grad, v.grad, sinks.grad
