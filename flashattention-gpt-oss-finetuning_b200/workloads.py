"""Seeded synthetic workloads with the shapes and value distributions of the benchmark configs.

The reference's own benchmark draws ``torch.randn`` inputs (benchmark_backward_speed.py:646-674);
these are the five configurations the B200 build is measured and checked on.  Inputs are drawn
on the CPU from one ``torch.Generator`` in the order q, k, v, dO (fp32), then scaled or
perturbed, then cast, so that a CPU checker and the GPU see identical values.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    n_q_heads: int
    n_kv_heads: int
    seq_len: int
    head_dim: int
    window_size: int
    sink_size: int
    dtype: torch.dtype
    seed: int
    input_scale: float = 1.0
    outlier_frac: float = 0.0     # fraction of q/k entries replaced by +-8

    def replace(self, **kw) -> "Workload":
        return dataclasses.replace(self, **kw)

    @property
    def group(self) -> int:
        return self.n_q_heads // self.n_kv_heads

    def describe(self) -> dict:
        return dict(workload=self.name, B=self.batch, Hq=self.n_q_heads, Hkv=self.n_kv_heads,
                    L=self.seq_len, D=self.head_dim, W=self.window_size, S=self.sink_size,
                    dtype=str(self.dtype).replace("torch.", ""), seed=self.seed)


CONFIGS = {
    # 0: the reference's own benchmark shape (README.md:35; benchmark_backward_speed.py:832)
    "cfg1_ref_bench": Workload("cfg1_ref_bench", 1, 16, 16, 4096, 16, 256, 4, torch.float16, 0),
    # 1: GPT-OSS-style sliding-window layer (the headline workload)
    "cfg2_gptoss_swa": Workload("cfg2_gptoss_swa", 4, 64, 8, 4096, 64, 128, 4, torch.bfloat16, 1,
                                input_scale=0.5),
    # 2: full causal layer (window disabled, W = L)
    "cfg3_full_causal": Workload("cfg3_full_causal", 2, 64, 8, 8192, 64, 8192, 4, torch.bfloat16, 2),
    # 3: long-context sliding window, sharded by KV head across GPUs
    "cfg4_long_swa": Workload("cfg4_long_swa", 1, 64, 8, 131072, 64, 128, 4, torch.bfloat16, 3),
    # 4: ragged length, large head dim, outliers; swept over S in {0, 16}
    "cfg5_ragged_s0": Workload("cfg5_ragged_s0", 8, 32, 4, 3000, 128, 1024, 0, torch.float16, 4,
                               outlier_frac=0.01),
    "cfg5_ragged_s16": Workload("cfg5_ragged_s16", 8, 32, 4, 3000, 128, 1024, 16, torch.float16, 4,
                                outlier_frac=0.01),
}


def make_inputs(w: Workload, device: Optional[torch.device] = None, kv_heads=None, batches=None):
    """(q, k, v, dO) for workload ``w``.

    ``batches`` / ``kv_heads``: optional index lists selecting a sub-problem (the draws are for
    the full problem, then sliced), so a shard sees exactly the values of the full workload.
    """
    g = torch.Generator().manual_seed(w.seed)
    qs = (w.batch, w.n_q_heads, w.seq_len, w.head_dim)
    ks = (w.batch, w.n_kv_heads, w.seq_len, w.head_dim)
    q = torch.randn(qs, generator=g)
    k = torch.randn(ks, generator=g)
    v = torch.randn(ks, generator=g)
    do = torch.randn(qs, generator=g)
    if w.input_scale != 1.0:
        q, k, v, do = (t * w.input_scale for t in (q, k, v, do))
    if w.outlier_frac > 0:
        for t in (q, k):
            flat = t.view(-1)
            n = int(round(w.outlier_frac * flat.numel()))
            idx = torch.randperm(flat.numel(), generator=g)[:n]
            sign = torch.randint(0, 2, (n,), generator=g).float() * 2 - 1
            flat[idx] = 8.0 * sign
    if batches is not None:
        q, k, v, do = (t[list(batches)] for t in (q, k, v, do))
    if kv_heads is not None:
        kvh = list(kv_heads)
        qh = [h * w.group + i for h in kvh for i in range(w.group)]
        q, do = q[:, qh], do[:, qh]
        k, v = k[:, kvh], v[:, kvh]
    out = tuple(t.to(w.dtype).contiguous() for t in (q, k, v, do))
    if device is not None:
        out = tuple(t.to(device) for t in out)
    return out


def visible_pairs_per_head(seq_len: int, window_size: int, sink_size: int) -> int:
    """sum_i [min(i+1, W) + max(0, min(S, i-W+1))]: the (query, key) pairs one head computes."""
    w = max(0, int(window_size))
    s = max(0, int(sink_size))
    i = np.arange(seq_len, dtype=np.int64)
    return int((np.minimum(i + 1, w) + np.maximum(0, np.minimum(s, i - w + 1))).sum())


def useful_flops(w: Workload, which: str = "fwd+bwd", batch: Optional[int] = None) -> float:
    """Useful FLOPs (window + sink pairs only): fwd 4*D, bwd 10*D, fwd+bwd 14*D per pair."""
    b = w.batch if batch is None else batch
    pairs = b * w.n_q_heads * visible_pairs_per_head(w.seq_len, w.window_size, w.sink_size)
    return float({"fwd": 4, "bwd": 10, "fwd+bwd": 14}[which] * w.head_dim * pairs)
