"""Pin the CPU oracle against fixtures produced by the reference project itself."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import swa_oracle as orc

FILES = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f)[7:-4] for f in FILES])
def test_oracle_matches_reference_naive(path):
    z = np.load(path)
    b, hq, hkv, l, d, w, s, _ = z["shape"]
    q, k, v, do = (torch.from_numpy(z[n]) for n in ("q", "k", "v", "do"))
    o, dq, dk, dv = orc.backward(q, k, v, do, int(w), int(s))
    for name, ours in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        ref = z["naive_" + name]
        assert _rel(ours.numpy(), ref) < 1e-5, name
        if "kernel_" + name in z:
            # the reference's fused Triton kernel (CPU interpreter); its backward divides
            # by l + 1e-6 (flash_attention_gpt_oss.py:293), hence the looser bound
            assert _rel(ours.numpy(), z["kernel_" + name]) < 1e-4, name


def test_forward_matches_backward_output():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 4, 70, 16, generator=g)
    k = torch.randn(1, 2, 70, 16, generator=g)
    v = torch.randn(1, 2, 70, 16, generator=g)
    o1, lse = orc.forward(q, k, v, 9, 3)
    o2 = orc.backward(q, k, v, torch.ones_like(q), 9, 3)[0]
    assert torch.allclose(o1, o2)
    assert torch.isfinite(lse).all()


def test_empty_rows_zero_vs_nan():
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 1, 8, 16, generator=g) for _ in range(3))
    o, lse = orc.forward(q, k, v, 0, 0)
    assert (o == 0).all() and torch.isneginf(lse).all()
    o_nan, _ = orc.forward(q, k, v, 0, 0, empty_rows="nan")
    assert torch.isnan(o_nan).all()


def test_useful_pairs_closed_form():
    for (l, w, s) in [(4096, 256, 4), (100, 1, 3), (64, 0, 5), (50, 1000, 70), (300, 17, 0)]:
        m = orc.visible_mask(l, w, s)
        assert int(m.sum()) == orc.visible_pairs_per_head(l, w, s)
    # published accounting: config 2 has 136,198,656 useful pairs
    assert 4 * 64 * orc.visible_pairs_per_head(4096, 128, 4) == 136198656


def test_sink_logits_oracle_reduces_to_token_sinks():
    # a sink logit of -inf is no sink at all; a finite one only rescales each row's weights
    g = torch.Generator().manual_seed(3)
    q, k, v, do = (torch.randn(s, generator=g, dtype=torch.float64)
                   for s in ((1, 4, 70, 16), (1, 2, 70, 16), (1, 2, 70, 16), (1, 4, 70, 16)))
    o0, dq0, dk0, dv0 = orc.backward(q, k, v, do, 20, 3)
    o1, dq1, dk1, dv1, ds1 = orc.backward_sink_logits(q, k, v, do, 20, 3, torch.full((4,), -float("inf")))
    for a, b in zip((o0, dq0, dk0, dv0), (o1, dq1, dk1, dv1)):
        assert torch.allclose(a, b, atol=1e-12)
    sinks = torch.tensor([-1.0, 0.0, 0.5, 2.0], dtype=torch.float64)
    o2, _, _, _, ds2 = orc.backward_sink_logits(q, k, v, do, 20, 3, sinks)
    _, lse0 = orc.forward(q, k, v, 20, 3)
    w = 1.0 / (1.0 + torch.exp(sinks.reshape(1, 4, 1) - lse0))   # share kept by the keys
    assert torch.allclose(o2, o0 * w[..., None], atol=1e-12)
    # d loss / d sink_h = -sum_i P_i,sink Delta_i with Delta_i = rowsum(dO * O)
    p_sink = torch.exp(sinks.reshape(1, 4, 1) - torch.logaddexp(lse0, sinks.reshape(1, 4, 1)))
    delta = (do * o2).sum(-1)
    assert torch.allclose(ds2, -(p_sink * delta).sum((0, 2)), atol=1e-10)
