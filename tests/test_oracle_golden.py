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
