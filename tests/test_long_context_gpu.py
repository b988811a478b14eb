"""Full-size long-context parity (B=1, Hq=64, Hkv=8, L=131072, D=64,
W=128, S=4, bf16) through size-independent checks:

* O and dQ of sampled 128-row blocks, exact against the windowed oracle;
* dK and dV of sampled non-sink 64-key blocks, exact: the windowed oracle over every query
  row (of every head of the GQA group) that can see the block;
* sum_j dV_j = sum over the group's query rows of dO_i (each softmax row sums to one) and
  sum_j dK_j = 0 (each row of dS sums to zero), which also covers the sink keys.
Tolerance: 1.5e-2 of the reference block's max-abs (bf16), as in the other parity tests.
"""
import pytest
import torch

from oracle import swa_oracle as orc
from tests._pkg import pkg, submodule

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

TOL = 1.5e-2


def _rel(a, r):
    a = a.double().cpu()
    r = r.double().cpu()
    return (a - r).abs().max().item() / max(r.abs().max().item(), 1e-30)


def test_cfg4_full_size_sampled_and_checksums():
    wl = submodule("workloads")
    w = wl.CONFIGS["cfg4_long_swa"]
    W, S, G = w.window_size, w.sink_size, w.group
    q, k, v, do = wl.make_inputs(w)
    dev = torch.device("cuda:0")
    qd, kd, vd = (t.to(dev).requires_grad_() for t in (q, k, v))
    o = pkg().flash_swda_with_sink(qd, kd, vd, W, S)
    o.backward(do.to(dev))
    torch.cuda.synchronize()
    L_ = submodule("_lib")
    assert L_.lib().swa_check_device(torch.cuda.current_stream(dev).cuda_stream) == L_.SWA_OK
    o, dq, dk, dv = (t.detach().float().cpu() for t in (o, qd.grad, kd.grad, vd.grad))
    for t in (o, dq, dk, dv):
        assert torch.isfinite(t).all()

    Lq = w.seq_len
    # 1) sampled query row blocks (first, near the sinks, middle, last)
    for h in (0, 37, 63):
        kvh = h // G
        for r0 in (0, 128, 65536, Lq - 128):
            ro, rdq, _, _, _ = orc.rows_backward(q[0, h], k[0, kvh], v[0, kvh], do[0, h],
                                                 r0, r0 + 128, W, S)
            assert _rel(o[0, h, r0:r0 + 128], ro) <= TOL, ("o", h, r0)
            assert _rel(dq[0, h, r0:r0 + 128], rdq) <= TOL, ("dq", h, r0)

    # 2) sampled non-sink key blocks: every row that sees them, for all G heads
    for kvh in (0, 5):
        for j0 in (64, 70000, Lq - 64):
            j1 = j0 + 64
            r1 = min(Lq, j1 + W - 1)
            rdk = torch.zeros(64, w.head_dim, dtype=torch.float64)
            rdv = torch.zeros_like(rdk)
            for g in range(G):
                h = kvh * G + g
                _, _, keys, p, ds = orc.rows_backward(q[0, h], k[0, kvh], v[0, kvh], do[0, h],
                                                      j0, r1, W, S)
                sel = (keys >= j0) & (keys < j1)
                qrows = q[0, h, j0:r1].double()
                dorows = do[0, h, j0:r1].double()
                rdk += (ds[:, sel].T @ qrows) / (w.head_dim ** 0.5)
                rdv += p[:, sel].T @ dorows
            assert _rel(dk[0, kvh, j0:j1], rdk) <= TOL, ("dk", kvh, j0)
            assert _rel(dv[0, kvh, j0:j1], rdv) <= TOL, ("dv", kvh, j0)

    # 3) identities over all keys (sinks included)
    for kvh in range(w.n_kv_heads):
        heads = slice(kvh * G, (kvh + 1) * G)
        sum_dv = dv[0, kvh].double().sum(0)
        ref_dv = do[0, heads].double().sum((0, 1))
        assert (sum_dv - ref_dv).abs().max().item() <= TOL * ref_dv.abs().max().item() + 1.0
        sum_dk = dk[0, kvh].double().sum(0)
        scale_dk = dk[0, kvh].double().abs().sum(0).max().item()
        assert sum_dk.abs().max().item() <= 1e-2 * scale_dk
