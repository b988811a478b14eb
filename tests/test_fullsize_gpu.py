"""Parity at the benchmark's full sizes (3 and 5, not reduced).

The whole problem runs on the GPU through the drop-in autograd Function; sampled
(batch, KV head) units -- the first, a middle one and the last -- are then checked against the
fp64 CPU oracle over the unit's whole GQA group and all of its rows and keys (sink keys
included: every unit holds its own sink keys).  The oracle runs one query head at a time
(``orc.backward`` on a [1, 1, L, D] slice against the unit's K/V), summing dK/dV over the
group, which bounds its memory at L x L fp64 per matrix.

Config 2 is the shape ``bench.py`` quotes its headline on (B=4, Hq=64, Hkv=8, L=4096, D=64,
W=128, S=4, bf16), so its persistent kernels wrap their item queues over the 148 SMs the same
number of times as in the benchmark.

Also here: the standalone Delta path (swa_bwd_preprocess, then swa_bwd_dkdv) against the
oracle's Delta and dK/dV.

Bar: max|x - ref| / max|ref| <= 2e-3 (fp16), <= 1.5e-2 (bf16), per tensor and unit.
"""
import ctypes

import pytest
import torch

from oracle import swa_oracle as orc
from tests._pkg import pkg, submodule

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

TOL = {torch.float16: 2e-3, torch.bfloat16: 1.5e-2}


def _rel(x, ref):
    x = x.double()
    ref = ref.double()
    den = ref.abs().max().item()
    return (x - ref).abs().max().item() / den if den > 0 else x.abs().max().item()


def _unit_reference(q, k, v, do, b, kvh, G, W, S):
    """fp64 (o, dq, dk, dv) of unit (b, kvh): o/dq [G, L, D], dk/dv [L, D]."""
    ks, vs = k[b:b + 1, kvh:kvh + 1], v[b:b + 1, kvh:kvh + 1]
    os_, dqs = [], []
    dk = dv = None
    for g in range(G):
        h = kvh * G + g
        o, dq, dk_h, dv_h = orc.backward(q[b:b + 1, h:h + 1], ks, vs, do[b:b + 1, h:h + 1], W, S)
        os_.append(o[0, 0])
        dqs.append(dq[0, 0])
        dk = dk_h[0, 0] if dk is None else dk + dk_h[0, 0]
        dv = dv_h[0, 0] if dv is None else dv + dv_h[0, 0]
    return torch.stack(os_), torch.stack(dqs), dk, dv


def _run_full(w):
    wl = submodule("workloads")
    q, k, v, do = wl.make_inputs(w)
    dev = torch.device("cuda:0")
    qd, kd, vd = (t.to(dev).requires_grad_() for t in (q, k, v))
    o = pkg().flash_swda_with_sink(qd, kd, vd, w.window_size, w.sink_size)
    o.backward(do.to(dev))
    torch.cuda.synchronize()
    L_ = submodule("_lib")
    assert L_.lib().swa_check_device(torch.cuda.current_stream(dev).cuda_stream) == L_.SWA_OK
    outs = tuple(t.detach().cpu() for t in (o, qd.grad, kd.grad, vd.grad))
    for n, t in zip(("o", "dq", "dk", "dv"), outs):
        assert torch.isfinite(t).all(), n
    return (q, k, v, do), outs


def _check_units(w, units):
    (q, k, v, do), (o, dq, dk, dv) = _run_full(w)
    G = w.group
    tol = TOL[w.dtype]
    errs = {}
    for b, kvh in units:
        ro, rdq, rdk, rdv = _unit_reference(q.float(), k.float(), v.float(), do.float(), b, kvh, G,
                                            w.window_size, w.sink_size)
        hs = slice(kvh * G, (kvh + 1) * G)
        e = {"o": _rel(o[b, hs], ro), "dq": _rel(dq[b, hs], rdq), "dk": _rel(dk[b, kvh], rdk),
             "dv": _rel(dv[b, kvh], rdv)}
        errs[(b, kvh)] = e
        bad = {n: x for n, x in e.items() if not x <= tol}
        assert not bad, f"unit {(b, kvh)}: tolerance {tol} exceeded: {e}"
    return errs


def test_cfg2_full_size_headline_shape():
    w = submodule("workloads").CONFIGS["cfg2_gptoss_swa"]
    _check_units(w, [(0, 0), (1, 5), (w.batch - 1, w.n_kv_heads - 1)])


def test_cfg3_full_size_full_causal():
    w = submodule("workloads").CONFIGS["cfg3_full_causal"]
    _check_units(w, [(0, 0), (w.batch - 1, w.n_kv_heads - 1)])


@pytest.mark.parametrize("name", ["cfg5_ragged_s0", "cfg5_ragged_s16"])
def test_cfg5_full_size_ragged(name):
    w = submodule("workloads").CONFIGS[name]
    _check_units(w, [(0, 0), (3, 2), (w.batch - 1, w.n_kv_heads - 1)])


def test_standalone_preprocess_then_dkdv():
    """swa_bwd_preprocess writes Delta to the workspace; swa_bwd_dkdv then reads it (the dQ
    pass, which also writes Delta, is not run)."""
    f = submodule("flash_attention_gpt_oss")
    L = submodule("_lib")
    lib = L.lib()
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(31)
    B, Hq, Hkv, Lq, D, W, S = 2, 8, 2, 1000, 64, 128, 4
    q, do = (torch.randn(B, Hq, Lq, D, generator=g).to(torch.bfloat16) for _ in range(2))
    k, v = (torch.randn(B, Hkv, Lq, D, generator=g).to(torch.bfloat16) for _ in range(2))
    qd, kd, vd, dod = (t.to(dev) for t in (q, k, v, do))
    o, lse = f.swa_forward(qd, kd, vd, W, S)
    lse = f._padded_lse(lse, Lq)
    dq, dk, dv = torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)
    prob = f._problem(qd, kd, W, S, D ** -0.5, D)
    nws = lib.swa_bwd_workspace_size(ctypes.byref(prob))
    ws = torch.full((nws,), 0xFF, dtype=torch.uint8, device=dev)
    args = L.SwaBwdArgs(prob, f._tensor(qd), f._tensor(kd), f._tensor(vd), f._tensor(o),
                        f._tensor(dod), lse.data_ptr(), f._tensor(dq), f._tensor(dk),
                        f._tensor(dv), ws.data_ptr(), nws)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.swa_bwd_preprocess(ctypes.byref(args), stream) == L.SWA_OK
    assert lib.swa_bwd_dkdv(ctypes.byref(args), stream) == L.SWA_OK
    torch.cuda.synchronize()
    assert lib.swa_check_device(stream) == L.SWA_OK
    ld = f.lse_row_stride(Lq)
    delta = ws[:B * Hq * ld * 4].view(torch.float32).view(B, Hq, ld).cpu()
    # Delta of the kernel's own O (bf16) and dO, in fp64
    ref_delta = (o.double() * dod.double()).sum(-1).cpu()
    assert _rel(delta[..., :Lq], ref_delta) <= 1e-5
    assert (delta[..., Lq:] == 0).all()
    _, _, rdk, rdv = orc.backward(q.float(), k.float(), v.float(), do.float(), W, S)
    assert _rel(dk.cpu(), rdk) <= TOL[torch.bfloat16]
    assert _rel(dv.cpu(), rdv) <= TOL[torch.bfloat16]
