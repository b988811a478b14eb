"""GPU checks of the packed variable-length mode (an additional mode; the reference takes dense
[B, H, L, D] only).  Each sequence of a packed batch must give exactly what the dense entry
point gives for that sequence alone (same kernels, bit-identical), and match the fp64 oracle
per sequence at the usual bar (2e-3 fp16, 1.5e-2 bf16, relative to max|ref|).
"""
import pytest
import torch

from oracle import swa_oracle as orc
from tests._pkg import pkg, submodule
from tests.test_parity_gpu import TOL, _rel, assert_device_ok

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def packed_inputs(lens, hq, hkv, d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    t = sum(lens)
    q = torch.randn(t, hq, d, generator=g).to(dtype)
    k = torch.randn(t, hkv, d, generator=g).to(dtype)
    v = torch.randn(t, hkv, d, generator=g).to(dtype)
    do = torch.randn(t, hq, d, generator=g).to(dtype)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    return q, k, v, do, cu


def run_varlen(q, k, v, do, cu, w, s, sinks=None):
    V = submodule("varlen")
    q, k, v = (x.to(DEV).detach().requires_grad_() for x in (q, k, v))
    sl = None if sinks is None else sinks.to(DEV).detach().requires_grad_()
    o = V.flash_swda_with_sink_varlen(q, k, v, cu, w, s, sinks=sl)
    o.backward(do.to(DEV))
    assert_device_ok(DEV)
    out = [o.detach(), q.grad, k.grad, v.grad]
    return out + ([sl.grad] if sl is not None else [])


def run_dense_seq(q, k, v, do, w, s, sinks=None):
    """One sequence ([L, H, D] slices) through the dense entry point as a [1, H, L, D] batch."""
    to4 = lambda x: x.transpose(0, 1).unsqueeze(0).contiguous().to(DEV)
    q4, k4, v4 = (to4(x).requires_grad_() for x in (q, k, v))
    sl = None if sinks is None else sinks.to(DEV).detach().requires_grad_()
    o = pkg().flash_swda_with_sink(q4, k4, v4, w, s, sinks=sl)
    o.backward(to4(do))
    back = lambda x: x[0].transpose(0, 1)
    out = [back(o.detach()), back(q4.grad), back(k4.grad), back(v4.grad)]
    return out + ([sl.grad] if sl is not None else [])


@pytest.mark.parametrize("lens,d,w,s", [
    ([300, 1, 129, 64, 777], 64, 96, 4),
    ([128, 0, 513, 255], 128, 1000, 16),   # an empty sequence; full causal
    ([70, 33, 200], 48, 40, 2),           # head dim padded to 64
])
def test_varlen_equals_dense_per_sequence(lens, d, w, s):
    q, k, v, do, cu = packed_inputs(lens, 8, 2, d, torch.bfloat16, seed=sum(lens))
    ours = run_varlen(q, k, v, do, cu, w, s)
    for b, n in enumerate(lens):
        if n == 0:
            continue
        sl = slice(cu[b], cu[b + 1])
        ref = run_dense_seq(q[sl], k[sl], v[sl], do[sl], w, s)
        for name, x, y in zip(("o", "dq", "dk", "dv"), ours, ref):
            assert torch.equal(x[sl], y), (b, name)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_varlen_oracle_parity(dtype):
    lens = [257, 64, 1000, 3]
    q, k, v, do, cu = packed_inputs(lens, 8, 4, 64, dtype, seed=7)
    ours = run_varlen(q, k, v, do, cu, 128, 4)
    for b in range(len(lens)):
        sl = slice(cu[b], cu[b + 1])
        to4 = lambda x: x[sl].transpose(0, 1).unsqueeze(0).float()
        ref = orc.backward(to4(q), to4(k), to4(v), to4(do), 128, 4)
        for name, x, r in zip(("o", "dq", "dk", "dv"), ours, ref):
            e = _rel(x[sl].transpose(0, 1).unsqueeze(0), r)
            assert e <= TOL[dtype], (b, name, e)


def test_varlen_with_sink_logits():
    lens = [190, 0, 64, 401]
    q, k, v, do, cu = packed_inputs(lens, 4, 2, 64, torch.bfloat16, seed=5)
    sinks = torch.tensor([-1.0, 0.0, 1.5, 3.0])
    ours = run_varlen(q, k, v, do, cu, 50, 3, sinks)
    total = torch.zeros(4)
    for b, n in enumerate(lens):
        if n == 0:
            continue
        sl = slice(cu[b], cu[b + 1])
        ref = run_dense_seq(q[sl], k[sl], v[sl], do[sl], 50, 3, sinks)
        for name, x, y in zip(("o", "dq", "dk", "dv"), ours[:4], ref[:4]):
            assert torch.equal(x[sl], y), (b, name)
        total = total + ref[4].float().cpu()
    assert torch.allclose(ours[4].float().cpu(), total, rtol=1e-5, atol=1e-6)


def test_varlen_empty_batch():
    V = submodule("varlen")
    q = torch.zeros(0, 4, 64, device=DEV, dtype=torch.float16, requires_grad=True)
    k = torch.zeros(0, 2, 64, device=DEV, dtype=torch.float16, requires_grad=True)
    v = torch.zeros(0, 2, 64, device=DEV, dtype=torch.float16, requires_grad=True)
    o = V.flash_swda_with_sink_varlen(q, k, v, [0, 0, 0], 16, 2)
    assert o.shape == (0, 4, 64)
    o.sum().backward()
    assert q.grad.shape == q.shape
