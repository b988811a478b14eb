"""GPU parity of the learned per-head sink-logit mode (GPT-OSS's form of attention sinks, an
additional mode beside the reference's sink tokens) against the fp64 oracle
(``oracle.swa_oracle.backward_sink_logits``), through the autograd API and the C ABI.

O, dQ, dK, dV: the same bar as the token-sink path (max|x - ref| / max|ref| <= 2e-3 fp16,
<= 1.5e-2 bf16).  d sink_h is a signed sum of B*L terms P_sink * Delta that cancel, so its
error is measured against the sum of the terms' magnitudes, with the same tolerances.
"""
import math

import pytest
import torch

from oracle import swa_oracle as orc
from tests._pkg import pkg
from tests.test_parity_gpu import TOL, _rel, assert_device_ok, rand

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def run_ours(q, k, v, do, sinks, w, s, scale=None):
    q, k, v = (t.to(DEV).detach().requires_grad_() for t in (q, k, v))
    sl = sinks.to(DEV).detach().requires_grad_()
    o = pkg().flash_swda_with_sink(q, k, v, w, s, True, scale, sinks=sl)
    o.backward(do.to(DEV))
    assert_device_ok(DEV)
    return o.detach(), q.grad, k.grad, v.grad, sl.grad


def sink_term_scale(q, k, v, do, sinks, w, s, scale):
    """Per head: sum over (b, i) of |P_sink * Delta| (the magnitude dsink is a signed sum of)."""
    o, lse = orc.forward_sink_logits(q, k, v, w, s, sinks, scale)
    delta = (do.double() * o).sum(-1)
    p_sink = torch.exp(sinks.double().reshape(1, -1, 1) - lse)
    return (p_sink * delta).abs().sum((0, 2))


def check(q, k, v, do, sinks, w, s, scale=None):
    tol = TOL[q.dtype]
    ours = run_ours(q, k, v, do, sinks, w, s, scale)
    ref = orc.backward_sink_logits(q.float(), k.float(), v.float(), do.float(), w, s,
                                   sinks.double(), scale)
    for n, a in zip(("o", "dq", "dk", "dv", "dsinks"), ours):
        assert torch.isfinite(a).all(), f"{n} has non-finite values"
    errs = {n: _rel(a, b) for n, a, b in zip(("o", "dq", "dk", "dv"), ours[:4], ref[:4])}
    den = sink_term_scale(q.float(), k.float(), v.float(), do.float(), sinks, w, s, scale)
    ds_err = ((ours[4].double().cpu() - ref[4]).abs() / den.clamp_min(1e-30)).max().item()
    errs["dsinks"] = ds_err
    bad = {n: e for n, e in errs.items() if not e <= tol}
    assert not bad, f"tolerance {tol} exceeded: {errs}"
    return errs


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("l,d,hq,hkv,w,s", [
    (300, 64, 8, 2, 64, 4),      # ragged L, GQA 4, window + token sinks + sink logits
    (256, 128, 4, 4, 1000, 0),   # full causal, no token sinks
    (129, 32, 8, 1, 1, 0),       # window 1: the sink column competes with one key
    (200, 16, 4, 2, 40, 16),     # D = 16, many token sinks
])
def test_sink_logits_parity(dtype, l, d, hq, hkv, w, s):
    q, k, v, do = rand((2, hq, l, d), (2, hkv, l, d), dtype, seed=l + d)
    sinks = torch.linspace(-3.0, 4.0, hq)
    check(q, k, v, do, sinks, w, s)


def test_sink_logits_gptoss_layer_reduced():
    # the GPT-OSS layer's head layout (Hq 64, Hkv 8, D 64, W 128, S 4), shorter sequence
    q, k, v, do = rand((1, 64, 512, 64), (1, 8, 512, 64), torch.bfloat16, seed=1, scale=0.5)
    g = torch.Generator().manual_seed(5)
    sinks = torch.randn(64, generator=g) * 2.0
    check(q, k, v, do, sinks, 128, 4)


def test_minus_inf_sink_is_the_token_sink_path():
    # a sink logit of -inf is no sink: same bits as flash_swda_with_sink without sinks
    q, k, v, do = rand((1, 4, 190, 64), (1, 2, 190, 64), torch.bfloat16, seed=9)
    a = run_ours(q, k, v, do, torch.full((4,), -math.inf), 50, 3)
    qd, kd, vd = (t.to(DEV).detach().requires_grad_() for t in (q, k, v))
    o = pkg().flash_swda_with_sink(qd, kd, vd, 50, 3)
    o.backward(do.to(DEV))
    for x, y in zip(a[:4], (o.detach(), qd.grad, kd.grad, vd.grad)):
        assert torch.equal(x, y)
    assert torch.equal(a[4].cpu(), torch.zeros(4))


def test_rows_without_keys_and_large_sinks():
    # W = 0, S = 0: no key is visible, the sink takes every row (O = 0, lse = sink, no NaN);
    # a very large logit drives O to 0 without overflow
    f = pkg()
    q, k, v, do = rand((1, 2, 70, 32), (1, 2, 70, 32), torch.float16, seed=3)
    sl = torch.tensor([0.5, -2.0], device=DEV)
    o, lse = f.swa_forward(q.to(DEV), k.to(DEV), v.to(DEV), 0, 0, sink_logits=sl)
    assert torch.equal(o, torch.zeros_like(o))
    assert torch.allclose(lse.cpu(), (sl.cpu() / math.log(2)).reshape(1, 2, 1).expand(1, 2, 70))
    ours = run_ours(q, k, v, do, torch.tensor([0.5, -2.0]), 0, 0)
    for x in ours[1:]:
        assert torch.equal(x.cpu(), torch.zeros_like(x.cpu()))
    # head 0: P_sink ~ 1 and O ~ e^-60 underflows in fp16, so Delta (formed from the stored
    # fp16 O, like the token-sink path's) is 0 and so is d sink_0; head 1 is an ordinary head
    big = torch.tensor([60.0, 0.0])
    ours = run_ours(q, k, v, do, big, 20, 2)
    ref = orc.backward_sink_logits(q.float(), k.float(), v.float(), do.float(), 20, 2,
                                   big.double())
    for n, a, b in zip(("o", "dq", "dk", "dv"), ours[:4], ref[:4]):
        assert torch.isfinite(a).all(), n
        assert _rel(a, b) <= TOL[torch.float16], n
    assert ours[4][0].item() == 0.0 and abs(ref[4][0].item()) < 1e-20
    den = sink_term_scale(q.float(), k.float(), v.float(), do.float(), big, 20, 2, None)
    assert abs(ours[4][1].item() - ref[4][1].item()) <= TOL[torch.float16] * den[1].item()


def test_sink_logits_deterministic():
    q, k, v, do = rand((2, 8, 333, 64), (2, 2, 333, 64), torch.bfloat16, seed=11)
    sinks = torch.linspace(-1.0, 1.0, 8)
    a = run_ours(q, k, v, do, sinks, 96, 4)
    b = run_ours(q, k, v, do, sinks, 96, 4)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
