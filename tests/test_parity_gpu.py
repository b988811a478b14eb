"""GPU parity: the CUDA kernels (through the drop-in autograd Function, i.e. the C-ABI
library) against the CPU oracle on the same seeded, dtype-rounded inputs.

Bar (tolerance of the task statement): max|x - ref| / max|ref| <= 2e-3 for fp16 and
<= 1.5e-2 for bf16, for O, dQ, dK and dV, the oracle computing in fp64.
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import swa_oracle as orc
from tests._pkg import pkg, submodule

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1.5e-2}
GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


def _rel(x, ref):
    x = x.detach().double().cpu()
    ref = ref.detach().double().cpu()
    den = ref.abs().max().item()
    if den == 0:
        return x.abs().max().item()
    return (x - ref).abs().max().item() / den


def run_ours(q, k, v, do, w, s, scale=None):
    dev = torch.device("cuda:0")
    q, k, v = (t.to(dev).detach().requires_grad_() for t in (q, k, v))
    o = pkg().flash_swda_with_sink(q, k, v, w, s, True, scale)
    o.backward(do.to(dev))
    assert_device_ok(dev)
    return o.detach(), q.grad, k.grad, v.grad


def assert_device_ok(dev):
    L = submodule("_lib")
    st = L.lib().swa_check_device(torch.cuda.current_stream(dev).cuda_stream)
    assert st == L.SWA_OK, f"device status {st}: {L.STATUS_NAMES.get(st)}"


def check(q, k, v, do, w, s, scale=None, tol=None, chunked=False):
    tol = tol or TOL[q.dtype]
    ours = run_ours(q, k, v, do, w, s, scale)
    if chunked:
        ref = orc.backward_chunked(q.float(), k.float(), v.float(), do.float(), w, s, scale,
                                   compute_dtype=torch.float64)
    else:
        ref = orc.backward(q.float(), k.float(), v.float(), do.float(), w, s, scale)
    errs = {n: _rel(a, b) for n, a, b in zip(("o", "dq", "dk", "dv"), ours, ref)}
    for n, a in zip(("o", "dq", "dk", "dv"), ours):
        assert torch.isfinite(a).all(), f"{n} has non-finite values"
    bad = {n: e for n, e in errs.items() if not e <= tol}
    assert not bad, f"tolerance {tol} exceeded: {errs}"
    return errs


def rand(shape_q, shape_k, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(shape_q, generator=g) * scale
    k = torch.randn(shape_k, generator=g) * scale
    v = torch.randn(shape_k, generator=g) * scale
    do = torch.randn(shape_q, generator=g) * scale
    return tuple(t.to(dtype) for t in (q, k, v, do))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(f)[7:-4] for f in GOLDEN])
def test_golden_cases(path, dtype):
    z = np.load(path)
    b, hq, hkv, l, d, w, s, _ = (int(x) for x in z["shape"])
    q, k, v, do = (torch.from_numpy(z[n]).to(dtype) for n in ("q", "k", "v", "do"))
    check(q, k, v, do, w, s)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("L", [1, 2, 63, 64, 65, 127, 128, 129, 255, 300])
def test_ragged_lengths(L, dtype):
    q, k, v, do = rand((2, 4, L, 64), (2, 2, L, 64), dtype, L)
    check(q, k, v, do, 37, 3)


@pytest.mark.parametrize("d", [16, 32, 64, 128])
@pytest.mark.parametrize("w,s", [(1, 0), (1, 5), (0, 3), (64, 4), (130, 70), (10**9, 0),
                                 (200, 200), (5, 1000)])
def test_window_sink_grid(d, w, s):
    q, k, v, do = rand((1, 4, 211, d), (1, 1, 211, d), torch.float16, d * 1000 + w % 997 + s)
    check(q, k, v, do, w, s)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("w,s", [(160, 4), (100, 1), (64, 16), (200, 17), (96, 32), (96, 33),
                                 (0, 20), (1, 8)])
def test_far_sink_pairs(d, w, s):
    # sink keys seen by rows far past their window: the far-chunk items of the dK/dV pass
    # and the sink-row reduction (W = 160 puts the near/far boundary inside a 128-row tile)
    dtype = torch.bfloat16 if (w + s) % 2 else torch.float16
    q, k, v, do = rand((2, 4, 1000, d), (2, 2, 1000, d), dtype, 7000 + d + w + s)
    check(q, k, v, do, w, s)


def test_no_visible_keys_gives_zero():
    q, k, v, do = rand((1, 2, 70, 32), (1, 2, 70, 32), torch.bfloat16, 9)
    o, dq, dk, dv = run_ours(q, k, v, do, 0, 0)
    for t in (o, dq, dk, dv):
        assert (t == 0).all()


@pytest.mark.parametrize("hq,hkv", [(16, 1), (8, 8), (12, 3)])
def test_gqa_groups(hq, hkv):
    q, k, v, do = rand((2, hq, 160, 64), (2, hkv, 160, 64), torch.bfloat16, hq * 10 + hkv)
    check(q, k, v, do, 48, 4)


@pytest.mark.parametrize("d", [8, 48, 80, 96, 112])
def test_head_dims_padded(d):
    q, k, v, do = rand((1, 4, 150, d), (1, 2, 150, d), torch.float16, d)
    check(q, k, v, do, 40, 4)


def test_custom_scale():
    q, k, v, do = rand((1, 4, 130, 64), (1, 2, 130, 64), torch.float16, 11)
    check(q, k, v, do, 50, 2, scale=0.3)


def test_non_contiguous_layouts():
    # [B, L, H, D] storage viewed as [B, H, L, D] (strided heads), as from a fused QKV projection
    g = torch.Generator().manual_seed(5)
    base_q = torch.randn(2, 190, 8, 64, generator=g).to(torch.bfloat16)
    base_k = torch.randn(2, 190, 2, 64, generator=g).to(torch.bfloat16)
    base_v = torch.randn(2, 190, 2, 64, generator=g).to(torch.bfloat16)
    do = torch.randn(2, 8, 190, 64, generator=g).to(torch.bfloat16)
    q, k, v = (t.transpose(1, 2) for t in (base_q, base_k, base_v))
    dev = torch.device("cuda:0")
    qd, kd, vd = (t.to(dev).transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    assert not qd.is_contiguous()
    qd, kd, vd = (t.detach().requires_grad_() for t in (qd, kd, vd))
    o = pkg().flash_swda_with_sink(qd, kd, vd, 33, 4)
    o.backward(do.to(dev))
    ref = orc.backward(q.float(), k.float(), v.float(), do.float(), 33, 4)
    for a, r in zip((o, qd.grad, kd.grad, vd.grad), ref):
        assert _rel(a, r) <= TOL[torch.bfloat16]


def test_backward_is_deterministic():
    q, k, v, do = rand((2, 8, 700, 64), (2, 2, 700, 64), torch.bfloat16, 21)
    r1 = run_ours(q, k, v, do, 100, 4)
    r2 = run_ours(q, k, v, do, 100, 4)
    for a, b in zip(r1, r2):
        assert torch.equal(a, b)


def test_forward_lse_matches_oracle():
    f = submodule("flash_attention_gpt_oss")
    q, k, v, _ = rand((1, 4, 300, 64), (1, 2, 300, 64), torch.float16, 3)
    dev = torch.device("cuda:0")
    o, lse2 = f.swa_forward(q.to(dev), k.to(dev), v.to(dev), 77, 5)
    ref_o, ref_lse = orc.forward(q.float(), k.float(), v.float(), 77, 5)
    assert _rel(o, ref_o) <= 2e-3
    lse_nat = lse2.double().cpu() / orc.LOG2E
    assert (lse_nat - ref_lse).abs().max().item() < 1e-3


@pytest.mark.parametrize("name", ["cfg1_ref_bench"])
def test_baseline_config_full(name):
    wl = submodule("workloads")
    w = wl.CONFIGS[name]
    q, k, v, do = wl.make_inputs(w)
    check(q, k, v, do, w.window_size, w.sink_size, chunked=True)


@pytest.mark.parametrize("name,kw", [
    ("cfg2_gptoss_swa", dict(batch=1, n_q_heads=16, n_kv_heads=2, seq_len=1024)),
    ("cfg3_full_causal", dict(batch=1, n_q_heads=8, n_kv_heads=1, seq_len=1024, window_size=1024)),
    ("cfg4_long_swa", dict(n_q_heads=8, n_kv_heads=1, seq_len=4096)),
    ("cfg5_ragged_s0", dict(batch=1, n_q_heads=8, n_kv_heads=1)),
    ("cfg5_ragged_s16", dict(batch=1, n_q_heads=8, n_kv_heads=1)),
])
def test_baseline_configs_reduced(name, kw):
    wl = submodule("workloads")
    w = wl.CONFIGS[name].replace(**kw)
    q, k, v, do = wl.make_inputs(w)
    check(q, k, v, do, w.window_size, w.sink_size, chunked=True)


def test_pinned_host_step_through_autograd():
    # a training step as a user runs it: pinned host inputs copied without blocking, forward
    # and backward through the autograd Function (the backward runs on autograd's own thread)
    q, k, v, do = (t.pin_memory() for t in rand((1, 8, 700, 64), (1, 2, 700, 64), torch.bfloat16, 77))
    dev = torch.device("cuda:0")
    qd, kd, vd, dod = (t.to(dev, non_blocking=True) for t in (q, k, v, do))
    for t in (qd, kd, vd):
        t.requires_grad_()
    o = pkg().flash_swda_with_sink(qd, kd, vd, 64, 4)
    o.backward(dod)
    assert_device_ok(dev)
    ref = orc.backward(q.float(), k.float(), v.float(), do.float(), 64, 4)
    for a, r in zip((o, qd.grad, kd.grad, vd.grad), ref):
        assert _rel(a, r) <= TOL[torch.bfloat16]


def test_backward_from_a_fresh_host_thread():
    # a thread that has made no CUDA runtime call of its own (as autograd's worker is when it
    # runs the first backward) has no current context; the library must bind one before it
    # encodes its TMA descriptors
    import threading
    f = submodule("flash_attention_gpt_oss")
    q, k, v, do = rand((1, 4, 300, 32), (1, 2, 300, 32), torch.float16, 78)
    dev = torch.device("cuda:0")
    qd, kd, vd, dod = (t.to(dev) for t in (q, k, v, do))
    o, lse = f.swa_forward(qd, kd, vd, 50, 4)
    out = {}

    def work():
        try:
            out["grads"] = f.swa_backward(qd, kd, vd, o, lse, dod, 50, 4)
            torch.cuda.synchronize(dev)
        except Exception as e:  # reported below, in the test's own thread
            out["error"] = e

    th = threading.Thread(target=work)
    th.start()
    th.join()
    assert "error" not in out, out.get("error")
    ref = orc.backward(q.float(), k.float(), v.float(), do.float(), 50, 4)
    for a, r in zip(out["grads"], ref[1:]):
        assert _rel(a, r) <= TOL[torch.float16]


def test_cuda_graph_replay_matches_eager():
    # one fwd + bwd captured once and replayed over refilled inputs
    plan = submodule("plan")
    dev = torch.device("cuda:0")
    q, k, v, do = (t.to(dev) for t in rand((2, 8, 640, 64), (2, 2, 640, 64), torch.bfloat16, 91))
    qb, kb, vb, dob = (t.clone() for t in (q, k, v, do))
    p = plan.SwaPlan(qb, kb, vb, 128, 4, dout=dob)
    g = p.capture()
    for seed in (92, 93):
        q2, k2, v2, do2 = (t.to(dev) for t in rand((2, 8, 640, 64), (2, 2, 640, 64), torch.bfloat16, seed))
        for dst, src in zip((qb, kb, vb, dob), (q2, k2, v2, do2)):
            dst.copy_(src)
        g.replay()
        torch.cuda.synchronize(dev)
        assert_device_ok(dev)
        ref = orc.backward(q2.float().cpu(), k2.float().cpu(), v2.float().cpu(), do2.float().cpu(), 128, 4)
        for a, r in zip((p.o, p.dq, p.dk, p.dv), ref):
            assert _rel(a, r) <= TOL[torch.bfloat16]
