"""swa_bwd_no_alloc: the backward for callers that cannot allocate device memory.

Some hosts cannot call cudaMalloc: an FFI/ctypes binding that only receives tensors and has no
device allocator of its own, or an engine whose fixed memory pool forbids side allocations.
For them the library offers swa_bwd_no_alloc, whose scratch lives in a static device array.
This test calls it through the C ABI and checks that its dq/dk/dv are bit-identical to the
regular swa_bwd (caller-provided workspace, pre-filled with 0xFF bytes so that a read of an
unwritten scratch byte would show) on the same inputs: both run the same deterministic
kernels.  It calls the entry point twice on the checked problem, with a call on a different
problem (other length, window, sink count, GQA group) in between, so that bytes a previous
call left in the shared array cannot pass for correct ones.  It runs last (file name) so a
``-x`` run has already run every other test when it starts; it also passes alone in a fresh
process, where its first call performs the per-device set-up.
"""
import ctypes

import pytest
import torch

from tests._pkg import submodule

pytestmark = pytest.mark.gpu


def _bwd_args(f, L, q, k, v, o, lse, do, dq, dk, dv, w, s, ws=None):
    prob = f._problem(q, k, w, s, 1.0 / q.shape[-1] ** 0.5, q.shape[-1])
    ws_ptr, ws_bytes = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    return L.SwaBwdArgs(prob, f._tensor(q), f._tensor(k), f._tensor(v), f._tensor(o),
                        f._tensor(do), lse.data_ptr(), f._tensor(dq), f._tensor(dk),
                        f._tensor(dv), ws_ptr, ws_bytes)


def _problem_inputs(f, dev, seed, b, hq, hkv, l, d, w, s):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, l, d, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(b, hkv, l, d, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(b, hkv, l, d, generator=g).to(torch.bfloat16).to(dev)
    do = torch.randn(b, hq, l, d, generator=g).to(torch.bfloat16).to(dev)
    o, lse = f.swa_forward(q, k, v, w, s)
    return q, k, v, do, o, lse


def _no_alloc(f, L, lib, stream, q, k, v, do, o, lse, w, s):
    out = [torch.full_like(t, float("nan")) for t in (q, k, v)]
    b = _bwd_args(f, L, q, k, v, o, lse, do, *out, w, s)     # no workspace given
    st = lib.swa_bwd_no_alloc(ctypes.byref(b), stream)
    assert st == L.SWA_OK, (lib.swa_status_string(st), lib.swa_last_cuda_error())
    torch.cuda.synchronize()
    return out


def test_no_alloc_is_bit_identical_to_workspace_backward_twice():
    f = submodule("flash_attention_gpt_oss")
    L = submodule("_lib")
    lib = L.lib()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    w, s = 96, 4
    q, k, v, do, o, lse = _problem_inputs(f, dev, 123, 2, 8, 2, 777, 64, w, s)

    # the existing entry point, with a caller-provided workspace full of 0xFF bytes
    ref = [torch.empty_like(t) for t in (q, k, v)]
    prob = f._problem(q, k, w, s, 0.125, 64)
    ws = torch.full((lib.swa_bwd_workspace_size(ctypes.byref(prob)),), 0xFF, dtype=torch.uint8,
                    device=dev)
    a = _bwd_args(f, L, q, k, v, o, lse, do, *ref, w, s, ws)
    assert lib.swa_bwd(ctypes.byref(a), stream) == L.SWA_OK
    torch.cuda.synchronize()
    for x in ref:
        assert torch.isfinite(x).all()

    # another problem in between: different length, window, sink count and GQA group
    other = _problem_inputs(f, dev, 7, 1, 16, 2, 1300, 64, 300, 16)
    for call in range(2):
        out = _no_alloc(f, L, lib, stream, q, k, v, do, o, lse, w, s)
        for name, x, r in zip(("dq", "dk", "dv"), out, ref):
            assert torch.equal(x, r), (call, name, (x.float() - r.float()).abs().max().item())
        if call == 0:
            oq, ok_, ov, odo, oo, olse = other
            _no_alloc(f, L, lib, stream, oq, ok_, ov, odo, oo, olse, 300, 16)


def test_no_alloc_rejects_problems_beyond_its_scratch():
    f = submodule("flash_attention_gpt_oss")
    L = submodule("_lib")
    lib = L.lib()
    dev = torch.device("cuda:0")
    # Delta alone needs B * Hq * round_up(L, 64) * 4 bytes: 64 * 64 * 4096 * 4 = 64 MiB > 16 MiB
    q = torch.empty(64, 64, 4096, 64, dtype=torch.bfloat16, device="meta")
    k = torch.empty(64, 8, 4096, 64, dtype=torch.bfloat16, device="meta")
    prob = f._problem(q, k, 128, 4, 0.125, 64)
    assert lib.swa_bwd_workspace_size(ctypes.byref(prob)) > L.SWA_NO_ALLOC_SCRATCH_BYTES
    t = L.SwaTensor(1 << 20, 1 << 20, 1 << 14, 64)
    args = L.SwaBwdArgs(prob, t, t, t, t, t, 1 << 20, t, t, t, None, 0)
    assert lib.swa_bwd_no_alloc(ctypes.byref(args), None) == L.SWA_ERR_TOO_LARGE
    del dev
