"""swa_bwd_no_alloc: the backward for callers that cannot allocate device memory.

Some hosts cannot call cudaMalloc: an FFI/ctypes binding that only receives tensors and has no
device allocator of its own, or an engine whose fixed memory pool forbids side allocations.
For them the library offers swa_bwd_no_alloc, whose scratch lives in a static device array.
This test calls it through the C ABI, twice in a row, and checks its dq/dk/dv against the
regular swa_bwd (caller-provided workspace) on the same inputs.  It runs last (file name) so a
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


def test_no_alloc_matches_workspace_backward_twice():
    f = submodule("flash_attention_gpt_oss")
    L = submodule("_lib")
    lib = L.lib()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = torch.Generator().manual_seed(123)
    w, s = 96, 4
    q = torch.randn(2, 8, 777, 64, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(2, 2, 777, 64, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(2, 2, 777, 64, generator=g).to(torch.bfloat16).to(dev)
    do = torch.randn(2, 8, 777, 64, generator=g).to(torch.bfloat16).to(dev)
    o, lse = f.swa_forward(q, k, v, w, s)
    stream = torch.cuda.current_stream(dev).cuda_stream

    # the existing entry point, with a caller-provided workspace
    ref = [torch.empty_like(t) for t in (q, k, v)]
    prob = f._problem(q, k, w, s, 0.125, 64)
    ws = torch.empty(lib.swa_bwd_workspace_size(ctypes.byref(prob)), dtype=torch.uint8, device=dev)
    a = _bwd_args(f, L, q, k, v, o, lse, do, *ref, w, s, ws)
    assert lib.swa_bwd(ctypes.byref(a), stream) == L.SWA_OK
    torch.cuda.synchronize()

    for call in range(2):
        out = [torch.full_like(t, float("nan")) for t in (q, k, v)]
        b = _bwd_args(f, L, q, k, v, o, lse, do, *out, w, s)     # no workspace given
        st = lib.swa_bwd_no_alloc(ctypes.byref(b), stream)
        assert st == L.SWA_OK, (call, lib.swa_status_string(st), lib.swa_last_cuda_error())
        torch.cuda.synchronize()
        for name, x, r in zip(("dq", "dk", "dv"), out, ref):
            assert torch.isfinite(x).all(), (call, name)
            err = (x.float() - r.float()).abs().max().item() / r.float().abs().max().item()
            assert err <= 1.5e-2, (call, name, err)
