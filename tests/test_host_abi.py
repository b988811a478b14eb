"""CPU-only checks of the C-ABI library and the host-side mirror (no kernel is launched)."""
import ctypes
import os
import re
import subprocess

import pytest
import torch

from tests._pkg import pkg, submodule

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "swa_attn.h")).read()
    return sorted(set(re.findall(r"SWA_API\s+[\w\s\*]+?\b(swa_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = pkg().lib()
    declared = _declared_symbols()
    assert declared, "no declarations parsed"
    assert sorted(submodule("_lib").EXPORTED_SYMBOLS) == declared
    out = subprocess.run(["nm", "-D", "--defined-only", pkg().lib_path()], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (swa_\w+)", out))
    for name in declared:
        assert name in exported, name
        assert getattr(lib, name) is not None


def test_status_strings_and_version():
    lib = pkg().lib()
    assert lib.swa_version() >= 100
    L = submodule("_lib")
    for st, name in L.STATUS_NAMES.items():
        assert lib.swa_status_string(st).decode() == name


def _problem(**kw):
    L = submodule("_lib")
    base = dict(batch=1, n_q_heads=4, n_kv_heads=2, seq_len=128, head_dim=64, window_size=16,
                sink_size=4, dtype=L.SWA_BF16, softmax_scale=0.125)
    base.update(kw)
    return L.SwaProblem(**base)


def _fwd_args(prob, ptr=16 * 1024):
    L = submodule("_lib")
    t = L.SwaTensor(ptr, 1 << 20, 1 << 14, prob.head_dim)
    return L.SwaFwdArgs(prob, t, t, t, t, ptr)


@pytest.mark.parametrize("kw,status", [
    (dict(n_q_heads=6, n_kv_heads=4), 1),       # Hq % Hkv (flash_attention_gpt_oss.py:354)
    (dict(head_dim=160), 1),                    # D > 128 (:353)
    (dict(head_dim=48), 2),                     # kernel sizes are 16/32/64/128
    (dict(dtype=7), 2),
    (dict(sink_size=-1), 1),
    (dict(seq_len=-5), 1),
    (dict(softmax_scale=float("nan")), 1),
])
def test_fwd_rejects_bad_problems_before_launch(kw, status):
    lib = pkg().lib()
    args = _fwd_args(_problem(**kw))
    assert lib.swa_fwd(ctypes.byref(args), None) == status


def test_fwd_rejects_null_and_misaligned():
    L = submodule("_lib")
    lib = pkg().lib()
    assert lib.swa_fwd(None, None) == L.SWA_ERR_INVALID_ARG
    args = _fwd_args(_problem(), ptr=16 * 1024 + 2)    # not 16-byte aligned
    assert lib.swa_fwd(ctypes.byref(args), None) == L.SWA_ERR_UNSUPPORTED
    args = _fwd_args(_problem())
    args.q.stride_l = 66                              # row pitch not a multiple of 16 bytes
    assert lib.swa_fwd(ctypes.byref(args), None) == L.SWA_ERR_UNSUPPORTED
    args = _fwd_args(_problem())
    args.lse = None
    assert lib.swa_fwd(ctypes.byref(args), None) == L.SWA_ERR_INVALID_ARG


def test_bwd_workspace_contract():
    L = submodule("_lib")
    lib = pkg().lib()
    prob = _problem()
    need = lib.swa_bwd_workspace_size(ctypes.byref(prob))
    assert need >= 1 * 4 * 128 * 4 and need % 256 == 0
    t = L.SwaTensor(1 << 20, 1 << 20, 1 << 14, 64)
    args = L.SwaBwdArgs(prob, t, t, t, t, t, 1 << 20, t, t, t, None, 0)
    for fn in ("swa_bwd", "swa_bwd_preprocess", "swa_bwd_dq", "swa_bwd_dkdv"):
        assert getattr(lib, fn)(ctypes.byref(args), None) == L.SWA_ERR_WORKSPACE
    args.workspace, args.workspace_bytes = 1 << 21, need - 1
    assert lib.swa_bwd(ctypes.byref(args), None) == L.SWA_ERR_WORKSPACE
    args.workspace, args.workspace_bytes = (1 << 21) + 16, need
    assert lib.swa_bwd(ctypes.byref(args), None) == L.SWA_ERR_WORKSPACE


def test_python_validation_matches_reference_asserts():
    f = submodule("flash_attention_gpt_oss")
    q = torch.zeros(1, 4, 8, 16, dtype=torch.float16)
    k = torch.zeros(1, 2, 8, 16, dtype=torch.float16)
    with pytest.raises(AssertionError):
        f.flash_swda_with_sink(q, k, k, 4, 0, is_causal=False)
    with pytest.raises(AssertionError):
        f.flash_swda_with_sink(q, torch.zeros(1, 3, 8, 16, dtype=torch.float16),
                               torch.zeros(1, 3, 8, 16, dtype=torch.float16), 4)
    with pytest.raises(AssertionError):
        f.flash_swda_with_sink(torch.zeros(1, 4, 8, 160), torch.zeros(1, 2, 8, 160),
                               torch.zeros(1, 2, 8, 160), 4)
    with pytest.raises(AssertionError):
        f.flash_swda_with_sink(q, k, torch.zeros(1, 2, 9, 16, dtype=torch.float16), 4)
    with pytest.raises(TypeError):
        f.flash_swda_with_sink(q.float(), k.float(), k.float(), 4)
    with pytest.raises(ValueError):     # CPU tensors: no CPU path exists
        f.flash_swda_with_sink(q, k, k, 4)


def test_kernel_head_dim_padding_rule():
    f = submodule("flash_attention_gpt_oss")
    assert [f._kernel_head_dim(d) for d in (1, 16, 17, 48, 64, 80, 128)] == [16, 16, 32, 64, 64, 128, 128]


def test_no_alloc_rejects_problems_beyond_its_static_scratch():
    L = submodule("_lib")
    lib = pkg().lib()
    big = _problem(n_q_heads=64, n_kv_heads=8, seq_len=131072)   # 32 MiB of Delta rows
    assert lib.swa_bwd_workspace_size(ctypes.byref(big)) > L.SWA_NO_ALLOC_SCRATCH_BYTES
    t = L.SwaTensor(1 << 20, 1 << 20, 1 << 14, 64)
    args = L.SwaBwdArgs(big, t, t, t, t, t, 1 << 20, t, t, t, None, 0)
    assert lib.swa_bwd_no_alloc(ctypes.byref(args), None) == L.SWA_ERR_TOO_LARGE
    assert lib.swa_bwd_no_alloc(None, None) == L.SWA_ERR_INVALID_ARG


def test_dkdv_launch_count():
    L = submodule("_lib")
    lib = pkg().lib()
    count = lambda **kw: lib.swa_bwd_dkdv_launch_count(ctypes.byref(_problem(**kw)))
    # sinks seen from far past the window, D >= 64: dK/dV, far sink-pair kernel, reduction
    assert count(n_q_heads=64, n_kv_heads=8, seq_len=4096, head_dim=64, window_size=128, sink_size=4) == 3
    assert count(n_q_heads=64, n_kv_heads=8, seq_len=4096, head_dim=64, window_size=128, sink_size=0) == 1
    # D = 32 keeps the far pairs as dK/dV items: dK/dV and the reduction
    assert count(n_q_heads=8, n_kv_heads=8, seq_len=4096, head_dim=32, window_size=128, sink_size=4) == 2
    # the window reaches every sink: no far pairs
    assert count(n_q_heads=8, n_kv_heads=8, seq_len=256, head_dim=64, window_size=512, sink_size=4) == 2
    assert count(head_dim=24) == 0
    assert lib.swa_bwd_dkdv_launch_count(None) == 0


def test_varlen_sizes_and_argument_errors():
    # host-only entry points: lse blocks per sequence, the largest one-sequence workspace
    import numpy as np
    L = submodule("_lib")
    lib = pkg().lib()
    prob = _problem(batch=4, seq_len=0)
    cu = np.array([0, 100, 100, 229, 1029], dtype=np.int32)
    floats = lib.swa_varlen_lse_floats(ctypes.byref(prob), cu.ctypes.data)
    assert floats == 4 * (128 + 0 + 192 + 832)
    ws = lib.swa_varlen_bwd_workspace_size(ctypes.byref(prob), cu.ctypes.data)
    # every non-empty sequence owns a 256-byte aligned region (sequences may overlap in time)
    one = lambda n: (lib.swa_bwd_workspace_size(ctypes.byref(_problem(batch=1, seq_len=n)))
                     + 255) // 256 * 256
    assert ws == one(100) + one(129) + one(800)
    bad = np.array([0, 100, 50, 60, 70], dtype=np.int32)   # decreasing offsets
    assert lib.swa_varlen_lse_floats(ctypes.byref(prob), bad.ctypes.data) == 0
    args = L.SwaVarlenFwdArgs(prob, bad.ctypes.data)
    assert lib.swa_varlen_fwd(ctypes.byref(args), None) == L.SWA_ERR_INVALID_ARG
    args = L.SwaVarlenFwdArgs(prob, None)
    assert lib.swa_varlen_fwd(ctypes.byref(args), None) == L.SWA_ERR_INVALID_ARG
    # no tokens at all: nothing to do, no pointer needed
    empty = np.zeros(5, dtype=np.int32)
    args = L.SwaVarlenFwdArgs(prob, empty.ctypes.data)
    assert lib.swa_varlen_fwd(ctypes.byref(args), None) == L.SWA_OK
    bargs = L.SwaVarlenBwdArgs(prob, empty.ctypes.data)
    assert lib.swa_varlen_bwd(ctypes.byref(bargs), None) == L.SWA_OK


def test_varlen_cu_seqlens_validation():
    import numpy as np
    V = submodule("varlen")
    assert V._host_cu([0, 3, 3, 10], 10).dtype == np.int32
    assert list(V._host_cu(torch.tensor([0, 5]), 5)) == [0, 5]
    for cu, total in (([1, 5], 5), ([0, 5, 4], 5), ([0, 5], 6), ([[0, 5]], 5)):
        with pytest.raises(ValueError):
            V._host_cu(cu, total)
