"""ctypes binding of ``lib/libswa_attn.so`` (declared in ``include/swa_attn.h``).

The library is the only compute path: when it is missing, :func:`lib` raises, so no call can
silently fall back to CPU or eager PyTorch arithmetic.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libswa_attn.so")

SWA_OK = 0
SWA_ERR_INVALID_ARG = 1
SWA_ERR_UNSUPPORTED = 2
SWA_ERR_LAUNCH = 3
SWA_ERR_DEVICE_TIMEOUT = 4
SWA_ERR_WORKSPACE = 5
SWA_ERR_TOO_LARGE = 6
SWA_NO_ALLOC_SCRATCH_BYTES = 16 << 20

SWA_F16 = 0
SWA_BF16 = 1

# Every extern "C" symbol include/swa_attn.h declares.
EXPORTED_SYMBOLS = (
    "swa_fwd", "swa_bwd", "swa_bwd_preprocess", "swa_bwd_dq", "swa_bwd_dkdv",
    "swa_bwd_workspace_size", "swa_bwd_dkdv_launch_count", "swa_bwd_launch_count", "swa_bwd_no_alloc", "swa_check_device",
    "swa_status_string", "swa_last_cuda_error", "swa_version", "swa_lse_row_stride",
    "swa_selftest_wait_timeout", "swa_fwd_sink_logits", "swa_bwd_sink_logits",
    "swa_varlen_lse_floats", "swa_varlen_bwd_workspace_size", "swa_varlen_fwd", "swa_varlen_bwd",
    "swa_device_status_async",
)


class SwaProblem(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("n_q_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
        ("seq_len", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("window_size", ctypes.c_int32),
        ("sink_size", ctypes.c_int32), ("dtype", ctypes.c_int32), ("softmax_scale", ctypes.c_float),
    ]


class SwaTensor(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("stride_b", ctypes.c_int64),
                ("stride_h", ctypes.c_int64), ("stride_l", ctypes.c_int64)]


class SwaFwdArgs(ctypes.Structure):
    _fields_ = [("p", SwaProblem), ("q", SwaTensor), ("k", SwaTensor), ("v", SwaTensor),
                ("o", SwaTensor), ("lse", ctypes.c_void_p)]


class SwaBwdArgs(ctypes.Structure):
    _fields_ = [("p", SwaProblem), ("q", SwaTensor), ("k", SwaTensor), ("v", SwaTensor),
                ("o", SwaTensor), ("dout", SwaTensor), ("lse", ctypes.c_void_p),
                ("dq", SwaTensor), ("dk", SwaTensor), ("dv", SwaTensor),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


class SwaPackedTensor(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("stride_t", ctypes.c_int64), ("stride_h", ctypes.c_int64)]


class SwaVarlenFwdArgs(ctypes.Structure):
    _fields_ = [("p", SwaProblem), ("cu_seqlens", ctypes.c_void_p), ("q", SwaPackedTensor),
                ("k", SwaPackedTensor), ("v", SwaPackedTensor), ("o", SwaPackedTensor),
                ("lse", ctypes.c_void_p), ("sink_logits", ctypes.c_void_p)]


class SwaVarlenBwdArgs(ctypes.Structure):
    _fields_ = [("p", SwaProblem), ("cu_seqlens", ctypes.c_void_p), ("q", SwaPackedTensor),
                ("k", SwaPackedTensor), ("v", SwaPackedTensor), ("o", SwaPackedTensor),
                ("dout", SwaPackedTensor), ("lse", ctypes.c_void_p), ("dq", SwaPackedTensor),
                ("dk", SwaPackedTensor), ("dv", SwaPackedTensor), ("sink_logits", ctypes.c_void_p),
                ("dsink_logits", ctypes.c_void_p), ("workspace", ctypes.c_void_p),
                ("workspace_bytes", ctypes.c_size_t)]


class SwaError(RuntimeError):
    """A non-zero SwaStatus from the library."""

    def __init__(self, status: int, where: str, detail: str = ""):
        self.status = status
        msg = f"{where}: {STATUS_NAMES.get(status, 'unknown status')} (status {status})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


class SwaDeviceTimeout(SwaError):
    """An on-device bounded wait gave up (SWA_ERR_DEVICE_TIMEOUT)."""


STATUS_NAMES = {
    SWA_OK: "ok", SWA_ERR_INVALID_ARG: "invalid argument",
    SWA_ERR_UNSUPPORTED: "unsupported shape, dtype or layout", SWA_ERR_LAUNCH: "CUDA launch failed",
    SWA_ERR_DEVICE_TIMEOUT: "on-device wait timed out",
    SWA_ERR_WORKSPACE: "workspace missing, misaligned or too small",
    SWA_ERR_TOO_LARGE: "problem needs more scratch than the static no-alloc workspace",
}

_lib = None
_lock = threading.Lock()


def _declare(l):
    P = ctypes.POINTER
    l.swa_fwd.argtypes = [P(SwaFwdArgs), ctypes.c_void_p]
    for name in ("swa_bwd", "swa_bwd_preprocess", "swa_bwd_dq", "swa_bwd_dkdv", "swa_bwd_no_alloc"):
        getattr(l, name).argtypes = [P(SwaBwdArgs), ctypes.c_void_p]
        getattr(l, name).restype = ctypes.c_int
    l.swa_fwd.restype = ctypes.c_int
    l.swa_fwd_sink_logits.argtypes = [P(SwaFwdArgs), ctypes.c_void_p, ctypes.c_void_p]
    l.swa_fwd_sink_logits.restype = ctypes.c_int
    l.swa_bwd_sink_logits.argtypes = [P(SwaBwdArgs), ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_void_p]
    l.swa_bwd_sink_logits.restype = ctypes.c_int
    for name in ("swa_varlen_lse_floats", "swa_varlen_bwd_workspace_size"):
        getattr(l, name).argtypes = [P(SwaProblem), ctypes.c_void_p]
        getattr(l, name).restype = ctypes.c_size_t
    l.swa_varlen_fwd.argtypes = [P(SwaVarlenFwdArgs), ctypes.c_void_p]
    l.swa_varlen_fwd.restype = ctypes.c_int
    l.swa_varlen_bwd.argtypes = [P(SwaVarlenBwdArgs), ctypes.c_void_p]
    l.swa_varlen_bwd.restype = ctypes.c_int
    l.swa_bwd_workspace_size.argtypes = [P(SwaProblem)]
    l.swa_bwd_workspace_size.restype = ctypes.c_size_t
    for name in ("swa_bwd_dkdv_launch_count", "swa_bwd_launch_count"):
        getattr(l, name).argtypes = [P(SwaProblem)]
        getattr(l, name).restype = ctypes.c_int
    l.swa_check_device.argtypes = [ctypes.c_void_p]
    l.swa_check_device.restype = ctypes.c_int
    l.swa_status_string.argtypes = [ctypes.c_int]
    l.swa_status_string.restype = ctypes.c_char_p
    l.swa_last_cuda_error.argtypes = []
    l.swa_last_cuda_error.restype = ctypes.c_char_p
    l.swa_device_status_async.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    l.swa_device_status_async.restype = ctypes.c_int
    l.swa_selftest_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_void_p]
    l.swa_selftest_wait_timeout.restype = ctypes.c_int
    l.swa_lse_row_stride.argtypes = [ctypes.c_int]
    l.swa_lse_row_stride.restype = ctypes.c_int
    l.swa_version.argtypes = []
    l.swa_version.restype = ctypes.c_int


def lib_path() -> str:
    return LIB_PATH


def lib():
    """Load (once) and return the C-ABI library; raises if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python flashattention-gpt-oss-finetuning_b200/build.py` "
                        "(there is no CPU or eager fallback)")
                l = ctypes.CDLL(LIB_PATH)
                _declare(l)
                _lib = l
    return _lib


def check(status: int, where: str):
    if status == SWA_OK:
        return
    detail = ""
    if status == SWA_ERR_LAUNCH:
        detail = lib().swa_last_cuda_error().decode()
    cls = SwaDeviceTimeout if status == SWA_ERR_DEVICE_TIMEOUT else SwaError
    raise cls(status, where, detail)


# ---------------------------------------------------------------------------------------
# Timeout monitor: surfaces an on-device wait that gave up without synchronising each call.
#
# After every launch sequence the Python API enqueues (swa_device_status_async) a copy of the
# device's error flag into a pinned host word and records an event behind it.  The next call
# on that device first looks at the word if the event has completed: a set flag means that an
# earlier launch's outputs are invalid (and that the kernels skip their work until the flag is
# cleared), so the call clears it (swa_check_device, which synchronises) and raises
# SwaDeviceTimeout instead of returning zeros.  Nothing is enqueued while a stream is being
# captured into a CUDA graph.
# ---------------------------------------------------------------------------------------

class _Monitor:
    def __init__(self, dev):
        import torch
        self.flag = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = torch.cuda.Event()
        self.armed = False
        self.dev = dev


_monitors = {}


def _monitor(dev):
    m = _monitors.get(dev.index)
    if m is None:
        with _lock:
            m = _monitors.get(dev.index)
            if m is None:
                m = _monitors[dev.index] = _Monitor(dev)
    return m


def _capturing(dev) -> bool:
    import torch
    return torch.cuda.is_current_stream_capturing()


def raise_if_device_timed_out(dev, stream_handle: int, where: str):
    """Raise SwaDeviceTimeout when a launch polled earlier on ``dev`` has reported a timeout."""
    if _capturing(dev):
        return
    m = _monitor(dev)
    if not m.armed or not m.event.query():
        return
    m.armed = False
    if int(m.flag[0]) == 0:
        return
    m.flag[0] = 0
    lib().swa_check_device(stream_handle)  # synchronises and clears the device flag
    raise SwaDeviceTimeout(SWA_ERR_DEVICE_TIMEOUT, where,
                           "an on-device wait of an earlier launch on this device gave up; "
                           "that launch's outputs are invalid")


def poll_device_status(dev, stream):
    """Enqueue the error-flag copy behind the launches just made on ``stream``."""
    if _capturing(dev):
        return
    m = _monitor(dev)
    check(lib().swa_device_status_async(m.flag.data_ptr(), stream.cuda_stream),
          "swa_device_status_async")
    m.event.record(stream)
    m.armed = True


def selftest_wait_timeout(limit_us: int, dev, stream=None):
    """Launch the failure-path self-test kernel (a bounded wait that gives up after
    ``limit_us``) and poll its status like any API call, so the next API call on ``dev``
    raises SwaDeviceTimeout."""
    import torch
    st = stream or torch.cuda.current_stream(dev)
    check(lib().swa_selftest_wait_timeout(int(limit_us), st.cuda_stream),
          "swa_selftest_wait_timeout")
    poll_device_status(dev, st)
