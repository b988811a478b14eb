"""Variable-length (packed) batches for the sliding-window + sink attention.

An additional mode with no counterpart in the reference, whose entry point takes dense
``[B, H, L, D]`` tensors only (flash_attention_gpt_oss.py:348).  Fine-tuning batches are
usually packed instead: ``batch`` sequences of different lengths laid end to end along one
token axis, with ``cu_seqlens`` (``batch + 1`` cumulative offsets, starting at 0) marking where
each one starts.  Layout (the common packed convention): q, o ``[T, Hq, D]``; k, v
``[T, Hkv, D]``.  A sequence attends only inside itself, with the reference's mask in its own
positions.  The compute is the C-ABI library's ``swa_varlen_fwd`` / ``swa_varlen_bwd``.

``cu_seqlens`` is read on the host: a CUDA tensor is copied to the host (one synchronising
copy); pass a list or a CPU tensor to avoid it.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence, Union

import numpy as np
import torch

from . import _lib
from .flash_attention_gpt_oss import (_DTYPES, _kernel_head_dim, _sink_logits_f32, _stream)

CuSeqlens = Union[Sequence[int], torch.Tensor, np.ndarray]


def _host_cu(cu_seqlens: CuSeqlens, total: int) -> np.ndarray:
    if isinstance(cu_seqlens, torch.Tensor):
        cu_seqlens = cu_seqlens.detach().cpu().numpy()
    cu = np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.int64))
    if cu.ndim != 1 or cu.size < 1 or cu[0] != 0 or np.any(np.diff(cu) < 0):
        raise ValueError("cu_seqlens must be 1-D, start at 0 and be non-decreasing")
    if cu[-1] != total:
        raise ValueError(f"cu_seqlens ends at {int(cu[-1])} but the tensors hold {total} tokens")
    if cu[-1] >= 2**31:
        raise ValueError("more than 2^31 - 1 tokens")
    return cu.astype(np.int32)


def _validate(q, k, v, is_causal):
    assert is_causal, "Currently, only causal attention is supported"
    assert q.dim() == 3 and k.dim() == 3 and v.dim() == 3, "packed q, k, v must be [T, H, D]"
    assert q.shape[0] == v.shape[0] and q.shape[2] == v.shape[2], \
        "Query and Value shapes must be compatible except for num_heads"
    assert k.shape == v.shape, "Key and Value shapes must be the same"
    assert q.shape[-1] <= 128, "Head dimension must be less than or equal to 128"
    assert q.shape[1] % k.shape[1] == 0, \
        "Number of query heads must be divisible by number of K/V heads"
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"q, k, v must share one dtype in (float16, bfloat16); got "
                        f"{q.dtype}, {k.dtype}, {v.dtype}")
    if not (q.is_cuda and k.device == q.device and v.device == q.device):
        raise ValueError("q, k, v must be on the same CUDA device")


def _prep(t: torch.Tensor, d_kernel: int) -> torch.Tensor:
    if t.shape[-1] != d_kernel:
        t = torch.nn.functional.pad(t, (0, d_kernel - t.shape[-1]))
    ok = (t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.stride(1) % 8 == 0
          and t.data_ptr() % 16 == 0)
    return t if ok else t.contiguous()


def _packed(t: torch.Tensor) -> _lib.SwaPackedTensor:
    return _lib.SwaPackedTensor(t.data_ptr(), t.stride(0), t.stride(1))


def _problem(q, k, n_seq, window_size, sink_size, scale, d_kernel) -> _lib.SwaProblem:
    w = max(-1, min(int(window_size), 2**31 - 1))
    return _lib.SwaProblem(n_seq, q.shape[1], k.shape[1], 0, d_kernel, w, int(sink_size),
                           _DTYPES[q.dtype], float(scale))


def swa_varlen_forward(q, k, v, cu_seqlens: CuSeqlens, window_size: int, sink_size: int = 0,
                       softmax_scale: Optional[float] = None,
                       sink_logits: Optional[torch.Tensor] = None):
    """Returns ``(o, lse, cu)``: o ``[T, Hq, D]``; ``lse`` the library's private per-sequence
    base-2 log-sum-exp blocks; ``cu`` the host int32 offsets.  Pass ``lse`` and ``cu``
    unchanged to :func:`swa_varlen_backward`."""
    _validate(q, k, v, True)
    cu = _host_cu(cu_seqlens, q.shape[0])
    d = q.shape[-1]
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    dk_ = _kernel_head_dim(d)
    qp, kp, vp = (_prep(t, dk_) for t in (q, k, v))
    prob = _problem(q, k, cu.size - 1, window_size, sink_size, softmax_scale, dk_)
    lib = _lib.lib()
    n_lse = lib.swa_varlen_lse_floats(ctypes.byref(prob), cu.ctypes.data)
    o = torch.empty((q.shape[0], q.shape[1], dk_), device=q.device, dtype=q.dtype)
    lse = torch.empty(max(n_lse, 1), device=q.device, dtype=torch.float32)
    sl = None if sink_logits is None else _sink_logits_f32(sink_logits, _as4(q))
    args = _lib.SwaVarlenFwdArgs(prob, cu.ctypes.data, _packed(qp), _packed(kp), _packed(vp),
                                 _packed(o), lse.data_ptr(), None if sl is None else sl.data_ptr())
    with torch.cuda.device(q.device):
        _lib.raise_if_device_timed_out(q.device, _stream(q.device), "swa_varlen_fwd")
        _lib.check(lib.swa_varlen_fwd(ctypes.byref(args), _stream(q.device)), "swa_varlen_fwd")
        _lib.poll_device_status(q.device, torch.cuda.current_stream(q.device))
    if dk_ != d:
        o = o[..., :d]
    return o, lse, cu


def _as4(q):
    """A [1, Hq, T, D] view (the sink-logit check reads the head count from dim 1)."""
    return q.transpose(0, 1).unsqueeze(0)


def swa_varlen_backward(q, k, v, o, lse, cu: np.ndarray, do, window_size: int,
                        sink_size: int = 0, softmax_scale: Optional[float] = None,
                        sink_logits: Optional[torch.Tensor] = None):
    """Returns ``(dq, dk, dv)`` (packed, input dtype, deterministic), plus ``dsink_logits``
    (fp32 ``[Hq]``) when ``sink_logits`` is given."""
    d = q.shape[-1]
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    dk_ = _kernel_head_dim(d)
    if do.dtype != q.dtype:
        do = do.to(q.dtype)
    qp, kp, vp, op, dop = (_prep(t, dk_) for t in (q, k, v, o, do))
    prob = _problem(q, k, cu.size - 1, window_size, sink_size, softmax_scale, dk_)
    lib = _lib.lib()
    dq = torch.empty((q.shape[0], q.shape[1], dk_), device=q.device, dtype=q.dtype)
    dk = torch.empty((k.shape[0], k.shape[1], dk_), device=q.device, dtype=q.dtype)
    dv = torch.empty_like(dk)
    ws_bytes = lib.swa_varlen_bwd_workspace_size(ctypes.byref(prob), cu.ctypes.data)
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    sl = dsl = None
    if sink_logits is not None:
        sl = _sink_logits_f32(sink_logits, _as4(q))
        dsl = torch.empty_like(sl)
    args = _lib.SwaVarlenBwdArgs(prob, cu.ctypes.data, _packed(qp), _packed(kp), _packed(vp),
                                 _packed(op), _packed(dop), lse.data_ptr(), _packed(dq),
                                 _packed(dk), _packed(dv), None if sl is None else sl.data_ptr(),
                                 None if dsl is None else dsl.data_ptr(), ws.data_ptr(), ws_bytes)
    with torch.cuda.device(q.device):
        _lib.raise_if_device_timed_out(q.device, _stream(q.device), "swa_varlen_bwd")
        _lib.check(lib.swa_varlen_bwd(ctypes.byref(args), _stream(q.device)), "swa_varlen_bwd")
        _lib.poll_device_status(q.device, torch.cuda.current_stream(q.device))
    if dk_ != d:
        dq, dk, dv = dq[..., :d], dk[..., :d], dv[..., :d]
    return (dq, dk, dv) if dsl is None else (dq, dk, dv, dsl)


class FlashSWDAWithSinkVarlen(torch.autograd.Function):
    """Packed variable-length form of FlashSWDAWithSink (optionally with learned sink
    logits ``sinks``, ``[Hq]``, which then get a gradient)."""

    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, window_size, sink_size, is_causal=True,
                softmax_scale=None, sinks=None):
        _validate(q, k, v, is_causal)
        if softmax_scale is None:
            softmax_scale = 1.0 / math.sqrt(q.shape[-1])
        o, lse, cu = swa_varlen_forward(q, k, v, cu_seqlens, window_size, sink_size,
                                        softmax_scale, sink_logits=sinks)
        if sinks is None:
            ctx.save_for_backward(q, k, v, o, lse)
        else:
            ctx.save_for_backward(q, k, v, o, lse, sinks)
        ctx.cu = cu
        ctx.softmax_scale = softmax_scale
        ctx.window_size = window_size
        ctx.sink_size = sink_size
        return o

    @staticmethod
    def backward(ctx, do):
        saved = ctx.saved_tensors
        q, k, v, o, lse = saved[:5]
        sinks = saved[5] if len(saved) > 5 else None
        r = swa_varlen_backward(q, k, v, o, lse, ctx.cu, do, ctx.window_size, ctx.sink_size,
                                ctx.softmax_scale, sink_logits=sinks)
        dsinks = r[3].to(sinks.dtype) if sinks is not None else None
        return r[0], r[1], r[2], None, None, None, None, None, dsinks


def flash_swda_with_sink_varlen(q, k, v, cu_seqlens: CuSeqlens, window_size: int,
                                sink_size: int = 0, is_causal: bool = True,
                                scale: Optional[float] = None,
                                sinks: Optional[torch.Tensor] = None):
    """``flash_swda_with_sink`` over packed sequences: q ``[T, Hq, D]``, k, v ``[T, Hkv, D]``,
    ``cu_seqlens`` ``batch + 1`` offsets; returns o ``[T, Hq, D]``."""
    return FlashSWDAWithSinkVarlen.apply(q, k, v, cu_seqlens, window_size, sink_size, is_causal,
                                         scale, sinks)
