"""Drop-in replacement for the reference module ``flash_attention_gpt_oss.py``.

Same public names, signatures, argument meaning and error behaviour as the reference
(junhown3/FlashAttention-GPT-OSS-finetuning, flash_attention_gpt_oss.py:340-438):

    FlashSWDAWithSink.apply(q, k, v, window_size, sink_size, is_causal=True, softmax_scale=None)
    flash_swda_with_sink(q, k, v, window_size, sink_size=0, is_causal=True, scale=None)

``q: [B, Hq, L, D]``, ``k, v: [B, Hkv, L, D]`` (fp16 or bf16, on a CUDA device), output
``[B, Hq, L, D]``.  Query head ``h`` reads KV head ``h // (Hq // Hkv)``; key ``j`` is visible
to query ``i`` iff ``j <= i`` and (``i - j < window_size`` or ``j < sink_size``).

Underneath, the reference's Triton kernels are replaced by the C-ABI library
``lib/libswa_attn.so`` (sm_100a CUDA kernels); this module only validates, allocates with the
torch caching allocator and passes raw pointers, element strides and the current CUDA stream.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from . import _lib

_DTYPES = {torch.float16: _lib.SWA_F16, torch.bfloat16: _lib.SWA_BF16}
_KERNEL_HEAD_DIMS = (16, 32, 64, 128)


def _kernel_head_dim(d: int) -> int:
    for k in _KERNEL_HEAD_DIMS:
        if d <= k:
            return k
    raise AssertionError("Head dimension must be less than or equal to 128")


def _prep(t: torch.Tensor, d_kernel: int) -> torch.Tensor:
    """Zero-pad the head dim to a kernel size and make rows 16-byte aligned if needed."""
    if t.shape[-1] != d_kernel:
        t = torch.nn.functional.pad(t, (0, d_kernel - t.shape[-1]))
    ok = (t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:3])
          and t.data_ptr() % 16 == 0)
    return t if ok else t.contiguous()


def _tensor(t: Optional[torch.Tensor]) -> _lib.SwaTensor:
    if t is None:
        return _lib.SwaTensor(None, 0, 0, 0)
    s = t.stride()
    return _lib.SwaTensor(t.data_ptr(), s[0], s[1], s[2])


def _problem(q, k, window_size, sink_size, scale, d_kernel) -> _lib.SwaProblem:
    b, hq, l, _ = q.shape
    w = int(window_size)
    w = max(-1, min(w, 2**31 - 1))
    return _lib.SwaProblem(b, hq, k.shape[1], l, d_kernel, w, int(sink_size), _DTYPES[q.dtype],
                           float(scale))


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def lse_row_stride(seq_len: int) -> int:
    """Row stride of the LSE buffer: seq_len rounded up to 64."""
    return (seq_len + 63) // 64 * 64


def _padded_lse(lse: torch.Tensor, seq_len: int) -> torch.Tensor:
    """The LSE storage the kernels expect ([B, Hq, lse_row_stride(L)] rows, +inf padding)."""
    ld = lse_row_stride(seq_len)
    if lse.dim() == 3 and lse.stride() == (lse.shape[1] * ld, ld, 1) and lse.dtype == torch.float32:
        return lse
    full = torch.full((lse.shape[0], lse.shape[1], ld), float("inf"), device=lse.device,
                      dtype=torch.float32)
    full[..., :seq_len] = lse[..., :seq_len]
    return full


def _validate(q, k, v, is_causal):
    """The reference's checks (flash_attention_gpt_oss.py:343-354), same exception type."""
    assert is_causal, "Currently, only causal attention is supported"
    assert q.dim() == 4 and k.dim() == 4 and v.dim() == 4, "q, k, v must be [B, H, L, D]"
    assert q.shape[0] == v.shape[0] and q.shape[2] == v.shape[2] and q.shape[3] == v.shape[3], \
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


def _sink_logits_f32(sinks: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """Learned sink logits as the contiguous fp32 [Hq] device array the library reads."""
    if not isinstance(sinks, torch.Tensor) or sinks.numel() != q.shape[1] or sinks.dim() != 1:
        raise ValueError(f"sinks must be a 1-D tensor of {q.shape[1]} (query heads) logits")
    if sinks.device != q.device:
        raise ValueError("sinks must be on the device of q")
    return sinks.detach().to(torch.float32).contiguous()


def swa_forward(q, k, v, window_size: int, sink_size: int = 0,
                softmax_scale: Optional[float] = None,
                sink_logits: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Forward only: returns ``(o, lse)`` where ``lse`` is the base-2 row log-sum-exp
    ([B, Hq, L] fp32 view of a buffer whose rows are padded to a multiple of 64; -inf for a
    row that sees no key).  Pass it unchanged to :func:`swa_backward`.

    ``sink_logits`` ([Hq], natural-log units, not scaled by ``softmax_scale``): learned
    per-head sink logits, GPT-OSS's form, an additional mode beside the reference's sink
    tokens.  Each row's softmax gets one more column of that value with no value vector;
    ``lse`` then includes it."""
    _validate(q, k, v, True)
    d = q.shape[-1]
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    dk_ = _kernel_head_dim(d)
    qp, kp, vp = (_prep(t, dk_) for t in (q, k, v))
    b, hq, l, _ = q.shape
    o = torch.empty((b, hq, l, dk_), device=q.device, dtype=q.dtype)
    lse = torch.empty((b, hq, lse_row_stride(l)), device=q.device, dtype=torch.float32)
    args = _lib.SwaFwdArgs(_problem(q, k, window_size, sink_size, softmax_scale, dk_),
                           _tensor(qp), _tensor(kp), _tensor(vp), _tensor(o), lse.data_ptr())
    with torch.cuda.device(q.device):
        _lib.raise_if_device_timed_out(q.device, _stream(q.device), "swa_fwd")
        if sink_logits is None:
            _lib.check(_lib.lib().swa_fwd(ctypes.byref(args), _stream(q.device)), "swa_fwd")
        else:
            sl = _sink_logits_f32(sink_logits, q)
            _lib.check(_lib.lib().swa_fwd_sink_logits(ctypes.byref(args), sl.data_ptr(),
                                                      _stream(q.device)), "swa_fwd_sink_logits")
        _lib.poll_device_status(q.device, torch.cuda.current_stream(q.device))
    if dk_ != d:
        o = o[..., :d]
    return o, lse[..., :l]


def swa_backward(q, k, v, o, lse, do, window_size: int, sink_size: int = 0,
                 softmax_scale: Optional[float] = None,
                 sink_logits: Optional[torch.Tensor] = None):
    """Backward: returns ``(dq, dk, dv)`` in the input dtype (deterministic).  With
    ``sink_logits`` (the forward's), returns ``(dq, dk, dv, dsink_logits)``, the last one
    fp32 [Hq]."""
    d = q.shape[-1]
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    dk_ = _kernel_head_dim(d)
    if do.dtype != q.dtype:
        do = do.to(q.dtype)
    qp, kp, vp, op, dop = (_prep(t, dk_) for t in (q, k, v, o, do))
    b, hq, l, _ = q.shape
    dq = torch.empty((b, hq, l, dk_), device=q.device, dtype=q.dtype)
    dk = torch.empty((b, k.shape[1], l, dk_), device=q.device, dtype=q.dtype)
    dv = torch.empty_like(dk)
    prob = _problem(q, k, window_size, sink_size, softmax_scale, dk_)
    lse = _padded_lse(lse, l)
    lib = _lib.lib()
    ws_bytes = lib.swa_bwd_workspace_size(ctypes.byref(prob))
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    args = _lib.SwaBwdArgs(prob, _tensor(qp), _tensor(kp), _tensor(vp), _tensor(op), _tensor(dop),
                           lse.data_ptr(), _tensor(dq), _tensor(dk), _tensor(dv),
                           ws.data_ptr(), ws_bytes)
    dsl = None
    with torch.cuda.device(q.device):
        _lib.raise_if_device_timed_out(q.device, _stream(q.device), "swa_bwd")
        if sink_logits is None:
            _lib.check(lib.swa_bwd(ctypes.byref(args), _stream(q.device)), "swa_bwd")
        else:
            sl = _sink_logits_f32(sink_logits, q)
            dsl = torch.empty_like(sl)
            _lib.check(lib.swa_bwd_sink_logits(ctypes.byref(args), sl.data_ptr(), dsl.data_ptr(),
                                               _stream(q.device)), "swa_bwd_sink_logits")
        _lib.poll_device_status(q.device, torch.cuda.current_stream(q.device))
    if dk_ != d:
        dq, dk, dv = dq[..., :d], dk[..., :d], dv[..., :d]
    return (dq, dk, dv) if dsl is None else (dq, dk, dv, dsl)


class FlashSWDAWithSink(torch.autograd.Function):
    """Causal sliding-window + sink-token + GQA attention (flash_attention_gpt_oss.py:340)."""

    @staticmethod
    def forward(ctx, q, k, v, window_size, sink_size, is_causal=True, softmax_scale=None):
        _validate(q, k, v, is_causal)
        if softmax_scale is None:
            softmax_scale = 1.0 / math.sqrt(q.shape[-1])
        o, lse = swa_forward(q, k, v, window_size, sink_size, softmax_scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.softmax_scale = softmax_scale
        ctx.window_size = window_size
        ctx.sink_size = sink_size
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = swa_backward(q, k, v, o, lse, do, ctx.window_size, ctx.sink_size,
                                  ctx.softmax_scale)
        return dq, dk, dv, None, None, None, None


class FlashSWDAWithSinkLogits(torch.autograd.Function):
    """FlashSWDAWithSink plus learned per-head sink logits (GPT-OSS's form of attention
    sinks; no counterpart in the reference).  ``sinks``: [Hq] logits, natural-log units, not
    scaled by ``softmax_scale``; gets a gradient in its own dtype."""

    @staticmethod
    def forward(ctx, q, k, v, sinks, window_size, sink_size, is_causal=True, softmax_scale=None):
        _validate(q, k, v, is_causal)
        if softmax_scale is None:
            softmax_scale = 1.0 / math.sqrt(q.shape[-1])
        o, lse = swa_forward(q, k, v, window_size, sink_size, softmax_scale, sink_logits=sinks)
        ctx.save_for_backward(q, k, v, o, lse, sinks)
        ctx.softmax_scale = softmax_scale
        ctx.window_size = window_size
        ctx.sink_size = sink_size
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, sinks = ctx.saved_tensors
        dq, dk, dv, dsl = swa_backward(q, k, v, o, lse, do, ctx.window_size, ctx.sink_size,
                                       ctx.softmax_scale, sink_logits=sinks)
        return dq, dk, dv, dsl.to(sinks.dtype), None, None, None, None


def flash_swda_with_sink(q, k, v, window_size: int, sink_size: int = 0, is_causal: bool = True,
                         scale: Optional[float] = None, sinks: Optional[torch.Tensor] = None):
    """Same signature as the reference (flash_attention_gpt_oss.py:437-438), plus the
    optional keyword ``sinks`` ([Hq] learned sink logits, see FlashSWDAWithSinkLogits)."""
    if sinks is not None:
        return FlashSWDAWithSinkLogits.apply(q, k, v, sinks, window_size, sink_size, is_causal,
                                             scale)
    return FlashSWDAWithSink.apply(q, k, v, window_size, sink_size, is_causal, scale)
