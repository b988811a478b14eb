"""Pre-bound launches for a fixed set of device buffers.

``SwaPlan`` owns the outputs and the backward workspace of one problem and keeps the C-ABI
argument blocks built once, so that repeated steps (a training loop, a benchmark, a CUDA-graph
capture) pay no per-call Python shape logic.  Each method launches exactly one kernel on the
given stream (the current torch stream when omitted); ``launches`` counts them.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib
from .flash_attention_gpt_oss import _DTYPES, _problem, _tensor, _validate


class SwaPlan:
    def __init__(self, q, k, v, window_size: int, sink_size: int = 0,
                 softmax_scale: Optional[float] = None, dout: Optional[torch.Tensor] = None):
        _validate(q, k, v, True)
        d = q.shape[-1]
        if d not in (16, 32, 64, 128):
            raise NotImplementedError("SwaPlan takes kernel head dims 16/32/64/128 directly")
        for t in (q, k, v) + ((dout,) if dout is not None else ()):
            if t.stride(-1) != 1:
                raise ValueError("last dimension must be contiguous")
        if softmax_scale is None:
            softmax_scale = 1.0 / math.sqrt(d)
        self.q, self.k, self.v = q, k, v
        self.dout = dout if dout is not None else torch.empty_like(q)
        self.o = torch.empty_like(q)
        b, hq, l = q.shape[:3]
        self.lse = torch.empty((b, hq, (l + 63) // 64 * 64), device=q.device, dtype=torch.float32)
        self.dq = torch.empty_like(q)
        self.dk = torch.empty_like(k)
        self.dv = torch.empty_like(v)
        self.problem = _problem(q, k, window_size, sink_size, softmax_scale, d)
        self.lib = _lib.lib()
        ws = self.lib.swa_bwd_workspace_size(ctypes.byref(self.problem))
        self.workspace = torch.empty(max(ws, 1), device=q.device, dtype=torch.uint8)
        self.fwd_args = _lib.SwaFwdArgs(self.problem, _tensor(q), _tensor(k), _tensor(v),
                                        _tensor(self.o), self.lse.data_ptr())
        self.bwd_args = _lib.SwaBwdArgs(self.problem, _tensor(q), _tensor(k), _tensor(v),
                                        _tensor(self.o), _tensor(self.dout), self.lse.data_ptr(),
                                        _tensor(self.dq), _tensor(self.dk), _tensor(self.dv),
                                        self.workspace.data_ptr(), ws)
        self._fa = ctypes.byref(self.fwd_args)
        self._ba = ctypes.byref(self.bwd_args)
        self.device = q.device
        self.launches = 0
        # swa_bwd_dkdv also launches the far sink-pair kernel and the sink-row reduction;
        # swa_bwd may fold the far sink pairs into its dQ kernel
        self._dkdv_kernels = self.lib.swa_bwd_dkdv_launch_count(ctypes.byref(self.problem))
        self._bwd_kernels = self.lib.swa_bwd_launch_count(ctypes.byref(self.problem))

    def _s(self, stream) -> int:
        return (stream or torch.cuda.current_stream(self.device)).cuda_stream

    def fwd(self, stream=None):
        _lib.check(self.lib.swa_fwd(self._fa, self._s(stream)), "swa_fwd")
        self.launches += 1

    def bwd_preprocess(self, stream=None):
        _lib.check(self.lib.swa_bwd_preprocess(self._ba, self._s(stream)), "swa_bwd_preprocess")
        self.launches += 1

    def bwd_dkdv(self, stream=None):
        _lib.check(self.lib.swa_bwd_dkdv(self._ba, self._s(stream)), "swa_bwd_dkdv")
        self.launches += self._dkdv_kernels

    def bwd_dq(self, stream=None):
        _lib.check(self.lib.swa_bwd_dq(self._ba, self._s(stream)), "swa_bwd_dq")
        self.launches += 1

    def bwd(self, stream=None):
        """The whole backward (swa_bwd): dQ (which also writes Delta to the workspace), then
        dK / dV."""
        _lib.check(self.lib.swa_bwd(self._ba, self._s(stream)), "swa_bwd")
        self.launches += self._bwd_kernels

    def step(self, stream=None):
        """One forward + backward over the bound buffers.  Raises SwaDeviceTimeout when an
        earlier step's on-device wait gave up (polled without a host synchronisation)."""
        st = stream or torch.cuda.current_stream(self.device)
        _lib.raise_if_device_timed_out(self.device, st.cuda_stream, "SwaPlan.step")
        self.fwd(st)
        self.bwd(st)
        _lib.poll_device_status(self.device, st)

    def capture(self) -> "torch.cuda.CUDAGraph":
        """Record one forward + backward (``step``) into a CUDA graph over the bound buffers.

        The library allocates nothing and takes every pointer, size and TMA descriptor at
        launch time, so the graph replays the same kernels on the same buffers: refill
        ``q, k, v, dout`` in place and call ``replay()``.  The first ``step`` runs eagerly
        before the capture (one-time kernel attribute set-up stays out of the graph)."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.step(side)  # warm-up outside the graph
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.step()
        return graph
