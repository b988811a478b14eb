"""Benchmark: fwd+bwd of causal sliding-window + sink + GQA attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2_gptoss_swa]
    python bench.py --impl reference ...      # the CPU reference arm (oracle port, host cores)
    torchrun --nproc-per-node N bench.py --gpus N ...

Metric: effective TFLOP/s of fwd+bwd counting only useful (window + sink) FLOPs
(14 * D per visible (query, key) pair), whole job over all ranks.  Work is partitioned by
independent (batch, KV head) units with no collective on the data path; the barrier and the
max-over-ranks device time are the only cross-rank traffic.
  --scaling strong (default) the workload is fixed and its (batch, KV head) units are split
                   over the ranks (cfg2: 32 units, 4 per GPU at N = 8);
  --scaling weak   every rank runs its own full copy of the workload's shape
                   (global batch = N x B).
  --scaling seq    the workload is fixed and its sequence is split over the ranks
                   (seqsplit.py: K/V halo and sink rows exchanged over NCCL inside the timed
                   step, halo dK/dV and sink partials sent back).

Prints ONE JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = importlib.import_module("flashattention-gpt-oss-finetuning_b200")
wl = importlib.import_module("flashattention-gpt-oss-finetuning_b200.workloads")
plan_mod = importlib.import_module("flashattention-gpt-oss-finetuning_b200.plan")
sh_mod = importlib.import_module("flashattention-gpt-oss-finetuning_b200.sharding")
seq_mod = importlib.import_module("flashattention-gpt-oss-finetuning_b200.seqsplit")

METRIC = "fwd+bwd effective TFLOP/s (window+sink FLOPs only)"
UNIT = "TFLOP/s"
L2_BYTES = 126 * 2**20


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j["hbm_gbs"], j["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------------------
# Algorithmic work per kernel (per launch over the whole problem)
# ---------------------------------------------------------------------------------------

def kernel_work(w: wl.Workload, batch: int):
    e = 2
    pairs = batch * w.n_q_heads * wl.visible_pairs_per_head(w.seq_len, w.window_size, w.sink_size)
    d = w.head_dim
    qbytes = batch * w.n_q_heads * w.seq_len * d * e
    kbytes = batch * w.n_kv_heads * w.seq_len * d * e
    rows = batch * w.n_q_heads * w.seq_len * 4
    return {
        "fwd": dict(flops=4 * d * pairs, bytes=qbytes + 2 * kbytes + qbytes + rows),
        "bwd_preprocess": dict(flops=2 * qbytes // e, bytes=2 * qbytes + rows),
        "bwd_dkdv": dict(flops=8 * d * pairs, bytes=2 * qbytes + 2 * kbytes + 2 * rows + 2 * kbytes),
        # dQ pass: Q, dO, O, K, V, LSE read; dQ and Delta written
        "bwd_dq": dict(flops=6 * d * pairs, bytes=3 * qbytes + 2 * kbytes + 2 * rows + qbytes),
        # whole backward (swa_bwd): Q, dO, O, K, V, LSE read once, dQ, dK, dV written once
        "bwd": dict(flops=10 * d * pairs, bytes=3 * qbytes + 2 * kbytes + rows + qbytes + 2 * kbytes),
    }


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for n, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# CPU arm: the oracle port of the reference's naive attention on the host cores
# ---------------------------------------------------------------------------------------

def cpu_sample_time(w: wl.Workload, steps: int, warmup: int):
    """Time fwd+bwd of the oracle on one (batch, query head) slice of ``w`` per step."""
    from oracle import swa_oracle as orc   # the checker / CPU baseline only
    torch.set_num_threads(os.cpu_count() or 1)
    sample = w.replace(batch=1, n_q_heads=1, n_kv_heads=1)
    q, k, v, do = (t.float() for t in wl.make_inputs(w.replace(batch=1), kv_heads=[0])[:4])
    q, do = q[:, :1].contiguous(), do[:, :1].contiguous()
    for _ in range(warmup):
        orc.backward(q, k, v, do, w.window_size, w.sink_size, compute_dtype=torch.float32)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        orc.backward(q, k, v, do, w.window_size, w.sink_size, compute_dtype=torch.float32)
        times.append(time.perf_counter() - t0)
    flops = wl.useful_flops(sample)
    t = statistics.median(times)
    return {
        "value": flops / t / 1e12, "unit": UNIT, "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": (f"oracle (fp32 torch-CPU restatement of pytorch_naive_attention + its "
                   f"gradient) on 1 of {w.batch * w.n_q_heads} (batch, query head) slices of "
                   f"{w.name}, fwd+bwd, median of {steps}"),
        "ms_per_sample": t * 1e3,
    }


def run_reference(args, w, rank, world):
    if rank != 0:
        return
    steps, warmup = max(1, min(args.steps, 10)), max(1, min(args.warmup, 3))
    cb = cpu_sample_time(w, steps, warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
        "ms_per_step": cb["ms_per_sample"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded randn, BASELINE shapes)",
        "config": dict(w.describe(), sample="1 (batch, query head) slice per step"),
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_profile_phase(args, w, local_rank):
    """Run one phase of the workload alone, for a profiler to capture."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    q, k, v, do = wl.make_inputs(w, device=dev)
    plan = plan_mod.SwaPlan(q, k, v, w.window_size, w.sink_size, None, dout=do)
    for _ in range(args.warmup):
        plan.step()
    fn = {"fwd": plan.fwd, "bwd": plan.bwd, "bwd_dq": plan.bwd_dq,
          "bwd_dkdv": plan.bwd_dkdv}[args.profile_phase]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    print(json.dumps({"profile_phase": args.profile_phase, "workload": w.name,
                      "ms_per_launch_set": e0.elapsed_time(e1) / args.steps}), flush=True)


def run_reference_triton(args, w, rank, local_rank):
    """One line for the reference's Triton kernels on one GPU (rank 0 only)."""
    if rank != 0:
        return
    line = {"impl": "reference_triton", "metric": METRIC, "unit": UNIT, "n_gpus": 1,
            "higher_is_better": True, "config": w.describe()}
    if not torch.cuda.is_available():
        line["unavailable"] = "no CUDA device"
    else:
        dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(dev)
        r = reference_triton_timed(w, dev, args.steps, args.warmup)
        line.update(r)
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------

def device_timed(w, dev, rank, steps, warmup):
    q, k, v, do = wl.make_inputs(w, device=dev)
    plan = plan_mod.SwaPlan(q, k, v, w.window_size, w.sink_size, None, dout=do)
    stream = torch.cuda.current_stream(dev)
    # the backward as one call (swa_bwd: dQ, dK/dV and the sink-row reduction)
    phases = ("fwd", "bwd")
    fns = (plan.fwd, plan.bwd)
    for _ in range(warmup):
        plan.step(stream)
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(fns) + 1)]
           for _ in range(steps)]
    launches0 = plan.launches
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(steps):
        evs[s][0].record(stream)
        for i, fn in enumerate(fns):
            fn(stream)
            evs[s][i + 1].record(stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    total_ms = start.elapsed_time(end)
    per_phase = {p: sum(evs[s][i].elapsed_time(evs[s][i + 1]) for s in range(steps)) / steps
                 for i, p in enumerate(phases)}
    launches = plan.launches - launches0
    # the same step replayed from a CUDA graph (launch overhead out of the picture)
    graph = plan.capture()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize(dev)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    start.record(stream)
    for _ in range(steps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize(dev)
    graph_ms = start.elapsed_time(end)
    return total_ms, per_phase, launches, graph_ms


def e2e_timed(w, dev, rank, steps, warmup):
    """Public API (autograd Function) with pinned host buffers, copies inside the timed region.

    Every step copies its q, k, v, dO in from pinned host memory and o, dq, dk, dv back out, as
    a training loop with a pinned-memory loader does: the input copy of step i + 1 runs on a
    copy stream while step i computes (two device input slots), and the output copies run on a
    second copy stream, so the host link carries both directions at once.  The timed region
    spans from before the first step's input copy to the last step's outputs in host memory.
    """
    q, k, v, do = (t.pin_memory() for t in wl.make_inputs(w))
    host_in = (q, k, v, do)
    outs = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (q, q, k, v)]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in outs)
    main = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    slots = [[torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host_in] for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    slot_free = [torch.cuda.Event() for _ in range(2)]
    for e in slot_free:
        e.record(main)

    def copy_in(i):
        sl = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(slot_free[sl])  # the step that used this slot has finished with it
            for d, h in zip(slots[sl], host_in):
                d.copy_(h, non_blocking=True)
            in_ready[sl].record(s_in)

    def compute_and_copy_out(i):
        sl = i % 2
        main.wait_event(in_ready[sl])
        qd, kd, vd, dod = (t.detach().requires_grad_(r) for t, r in zip(slots[sl], (True, True, True, False)))
        o = PKG.flash_swda_with_sink(qd, kd, vd, w.window_size, w.sink_size)
        o.backward(dod)
        res = (o.detach(), qd.grad, kd.grad, vd.grad)
        done = torch.cuda.Event()
        done.record(main)
        slot_free[sl].record(main)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for dst, src in zip(outs, res):
                dst.copy_(src, non_blocking=True)
                src.record_stream(s_out)

    def run(n):
        copy_in(0)
        for i in range(n):
            if i + 1 < n:
                copy_in(i + 1)
            compute_and_copy_out(i)
        main.wait_stream(s_out)

    run(warmup)
    torch.cuda.synchronize(dev)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(main)
    s_in.wait_stream(main)
    run(steps)
    b.record(main)
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b), h2d, d2h


def copy_floor_timed(w, dev, steps):
    """The host link's own floor for the e2e step: the same pinned input bytes host->device on
    one stream and the same output bytes device->host on another, both directions at once,
    nothing else running.  Returns ms per step."""
    qs = (w.batch, w.n_q_heads, w.seq_len, w.head_dim)
    ks = (w.batch, w.n_kv_heads, w.seq_len, w.head_dim)
    host_in = [torch.empty(sh, dtype=w.dtype).pin_memory() for sh in (qs, ks, ks, qs)]
    host_out = [torch.empty(sh, dtype=w.dtype).pin_memory() for sh in (qs, qs, ks, ks)]
    dev_in = [torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host_in]
    dev_out = [torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host_out]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    main = torch.cuda.current_stream(dev)

    def run(n):
        s_in.wait_stream(main)
        s_out.wait_stream(main)
        for _ in range(n):
            with torch.cuda.stream(s_in):
                for d, h in zip(dev_in, host_in):
                    d.copy_(h, non_blocking=True)
            with torch.cuda.stream(s_out):
                for h, d in zip(host_out, dev_out):
                    h.copy_(d, non_blocking=True)
        main.wait_stream(s_in)
        main.wait_stream(s_out)

    run(2)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(main)
    run(steps)
    b.record(main)
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / steps


def _load_reference_triton():
    """The reference's own module (unmodified), installed under baseline/_ref, or the
    directory named by SWA_REFERENCE_DIR.  Returns (module, None) or (None, reason)."""
    import importlib.util
    cands = [os.environ.get("SWA_REFERENCE_DIR"), os.path.join(ROOT, "baseline", "_ref")]
    for d in cands:
        if not d:
            continue
        path = os.path.join(d, "flash_attention_gpt_oss.py")
        if os.path.exists(path):
            try:
                spec = importlib.util.spec_from_file_location("_reference_flash_attention_gpt_oss", path)
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                return mod, None
            except Exception as e:  # import error (e.g. no triton): reported, not raised
                return None, f"importing the reference from {d} failed: {type(e).__name__}: {e}"
    return None, ("the reference is not installed on this box (baseline/_ref is absent and "
                  "SWA_REFERENCE_DIR is unset)")


def reference_triton_timed(w, dev, steps, warmup):
    """The reference's Triton kernels (FlashSWDAWithSink, flash_attention_gpt_oss.py:340-438)
    on this GPU through its own autograd Function, fwd+bwd of ``w``, CUDA events on the
    launching stream.  Returns a dict for the JSON line (or {"unavailable": reason})."""
    mod, why = _load_reference_triton()
    if mod is None:
        return {"unavailable": why}
    q, k, v, do = wl.make_inputs(w, device=dev)
    qd, kd, vd = (t.detach().requires_grad_() for t in (q, k, v))
    stream = torch.cuda.current_stream(dev)

    def step():
        for t in (qd, kd, vd):
            t.grad = None
        o = mod.flash_swda_with_sink(qd, kd, vd, w.window_size, w.sink_size)
        o.backward(do)
        return o

    try:
        for _ in range(warmup):
            o = step()
        torch.cuda.synchronize(dev)
    except Exception as e:
        return {"unavailable": f"the reference's Triton kernels failed here: {type(e).__name__}: "
                               f"{str(e).splitlines()[0][:200] if str(e) else ''}"}
    # the same inputs through this library's drop-in Function, for a sanity comparison
    qo, ko, vo = (t.detach().clone().requires_grad_() for t in (q, k, v))
    oo = PKG.flash_swda_with_sink(qo, ko, vo, w.window_size, w.sink_size)
    oo.backward(do)
    ours = (oo, qo.grad, ko.grad, vo.grad)
    diffs = {}
    for n, a, b in zip(("o", "dq", "dk", "dv"), (o, qd.grad, kd.grad, vd.grad), ours):
        a, b = a.detach().float(), b.detach().float()
        diffs[n] = (a - b).abs().max().item() / max(b.abs().max().item(), 1e-30)
    del ours, oo, qo, ko, vo
    a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a_ev.record(stream)
    for _ in range(steps):
        step()
    b_ev.record(stream)
    torch.cuda.synchronize(dev)
    ms = a_ev.elapsed_time(b_ev) / steps
    return {"value": wl.useful_flops(w) / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms,
            "steps": steps, "warmup": warmup,
            "path": "reference FlashSWDAWithSink (Triton) from baseline/_ref, autograd fwd+bwd, "
                    "inputs resident on the GPU, CUDA events",
            "max_rel_diff_vs_ours": diffs}


def gather_over_ranks(x: float, dev) -> list:
    if not torch.distributed.is_initialized():
        return [x]
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    out = [torch.zeros_like(t) for _ in range(torch.distributed.get_world_size())]
    torch.distributed.all_gather(out, t)
    return [float(o.item()) for o in out]


def max_over_ranks(x: float, dev) -> float:
    if not torch.distributed.is_initialized():
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def rank_workload(w, rank, world, scaling):
    """This rank's share: its own copy (weak) or its (batch, KV head) units (strong), the
    units repacked as a batch of single-KV-head problems."""
    if scaling == "weak" or world == 1:
        return w.replace(seed=w.seed + 1000 * rank)
    units = sh_mod.plan_units(w.batch, w.n_kv_heads, world)[rank]
    return w.replace(batch=max(len(units), 1), n_q_heads=w.group, n_kv_heads=1,
                     seed=w.seed + 1000 * rank)


def run_ours(args, w_job, rank, world, local_rank):
    w = rank_workload(w_job, rank, world, args.scaling)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hbm_peak, tf_peak, peak_kind = _peaks()
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks:
        clocks.start()
    total_ms, per_phase, launches, graph_ms = device_timed(w, dev, rank, args.steps, args.warmup)
    graph_ms = max_over_ranks(graph_ms, dev) / args.steps
    clk = clocks.stop() if clocks else None
    per_rank_ms = [x / args.steps for x in gather_over_ranks(total_ms, dev)]
    per_rank_units = [len(u) for u in sh_mod.plan_units(w_job.batch, w_job.n_kv_heads, world)] \
        if args.scaling == "strong" else [w_job.batch * w_job.n_kv_heads] * world
    total_ms = max_over_ranks(total_ms, dev)
    ms = total_ms / args.steps
    flops_job = wl.useful_flops(w_job) * (world if args.scaling == "weak" else 1)
    value = flops_job / (ms * 1e-3) / 1e12

    e2e = None
    if not args.no_e2e:
        e_steps = max(3, min(args.steps, 10))
        e_ms, h2d, d2h = e2e_timed(w, dev, rank, e_steps, max(3, min(args.warmup, 3)))
        e_ms = max_over_ranks(e_ms, dev) / e_steps
        floor_ms = max_over_ranks(copy_floor_timed(w, dev, e_steps), dev)
        e2e = {"value": flops_job / (e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e_ms,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "copy_floor_ms": floor_ms, "frac_of_copy_floor": floor_ms / e_ms,
               "path": "flash_swda_with_sink autograd, pinned host in/out, copies overlapped across steps",
               "copy_floor": "the same pinned bytes in and out on two streams at once, no compute"}
    ref_triton = None
    if world == 1 and not args.no_reference_triton:
        ref_triton = reference_triton_timed(w, dev, max(3, min(args.steps, 10)), 3)

    if rank != 0:
        return
    work = kernel_work(w, w.batch)
    dom = max(per_phase, key=per_phase.get)
    kw = work[dom]
    t_s = per_phase[dom] * 1e-3
    t_tensor = kw["flops"] / (tf_peak * 1e12)
    t_hbm = kw["bytes"] / (hbm_peak * 1e9)
    if t_tensor >= t_hbm:
        roof = {"bound": "tensor", "achieved": kw["flops"] / t_s / 1e12, "peak": tf_peak,
                "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": kw["bytes"] / t_s / 1e9, "peak": hbm_peak,
                "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof.update(kernel=dom, peak_source=f"MEASURED_PEAKS.json burst ({peak_kind})",
                algorithmic_flops=kw["flops"], algorithmic_bytes=kw["bytes"],
                kernel_ms=per_phase[dom],
                traffic=TRAFFIC.get((kernel_sources_sha(), w_job.name, dom)) if world == 1 else None,
                kernel_sources_sha=kernel_sources_sha(),
                tensor_frac=(kw["flops"] / t_s / 1e12) / tf_peak,
                hbm_frac=(kw["bytes"] / t_s / 1e9) / hbm_peak)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": str(w.dtype).replace("torch.", "").replace("bfloat16", "bf16").replace("float16", "f16"),
        "data": "synthetic (seeded randn of the workload's shape; no dataset)",
        "config": dict(w_job.describe(), global_batch=w_job.batch * (world if args.scaling == "weak" else 1),
                       per_rank=w.describe(), parallelism=f"dp{world} by (batch, kv_head) units",
                       l2="inputs larger than L2 (q, dO 134 MB each + k, v, o, grads)"),
        "phase_ms": per_phase,
        "per_rank": {"ms_per_step": per_rank_ms, "units": per_rank_units},
        "gpu_launches": launches,
        "cuda_graph": {"ms_per_step": graph_ms, "value": flops_job / (graph_ms * 1e-3) / 1e12,
                       "note": "same step captured once (SwaPlan.capture) and replayed"},
        "roofline": roof,
        "clocks": clk,
        "e2e": e2e,
        "reference_triton": ref_triton,
    }
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_sample_time(w, 3, 1)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)


def run_seq(args, w, rank, world, local_rank):
    """Sequence split: rank r holds rows split_bounds(L, world)[r] of the whole workload."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    a, b = seq_mod.split_bounds(w.seq_len, world)[rank]
    q, k, v, do = (t[:, :, a:b].contiguous().to(dev) for t in wl.make_inputs(w))
    stream = torch.cuda.current_stream(dev)

    def step():
        o, st = seq_mod.seq_sharded_forward(q, k, v, w.seq_len, w.window_size, w.sink_size)
        return seq_mod.seq_sharded_backward(st, do)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks:
        clocks.start()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    clk = clocks.stop() if clocks else None
    ms = max_over_ranks(e0.elapsed_time(e1), dev) / args.steps
    if rank != 0:
        return
    value = wl.useful_flops(w) / (ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else "f16",
        "data": "synthetic (seeded randn of the workload's shape; no dataset)",
        "config": dict(w.describe(), parallelism=f"seq{world}: sequence split, K/V halo over NCCL",
                       rows_per_rank=b - a),
        "clocks": clk, "e2e": None, "roofline": None,
        "note": "secondary mode; exchanges (sink broadcast, halo send/recv, halo dK/dV return, "
                "sink reduce) and the local prefix copies are inside the timed step",
    }
    print(json.dumps(line), flush=True)


def run_variant(args, w, local_rank):
    """1-GPU lines for the additional modes (not the headline): learned sink logits on the
    workload's shape, or a packed variable-length batch of the workload's head layout."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    F = PKG.flash_attention_gpt_oss
    V = importlib.import_module("flashattention-gpt-oss-finetuning_b200.varlen")
    stream = torch.cuda.current_stream(dev)
    extra = {}
    if args.variant == "sink_logits":
        q, k, v, do = wl.make_inputs(w, device=dev)
        g = torch.Generator().manual_seed(w.seed)
        sl = (torch.randn(w.n_q_heads, generator=g) * 2).to(dev)
        flops = wl.useful_flops(w)

        def step():
            o, lse = F.swa_forward(q, k, v, w.window_size, w.sink_size, sink_logits=sl)
            F.swa_backward(q, k, v, o, lse, do, w.window_size, w.sink_size, sink_logits=sl)
        cfg = dict(w.describe(), variant="learned per-head sink logits + token sinks")
    else:
        g = torch.Generator().manual_seed(w.seed)
        n_seq = 32
        lens = torch.randint(128, w.seq_len // 2 + 1, (n_seq,), generator=g).tolist()
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        t = cu[-1]
        q, do = ((torch.randn(t, w.n_q_heads, w.head_dim, generator=g) * w.input_scale)
                 .to(w.dtype).to(dev) for _ in range(2))
        k, v = ((torch.randn(t, w.n_kv_heads, w.head_dim, generator=g) * w.input_scale)
                .to(w.dtype).to(dev) for _ in range(2))
        flops = sum(wl.useful_flops(w.replace(batch=1, seq_len=n)) for n in lens)

        def step():
            o, lse, cuh = V.swa_varlen_forward(q, k, v, cu, w.window_size, w.sink_size)
            V.swa_varlen_backward(q, k, v, o, lse, cuh, do, w.window_size, w.sink_size)
        # the same sequences padded to a dense batch, as without the packed mode
        lmax = max(lens)
        qd = torch.zeros(n_seq, w.n_q_heads, lmax, w.head_dim, dtype=w.dtype, device=dev)
        kd = torch.zeros(n_seq, w.n_kv_heads, lmax, w.head_dim, dtype=w.dtype, device=dev)
        vd, dod = torch.zeros_like(kd), torch.zeros_like(qd)
        for i, n in enumerate(lens):
            a = cu[i]
            qd[i, :, :n] = q[a:a + n].transpose(0, 1)
            kd[i, :, :n] = k[a:a + n].transpose(0, 1)
            vd[i, :, :n] = v[a:a + n].transpose(0, 1)
            dod[i, :, :n] = do[a:a + n].transpose(0, 1)

        def dense_step():
            o, lse = F.swa_forward(qd, kd, vd, w.window_size, w.sink_size)
            F.swa_backward(qd, kd, vd, o, lse, dod, w.window_size, w.sink_size)
        for _ in range(args.warmup):
            dense_step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            dense_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        dms = e0.elapsed_time(e1) / args.steps
        extra["padded_dense"] = {"ms_per_step": dms, "value": flops / (dms * 1e-3) / 1e12,
                                 "note": "same sequences zero-padded to [32, H, max_len, D]"}
        cfg = dict(w.describe(), variant="packed variable-length batch", n_seq=n_seq,
                   total_tokens=t, min_len=min(lens), max_len=lmax)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local_rank)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    line = {
        "metric": METRIC, "value": flops / (ms * 1e-3) / 1e12, "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if w.dtype == torch.bfloat16 else "f16",
        "data": "synthetic (seeded randn; no dataset)", "config": cfg, "clocks": clk,
        "e2e": None, "roofline": None, **extra,
        "note": "additional mode (not the headline); Python API with inputs resident on the GPU",
    }
    print(json.dumps(line), flush=True)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum, summed over the phase's kernels)
# per step of a phase, from one ncu capture of `bench.py --steps 1 --warmup 3`, keyed by
# (hash of the kernel sources, workload, phase).  A figure taken on other kernel sources is
# never reported: the line then carries traffic = null.
TRAFFIC: dict = {
    # bwd = bwd_dq_gqa 560.7 MB + bwd_dkdv 345.2 MB + bwd_sink_reduce 2.2 MB; fwd = fwd_gqa
    ("6bc957277f57", "cfg2_gptoss_swa", "bwd"): 560_742_400 + 345_186_490 + 2_174_999,
    ("6bc957277f57", "cfg2_gptoss_swa", "fwd"): 262_824_308,
}


def kernel_sources_sha() -> str:
    import hashlib
    csrc = os.path.join(ROOT, "flashattention-gpt-oss-finetuning_b200", "csrc")
    h = hashlib.sha256()
    for name in sorted(os.listdir(csrc)):
        if name.endswith((".cu", ".cuh", ".h")):
            with open(os.path.join(csrc, name), "rb") as f:
                h.update(name.encode() + b"\0" + f.read())
    return h.hexdigest()[:12]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "reference_triton"], default="ours",
                    help="reference: the CPU reference arm; reference_triton: the reference's "
                         "Triton kernels on one GPU (the second comparison point)")
    ap.add_argument("--workload", default="cfg2_gptoss_swa", choices=sorted(wl.CONFIGS))
    ap.add_argument("--scaling", choices=["weak", "strong", "seq"], default="strong")
    ap.add_argument("--variant", choices=["plain", "sink_logits", "varlen"], default="plain",
                    help="additional modes, 1 GPU (default: the headline path)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-triton", action="store_true")
    ap.add_argument("--profile-phase", choices=["fwd", "bwd", "bwd_dq", "bwd_dkdv"], default=None,
                    help="profiling driver: `--warmup` full steps, then `--steps` launches of "
                         "this phase only (for an ncu capture with -k / -s / -c); prints one line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    w = wl.CONFIGS[args.workload]
    if args.impl == "reference":
        run_reference(args, w, rank, world)
        return
    if args.profile_phase:
        run_profile_phase(args, w, local_rank)
        return
    if args.impl == "reference_triton":
        run_reference_triton(args, w, rank, local_rank)
        return
    if world > 1:
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        if args.variant != "plain":
            run_variant(args, w, local_rank)
        elif args.scaling == "seq":
            run_seq(args, w, rank, world, local_rank)
        else:
            run_ours(args, w, rank, world, local_rank)
    finally:
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
