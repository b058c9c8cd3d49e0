#!/usr/bin/env python
"""Benchmark of the torch.ops.kp hot path on B200s: prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload KEY] [--impl ours|reference]

A step is one call of the op on the whole synthetic job (default: full sum of one
vector of 2^28+1 fp32 values drawn U(-1,1), the reduction headline configuration).
Under torchrun the ONE job is split N ways along the op's natural axis (strong
scaling): the reduction into contiguous chunks, softmax and LayerNorm into row
blocks, GEMM into M-blocks of A with B replicated, attention into (batch, head)
slices. Every rank draws the same global input from the same seed and keeps its
shard. The reduction's one exchange step (the sum of the per-GPU partials) runs in
its finishing kernel over NVLink peer memory inside the timed step; the other ops
need no exchange (an all_gather would only assemble outputs).

value      whole-job algorithmic bytes (or FLOPs) / max-over-ranks device time, inputs
           resident in HBM; per-step CUDA events; when a rank's working set is under
           twice the L2, L2 is flushed between steps outside the events (256 MB
           written, then read back so no dirty lines are left for the timed kernel;
           for the reduction at N > 1 a one-element NCCL all_reduce after the flush
           re-aligns the ranks, whose in-kernel exchange would otherwise time the
           flushes' skew).
e2e        the same metric through the public API (torch.ops.kp, and the peer-sum
           object at N > 1) with each rank's inputs copied from pinned host memory and
           the result copied back inside the timed region.
roofline   rank 0's algorithmic bytes/FLOPs per call over its measured device time,
           against MEASURED_PEAKS.json (HBM copy GB/s, or cuBLAS bf16 TFLOP/s).
check      the reduction's result against the float64 sum of the global vector (the
           ranks' float64 shard sums, all-reduced), with the spec's tolerance.
configs    the other headline workloads, split the same way, device-timed; at N = 1
           each row also carries its e2e number, the reference's CPU path and the
           reference's own Triton kernels for the op timed on the same inputs
           ("triton_twins", a comparison, not this library).
cpu_baseline  the reference's CPU path (the PyTorch built-in its spec names as
           ``baseline``) on this box's host cores, rank 0 at N=1 only.
--impl reference  runs only that CPU path, on the same job, and prints its line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from kernelpilot_b200 import dist as kdist  # noqa: E402
from kernelpilot_b200.specs import CONFIGS, Workload  # noqa: E402

METRIC = "achieved HBM TB/s (softmax/reduce) and BF16 TFLOPS (GEMM/attn), % of peak"
DEFAULT_WORKLOAD = "reduce_f32_2p28p1"
L2_BYTES = 126 * 1024 * 1024
DTYPE_NAMES = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def launches_per_call(w: Workload) -> int:
    """Kernels of ours one call of the best variant launches on this workload."""
    if w.kernel == "reduce_sum":
        return 2  # persistent level + one-CTA finish (with the peer exchange at N > 1)
    if w.kernel == "matmul":
        M, N, K = w.shape
        # tensor-core GEMM, plus a pitch-padding copy per operand TMA cannot describe
        return 1 + int((K * 2) % 16 != 0) + int((N * 2) % 16 != 0)
    if w.kernel == "attention_causal":
        return 2 if w.shape[2] > 256 else 1  # main grid + the few-key-rows grid
    return 1


# ------------------------------------------------------------------ helpers

def work_per_call(w: Workload) -> float:
    """Algorithmic bytes (hbm-bound) or FLOPs (tensor-bound) of one call."""
    s = w.spec
    return s.bytes_moved(w.shape, w.dtype) if w.bound == "hbm" else s.flops(w.shape)


def unit_of(w: Workload) -> str:
    return "TB/s" if w.bound == "hbm" else "TFLOPS"


def rate(w: Workload, ms: float) -> float:
    return work_per_call(w) / (ms / 1e3) / 1e12


def local_workload(w: Workload, rank: int, world: int) -> Workload:
    """The shard of the job this rank computes, as a workload of its own shape."""
    import dataclasses

    return dataclasses.replace(w, shape=kdist.local_shape(w.kernel, w.shape, rank, world))


def job_config(w: Workload, world: int) -> dict:
    """The ``config`` of the JSON line; both arms print exactly this dict."""
    shapes = sorted({kdist.local_shape(w.kernel, w.shape, r, world) for r in range(world)})
    return {"workload": w.key, "shape": list(w.shape), "dtype": DTYPE_NAMES[w.dtype],
            "description": w.description, "partition": kdist.PARTITION[w.kernel],
            "per_rank": [list(s) for s in shapes], "parallelism": f"dp{world}"}


def measured_peaks() -> dict:
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def roofline_peak(w: Workload) -> tuple[float, str]:
    """(peak, where it came from) in GB/s or TFLOP/s."""
    mp = measured_peaks()
    if w.bound == "hbm":
        if "hbm_gbs" in mp:
            return float(mp["hbm_gbs"]), "measured copy bandwidth (read + write)"
        return 6650.0, "fallback"
    if "bf16_tflops" in mp:
        return float(mp["bf16_tflops"]), "measured cuBLAS bf16 GEMM, burst"
    return 1590.0, "fallback"


def profiled_traffic(w: Workload) -> float | None:
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary
    (a line ``traffic_per_launch_bytes: <int>`` in profiles/<workload>.md)."""
    p = REPO / "profiles" / f"{w.key}.md"
    try:
        m = re.search(r"traffic_per_launch_bytes:\s*([0-9]+)", p.read_text())
    except OSError:
        return None
    return float(m.group(1)) if m else None


def rounded(d: dict, nd: int = 5) -> dict:
    return {k: (round(v, nd) if isinstance(v, float) else v) for k, v in d.items()}


class ClockSampler:
    """nvidia-smi clock/throttle samples every 50 ms while the timed region runs. The
    summary keeps the samples taken inside the window given to ``load`` (the steps
    under load, by the host's clock), or the one nearest to it when the window is
    shorter than the sampling period."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.out = ""
        self.window = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def load(self, t0: float, t1: float) -> None:
        """The wall-clock window (time.time()) in which the GPU ran the steps."""
        self.window = (t0, t1)

    def summary(self) -> dict:
        import datetime

        rows = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]),
                             {n for n, v in zip(names, parts[6:10], strict=False)
                              if v.lower() == "active"}))
            except ValueError:
                continue
        kept = rows
        if self.window is not None and rows:
            t0, t1 = self.window
            kept = [r for r in rows if t0 <= r[0] <= t1]
            if not kept:
                mid = (t0 + t1) / 2
                kept = [min(rows, key=lambda r: abs(r[0] - mid))]
        sm = [r[1] for r in kept]
        reasons = set().union(*(r[3] for r in kept)) if kept else set()
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_mhz_min": min(sm) if sm else None,
                "sm_max_mhz": kept[-1][2] if kept else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "samples_total": len(rows)}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ------------------------------------------------------------------ op plumbing

def reduce_exchange(rk: kdist.Rank):
    """(callable, description) of the reduction over the shards at world > 1: the
    in-kernel peer-memory combine when every rank can map its peers' memory, else one
    NCCL all_reduce of the fp32 partial (decided collectively)."""
    from kernelpilot_b200 import registry

    fn = registry.best("reduce_sum")
    if rk.world > 1:
        try:
            return kdist.PeerSum(), "in the finishing kernel: partials stored into every " \
                "rank's buffer over NVLink (CUDA IPC), summed in rank order"
        except RuntimeError:
            pass
    return (lambda x: kdist.sharded_reduce_sum(x, fn)), "all_reduce(SUM) of fp32 partials"


def make_step(w: Workload, inputs: tuple, exchange=None):
    """The timed unit: one call of the best variant on this rank's shard (+ the
    exchange step of the reduction, if any)."""
    from kernelpilot_b200 import registry

    fn = registry.best(w.kernel)
    if w.kernel == "reduce_sum" and exchange is not None:
        return lambda: exchange(inputs[0])
    return lambda: fn(*inputs)


def decide_flush(inputs: tuple, world: int) -> bool:
    """Flush L2 between steps when this job's inputs would otherwise stay in it: the
    largest rank's input bytes under twice the L2. Decided from the max over ranks, so
    every rank takes the same steps (the flush of an exchanging step is followed by a
    collective)."""
    nbytes = sum(t.numel() * t.element_size() for t in inputs)
    if world > 1:
        t = torch.tensor([float(nbytes)], dtype=torch.float64,
                         device=inputs[0].device if inputs else "cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        nbytes = int(t.item())
    return nbytes < 2 * L2_BYTES


def time_steps(step, steps: int, flush: bool, world: int, align: bool = False
               ) -> tuple[float, list[float]]:
    """(max-over-ranks total ms of the K steps, per-step ms on this rank).

    ``align`` is for steps that synchronise the ranks on the GPU (the reduction's
    in-kernel exchange): the ranks' streams reach the first step at host-dependent
    times, and every rank's exchange waits for the last one, so the first timed step
    would carry that launch skew (up to ~0.25 ms at N = 4). The stream first idles
    ~0.1 ms on the GPU, so the host can queue everything behind it, then runs one
    untimed step that brings the ranks together on the device; the timed steps
    follow it back to back. When the L2 is flushed between steps, each rank's flush
    ends at its own time, so an aligned step is also preceded by a one-element NCCL
    all_reduce (outside the timed region) that brings the ranks' streams together
    again before the idle work that lets the hosts queue the step."""
    from kernelpilot_b200.harness import flush_l2

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    rejoin = torch.zeros(1, device="cuda") if align and world > 1 else None
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    if align and world > 1:
        torch.cuda._sleep(200_000)
        step()
    for i in range(steps):
        if flush:
            flush_l2(clean=True)
            if rejoin is not None:
                torch.distributed.all_reduce(rejoin)
            # GPU-side idle work after the flush, outside the timed region, so the start
            # event, the step and the end event are already queued when the GPU reaches
            # them (a late host would otherwise be timed as an idle gap): ~50 us, or
            # ~0.5 ms after a re-alignment, where one rank's late host would also be
            # timed by every other rank's exchange
            torch.cuda._sleep(100_000 if rejoin is None else 1_000_000)
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends, strict=True)]
    total = torch.tensor([sum(per)], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(total, op=torch.distributed.ReduceOp.MAX)
    return float(total.item()), per


def time_e2e(w: Workload, local: tuple, steps: int, world: int, exchange=None) -> dict:
    """Public API with host buffers: H2D of this rank's inputs from pinned memory, the
    op, D2H of its result, all inside the timed region; value = the whole job over the
    max-over-ranks time."""
    from kernelpilot_b200 import registry

    op = registry.best(w.kernel)
    host = [t.cpu().pin_memory() for t in local]
    dev = [torch.empty_like(t) for t in local]
    out_host = None
    h2d = sum(t.numel() * t.element_size() for t in host)

    def one():
        nonlocal out_host
        for d, h in zip(dev, host, strict=True):
            d.copy_(h, non_blocking=True)
        r = exchange(dev[0]) if (w.kernel == "reduce_sum" and exchange is not None) \
            else op(*dev)
        if out_host is None:
            out_host = torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
        out_host.copy_(r, non_blocking=True)

    one()
    torch.cuda.synchronize()
    total, _ = time_steps(one, steps, flush=False, world=world)
    d2h = out_host.numel() * out_host.element_size()
    ms = total / steps
    del host, dev
    return {"value": rate(w, ms), "unit": unit_of(w), "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms}


def spot_check(w: Workload, local: tuple, out: torch.Tensor) -> dict:
    """The reference gate (kernelpilot's ``compare`` with the spec's tolerance) on a
    slice of this rank's output: 64 rows (softmax, LayerNorm, GEMM), one (batch,
    head) slice (attention), the first 2^20 elements (elementwise add), or the whole
    sum of this rank's shard (reduction)."""
    from kernelpilot_b200 import harness

    spec = w.spec
    if w.kernel in ("softmax", "layernorm"):
        n = min(64, local[0].shape[0])
        ins, got = (local[0][:n],) + tuple(local[1:]), out[:n]
        shape = (n,) + tuple(w.shape[1:])
    elif w.kernel == "matmul":
        n = min(64, local[0].shape[0])
        ins, got, shape = (local[0][:n], local[1]), out[:n], (n,) + tuple(w.shape[1:])
    elif w.kernel in ("attention", "attention_causal"):
        ins = tuple(t[:, :1] for t in local)
        got, shape = out[:, :1], (1, 1) + tuple(w.shape[2:])
    elif w.kernel == "vector_add":
        n = min(1 << 20, local[0].numel())
        ins, got, shape = tuple(t[:n] for t in local), out[:n], (n,)
    elif w.kernel == "reduce_sum":
        ins, got, shape = tuple(local), out.reshape(()), (local[0].numel(),)
    else:
        return {}
    tol = spec.tolerance(shape, w.dtype)
    info = harness.compare(got, spec.reference(*ins), tol.atol, tol.rtol)
    return {"what": f"{tuple(got.shape)} slice of rank 0's output vs float64",
            "max_abs_err": info["max_abs_err"], "ok": info["num_mismatched"] == 0}


# ------------------------------------------------------------------ CPU (reference) path

def reference_baseline(w: Workload):
    """(callable, kind): the reference's CPU implementation of this op: its
    ``spec.baseline`` (the PyTorch built-in, kernelpilot/specs.py:127,158,200,274)
    from the unmodified reference package the harness loads."""
    if w.kernel == "attention_causal":
        # the reference has no causal op: its attention baseline with the causal flag
        import torch.nn.functional as F

        return (lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True),
                "reference")
    from kernelpilot_b200 import harness

    return harness.reference().specs.get_spec(w.kernel).baseline, "reference"


def subset_workload(w: Workload, n: int) -> Workload:
    """The same workload with its leading dimension cut to n."""
    import dataclasses

    shape = (n,) + tuple(w.shape[1:])
    return dataclasses.replace(w, key=f"{w.key}[subset {n}]", shape=shape)


def cpu_sample(w: Workload) -> tuple[tuple, float, str]:
    """A bounded CPU sample of the workload: (inputs, fraction of one call, label)."""
    gen_cpu = torch.device("cpu")
    if w.kernel in ("reduce_sum", "vector_add"):
        return w.make_inputs(w.shape, w.dtype, gen_cpu, 0), 1.0, "the full instance"
    if w.kernel in ("softmax", "layernorm"):
        M, N = w.shape
        rows = min(M, max(1, (64 << 20) // (N * 4)))
        return w.make_inputs((rows, N), w.dtype, gen_cpu, 0), rows / M, f"{rows} of {M} rows"
    if w.kernel == "matmul":
        M, N, K = w.shape
        rows = min(M, 512)
        a, b = w.make_inputs((rows, N, K), w.dtype, gen_cpu, 0)
        return (a, b), rows / M, f"{rows} of {M} rows of A"
    B, H, S, D = w.shape
    q, k, v = w.make_inputs((1, 1, S, D), w.dtype, gen_cpu, 0)
    return (q, k, v), 1.0 / (B * H), f"1 of {B * H} (batch, head) slices"


def cpu_model() -> str:
    """The host CPU's model name (Linux /proc/cpuinfo), or the platform's processor."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def time_cpu(w: Workload, reps: int, budget_s: float = 20.0) -> dict:
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    fn, kind = reference_baseline(w)
    inputs, frac, label = cpu_sample(w)
    fn(*inputs)
    times = []
    t_start = time.perf_counter()
    for _ in range(max(1, reps)):
        t0 = time.perf_counter()
        fn(*inputs)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    sec = statistics.median(times) / frac  # scaled to one full call
    value = work_per_call(w) / sec / 1e12
    return {"value": value, "unit": unit_of(w), "cores": torch.get_num_threads(),
            "cpu_model": cpu_model(),
            "kind": kind, "sample": f"{label}, median of {len(times)} calls, "
                                   f"scaled to one full call",
            "ms_per_call": sec * 1e3}


def run_reference(args, rk: kdist.Rank) -> int:
    if rk.rank != 0:
        return 0
    w = CONFIGS[args.workload]
    from kernelpilot_b200 import harness

    if not harness.available():
        print(json.dumps({"impl": "reference", "unavailable":
                          f"the kernelpilot package is not installed under {harness.reference_root()}"}),
              flush=True)
        return 0
    cb = time_cpu(w, reps=args.steps + args.warmup)
    line = {"metric": METRIC, "value": cb["value"], "unit": cb["unit"], "n_gpus": rk.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["ms_per_call"],
            "higher_is_better": True, "scaling": "strong" if rk.world > 1 else "weak",
            "vs_baseline": None, "dtype": DTYPE_NAMES[w.dtype], "data": "synthetic",
            "config": job_config(w, rk.world),
            "impl": "reference", "cpu_baseline": rounded(cb),
            "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ Triton twins

def time_calls(fn, inputs: tuple, calls: int) -> tuple[float, object]:
    """Mean device ms per call of ``fn`` over ``calls`` back-to-back calls (inputs
    larger than L2 or flushed by the caller's convention), and the last output."""
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = None
    t0.record()
    for _ in range(calls):
        out = fn(*inputs)
    t1.record()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / calls, out


def triton_twins(w: Workload, inputs: tuple, peak: float) -> dict:
    """The reference's own Triton kernels for this op (kernelpilot/triton_kernels/*,
    registered as ``triton:<name>`` by kernelpilot/registry.py:58-65), compiled by
    Triton for this GPU and timed on the same inputs: a comparison row, not part of
    this library. Each gets the same spot check as our kernels."""
    from kernelpilot_b200 import harness

    if w.kernel == "attention_causal":
        return {"note": "the reference has no causal Triton kernel"}
    try:
        impls = harness.reference().registry.triton_impls(w.kernel)
    except Exception as e:  # reported, never hidden
        return {"error": f"{type(e).__name__}: {e}"[:200]}
    rows = {}
    scale = 1e3 if w.bound == "hbm" else 1.0
    for name, fn in impls.items():
        try:
            t_first = time.perf_counter()
            fn(*inputs)  # compiles (and autotunes) once
            torch.cuda.synchronize()
            first_s = time.perf_counter() - t_first
            est, _ = time_calls(fn, inputs, 1)
            calls = int(min(20, max(3, 5.0 / max(est, 1e-3))))
            time_calls(fn, inputs, 2)
            # timed exactly as our kernels are: per-call events, L2 flushed between
            # calls when the inputs would otherwise stay in it
            flush = sum(t.numel() * t.element_size() for t in inputs) < 2 * L2_BYTES
            total, _ = time_steps(lambda: fn(*inputs), calls, flush, world=1)
            ms = total / calls
            out = fn(*inputs)
            torch.cuda.synchronize()
            val = rate(w, ms)
            rows[name] = {"value": round(val, 4), "ms": round(ms, 5), "calls": calls,
                          "frac_of_peak": round(val * scale / peak, 4),
                          "first_call_s": round(first_s, 2),
                          "check": rounded(spot_check(w, inputs, out), 8)}
            del out
        except Exception as e:  # a Triton kernel that fails on this shape is reported
            rows[name] = {"error": f"{type(e).__name__}: {e}"[:200]}
        torch.cuda.empty_cache()
    return rows


# ------------------------------------------------------------------ the configs table

def time_assemble(w: Workload, out: torch.Tensor, world: int, calls: int = 5) -> dict:
    """The whole output gathered on every rank (``dist.assemble_rows``: one NCCL
    all_gather of the row / (batch, head) / element blocks): the median over
    ``calls`` timed calls of each call's max-over-ranks device time, after two
    untimed calls (the first in a process loads the copy kernels it uses and can take
    milliseconds of host time). Not part of the sharded step: an op's outputs stay
    sharded unless a caller asks for them whole."""
    units = w.shape[0] * w.shape[1] if w.kernel in ("attention", "attention_causal") \
        else w.shape[0]
    if w.kernel in ("attention", "attention_causal"):
        local = out.reshape(out.shape[1], -1)   # (1, B*H slices, S, D)
    elif w.kernel == "vector_add":
        local = out.reshape(-1, 1)
    else:
        local = out.reshape(out.shape[0], -1)   # rows
    local = local.contiguous()
    counts = kdist.row_counts(units, world)
    for _ in range(2):
        kdist.assemble_rows(local, counts)      # untimed
    per_call = []
    for _ in range(calls):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.distributed.barrier()
        torch.cuda.synchronize()
        e0.record()
        full = kdist.assemble_rows(local, counts)
        e1.record()
        torch.cuda.synchronize()
        got = full.numel() * full.element_size() - local.numel() * local.element_size()
        del full
        per_call.append(e0.elapsed_time(e1))
    ms = torch.tensor(per_call, dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    med = float(ms.median().item())
    return {"ms": round(med, 4), "ms_calls": [round(float(v), 4) for v in ms.tolist()],
            "bytes_in_per_rank": got, "GB_s_per_rank": round(got / (med / 1e3) / 1e9, 1),
            "how": "dist.assemble_rows: NCCL all_gather of the output blocks"}


def measure_row(w: Workload, rk: kdist.Rank, with_host: bool, warmup: int = 3,
                budget_ms: float = 5.0, min_steps: int = 10, max_steps: int = 50,
                with_triton: bool = False) -> dict:
    """One workload of the table, split over the ranks like the headline: the whole
    job's rate over the max-over-ranks mean call time, the median call time beside
    it. The call count fills about ``budget_ms`` of device time (within [min_steps,
    max_steps]), estimated after the warm-up: short kernels get enough calls for a
    stable mean, long tensor-core ones few enough that the table does not push the
    GPU into power capping and slow the rows after it. ``with_host`` adds the row's
    e2e number and the reference's CPU path (rank 0, one GPU)."""
    world = rk.world
    inputs = kdist.shard_inputs(w.kernel, w.inputs("cuda", seed=0), rk.rank, world)
    torch.cuda.empty_cache()
    exchange = reduce_exchange(rk)[0] if (w.kernel == "reduce_sum" and world > 1) else None
    step = make_step(w, inputs, exchange)
    for _ in range(warmup):
        step()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(2):
        step()
    t1.record()
    torch.cuda.synchronize()
    est = torch.tensor([max(t0.elapsed_time(t1) / 2, 1e-3)], device="cuda")
    if world > 1:  # every rank must time the same number of calls
        torch.distributed.all_reduce(est, op=torch.distributed.ReduceOp.MAX)
    steps = int(min(max_steps, max(min_steps, budget_ms / float(est.item()))))
    flush = decide_flush(inputs, world)
    total, per = time_steps(step, steps, flush, world, align=isinstance(exchange, kdist.PeerSum))
    ms = total / steps
    peak, src = roofline_peak(w)
    val = rate(w, ms)
    scale = 1e3 if w.bound == "hbm" else 1.0
    row = {"value": round(val, 4), "unit": unit_of(w), "ms": round(ms, 5),
           "ms_median_rank0": round(statistics.median(per), 5), "steps": steps,
           "frac_of_peak": round(val * scale / (peak * world), 4),
           "peak": f"{world} x {peak} ({src})",
           "per_rank": list(kdist.local_shape(w.kernel, w.shape, rk.rank, world)),
           "launches": launches_per_call(local_workload(w, rk.rank, world)) * steps}
    out = step()
    torch.cuda.synchronize()
    if rk.rank == 0:
        row["check"] = rounded(spot_check(w, inputs, out), 8)
    if world > 1 and w.kernel != "reduce_sum":
        row["assemble"] = time_assemble(w, out, world)
    del out
    if with_triton and world == 1:
        row["triton_twins"] = triton_twins(w, inputs, peak)
    if with_host:
        e2e = time_e2e(w, inputs, steps=3, world=world, exchange=exchange)
        row["e2e"] = rounded({k: v for k, v in e2e.items()}, 5)
        del inputs, step
        torch.cuda.empty_cache()
        row["cpu_baseline"] = rounded(time_cpu(w, reps=5, budget_s=4.0), 5)
    if isinstance(exchange, kdist.PeerSum):
        exchange.close()
    return row


# ------------------------------------------------------------------ main

def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(CONFIGS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the table of the other headline workloads")
    ap.add_argument("--configs", default="",
                    help="comma-separated workload keys for the table (default: all)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--no-triton", action="store_true",
                    help="skip the reference's Triton kernels in the configs table")
    ap.add_argument("--subset", type=int, default=0,
                    help="run a smaller instance: this many rows (softmax), rows of A (matmul), "
                         "batches (attention) or elements (reduce_sum); for profiling")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    rk = kdist.env_rank()
    if args.impl == "reference":
        return run_reference(args, rk)

    rk = kdist.init(timeout_s=300)
    torch.cuda.set_device(rk.local_rank)
    from kernelpilot_b200 import ext

    if not ext.load():
        raise RuntimeError("kernelpilot_b200 extension missing: run python -m kernelpilot_b200.build")
    w = CONFIGS[args.workload]
    if args.subset:
        w = subset_workload(w, args.subset)
    lw = local_workload(w, rk.rank, rk.world)
    inputs = kdist.shard_inputs(w.kernel, w.inputs("cuda", seed=0), rk.rank, rk.world)
    torch.cuda.empty_cache()
    flush = decide_flush(inputs, rk.world)
    exchange, exchange_desc = (None, "none")
    if w.kernel == "reduce_sum":
        exchange, exchange_desc = (reduce_exchange(rk) if rk.world > 1
                                   else (None, "none (one GPU)"))
    step = make_step(w, inputs, exchange)

    with ClockSampler(physical_gpu_index(rk.local_rank)) as clocks:
        t_load = time.time()
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        total_ms, per = time_steps(step, args.steps, flush, rk.world,
                                   align=isinstance(exchange, kdist.PeerSum))
        clocks.load(t_load, time.time())
    ms = total_ms / args.steps

    check = None
    if w.kernel == "reduce_sum":
        # one more call on every rank, outside the timing, against the float64 sum of
        # the global vector; no bounded wait (the peer exchange) may have given up
        import ctypes

        got = step().reshape(()).to(torch.float64)
        ref = inputs[0].double().sum().reshape(1)
        lo_hi = torch.stack([got, -got]).reshape(2)
        if rk.world > 1:
            torch.distributed.all_reduce(ref, op=torch.distributed.ReduceOp.SUM)
            torch.distributed.all_reduce(lo_hi, op=torch.distributed.ReduceOp.MAX)
        word = ctypes.c_uint(0)
        ext.capi_check(ext.capi().kpb_device_errors(ctypes.byref(word)))
        tol = w.spec.tolerance(w.shape, w.dtype)
        g, r = float(got), float(ref)
        err = abs(g - r)
        ok = (math.isfinite(g) and err <= tol.atol + tol.rtol * abs(r) and not word.value
              and float(lo_hi[0]) == -float(lo_hi[1]))
        check = {"result": g, "reference_f64": r, "max_abs_err": err, "atol": tol.atol,
                 "rtol": tol.rtol, "same_bits_on_every_rank": float(lo_hi[0]) == -float(lo_hi[1]),
                 "device_error_bits": word.value, "ok": ok}
        if not ok:
            raise RuntimeError(f"reduce_sum run invalid: {check}")

    value = rate(w, ms)
    peak, peak_src = roofline_peak(w)
    local_ms = statistics.mean(per)
    step_stats = {"mean": round(local_ms, 5), "median": round(statistics.median(per), 5),
                  "min": round(min(per), 5), "max": round(max(per), 5)}
    achieved = work_per_call(lw) / (local_ms / 1e3) / (1e9 if w.bound == "hbm" else 1e12)
    roof = {"bound": w.bound, "achieved": round(achieved, 2), "peak": peak,
            "unit": "GB/s" if w.bound == "hbm" else "TFLOP/s",
            "frac": round(achieved / peak, 4), "traffic": profiled_traffic(w),
            "peak_source": f"{peak_src} (MEASURED_PEAKS.json)" if peak_src != "fallback"
            else "fallback",
            "kernel": "rank 0's call on its shard, mean device time per call"}

    e2e = time_e2e(w, inputs, args.e2e_steps, rk.world, exchange) if args.e2e_steps > 0 else None
    twins = triton_twins(w, inputs, peak) if (rk.world == 1 and not args.no_triton) else None

    configs = {}
    configs_clocks = None
    if not args.no_configs:
        del inputs, step
        torch.cuda.empty_cache()
        keys = [k for k in (args.configs.split(",") if args.configs else CONFIGS) if k]
        with_host = rk.world == 1 and not args.no_cpu
        # clocks sampled over the whole table too: its numbers are only comparable
        # between runs at the same clocks
        with ClockSampler(physical_gpu_index(rk.local_rank)) as table_clocks:
            for key in keys:
                if key == w.key:
                    continue
                try:
                    configs[key] = measure_row(CONFIGS[key], rk, with_host,
                                               with_triton=not args.no_triton)
                except Exception as e:  # reported in the line, never hidden
                    configs[key] = {"error": f"{type(e).__name__}: {e}"[:300]}
                    if rk.world > 1:
                        raise  # the ranks would go out of step
                torch.cuda.empty_cache()
        configs_clocks = table_clocks.summary()

    cpu = None
    if rk.world == 1 and rk.rank == 0 and not args.no_cpu:
        cpu = time_cpu(w, reps=5)

    if rk.world > 1:
        torch.cuda.synchronize()
        torch.distributed.barrier()
        if isinstance(exchange, kdist.PeerSum):
            exchange.close()  # collective: synchronises and waits for every rank
        torch.distributed.destroy_process_group()
    if rk.rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": unit_of(w), "n_gpus": rk.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "step_ms_rank0": step_stats,
        "higher_is_better": True, "scaling": "strong" if rk.world > 1 else "weak",
        "vs_baseline": None, "dtype": DTYPE_NAMES[w.dtype], "data": "synthetic",
        "config": job_config(w, rk.world),
        "timing": {"l2": ("flushed between steps outside the events (256 MB written, then "
                          "read so no dirty lines remain)"
                          + ("; then a one-element NCCL all_reduce re-aligns the ranks "
                             "before the next step" if isinstance(exchange, kdist.PeerSum)
                             else "")) if flush else
                   "each rank's inputs larger than twice the L2",
                   "exchange": exchange_desc,
                   "ranks": "max over ranks of the summed per-step CUDA-event times"},
        "pct_of_peak": round(value * (1e3 if w.bound == "hbm" else 1.0) / (peak * rk.world), 4),
        "roofline": roof,
        "e2e": rounded(e2e) if e2e else None,
        "gpu_launches": launches_per_call(lw) * args.steps,
        "clocks": clocks.summary(),
    }
    if check:
        line["check"] = check
    if twins:
        line["triton_twins"] = twins
    if cpu:
        line["cpu_baseline"] = rounded(cpu)
    if configs:
        line["configs"] = configs
        line["configs_clocks"] = configs_clocks
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
