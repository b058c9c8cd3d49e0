"""Evaluates one candidate CUDA kernel for B200 in a process of its own.

    python -m kernelpilot_b200.agent.worker --kernel softmax --lang cuda \\
        --dtype bfloat16 --code cand.cu --out result.json [--build-dir D] [--bench-shapes JSON]

Follows kernelpilot/agent/worker.py (evaluate :99-186, main :189-204) with the HIP and
Triton paths replaced by one CUDA-only contract: the candidate source is compiled
with nvcc for sm_100a alone (``-gencode arch=compute_100a,code=sm_100a``), after
``<torch/extension.h>`` and ``kp_contract.cuh`` (the CUDA-only successor of
csrc/compat.h), into the candidate's own build directory. Then, in order:

1. compile      a compiler error ends the evaluation (stage "compile");
2. correctness  every test shape of the op's spec against the float64 reference, with
                the spec's tolerances (the reference harness's ``check_impl``);
3. benchmark    every benchmark shape, re-verified, timed against the PyTorch built-in
                the spec names as its baseline (the reference harness's ``bench_one``,
                with the B200 peaks of ``harness.gpu_info``);
4. profile      the kernels one call launches (torch.profiler) and, from ptxas, each
                kernel's registers, spills and static shared memory.

The sandbox (``sandbox.run_candidate``) runs this in a subprocess with a time limit,
so a hang, a crash or a GPU fault in generated code never reaches the caller.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import re
import sys
import tempfile
import time
import traceback
import uuid
from pathlib import Path

from .result import EvalResult

CONTRACT_DIR = Path(__file__).resolve().parent
CONTRACT_HEADER = "kp_contract.cuh"
PRELUDE = '#include <torch/extension.h>\n#include "kp_contract.cuh"\n'
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xptxas=-v",
              "-gencode", "arch=compute_100a,code=sm_100a"]
LANGS = ("cuda",)
MAX_LOG = 6000


def _tail(s: str, n: int = MAX_LOG) -> str:
    return s if len(s) <= n else "...(truncated)...\n" + s[-n:]


def arity(signature: str) -> int:
    """Tensor arguments of ``kernel_fn`` in a spec's Python signature."""
    return signature.split("->")[0].count("torch.Tensor")


def host_declaration(n: int) -> str:
    return "torch::Tensor kernel_fn(" + ", ".join(f"torch::Tensor x{i}" for i in range(n)) + ")"


@contextlib.contextmanager
def captured_output(path: Path):
    """Send this process's stdout and stderr (file descriptors 1 and 2, so the
    compiler processes' output as well) to `path` while the block runs."""
    sys.stdout.flush()
    sys.stderr.flush()
    saved = (os.dup(1), os.dup(2))
    with open(path, "wb") as f:
        os.dup2(f.fileno(), 1)
        os.dup2(f.fileno(), 2)
        try:
            yield
        finally:
            sys.stdout.flush()
            sys.stderr.flush()
            os.dup2(saved[0], 1)
            os.dup2(saved[1], 2)
            os.close(saved[0])
            os.close(saved[1])


_ENTRY = re.compile(r"Compiling entry function '([^']+)' for '(sm_\w+)'")
_USED = re.compile(r"Used (\d+) registers(?:.*?(\d+) bytes smem)?")
_SPILL = re.compile(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads")


def ptxas_resources(log: str) -> list[dict]:
    """Per-kernel resource usage from ``-Xptxas=-v`` output: registers per thread,
    spill bytes, static shared memory."""
    out: list[dict] = []
    cur: dict | None = None
    for line in log.splitlines():
        m = _ENTRY.search(line)
        if m:
            cur = {"kernel": m.group(1)[:120], "arch": m.group(2)}
            out.append(cur)
            continue
        if cur is None:
            continue
        m = _SPILL.search(line)
        if m:
            cur.update(stack_bytes=int(m.group(1)), spill_stores=int(m.group(2)),
                       spill_loads=int(m.group(3)))
        m = _USED.search(line)
        if m:
            cur["registers"] = int(m.group(1))
            if m.group(2) is not None:
                cur["smem_bytes"] = int(m.group(2))
    return out[:10]


def compile_candidate(code_path: Path, n_args: int, build_dir: Path):
    """Build the candidate as a PyTorch extension for sm_100a; returns
    (kernel_fn, compiler output). Raises with the compiler output on failure."""
    from torch.utils.cpp_extension import load_inline

    build_dir.mkdir(parents=True, exist_ok=True)
    log_path = build_dir / "compile.log"
    try:
        with captured_output(log_path):
            ext = load_inline(
                name=f"kpb_candidate_{uuid.uuid4().hex[:10]}",
                cpp_sources=host_declaration(n_args) + ";",
                cuda_sources=PRELUDE + code_path.read_text(),
                functions=["kernel_fn"],
                extra_include_paths=[str(CONTRACT_DIR)],
                extra_cuda_cflags=NVCC_FLAGS,
                build_directory=str(build_dir),
                verbose=True)
    except Exception as e:
        log = log_path.read_text(errors="replace") if log_path.exists() else ""
        raise RuntimeError(f"{type(e).__name__}: {e}\n{log}") from None
    return ext.kernel_fn, log_path.read_text(errors="replace")


def _profile(fn, inputs) -> list[dict]:
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn(*inputs)
        torch.cuda.synchronize()
    rows = []
    for ev in prof.key_averages():
        us = getattr(ev, "device_time_total", None) or getattr(ev, "cuda_time_total", 0)
        if us:
            rows.append({"name": ev.key[:120], "calls": ev.count, "device_us": round(us, 2)})
    rows.sort(key=lambda r: -r["device_us"])
    return rows[:8]


def evaluate(kernel: str, lang: str, dtype_name: str, code_path: Path, build_dir: Path,
             bench_shapes: list[tuple] | None = None) -> EvalResult:
    import torch

    from .. import harness
    from ..specs import get_spec

    check_impl = harness.check_impl
    bench_one = harness.reference().benchmark.bench_one

    t0 = time.monotonic()

    def done(**kw) -> EvalResult:
        return EvalResult(duration_s=time.monotonic() - t0, **kw)

    if lang not in LANGS:
        return done(stage="rejected",
                    error=f"language {lang!r} is not evaluated here: candidates are CUDA C++ "
                          "compiled for sm_100a (B200)")
    spec = get_spec(kernel)
    dtype = getattr(torch, dtype_name)
    if not torch.cuda.is_available():
        return done(stage="crash", error="no GPU available in the worker")
    cap = torch.cuda.get_device_capability()
    if cap != (10, 0):
        return done(stage="crash",
                    error=f"candidates are built for sm_100a only; this GPU is sm_{cap[0]}{cap[1]}")

    # 1. compile
    try:
        fn, compile_log = compile_candidate(code_path, arity(spec.signature), build_dir)
    except Exception as e:
        return done(stage="compile", error=_tail(str(e)))
    resources = ptxas_resources(compile_log)
    compile_log = _tail(compile_log, 3000)

    # 2. correctness on every test shape
    passed = 0
    for shape in spec.test_shapes:
        res = check_impl(spec, "candidate", fn, shape, dtype, "cuda")
        if not res.ok:
            return done(stage="correctness", error=res.summary(), failures=[res.to_dict()],
                        checks_passed=passed, compile_log=compile_log)
        passed += 1

    # 3. benchmark against the PyTorch built-in, every shape verified again
    gpu = harness.gpu_info()
    rows = []
    try:
        for shape in bench_shapes or spec.bench_shapes:
            cand = bench_one(spec, "candidate", fn, shape, dtype, gpu, verify=True)
            if not cand.correct:
                return done(stage="correctness", error=cand.note, checks_passed=passed,
                            compile_log=compile_log)
            base = bench_one(spec, "torch", spec.baseline, shape, dtype, gpu, verify=False)
            rows.append({"shape": list(shape), "ms": cand.ms, "torch_ms": base.ms,
                         "speedup": base.ms / cand.ms, "gbs": cand.gbs, "tflops": cand.tflops,
                         "pct_peak_bw": cand.pct_peak_bw,
                         "pct_peak_flops": cand.pct_peak_flops})
    except Exception:
        return done(stage="benchmark", error=_tail(traceback.format_exc()),
                    checks_passed=passed, compile_log=compile_log)

    # 4. profile one call at the first benchmark shape
    info: dict = {"ptxas": resources}
    try:
        shape = (bench_shapes or spec.bench_shapes)[0]
        info["gpu_kernels"] = _profile(fn, spec.make_inputs(shape, dtype, torch.device("cuda"), 0))
        info["gpu"] = gpu.describe()
    except Exception as e:
        info["error"] = f"{type(e).__name__}: {e}"
    return done(stage="ok", checks_passed=passed, bench=rows, profile=info,
                compile_log=compile_log)


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--kernel", required=True)
    p.add_argument("--lang", choices=LANGS, default="cuda")
    p.add_argument("--dtype", default="float32")
    p.add_argument("--code", required=True)
    dest = p.add_mutually_exclusive_group(required=True)
    dest.add_argument("--out", help="write the result JSON to this file")
    dest.add_argument("--result-fd", type=int, help="write the result JSON to this open fd")
    p.add_argument("--build-dir", default=None)
    p.add_argument("--bench-shapes", default=None, help="JSON list of shapes")
    a = p.parse_args(argv)
    code = Path(a.code)
    shapes = [tuple(s) for s in json.loads(a.bench_shapes)] if a.bench_shapes else None
    build = Path(a.build_dir) if a.build_dir else Path(tempfile.mkdtemp(prefix="kpb_build_"))
    try:
        res = evaluate(a.kernel, a.lang, a.dtype, code, build, shapes)
    except Exception:
        res = EvalResult(stage="crash", error=_tail(traceback.format_exc()))
    payload = json.dumps(res.to_dict())
    if a.out:
        Path(a.out).write_text(payload)
    else:
        with os.fdopen(a.result_fd, "w") as f:
            f.write(payload)
    return 0


if __name__ == "__main__":
    sys.exit(main())
