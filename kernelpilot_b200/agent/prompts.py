"""The contract a generated kernel must meet, as prompt text, plus the feedback
formatting and code extraction around it (kernelpilot/agent/prompts.py: SYSTEM and
HIP_CONTRACT :16-49, system_prompt :52-63, user_prompt :117-163, extract_code
:166-185).

The reference's HIP contract (``compat.h``, ``warpSize``, HIP names) is replaced by
one for CUDA C++ on B200: the file is compiled by nvcc for sm_100a only, after
``<torch/extension.h>`` and ``kp_contract.cuh``; a warp is 32 threads; the kernel
launches on PyTorch's current stream; tensor cores are reached through tcgen05/TMA
inline PTX, since the legacy mma.sync path cannot reach their throughput.
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass

from ..specs import KernelSpec
from .result import EvalResult
from .worker import arity, host_declaration

SYSTEM = """You are a GPU kernel engineer. You write correct, fast CUDA C++ kernels for \
an NVIDIA B200 (Blackwell, sm_100a) and improve them from benchmark and profiler \
feedback.

Rules:
- Answer with a short plan (what you change and why it should be faster, 2-5 \
sentences), then exactly ONE fenced code block holding the whole source file.
- Every result is checked against a float64 PyTorch reference on many shapes, \
including size 1, sizes that are not powers of two and large sizes. A wrong kernel is \
rejected however fast it is.
- Do not call the PyTorch operator you are implementing, or a library that implements \
it; your own kernels must do the work. Allocating outputs with torch::empty is fine.
- Never write to the input tensors.
{contract}"""

CUDA_CONTRACT = """- Language: CUDA C++17, compiled by nvcc for sm_100a only \
(-gencode arch=compute_100a,code=sm_100a, -O3) through PyTorch's cpp_extension. \
Included before your code: <torch/extension.h> and "kp_contract.cuh", which brings in \
the CUDA runtime, fp16 and bf16 headers and defines KP_SHFL_DOWN / KP_SHFL_XOR(v, \
delta), KP_CHECK_LAUNCH(), kp::kWarp (32: a warp has 32 threads), kp::kSms (148), \
kp::to_float / kp::from_float<T> for float, __half and __nv_bfloat16, kp::warp_sum, \
kp::warp_max and kp::block_reduce<is_max>(v, scratch[kp::kMaxWarps]).
- Define this host function (every argument a torch::Tensor, in this order):
    {host_decl}
  Its Python-side meaning: {signature}
- Inputs are contiguous CUDA tensors of dtype {dtype} (__half for float16, \
__nv_bfloat16 for bfloat16: reinterpret data_ptr). Launch on the current stream: include \
<ATen/cuda/CUDAContext.h> and use at::cuda::getCurrentCUDAStream(); call \
KP_CHECK_LAUNCH() after each launch.
- B200: 148 SMs, up to 227 KB of shared memory per block, HBM3e near 7.7 TB/s. \
Memory-bound kernels: 16-byte vector loads and stores, enough bytes in flight per SM, \
grids sized in multiples of 148. Matrix products: tensor cores through tcgen05.mma \
inline PTX with operands staged in shared memory by TMA (cp.async.bulk.tensor) and \
accumulators in tensor memory; wgmma does not exist on sm_100a."""


def system_prompt(spec: KernelSpec, lang: str = "cuda", dtype: str = "float32") -> str:
    if lang != "cuda":
        raise ValueError(f"unsupported language {lang!r}: candidates are CUDA C++ for sm_100a")
    contract = CUDA_CONTRACT.format(host_decl=host_declaration(arity(spec.signature)),
                                    signature=spec.signature, dtype=dtype)
    return SYSTEM.format(contract=contract)


@dataclass
class AttemptView:
    """What a prompt shows of an earlier attempt."""

    iteration: int
    code: str
    result: EvalResult


def _lines_tail(s: str, n: int) -> str:
    return "\n".join(s.strip().splitlines()[-n:])


def _fmt_bench(res: EvalResult) -> str:
    out = []
    for r in res.bench:
        peak = []
        if r.get("pct_peak_bw") is not None:
            peak.append(f"{r['pct_peak_bw']:.0f}% of peak HBM bandwidth")
        if r.get("pct_peak_flops") is not None:
            peak.append(f"{r['pct_peak_flops']:.0f}% of peak FLOPS")
        out.append(f"  shape={tuple(r['shape'])}: {r['ms']:.4f} ms vs PyTorch "
                   f"{r['torch_ms']:.4f} ms -> {r['speedup']:.2f}x; {r['gbs']:.0f} GB/s, "
                   f"{r['tflops']:.2f} TFLOPS ({', '.join(peak) or 'peak unknown'})")
    return "\n".join(out)


def _fmt_profile(res: EvalResult) -> str:
    p = res.profile or {}
    out = []
    if p.get("gpu_kernels"):
        out.append("Kernels one call launches (torch.profiler):\n" + "\n".join(
            f"  {k['name']}: {k['calls']} call(s), {k['device_us']} us" for k in p["gpu_kernels"]))
    if p.get("ptxas"):
        out.append("Resources per kernel (ptxas): " + json.dumps(p["ptxas"]))
    return "\n".join(out)


_LABELS = {
    "no_code": "No code block in your answer.",
    "rejected": "REJECTED before it ran.",
    "compile": "COMPILE ERROR.",
    "correctness": "WRONG RESULT (rejected).",
    "benchmark": "Crashed while being benchmarked.",
    "timeout": "TIMEOUT.",
    "crash": "The process crashed.",
}


def format_result(res: EvalResult) -> str:
    if res.ok:
        text = (f"Correct on all {res.checks_passed} test shapes. Score (geometric-mean "
                f"speed-up over PyTorch): {res.score:.3f}x\n{_fmt_bench(res)}")
        prof = _fmt_profile(res)
        return text + ("\n" + prof if prof else "")
    text = f"{_LABELS.get(res.stage, res.stage)}\n{res.error or ''}"
    if res.stage == "correctness" and res.checks_passed:
        text += f"\n(It passed {res.checks_passed} smaller shapes before failing.)"
    if res.stage == "compile" and res.compile_log and res.compile_log not in (res.error or ""):
        text += "\nCompiler output:\n" + _lines_tail(res.compile_log, 60)
    return text


def user_prompt(spec: KernelSpec, lang: str, dtype: str, gpu_desc: str,
                history: list[AttemptView], best: AttemptView | None,
                bench_shapes: list[tuple], recent: int = 3) -> str:
    parts = [
        f"## Task: {spec.name}",
        spec.description,
        f"Target GPU: {gpu_desc}",
        f"dtype: {dtype}",
        "Reference semantics (evaluated in float64):",
        f"```python\n{spec.reference_source().strip()}\n```",
        "Correctness shapes (" + ", ".join(spec.shape_names) + "): "
        + ", ".join(str(tuple(s)) for s in spec.test_shapes),
        "Benchmark shapes (what you optimise for): "
        + ", ".join(str(tuple(s)) for s in bench_shapes),
    ]
    if best is not None:
        parts += [f"## Best correct kernel so far (attempt {best.iteration})",
                  format_result(best.result), f"```cuda\n{best.code.strip()}\n```"]
    latest = [a for a in history if best is None or a.iteration != best.iteration][-recent:]
    if latest:
        parts.append("## Latest attempts")
        parts += [f"### Attempt {a.iteration}\n{format_result(a.result)}" for a in latest]
        last = history[-1]
        if not last.result.ok and (best is None or last.iteration != best.iteration):
            parts.append(f"Code of attempt {last.iteration} (fix it or try another approach):"
                         f"\n```cuda\n{last.code.strip()}\n```")
    if not history:
        parts.append("## Instructions\nWrite a correct, reasonably fast first version.")
    elif best is None:
        parts.append("## Instructions\nNo correct kernel yet: fix the errors above first; "
                     "correct before fast.")
    else:
        parts.append("## Instructions\nBeat the best kernel above. From the benchmark and "
                     "profiler numbers decide whether it is bound by HBM bandwidth, the "
                     "tensor cores or latency, and attack that limit.")
    return "\n\n".join(parts)


_FENCE = re.compile(r"```([A-Za-z0-9_+\-]*)[ \t]*\n(.*?)```", re.DOTALL)
_TAGS = {"cuda": {"cuda", "cu", "cpp", "c++", "c"}}


def extract_code(text: str, lang: str = "cuda") -> str | None:
    """The candidate source in an answer: the longest block tagged for `lang`, else
    the longest untagged block; None when there is none."""
    blocks = [(tag.lower(), body) for tag, body in _FENCE.findall(text)]
    tagged = [b for t, b in blocks if t in _TAGS[lang]]
    pool = tagged or [b for t, b in blocks if not t]
    code = max(pool, key=len).strip() if pool else ""
    return code or None
