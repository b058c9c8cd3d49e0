"""Candidate-kernel evaluation for the B200 contract, without a GPU: the contract
header compiles for sm_100a on its own, a compiler error is reported as such, code
extraction, the prompt text of the contract, the result record and the sandbox's
time limit (after kernelpilot's tests/cpu/test_agent.py: extraction :35-52, prompts
:81-96, sandbox :166-176)."""

import subprocess
from pathlib import Path

import pytest

from kernelpilot_b200.agent import worker
from kernelpilot_b200.agent.prompts import AttemptView, extract_code, system_prompt, user_prompt
from kernelpilot_b200.agent.result import EvalResult
from kernelpilot_b200.agent.sandbox import run_candidate
from kernelpilot_b200.specs import get_spec

CANDIDATES = Path(__file__).resolve().parent / "candidates"


def ok_result(speedup: float) -> EvalResult:
    return EvalResult(stage="ok", checks_passed=8, bench=[
        {"shape": [4096, 4096], "ms": 1.0 / speedup, "torch_ms": 1.0, "speedup": speedup,
         "gbs": 100.0, "tflops": 0.1, "pct_peak_bw": 30.0, "pct_peak_flops": 1.0}])


def reply(code: str, tag: str = "cuda") -> str:
    return f"Plan: one CTA per row.\n```{tag}\n{code}\n```\n"


# ----------------------------------------------------------------- extraction

def test_extract_code_tagged_and_longest():
    assert extract_code(reply("__global__ void k(){}")) == "__global__ void k(){}"
    text = "```bash\nls\n```\n```cu\nshort\n```\n```cpp\nmuch longer source\n```"
    assert extract_code(text) == "much longer source"


def test_extract_code_untagged_fallback_and_none():
    assert extract_code("```\nkernel\n```") == "kernel"
    assert extract_code("Use shared memory for the row.") is None
    assert extract_code("```python\nprint(1)\n```") is None


# ----------------------------------------------------------------- contract text

def test_system_prompt_states_the_sm100a_contract():
    p = system_prompt(get_spec("layernorm"), "cuda", "bfloat16")
    assert "torch::Tensor kernel_fn(torch::Tensor x0, torch::Tensor x1, torch::Tensor x2)" in p
    assert "sm_100a" in p and "kp_contract.cuh" in p and "getCurrentCUDAStream" in p
    assert "__nv_bfloat16" in p
    assert "warpSize" not in p and "HIP" not in p
    with pytest.raises(ValueError):
        system_prompt(get_spec("softmax"), "hip", "float32")


def test_user_prompt_carries_spec_feedback_and_best():
    spec = get_spec("softmax")
    bad = EvalResult(stage="correctness", error="softmax[candidate] MISMATCH max_abs_err=3.1e-01",
                     checks_passed=3)
    hist = [AttemptView(1, "BEST_CODE", ok_result(1.3)), AttemptView(2, "BROKEN_CODE", bad)]
    p = user_prompt(spec, "cuda", "float32", "NVIDIA B200", hist, hist[0], spec.bench_shapes)
    assert "def softmax_reference" in p
    assert "BEST_CODE" in p and "1.300x" in p
    assert "max_abs_err=3.1e-01" in p and "BROKEN_CODE" in p
    assert "passed 3 smaller shapes" in p
    first = user_prompt(spec, "cuda", "float32", "NVIDIA B200", [], None, spec.bench_shapes)
    assert "first version" in first


# ----------------------------------------------------------------- result record

def test_result_score_is_geometric_mean_and_only_for_ok():
    r = EvalResult(stage="ok", bench=[{"speedup": 2.0}, {"speedup": 8.0}])
    assert r.score == pytest.approx(4.0)
    assert EvalResult(stage="correctness", bench=[{"speedup": 100.0}]).score is None
    d = r.to_dict()
    assert d["score"] == pytest.approx(4.0)
    assert EvalResult.from_dict(d) == r
    with pytest.raises(ValueError):
        EvalResult(stage="finished")


# ----------------------------------------------------------------- worker pieces

def test_arity_and_host_declaration():
    assert worker.arity(get_spec("attention").signature) == 3
    assert worker.host_declaration(2) == "torch::Tensor kernel_fn(torch::Tensor x0, torch::Tensor x1)"


def test_ptxas_resources_parsed():
    log = """ptxas info    : Compiling entry function '_Z3subPKfS0_Pfl' for 'sm_100a'
ptxas info    : Function properties for _Z3subPKfS0_Pfl
    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Used 12 registers, used 0 barriers, 1024 bytes smem, 392 bytes cmem[0]
"""
    (r,) = worker.ptxas_resources(log)
    assert r["arch"] == "sm_100a" and r["registers"] == 12 and r["smem_bytes"] == 1024
    assert r["spill_stores"] == 0 and r["spill_loads"] == 0


def test_contract_header_compiles_for_sm100a(tmp_path):
    # the header stands alone: a kernel using every helper builds for sm_100a only
    src = tmp_path / "probe.cu"
    src.write_text('#include "kp_contract.cuh"\n'
                   "template <typename T> __global__ void k(const T* x, float* out, int n) {\n"
                   "  __shared__ float s[kp::kMaxWarps];\n"
                   "  float v = threadIdx.x < n ? kp::to_float(x[threadIdx.x]) : 0.f;\n"
                   "  v = kp::block_reduce<false>(v, s) + kp::block_reduce<true>(v, s);\n"
                   "  if (threadIdx.x == 0) out[0] = kp::warp_sum(v) + kp::warp_max(v) +\n"
                   "      kp::to_float(kp::from_float<T>(v)) + KP_SHFL_DOWN(v, 1);\n"
                   "}\n"
                   "template __global__ void k<float>(const float*, float*, int);\n"
                   "template __global__ void k<__half>(const __half*, float*, int);\n"
                   "template __global__ void k<__nv_bfloat16>(const __nv_bfloat16*, float*, int);\n"
                   "int launch() { k<float><<<1, 64>>>(nullptr, nullptr, 0); KP_CHECK_LAUNCH();"
                   " return kp::ceil_div(7, 2) + kp::kWarp + kp::kSms; }\n")
    out = subprocess.run(["nvcc", *worker.NVCC_FLAGS, f"-I{worker.CONTRACT_DIR}", "-c", str(src),
                          "-o", str(tmp_path / "probe.o")], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert any(r["arch"] == "sm_100a" for r in worker.ptxas_resources(out.stdout + out.stderr))


def test_compile_error_is_reported_with_compiler_output(tmp_path):
    with pytest.raises(RuntimeError) as e:
        worker.compile_candidate(CANDIDATES / "does_not_compile.cu", 1, tmp_path / "build")
    assert "error" in str(e.value)


# ----------------------------------------------------------------- sandbox

def test_sandbox_reports_missing_gpu_or_rejects_language(tmp_path):
    code = (CANDIDATES / "vector_add_wrong.cu").read_text()
    res = run_candidate(code, "vector_add", "cuda", "float32", timeout_s=180,
                        workdir=tmp_path / "a")
    import torch

    if not torch.cuda.is_available():
        assert res.stage == "crash" and "no GPU" in res.error
    res = run_candidate(code, "vector_add", "hip", "float32", timeout_s=180,
                        workdir=tmp_path / "b")
    assert res.stage == "crash" and "invalid choice" in res.error  # the CLI knows only cuda


def test_sandbox_timeout_ends_the_worker(tmp_path):
    res = run_candidate("x", "vector_add", "cuda", "float32", timeout_s=0.01, workdir=tmp_path)
    assert res.stage == "timeout"
