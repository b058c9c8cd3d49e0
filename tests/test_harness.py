"""CPU tests of the harness layer: the reference's own harness (kernelpilot's
correctness/benchmark/device modules, loaded unchanged) drives this library's specs,
the specs agree with the reference's on everything they share, and the pieces this
library adds (check_on_inputs, check_chunked, B200 peaks) behave like the reference's
gate."""

import math

import pytest
import torch

from kernelpilot_b200 import harness
from kernelpilot_b200.specs import CONFIGS, SPECS, get_spec

ref = harness.reference()


def test_reference_harness_is_the_installed_package():
    assert ref.correctness.__file__.startswith(str(harness.reference_root()))
    assert harness.compare.__module__ == "kernelpilot_b200.harness"
    # the functions the tests and bench use are the reference's own objects
    x = torch.randn(10)
    assert harness.compare(x, x.clone(), 0, 0) == ref.correctness.compare(x, x.clone(), 0, 0)


# ---------------------------------------------------------------- specs vs the reference

SHARED = ["vector_add", "reduce_sum", "softmax", "matmul", "layernorm", "attention"]


@pytest.mark.parametrize("name", SHARED)
def test_specs_match_the_reference_on_shared_dtypes(name):
    mine, theirs = get_spec(name), ref.specs.get_spec(name)
    assert mine.name == theirs.name and mine.shape_names == theirs.shape_names
    assert mine.test_shapes == theirs.test_shapes
    assert mine.bench_shapes == theirs.bench_shapes
    assert set(theirs.dtypes) <= set(mine.dtypes)
    assert torch.bfloat16 in mine.dtypes  # the one additive dtype
    for dtype in theirs.dtypes:
        assert mine.output_dtype(dtype) == theirs.output_dtype(dtype)
        for shape in mine.test_shapes + mine.bench_shapes:
            assert mine.flops(shape) == theirs.flops(shape)
            assert mine.bytes_moved(shape, dtype) == theirs.bytes_moved(shape, dtype)
            t0, t1 = mine.tolerance(shape, dtype), theirs.tolerance(shape, dtype)
            assert (t0.atol, t0.rtol) == (t1.atol, t1.rtol)


@pytest.mark.parametrize("name", SHARED)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_generators_and_references_match_the_reference(name, dtype):
    mine, theirs = get_spec(name), ref.specs.get_spec(name)
    shape = mine.test_shapes[min(2, len(mine.test_shapes) - 1)]
    a = mine.make_inputs(shape, dtype, torch.device("cpu"), 3)
    b = theirs.make_inputs(shape, dtype, torch.device("cpu"), 3)
    assert all(torch.equal(x, y) for x, y in zip(a, b, strict=True))
    assert torch.equal(mine.reference(*a), theirs.reference(*a))


def test_bf16_tolerances_take_the_reference_non_fp32_branch():
    for name in ("reduce_sum", "softmax", "matmul", "layernorm", "attention"):
        mine = get_spec(name)
        for shape in mine.test_shapes:
            assert mine.tolerance(shape, torch.bfloat16) == mine.tolerance(shape, torch.float16)
    # the one deliberate widening: one bf16 rounding of a sum is up to 2^-9 relative
    assert get_spec("vector_add").tolerance((7,), torch.bfloat16).rtol == 4e-3


# ---------------------------------------------------------------- the reference gate on our specs

@pytest.mark.parametrize("name", list(SPECS))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_torch_baseline_passes_the_reference_gate_on_cpu(name, dtype):
    spec = get_spec(name)
    shape = spec.test_shapes[min(2, len(spec.test_shapes) - 1)]
    res = harness.check_impl(spec, "torch", spec.baseline, shape, dtype, "cpu")
    assert res.ok, res.summary()


@pytest.mark.parametrize("name", list(SPECS))
def test_reference_gate_catches_a_wrong_kernel(name):
    spec = get_spec(name)
    shape = spec.test_shapes[min(2, len(spec.test_shapes) - 1)]

    def wrong(*xs):
        out = spec.baseline(*xs).clone()
        out.view(-1)[0] += 1.0
        return out

    res = harness.check_impl(spec, "wrong", wrong, shape, torch.float32, "cpu")
    assert not res.ok
    assert "MISMATCH" in res.summary() and "max_abs_err" in res.summary()


def test_check_on_inputs_uses_the_given_tensors():
    spec = get_spec("reduce_sum")
    x = torch.full((1000,), 0.5)
    seen = []

    def fn(t):
        seen.append(t)
        return t.sum(dtype=torch.float32)

    res = harness.check_on_inputs(spec, "torch", fn, (x,), (1000,), torch.float32)
    assert res.ok and seen[0] is x
    res = harness.check_on_inputs(spec, "off", lambda t: t.sum() + 1, (x,), (1000,),
                                  torch.float32)
    assert not res.ok
    res = harness.check_on_inputs(spec, "mut", lambda t: t.mul_(2).sum(), (x.clone(),), (1000,),
                                  torch.float32)
    assert not res.ok and "in place" in res.error


@pytest.mark.parametrize("name", ["softmax", "matmul", "attention", "attention_causal",
                                  "reduce_sum", "layernorm", "vector_add"])
def test_chunked_check_agrees_with_check_impl(name):
    spec = get_spec(name)
    shape = spec.test_shapes[3]
    inputs = spec.make_inputs(shape, torch.float32, torch.device("cpu"), 0)
    out = spec.baseline(*inputs)
    res = harness.check_chunked(spec, "torch", inputs, out, shape, torch.float32,
                                elems_per_chunk=64)
    assert res.ok, res.summary()
    bad = out.clone()
    bad.view(-1)[-1] += 1.0
    res = harness.check_chunked(spec, "bad", inputs, bad, shape, torch.float32,
                                elems_per_chunk=64)
    assert not res.ok and res.num_mismatched == 1
    # the worst element is reported by its index in the whole output
    if out.dim():
        assert res.worst_index == tuple(int(i) for i in torch.unravel_index(
            torch.tensor(out.numel() - 1), out.shape))


def test_chunked_check_rejects_the_wrong_dtype():
    spec = get_spec("softmax")
    x = torch.randn(4, 16)
    res = harness.check_chunked(spec, "f64", (x,), torch.softmax(x.double(), -1), (4, 16),
                                torch.float32)
    assert not res.ok and "dtype" in res.error


# ---------------------------------------------------------------- peaks

def test_b200_peaks_know_bf16(tmp_path, monkeypatch):
    for var in ("KP_PEAK_BW_GBS", "KP_PEAK_FP32_TFLOPS", "KP_PEAK_FP16_TFLOPS",
                "KP_PEAK_BF16_TFLOPS"):
        monkeypatch.delenv(var, raising=False)
    info = harness.b200_info(measured_path=tmp_path / "missing.json")
    assert info.source == "datasheet" and info.peak_bw_gbs == 7700.0
    assert info.peak_for(torch.bfloat16) == 2250.0 and info.peak_for(torch.float32) == 75.0
    # the reference's own class would give bf16 the fp32 CUDA-core peak
    plain = ref.device.GPUInfo("x", "nvidia", 1.0, {"float32": 75.0, "float16": 2250.0})
    assert plain.peak_for(torch.bfloat16) == 75.0
    p = tmp_path / "MEASURED_PEAKS.json"
    p.write_text('{"hbm_gbs": 6448.7, "bf16_tflops": 1676.2, "gpu_name": "NVIDIA B200"}')
    info = harness.b200_info(measured_path=p)
    assert info.peak_bw_gbs == 6448.7 and info.peak_for(torch.bfloat16) == 1676.2
    monkeypatch.setenv("KP_PEAK_BF16_TFLOPS", "1000")
    assert harness.b200_info(measured_path=p).peak_for(torch.bfloat16) == 1000.0


def test_reference_benchmark_rows_accept_the_b200_info():
    # bench_one's report path: rates and % of peak from our spec and the B200 peaks
    info = harness.b200_info()
    r = ref.benchmark.BenchResult("softmax", "cuda:staged_tma", "bfloat16", (8, 8), ms=1.0)
    md = ref.benchmark.to_markdown([r], info)
    assert "B200" in md and "### softmax" in md


# ---------------------------------------------------------------- headline workloads

@pytest.mark.parametrize("name", list(SPECS))
def test_specs_are_consistent(name):
    spec = get_spec(name)
    for shape in spec.test_shapes + spec.bench_shapes:
        assert len(shape) == len(spec.shape_names)
    for shape in spec.bench_shapes:
        for dt in spec.dtypes:
            assert spec.flops(shape) > 0 and spec.bytes_moved(shape, dt) > 0


def test_headline_configs_work_per_spec_formulas():
    w = CONFIGS["softmax_f32_4096x4097"]
    assert w.spec.bytes_moved(w.shape, w.dtype) == 134_250_496
    w = CONFIGS["reduce_f32_2p28p1"]
    assert w.spec.bytes_moved(w.shape, w.dtype) == 1_073_741_832
    w = CONFIGS["gemm_bf16_8192"]
    assert w.spec.flops(w.shape) == pytest.approx(1.0995e12, rel=1e-4)
    w = CONFIGS["attn_bf16_b8h32s4096d128"]
    assert w.spec.flops(w.shape) == pytest.approx(2.1990e12, rel=1e-4)
    wc = CONFIGS["attn_causal_bf16_b8h32s4096d128"]
    assert wc.spec.flops(wc.shape) == pytest.approx(w.spec.flops(w.shape) / 2, rel=1e-3)


def test_config_generators_have_the_stated_distributions():
    (x,) = CONFIGS["reduce_f32_2p28p1"].make_inputs((100000,), torch.float32, "cpu", 0)
    assert x.min() >= -1 and x.max() <= 1 and abs(float(x.mean())) < 0.02
    a, b = CONFIGS["gemm_bf16_8192"].make_inputs((64, 64, 4096), torch.float32, "cpu", 0)
    assert float(a.std()) == pytest.approx(1 / math.sqrt(4096), rel=0.05)
