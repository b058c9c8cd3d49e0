"""CPU tests of the harness mirror (kernelpilot tests/cpu/test_harness.py and
test_roofline.py): the comparator must catch wrong answers, NaNs, shape/dtype
mismatches and in-place mutation; specs stay consistent; peaks resolve."""

import math

import pytest
import torch

from kernelpilot_b200.benchmark import BenchResult, load_results, save_results, to_markdown
from kernelpilot_b200.correctness import KernelMismatch, check_chunked, check_impl, compare
from kernelpilot_b200.device import GPUInfo, lookup_peaks, measured_peaks
from kernelpilot_b200.specs import CONFIGS, SPECS, get_spec


def test_compare_exact():
    x = torch.randn(100)
    info = compare(x, x.clone(), 1e-6, 1e-6)
    assert info["num_mismatched"] == 0 and info["max_abs_err"] == 0


def test_compare_reports_worst_element():
    ref = torch.zeros(4, 5)
    out = ref.clone()
    out[2, 3] = 1.0
    info = compare(out, ref, 1e-3, 1e-3)
    assert info["num_mismatched"] == 1
    assert info["worst_index"] == (2, 3)
    assert info["max_abs_err"] == pytest.approx(1.0)


def test_compare_nan_is_error():
    assert compare(torch.tensor([1.0, float("nan"), 1.0]), torch.ones(3), 1e-3, 1e-3)[
        "num_mismatched"] == 1


def test_compare_matching_inf_is_ok():
    ref = torch.tensor([float("inf"), 1.0])
    assert compare(ref.clone(), ref, 0, 0)["num_mismatched"] == 0


def test_compare_shape_mismatch_raises():
    with pytest.raises(KernelMismatch):
        compare(torch.zeros(3), torch.zeros(4), 1, 1)


@pytest.mark.parametrize("name", list(SPECS))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_torch_baseline_passes_on_cpu(name, dtype):
    spec = get_spec(name)
    shape = spec.test_shapes[min(2, len(spec.test_shapes) - 1)]
    res = check_impl(spec, "torch", spec.baseline, shape, dtype, "cpu")
    assert res.ok, res.summary()


@pytest.mark.parametrize("name", list(SPECS))
def test_wrong_kernel_is_caught(name):
    spec = get_spec(name)
    shape = spec.test_shapes[min(2, len(spec.test_shapes) - 1)]

    def wrong(*xs):
        out = spec.baseline(*xs).clone()
        out.view(-1)[0] += 1.0
        return out

    res = check_impl(spec, "wrong", wrong, shape, torch.float32, "cpu")
    assert not res.ok
    assert "MISMATCH" in res.summary() and "max_abs_err" in res.summary()


def test_inplace_mutation_is_caught():
    spec = get_spec("softmax")

    def mutating(x):
        x.mul_(2)
        return torch.softmax(x, -1)

    res = check_impl(spec, "mut", mutating, (4, 16), torch.float32, "cpu")
    assert not res.ok and "in place" in res.error


def test_wrong_dtype_is_caught():
    spec = get_spec("softmax")
    res = check_impl(spec, "f32", lambda x: torch.softmax(x.float(), -1), (4, 16),
                     torch.float16, "cpu")
    assert not res.ok and "dtype" in res.error


def test_crash_is_reported_not_raised():
    spec = get_spec("softmax")

    def boom(x):
        raise RuntimeError("illegal memory access")

    res = check_impl(spec, "boom", boom, (4, 16), torch.float32, "cpu")
    assert not res.ok and "illegal memory access" in res.error


def test_peak_lookup():
    assert lookup_peaks("Tesla T4") == (320.0, 8.1, 65.0)
    assert lookup_peaks("NVIDIA L40S") is None
    assert lookup_peaks("NVIDIA H100 PCIe")[0] == 2000.0
    assert lookup_peaks("NVIDIA B200")[0] == 7700.0


def test_bf16_peak_is_not_the_fp32_peak():
    g = GPUInfo("NVIDIA B200", "nvidia", 7700.0,
                {"float32": 75.0, "float16": 2250.0, "bfloat16": 2250.0})
    assert g.peak_for(torch.bfloat16) == 2250.0 and g.peak_for(torch.float32) == 75.0


def test_measured_peaks_file_parses(tmp_path):
    p = tmp_path / "MEASURED_PEAKS.json"
    p.write_text('{"hbm_gbs": 6553.9, "bf16_tflops": 1651.9, "gpu_name": "NVIDIA B200"}')
    assert measured_peaks(p)["hbm_gbs"] == 6553.9
    assert measured_peaks(tmp_path / "missing.json") is None


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


@pytest.mark.parametrize("name", ["softmax", "matmul", "attention", "attention_causal",
                                  "reduce_sum"])
def test_chunked_check_agrees_with_check_impl(name):
    spec = get_spec(name)
    shape = spec.test_shapes[3]
    inputs = spec.make_inputs(shape, torch.float32, torch.device("cpu"), 0)
    out = spec.baseline(*inputs)
    res = check_chunked(spec, "torch", inputs, out, shape, torch.float32, elems_per_chunk=64)
    assert res.ok, res.summary()
    bad = out.clone()
    bad.view(-1)[-1] += 1.0
    res = check_chunked(spec, "bad", inputs, bad, shape, torch.float32, elems_per_chunk=64)
    assert not res.ok and res.num_mismatched == 1


def _fake_results():
    return [
        BenchResult("softmax", "torch", "float32", (4096, 4097), ms=0.05, gbs=2600,
                    tflops=1.6, arithmetic_intensity=0.6),
        BenchResult("matmul", "cuda:tcgen05", "bfloat16", (8192, 8192, 8192), ms=0.9,
                    gbs=440, tflops=1200, arithmetic_intensity=2731),
        BenchResult("softmax", "cuda:thread_row", "float32", (4096, 4096), ms=None,
                    correct=False),
    ]


def test_results_roundtrip_and_markdown(tmp_path):
    gpu = GPUInfo(name="Fake GPU", vendor="nvidia", peak_bw_gbs=300.0,
                  peak_tflops={"float32": 8.0, "float16": 65.0}, source="test")
    save_results(_fake_results(), gpu, tmp_path)
    g2, results = load_results(tmp_path / "bench.json")
    assert g2.name == "Fake GPU" and len(results) == 3
    md = to_markdown(results, g2)
    assert "FAILED correctness" in md and "### matmul" in md
