"""The CPU oracle, pinned against the reference: every function reproduces the
reference's float64 outputs stored in tests/golden (made by make_golden.py from the
reference package itself), and the comparator reproduces the reference harness's
known-answer cases (kernelpilot tests/cpu/test_harness.py:12-41)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
OPS = ["vector_add", "reduce_sum", "softmax", "matmul", "layernorm", "attention",
       "attention_causal"]


def golden_cases(op: str):
    blob = np.load(GOLDEN / f"{op}.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in blob.files})
    for key in keys:
        dtype, shape_s = key.split("|")
        shape = tuple(int(s) for s in shape_s.split(","))
        n_in = sum(1 for k in blob.files if k.startswith(key + "|in"))
        inputs = [blob[f"{key}|in{i}"] for i in range(n_in)]
        yield dtype, shape, inputs, blob[f"{key}|out"]


@pytest.mark.parametrize("op", OPS)
def test_oracle_matches_reference_golden(op):
    n = 0
    for dtype, shape, inputs, want in golden_cases(op):
        got = oracle.run(op, inputs, dtype)
        assert got.shape == want.shape, (op, dtype, shape)
        # float64 vs float64: only summation order differs
        np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12,
                                   err_msg=f"{op} {dtype} {shape}")
        n += 1
    assert n >= 15


def test_bf16_bits_roundtrip_matches_torch():
    x = torch.randn(4096) * 100
    x[:4] = torch.tensor([0.0, -0.0, float("inf"), -float("inf")])
    ours = oracle.f32_to_bf16_bits(x.numpy())
    theirs = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)
    back = oracle.bf16_bits_to_f32(ours)
    assert np.array_equal(back, x.to(torch.bfloat16).float().numpy())


def test_compare_exact():
    x = np.random.default_rng(0).standard_normal(100)
    info = oracle.compare(x, x.copy(), 1e-6, 1e-6)
    assert info["num_mismatched"] == 0 and info["max_abs_err"] == 0


def test_compare_reports_worst_element():
    ref = np.zeros((4, 5))
    out = ref.copy()
    out[2, 3] = 1.0
    info = oracle.compare(out, ref, 1e-3, 1e-3)
    assert info["num_mismatched"] == 1 and info["worst_index"] == (2, 3)
    assert info["max_abs_err"] == pytest.approx(1.0)


def test_compare_nan_is_error_and_matching_inf_is_ok():
    assert oracle.compare(np.array([1.0, np.nan, 1.0]), np.ones(3), 1e-3, 1e-3)[
        "num_mismatched"] == 1
    ref = np.array([np.inf, 1.0])
    assert oracle.compare(ref.copy(), ref, 0, 0)["num_mismatched"] == 0


def test_compare_shape_mismatch_raises():
    with pytest.raises(ValueError):
        oracle.compare(np.zeros(3), np.zeros(4), 1, 1)


@pytest.mark.parametrize("op", OPS)
def test_planted_error_is_caught(op):
    """A single wrong element in an otherwise exact answer fails the tolerance test."""
    dtype, shape, inputs, want = next(iter(golden_cases(op)))
    atol, rtol = oracle.tolerance(op, shape, "float32")
    bad = np.array(want, dtype=np.float64, copy=True)
    bad.reshape(-1)[0] += 1.0
    assert oracle.compare(bad, want, atol, rtol)["num_mismatched"] == 1


def test_tolerances_match_spec():
    from kernelpilot_b200.specs import get_spec
    for op, shape in [("reduce_sum", (65537,)), ("softmax", (3, 7)), ("matmul", (4, 5, 4096)),
                      ("attention", (1, 2, 7, 32)), ("attention_causal", (1, 2, 7, 32))]:
        spec = get_spec(op)
        for dt in spec.dtypes:
            t = spec.tolerance(shape, dt)
            assert oracle.tolerance(op, shape, str(dt)[6:]) == (t.atol, t.rtol)


def test_oracle_agrees_with_spec_reference_on_fresh_inputs():
    from kernelpilot_b200.specs import SPECS
    for name, spec in SPECS.items():
        shape = spec.test_shapes[2]
        inputs = spec.make_inputs(shape, torch.float32, torch.device("cpu"), 7)
        want = spec.reference(*inputs).numpy()
        got = oracle.run(name, [t.numpy() for t in inputs], "float32")
        np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)
