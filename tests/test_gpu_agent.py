"""Candidate kernels through the sandboxed worker on a B200: a correct candidate is
compiled for sm_100a, passes every correctness shape of its spec and is benchmarked
against the PyTorch built-in; a candidate that computes the wrong thing is stopped at
the correctness stage (kernelpilot/agent/worker.py:99-186 stage order)."""

from pathlib import Path

import pytest

from kernelpilot_b200.agent.sandbox import run_candidate
from kernelpilot_b200.specs import get_spec

pytestmark = pytest.mark.gpu

CANDIDATES = Path(__file__).resolve().parent / "candidates"


def test_correct_candidate_is_benchmarked(tmp_path):
    res = run_candidate((CANDIDATES / "softmax_block_row.cu").read_text(), "softmax", "cuda",
                        "bfloat16", timeout_s=600, bench_shapes=[(1024, 4096)], workdir=tmp_path)
    assert res.stage == "ok", f"{res.stage}: {res.error}\n{res.compile_log[-2000:]}"
    assert res.checks_passed == len(get_spec("softmax").test_shapes)
    (row,) = res.bench
    assert row["shape"] == [1024, 4096] and row["ms"] > 0 and row["speedup"] > 0
    assert res.score is not None
    kernels = [r["kernel"] for r in res.profile["ptxas"]]
    assert any("softmax_rows" in k for k in kernels)
    assert all(r["arch"] == "sm_100a" for r in res.profile["ptxas"])
    assert any("softmax_rows" in k["name"] for k in res.profile["gpu_kernels"])


def test_wrong_candidate_is_rejected(tmp_path):
    res = run_candidate((CANDIDATES / "vector_add_wrong.cu").read_text(), "vector_add", "cuda",
                        "float32", timeout_s=600, workdir=tmp_path)
    assert res.stage == "correctness", f"{res.stage}: {res.error}"
    assert res.score is None and not res.bench
    assert "MISMATCH" in res.error or "mismatch" in res.error.lower()
