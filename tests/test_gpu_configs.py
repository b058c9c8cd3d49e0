"""Parity at the headline workloads' full sizes: the B200 kernel on each
configuration's own seeded generator, checked element by element against the float64
reference (evaluated in row / head blocks so the reference fits in memory), plus the
size-independent properties each op has (softmax rows sum to one, LayerNorm rows
are standardised before the affine step, the reduction is linear in its input)."""

from __future__ import annotations

import pytest
import torch

from kernelpilot_b200 import registry
from kernelpilot_b200.harness import check_chunked
from kernelpilot_b200.specs import CONFIGS

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("key", list(CONFIGS))
def test_headline_workload_full_size(key):
    w = CONFIGS[key]
    inputs = w.inputs("cuda", seed=0)
    out = registry.best(w.kernel)(*inputs)
    torch.cuda.synchronize()
    res = check_chunked(w.spec, "best", inputs, out, w.shape, w.dtype)
    assert res.ok, res.summary()
    if w.kernel == "softmax":
        rows = out.float().sum(-1)
        tol = 1e-4 if w.dtype == torch.float32 else 2e-2
        assert float((rows - 1).abs().max()) < tol
    if w.kernel == "layernorm":
        # (y - b) / w has zero mean and unit (biased) variance in every row
        x, wt, bs = inputs
        z = (out.double() - bs.double()) / wt.double()
        tol = 1e-4 if w.dtype == torch.float32 else 5e-2
        assert float(z.mean(-1).abs().max()) < tol
        assert float((z.var(-1, unbiased=False) - 1).abs().max()) < 2 * tol
    del inputs, out
    torch.cuda.empty_cache()


def test_reduce_is_linear_at_full_size():
    w = CONFIGS["reduce_f32_2p28p1"]
    (x,) = w.inputs("cuda", seed=1)
    fn = registry.best("reduce_sum")
    s1 = float(fn(x))
    # halves summed separately add up to the whole (up to fp32 rounding)
    h = x.numel() // 2
    s2 = float(fn(x[:h].contiguous())) + float(fn(x[h:].contiguous()))
    assert abs(s1 - s2) < 1e-5 * x.numel() ** 0.5 + 1e-5
    # scaling by 2 is exact in binary floating point
    assert float(fn(x * 2)) == pytest.approx(2 * s1, abs=1e-6)
