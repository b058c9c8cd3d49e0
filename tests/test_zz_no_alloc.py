"""kpb_reduce_sum_noalloc, the full sum for callers that may not allocate device
memory when they call (fixed start-up budgets, memory owned by another allocator,
runtimes that forbid allocation after initialisation): called through the C ABI, its
result must be identical, bit for bit, to the allocating entry point kpb_reduce_sum's
(both run the same kernels and add the partials in the same fixed order), on two calls
in a row with different inputs: the built-in scratch keeps the previous call's
partials, so a stale or overlapping partial would show up in the second call. The
results are also within the reduction's tolerance of the float64 sum.

This file sorts last so that a run stopping at the first failure has already run every
other test; it also passes alone in a fresh process.
"""

import pytest
import torch

from kernelpilot_b200 import ext
from kernelpilot_b200.specs import get_spec

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,n", [(torch.float32, 2**28 + 1), (torch.bfloat16, 3_000_001),
                                     (torch.float16, 1000), (torch.float32, 7)])
def test_noalloc_matches_allocating_entry_point_twice(dtype, n):
    lib = ext.capi()
    spec = get_spec("reduce_sum")
    code = ext.DTYPE_CODES[dtype]
    dev = torch.device("cuda")
    tol = spec.tolerance((n,), dtype)
    first = spec.make_inputs((n,), dtype, dev, 0)[0]
    second = spec.make_inputs((n,), dtype, dev, 1)[0] * 3
    for x in (first, second):
        stream = ext.current_stream_ptr()
        want = torch.empty((), device=dev)
        ext.capi_check(lib.kpb_reduce_sum(2, code, x.data_ptr(), want.data_ptr(), n, stream))
        got = torch.full((), float("nan"), device=dev)
        ext.capi_check(lib.kpb_reduce_sum_noalloc(code, x.data_ptr(), got.data_ptr(), n,
                                                  stream))
        torch.cuda.synchronize()
        assert torch.equal(got, want), (str(dtype), n, float(got), float(want))
        exact = float(x.double().sum())
        assert abs(float(got) - exact) <= tol.atol + tol.rtol * abs(exact)


def test_noalloc_rejects_bad_arguments():
    lib = ext.capi()
    assert lib.kpb_reduce_sum_noalloc(7, None, None, 10, None) == 1
    assert b"dtype" in lib.kpb_last_error()
    assert lib.kpb_reduce_sum_noalloc(0, None, None, -1, None) == 1
