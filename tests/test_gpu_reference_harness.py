"""The drop-in claim, run as the reference runs it: kernelpilot's own GPU correctness
loop (tests/gpu/test_correctness.py:17-31 there: every ``hip:<stage>`` implementation
its registry lists x ``spec.dtypes`` x ``spec.test_shapes``, each through
``correctness.check_impl``) over the reference's own specs, with this library's
``libkernelpilot_ops.so`` in place of the HIP build. The library is loaded by the
reference's ``ext.load()`` through ``KP_EXT_PATH`` (kernelpilot/ext.py:15-33) and
called through the reference's ``registry._hip_impl`` (kernelpilot/registry.py:41-48),
so nothing of this package stands between the reference harness and the ops."""

import os

import pytest
import torch

from kernelpilot_b200 import ext as our_ext
from kernelpilot_b200 import harness
from kernelpilot_b200.registry import CUDA_STAGES

ref = harness.reference()


def _cases():
    for name, spec in ref.specs.SPECS.items():
        for stage in ref.registry.HIP_STAGES[name]:
            for dtype in spec.dtypes:
                for shape in spec.test_shapes:
                    yield pytest.param(name, f"hip:{stage}", dtype, shape,
                                       id=f"{name}-hip:{stage}-{str(dtype)[6:]}-{shape}",
                                       marks=pytest.mark.gpu)


@pytest.fixture(scope="module")
def reference_with_this_library():
    os.environ["KP_EXT_PATH"] = str(our_ext.LIB_DIR / our_ext.OPS_NAME)
    ref.ext.load.cache_clear()
    assert ref.ext.library_path() == our_ext.LIB_DIR / our_ext.OPS_NAME
    assert ref.ext.load(), "the reference's loader did not load this library"
    yield ref


def test_stage_counts_match_the_reference_registry():
    # a caller indexing the reference's stages reaches a kernel of the same rank here
    for name, stages in ref.registry.HIP_STAGES.items():
        assert len(CUDA_STAGES[name]) == len(stages), name


@pytest.mark.parametrize("kernel,impl,dtype,shape", list(_cases()))
def test_reference_correctness_loop_passes(reference_with_this_library, kernel, impl, dtype,
                                           shape):
    r = reference_with_this_library
    spec = r.specs.SPECS[kernel]
    fn = r.registry.get_impls(kernel, include=("hip",))[impl]
    res = r.correctness.check_impl(spec, impl, fn, shape, dtype, "cuda")
    assert res.ok, res.summary()


@pytest.mark.gpu
def test_reference_bench_one_times_this_library(reference_with_this_library):
    # the reference's benchmark entry point on one bench shape per op, verified first
    r = reference_with_this_library
    gpu = harness.gpu_info()
    for name, spec in r.specs.SPECS.items():
        best = f"hip:{r.registry.HIP_STAGES[name][-1]}"
        fn = r.registry.get_impls(name, include=("hip",))[best]
        res = r.benchmark.bench_one(spec, best, fn, spec.bench_shapes[0], torch.float16, gpu,
                                    warmup=2, iters=5)
        assert res.correct and res.ms and res.ms > 0, (name, res.note)
