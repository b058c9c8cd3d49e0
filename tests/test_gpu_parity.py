"""Parity of the sm_100a kernels with the float64 reference, on a GPU.

* every registered implementation x dtype x spec test shape through ``check_impl``
  (the reference's own gate, kernelpilot tests/gpu/test_correctness.py:17-31);
* the reference's golden vectors (tests/golden, made from the reference package)
  uploaded to the GPU, for every CUDA variant;
* B200-specific edges: rows that do not start on a 16-byte boundary, rows longer
  than one CTA holds, misaligned reduction inputs, GEMM shapes whose B rows are not
  16-byte aligned, partial tiles;
* the C ABI called directly with raw device pointers (ctypes);
* determinism of the reduction, and no kernel wait ever timing out.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from kernelpilot_b200 import ext, registry
from kernelpilot_b200.harness import check_impl, check_on_inputs, compare
from kernelpilot_b200.specs import SPECS, get_spec

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cases():
    for name, spec in SPECS.items():
        for impl in ["torch"] + [f"cuda:{s}" for s in registry.CUDA_STAGES[name]]:
            for dtype in spec.dtypes:
                for shape in spec.test_shapes:
                    yield pytest.param(name, impl, dtype, shape,
                                       id=f"{name}-{impl}-{str(dtype)[6:]}-{shape}")


def test_extension_built_and_in_tree():
    assert ext.load(), "extension missing: run python -m kernelpilot_b200.build"
    assert ext.library_path().parent == ext.LIB_DIR


@pytest.mark.parametrize("kernel,impl,dtype,shape", list(_cases()))
def test_kernel_matches_reference(kernel, impl, dtype, shape):
    spec = SPECS[kernel]
    fn = registry.get_impls(kernel)[impl]
    res = check_impl(spec, impl, fn, shape, dtype, "cuda")
    assert res.ok, res.summary()


# ------------------------------------------------------------------ golden vectors

def _golden(op):
    blob = np.load(GOLDEN / f"{op}.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in blob.files})
    for key in keys:
        dtype, shape_s = key.split("|")
        shape = tuple(int(s) for s in shape_s.split(","))
        n_in = sum(1 for k in blob.files if k.startswith(key + "|in"))
        yield dtype, shape, [blob[f"{key}|in{i}"] for i in range(n_in)], blob[f"{key}|out"]


def _to_device(a: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "bfloat16":
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(a.copy()).cuda()


@pytest.mark.parametrize("op", list(SPECS))
def test_golden_vectors_every_variant(op):
    spec = get_spec(op)
    for variant, stage in enumerate(registry.CUDA_STAGES[op]):
        fn = registry.get_impls(op)[f"cuda:{stage}"]
        for dtype, shape, ins, want in _golden(op):
            xs = [_to_device(a, dtype) for a in ins]
            out = fn(*xs)
            torch.cuda.synchronize()
            tol = spec.tolerance(shape, getattr(torch, dtype))
            info = compare(out.cpu(), torch.from_numpy(want), tol.atol, tol.rtol)
            assert info["num_mismatched"] == 0, (op, stage, dtype, shape, info)


# ------------------------------------------------------------------ B200 edges

EDGE = [
    ("softmax", (33, 4097), torch.float32),      # rows start at 4-byte offsets
    ("softmax", (7, 24577), torch.float32),      # just past one CTA's registers -> cluster of 2
    ("softmax", (3, 100003), torch.float32),     # long misaligned rows, cluster of 8
    ("softmax", (9, 32768), torch.bfloat16),     # staged, 4 vectors per thread
    ("softmax", (5, 32769), torch.bfloat16),     # cluster of 2, misaligned
    ("softmax", (64, 131072), torch.bfloat16),   # cluster of 4, aligned
    ("softmax", (64, 65537), torch.float32),     # cluster of 4, rows at 4-byte offsets
    ("softmax", (33, 100000), torch.float16),    # cluster of 4, 8 rows per cluster pass
    ("softmax", (7, 196608), torch.float32),     # cluster of 8, exactly full
    ("softmax", (3, 196609), torch.float32),     # one value past 8 CTAs -> two-pass
    ("softmax", (5, 262144), torch.bfloat16),    # cluster of 8, 16-bit limit
    ("softmax", (2, 262153), torch.bfloat16),    # past it, misaligned -> two-pass
    ("softmax", (1000, 40000), torch.bfloat16),  # more rows than resident clusters
    ("softmax", (300, 4095), torch.float16),     # odd rows, many CTAs per SM
    ("softmax", (1500, 1), torch.float32),       # one element per row
    ("layernorm", (33, 4097), torch.float32),    # rows at 4-byte offsets -> block per row
    ("layernorm", (7, 32768), torch.float32),    # longest fp32 row held in registers
    ("layernorm", (3, 32772), torch.float32),    # one vector past it -> block per row
    ("layernorm", (9, 32768), torch.bfloat16),   # 16 warps x 8 vectors per row
    ("layernorm", (5, 65536), torch.bfloat16),   # 32 warps x 8 vectors per row
    ("layernorm", (5, 32769), torch.bfloat16),   # block per row, misaligned
    ("layernorm", (300, 4095), torch.float16),   # odd rows
    ("layernorm", (1500, 1), torch.float32),     # one element per row: y = b
    ("layernorm", (1000, 8), torch.bfloat16),    # one vector per row, 8 rows per warp group
    ("layernorm", (4096, 4096), torch.bfloat16), # two rows per CTA
    ("vector_add", (2**24 + 3,), torch.float32),
    ("vector_add", (5_000_011,), torch.bfloat16),
    ("reduce_sum", (2**24 + 3,), torch.float32),
    ("reduce_sum", (5_000_011,), torch.bfloat16),
    ("matmul", (4097, 264, 256), torch.bfloat16),
    ("matmul", (300, 4097, 192), torch.bfloat16),  # B rows not 16-byte aligned
    ("matmul", (129, 257, 72), torch.float16),
    ("matmul", (512, 512, 4104), torch.bfloat16),
    # ragged M and N (N % 256 = 208), long K
    ("matmul", (1000, 2000, 3000), torch.bfloat16),
    # one-column and one-row edge tiles, B rows not 16-byte aligned, several tile waves
    ("matmul", (2049, 4097, 2048), torch.bfloat16),
    # ragged everything in fp16 (N % 256 = 76, K % 64 = 8)
    ("matmul", (777, 1100, 5000), torch.float16),
    # A rows not 16-byte aligned (K % 8 = 7): A staged alone, then A and B both staged
    ("matmul", (256, 512, 999), torch.float16),
    ("matmul", (300, 500, 1001), torch.bfloat16),
    # B rows not 16-byte aligned with one 128-row block (pitch copy of B) and with a
    # ragged K under several pair-tile waves (B rows staged by the GEMM itself)
    ("matmul", (100, 4097, 300), torch.bfloat16),
    ("matmul", (640, 3001, 1000), torch.float16),
    ("attention", (2, 3, 300, 128), torch.bfloat16),
    ("attention", (1, 4, 513, 64), torch.float16),
    ("attention_causal", (2, 3, 300, 128), torch.bfloat16),
    ("attention_causal", (1, 2, 1000, 64), torch.bfloat16),
    # D = 128: a single query, ragged S (partial K/V and query tiles), and many heads
    ("attention", (1, 1, 1, 128), torch.bfloat16),
    ("attention", (1, 2, 129, 128), torch.float16),
    ("attention", (3, 40, 384, 128), torch.bfloat16),
    ("attention_causal", (1, 3, 257, 128), torch.float16),
    ("attention_causal", (2, 40, 640, 128), torch.bfloat16),
]


@pytest.mark.parametrize("kernel,shape,dtype", EDGE,
                         ids=[f"{k}-{s}-{str(d)[6:]}" for k, s, d in EDGE])
def test_edge_shapes_best_variant(kernel, shape, dtype):
    res = check_impl(get_spec(kernel), "best", registry.best(kernel), shape, dtype, "cuda")
    assert res.ok, res.summary()


@pytest.mark.parametrize("a_off,b_off", [(1, 0), (0, 3), (5, 2)])
def test_matmul_misaligned_bases(a_off, b_off):
    # a base off a 16-byte boundary cannot be a TMA base: that operand is staged
    spec = get_spec("matmul")
    dev = torch.device("cuda")
    M, N, K = 384, 520, 640
    a0, b0 = spec.make_inputs((M + 1, N + 1, K + 1), torch.bfloat16, dev, 0)
    a = a0.flatten()[a_off:a_off + M * K].view(M, K)
    b = b0.flatten()[b_off:b_off + K * N].view(K, N)
    res = check_on_inputs(spec, "best", registry.best("matmul"), (a, b), (M, N, K),
                          torch.bfloat16)
    assert res.ok, res.summary()


@pytest.mark.parametrize("offset", [1, 2, 3])
def test_reduce_misaligned_input(offset):
    spec = get_spec("reduce_sum")
    base = spec.make_inputs((1_000_003,), torch.float32, torch.device("cuda"), 0)[0]
    x = base[offset:]
    assert x.data_ptr() % 16 != 0
    res = check_on_inputs(spec, "best", registry.best("reduce_sum"), (x,), (x.numel(),),
                          torch.float32)
    assert res.ok, res.summary()


@pytest.mark.parametrize("offset", [1, 3])
def test_softmax_misaligned_base(offset):
    spec = get_spec("softmax")
    flat = spec.make_inputs((64 * 1000 + offset,), torch.float32, torch.device("cuda"), 0)[0]
    x = flat[offset:].view(64, 1000)
    res = check_on_inputs(spec, "best", registry.best("softmax"), (x,), (64, 1000),
                          torch.float32)
    assert res.ok, res.summary()


@pytest.mark.parametrize("offsets", [(1, 1, 1), (1, 2, 3), (0, 0, 5), (3, 0, 0)])
def test_vector_add_misaligned(offsets):
    # equal offsets share a vector grid (scalar head + vector body); unequal ones do not
    spec = get_spec("vector_add")
    n = 1_000_003
    a0, b0 = spec.make_inputs((n + 8,), torch.float16, torch.device("cuda"), 0)
    a, b = a0[offsets[0]:offsets[0] + n], b0[offsets[1]:offsets[1] + n]
    c0 = torch.empty(n + 8, dtype=torch.float16, device="cuda")
    c = c0[offsets[2]:offsets[2] + n]
    ext.capi_check(ext.capi().kpb_vector_add(2, 1, a.data_ptr(), b.data_ptr(), c.data_ptr(), n,
                                             ext.current_stream_ptr()))
    torch.cuda.synchronize()
    assert torch.equal(c, (a.float() + b.float()).half())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("x_off,p_off", [(1, 1), (3, 3), (0, 1), (1, 0), (1, 2), (0, 3)])
def test_layernorm_misaligned_base_and_params(x_off, p_off, dtype):
    # rows, w and b each at their own offset from a 16-byte boundary: the rows-in-
    # registers kernel reads w/b as shifted pairs of aligned vectors
    spec = get_spec("layernorm")
    dev = torch.device("cuda")
    M, N = 64, 1000
    x0, w0, b0 = spec.make_inputs((M, N + 8), dtype, dev, 0)
    x = x0.flatten()[x_off:x_off + M * N].view(M, N)
    w, b = w0[p_off:p_off + N], b0[p_off:p_off + N]
    res = check_on_inputs(spec, "best", registry.best("layernorm"), (x, w, b), (M, N), dtype)
    assert res.ok, res.summary()


def test_layernorm_constant_rows_give_bias():
    # zero variance: (x - mean) is exactly 0, so y = b for any weight
    ops = ext.ops()
    x = torch.full((40, 3000), 7.25, device="cuda")
    w = torch.randn(3000, device="cuda")
    b = torch.randn(3000, device="cuda")
    for v in range(3):
        assert torch.equal(ops.layernorm(x, w, b, 1e-5, v), b.expand(40, 3000))


def test_reduce_is_deterministic():
    x = get_spec("reduce_sum").make_inputs((2**26 + 5,), torch.float32,
                                           torch.device("cuda"), 3)[0]
    fn = registry.best("reduce_sum")
    a = fn(x)
    b = fn(x)
    assert torch.equal(a, b)


def test_empty_inputs():
    ops = ext.ops()
    x = torch.empty(0, device="cuda")
    assert float(ops.reduce_sum(x, 2)) == 0.0
    assert ops.softmax(torch.empty(0, 5, device="cuda"), 2).shape == (0, 5)
    a = torch.randn(3, 0, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(0, 4, device="cuda", dtype=torch.bfloat16)
    assert torch.count_nonzero(ops.matmul(a, b, 3)) == 0
    assert ops.vector_add(x, x, 2).shape == (0,)
    e = torch.empty(0, 5, device="cuda")
    assert ops.layernorm(e, torch.ones(5, device="cuda"), torch.zeros(5, device="cuda"),
                         1e-5, 2).shape == (0, 5)


def test_bad_inputs_raise():
    ops = ext.ops()
    with pytest.raises(RuntimeError, match="contiguous"):
        ops.softmax(torch.randn(8, 8, device="cuda").t(), 2)
    with pytest.raises(RuntimeError, match="variant"):
        ops.softmax(torch.randn(8, 8, device="cuda"), 3)
    with pytest.raises(RuntimeError, match="float32, float16 and bfloat16"):
        ops.softmax(torch.randn(8, 8, device="cuda").double(), 2)
    with pytest.raises(RuntimeError, match="match in shape"):
        ops.vector_add(torch.randn(8, device="cuda"), torch.randn(9, device="cuda"), 2)
    with pytest.raises(RuntimeError, match="must have size"):
        ops.layernorm(torch.randn(4, 8, device="cuda"), torch.ones(7, device="cuda"),
                      torch.zeros(8, device="cuda"), 1e-5, 2)
    with pytest.raises(RuntimeError, match="share a dtype"):
        ops.layernorm(torch.randn(4, 8, device="cuda"), torch.ones(8, device="cuda").half(),
                      torch.zeros(8, device="cuda"), 1e-5, 2)
    with pytest.raises(RuntimeError, match="same dtype"):
        ops.matmul(torch.randn(8, 8, device="cuda"), torch.randn(8, 8, device="cuda").half(), 3)


# ------------------------------------------------------------------ C ABI directly

def _p(t: torch.Tensor) -> int:
    return t.data_ptr()


def test_capi_matches_torch_ops():
    lib = ext.capi()
    stream = ext.current_stream_ptr()
    dev = torch.device("cuda")
    ops = ext.ops()

    x = get_spec("reduce_sum").make_inputs((3_000_001,), torch.float32, dev, 0)[0]
    out = torch.empty((), device=dev)
    ext.capi_check(lib.kpb_reduce_sum(2, 0, _p(x), _p(out), x.numel(), stream))
    torch.cuda.synchronize()
    assert torch.equal(out, ops.reduce_sum(x, 2))

    x = get_spec("softmax").make_inputs((128, 4097), torch.bfloat16, dev, 0)[0]
    y = torch.empty_like(x)
    ext.capi_check(lib.kpb_softmax(2, 2, _p(x), _p(y), 128, 4097, stream))
    torch.cuda.synchronize()
    assert torch.equal(y, ops.softmax(x, 2))

    a, b = get_spec("matmul").make_inputs((256, 300, 128), torch.bfloat16, dev, 0)
    c = torch.empty(256, 300, dtype=torch.bfloat16, device=dev)
    ext.capi_check(lib.kpb_matmul(3, 2, _p(a), _p(b), _p(c), 256, 300, 128, stream))
    torch.cuda.synchronize()
    assert torch.equal(c, ops.matmul(a, b, 3))

    a, b = get_spec("vector_add").make_inputs((100_001,), torch.bfloat16, dev, 0)
    c = torch.empty_like(a)
    ext.capi_check(lib.kpb_vector_add(2, 2, _p(a), _p(b), _p(c), a.numel(), stream))
    torch.cuda.synchronize()
    assert torch.equal(c, ops.vector_add(a, b, 2))

    x, w, b = get_spec("layernorm").make_inputs((100, 3000), torch.float16, dev, 0)
    y = torch.empty_like(x)
    ext.capi_check(lib.kpb_layernorm(2, 1, _p(x), _p(w), _p(b), _p(y), 100, 3000,
                                     ctypes.c_float(1e-5), stream))
    torch.cuda.synchronize()
    assert torch.equal(y, ops.layernorm(x, w, b, 1e-5, 2))

    q, k, v = get_spec("attention").make_inputs((1, 2, 200, 128), torch.bfloat16, dev, 0)
    o = torch.empty_like(q)
    ext.capi_check(lib.kpb_attention(1, 2, _p(q), _p(k), _p(v), _p(o), 2, 200, 128, stream))
    ext.capi_check(lib.kpb_attention_causal(1, 2, _p(q), _p(k), _p(v), _p(o), 2, 200, 128,
                                            stream))
    torch.cuda.synchronize()
    assert torch.equal(o, ops.attention_causal(q, k, v, 1))


def test_no_kernel_wait_timed_out():
    lib = ext.capi()
    bits = ctypes.c_uint(0)
    ext.capi_check(lib.kpb_device_errors(ctypes.byref(bits)))
    assert bits.value == 0


@pytest.mark.gpu
def test_kernel_attributes_survive_smaller_launches_in_between():
    # the dynamic shared-memory opt-in of a kernel is one value: a launch asking for
    # less must not lower it under what an earlier, larger launch needed
    spec = get_spec("softmax")
    fn = registry.best("softmax")
    # rows of 16-bit values from 8K to 32K elements share one kernel instantiation and
    # need shared-memory stages of different sizes
    for shape in [(4, 32768), (4, 16384), (4, 32768), (4, 8192), (4, 24576), (4, 32768),
                  (4, 1024), (300, 4095), (4, 32768)]:
        res = check_impl(spec, "best", fn, shape, torch.bfloat16, "cuda")
        assert res.ok, res.summary()
