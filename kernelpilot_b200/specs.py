"""Op contracts for the ``torch.ops.kp`` suite: what each op computes (a float64
PyTorch reference), which shapes and dtypes it must accept, how much work one call
does (FLOPs, ideal bytes) and how close an answer must be.

Field-for-field the same contract as kernelpilot/specs.py:29-54 (``KernelSpec``),
with the same input generators (kernelpilot/specs.py:61-72), references, test shapes
and tolerances, so a result that passes here passes the reference harness. The
additions are all additive:

* ``torch.bfloat16`` in every ``dtypes`` list (bf16 takes the reference's non-fp32
  tolerance branch, exactly as the reference lambdas would give it);
* ``ATTENTION_CAUSAL``: the same attention with an upper-triangular mask; its
  ``flops`` counts only the useful (unmasked) half;
* ``VECTOR_ADD`` and ``LAYERNORM`` (kernelpilot/specs.py:77-101, 214-250), the
  reference's remaining ``kp`` ops, with the same additions;
* ``CONFIGS``: the headline workloads (the five of the reference's benchmark table,
  plus causal attention, a long-row softmax, the elementwise add and LayerNorm) with
  their own generators
  (U(-1,1) for the reduction and the add, N(0,1)/sqrt(K) for the GEMM) next to
  ``make_inputs``.
"""

from __future__ import annotations

import inspect
import math
from collections.abc import Callable
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

Shape = tuple[int, ...]
Inputs = tuple[torch.Tensor, ...]

HALF_TYPES = (torch.float16, torch.bfloat16)
ALL_DTYPES = [torch.float32, torch.float16, torch.bfloat16]


@dataclass(frozen=True)
class Tolerance:
    atol: float
    rtol: float


@dataclass
class KernelSpec:
    name: str
    description: str
    signature: str
    make_inputs: Callable[[Shape, torch.dtype, torch.device, int], Inputs]
    reference: Callable[..., torch.Tensor]
    baseline: Callable[..., torch.Tensor]
    test_shapes: list[Shape]
    bench_shapes: list[Shape]
    dtypes: list[torch.dtype]
    flops: Callable[[Shape], float]
    bytes_moved: Callable[[Shape, torch.dtype], float]
    tolerance: Callable[[Shape, torch.dtype], Tolerance]
    shape_names: tuple[str, ...]
    output_dtype: Callable[[torch.dtype], torch.dtype] = field(default=lambda dt: dt)

    def reference_source(self) -> str:
        return inspect.getsource(self.reference)

    def format_shape(self, shape: Shape) -> str:
        return ", ".join(f"{n}={v}" for n, v in zip(self.shape_names, shape, strict=True))


def element_size(dtype: torch.dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


def generator(device: torch.device | str, seed: int) -> torch.Generator:
    """Seeded generator on ``device`` (kernelpilot/specs.py:69-72). CPU and CUDA
    generators give different streams for one seed, so a check always evaluates the
    reference on the very tensors the kernel saw."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def randn(shape: Shape, dtype: torch.dtype, device, gen: torch.Generator,
          scale: float = 1.0) -> torch.Tensor:
    """N(0,1)*scale drawn in float32 on ``device`` and then cast, so every dtype of
    one seed sees the same values up to rounding (kernelpilot/specs.py:61-66)."""
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * scale
    return x.to(dtype)


def _half_or(fp32: Tolerance, other: Tolerance):
    return lambda s, dt: fp32 if dt == torch.float32 else other


# ------------------------------------------------------------------ vector add

def vector_add_reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return a.double() + b.double()


def _vector_add_inputs(shape, dtype, device, seed):
    g = generator(device, seed)
    return randn(shape, dtype, device, g), randn(shape, dtype, device, g)


VECTOR_ADD = KernelSpec(
    name="vector_add",
    description="Elementwise c = a + b over 1-D tensors.",
    signature="def kernel_fn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor  # same dtype as a",
    make_inputs=_vector_add_inputs,
    reference=vector_add_reference,
    baseline=torch.add,
    test_shapes=[(1,), (7,), (1000,), (1024,), (65537,), (1 << 20,), (3_000_001,)],
    bench_shapes=[(1 << 24,), (1 << 26,)],
    dtypes=list(ALL_DTYPES),
    flops=lambda s: float(s[0]),
    bytes_moved=lambda s, dt: 3.0 * s[0] * element_size(dt),
    # fp32 / fp16 as the reference (kernelpilot/specs.py:99-100); bf16 gets rtol 4e-3:
    # one bf16 rounding of the sum is already up to 2^-9 relative, above the fp16 1e-3
    tolerance=lambda s, dt: (Tolerance(1e-6, 1e-6) if dt == torch.float32 else
                             Tolerance(1e-3, 4e-3) if dt == torch.bfloat16 else
                             Tolerance(1e-3, 1e-3)),
    shape_names=("n",),
)


# ------------------------------------------------------------------ reduction

def reduce_sum_reference(x: torch.Tensor) -> torch.Tensor:
    return x.double().sum()


def _reduce_sum_inputs(shape, dtype, device, seed):
    return (randn(shape, dtype, device, generator(device, seed)),)


def _reduce_sum_tol(shape, dtype):
    # fp32 accumulation error of n O(1) terms grows like sqrt(n)*eps
    # (kernelpilot/specs.py:114-117).
    n = shape[0]
    return Tolerance(atol=1e-5 * math.sqrt(n) + 1e-5, rtol=1e-5)


REDUCE_SUM = KernelSpec(
    name="reduce_sum",
    description="Sum of all elements of a 1-D tensor, returned as a float32 scalar "
                "(0-dim tensor), accumulating in float32 regardless of input dtype.",
    signature="def kernel_fn(x: torch.Tensor) -> torch.Tensor  # 0-dim float32",
    make_inputs=_reduce_sum_inputs,
    reference=reduce_sum_reference,
    baseline=lambda x: x.sum(dtype=torch.float32),
    test_shapes=[(1,), (7,), (1000,), (1024,), (65537,), (1 << 20,), (3_000_001,)],
    bench_shapes=[(1 << 24,), (1 << 26,)],
    dtypes=list(ALL_DTYPES),
    flops=lambda s: float(s[0]),
    bytes_moved=lambda s, dt: float(s[0] * element_size(dt) + 4),
    tolerance=_reduce_sum_tol,
    shape_names=("n",),
    output_dtype=lambda dt: torch.float32,
)


# ------------------------------------------------------------------ softmax

def softmax_reference(x: torch.Tensor) -> torch.Tensor:
    return torch.softmax(x.double(), dim=-1)


def _softmax_inputs(shape, dtype, device, seed):
    # scale 30 overflows exp() in fp32 unless the row max is subtracted first
    return (randn(shape, dtype, device, generator(device, seed), scale=30.0),)


SOFTMAX = KernelSpec(
    name="softmax",
    description="Numerically stable softmax over the last dimension of a contiguous "
                "(M, N) tensor. Output has the input dtype.",
    signature="def kernel_fn(x: torch.Tensor) -> torch.Tensor  # same shape/dtype as x",
    make_inputs=_softmax_inputs,
    reference=softmax_reference,
    baseline=lambda x: torch.softmax(x, dim=-1),
    test_shapes=[(1, 1), (1, 7), (3, 1000), (17, 1024), (128, 4097), (64, 12288),
                 (4, 32768), (1000, 129)],
    bench_shapes=[(4096, 1024), (4096, 4096), (1024, 32768)],
    dtypes=list(ALL_DTYPES),
    flops=lambda s: 5.0 * s[0] * s[1],
    bytes_moved=lambda s, dt: 2.0 * s[0] * s[1] * element_size(dt),
    tolerance=_half_or(Tolerance(1e-6, 1e-5), Tolerance(1e-3, 1e-2)),
    shape_names=("M", "N"),
)


# ------------------------------------------------------------------ matmul

def matmul_reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return a.double() @ b.double()


def _matmul_inputs(shape, dtype, device, seed):
    M, N, K = shape
    g = generator(device, seed)
    return randn((M, K), dtype, device, g), randn((K, N), dtype, device, g)


def _matmul_tol(shape, dtype):
    # |C| grows like sqrt(K); fp32 accumulation error like K*eps
    # (kernelpilot/specs.py:183-190).
    K = shape[2]
    if dtype == torch.float32:
        return Tolerance(atol=2e-6 * K + 1e-5, rtol=1e-4)
    return Tolerance(atol=1e-3 * math.sqrt(K) + 1e-3, rtol=1e-2)


MATMUL = KernelSpec(
    name="matmul",
    description="C = A @ B for row-major A (M, K) and B (K, N). Output has the input dtype; "
                "accumulate in float32. TF32 is not allowed for float32 inputs.",
    signature="def kernel_fn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor  # (M, N)",
    make_inputs=_matmul_inputs,
    reference=matmul_reference,
    baseline=torch.matmul,
    test_shapes=[(1, 1, 1), (7, 13, 5), (64, 64, 64), (127, 129, 65), (256, 512, 128),
                 (33, 1000, 77), (512, 256, 1024), (1024, 1024, 1024)],
    bench_shapes=[(1024, 1024, 1024), (2048, 2048, 2048), (4096, 4096, 4096)],
    dtypes=list(ALL_DTYPES),
    flops=lambda s: 2.0 * s[0] * s[1] * s[2],
    bytes_moved=lambda s, dt: float((s[0] * s[2] + s[2] * s[1] + s[0] * s[1])
                                    * element_size(dt)),
    tolerance=_matmul_tol,
    shape_names=("M", "N", "K"),
)


# ------------------------------------------------------------------ attention

def attention_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    q, k, v = q.double(), k.double(), v.double()
    scores = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    return torch.softmax(scores, dim=-1) @ v


def attention_causal_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor
                               ) -> torch.Tensor:
    q, k, v = q.double(), k.double(), v.double()
    S = q.shape[-2]
    scores = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
    scores = scores.masked_fill(mask, float("-inf"))
    return torch.softmax(scores, dim=-1) @ v


def _attention_inputs(shape, dtype, device, seed):
    g = generator(device, seed)
    return tuple(randn(shape, dtype, device, g) for _ in range(3))


_ATTN_TEST_SHAPES = [(1, 1, 1, 16), (1, 2, 7, 32), (2, 4, 64, 64), (1, 2, 100, 64),
                     (2, 2, 128, 128), (1, 3, 50, 48)]
_ATTN_BENCH_SHAPES = [(8, 16, 128, 64), (8, 16, 256, 64), (4, 16, 512, 64)]
_ATTN_TOL = _half_or(Tolerance(1e-5, 1e-4), Tolerance(2e-3, 1e-2))

ATTENTION = KernelSpec(
    name="attention",
    description="Non-causal scaled dot-product attention softmax(Q K^T / sqrt(D)) V for "
                "contiguous (B, H, S, D) tensors. Output has the input dtype.",
    signature="def kernel_fn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor)"
              " -> torch.Tensor  # (B, H, S, D)",
    make_inputs=_attention_inputs,
    reference=attention_reference,
    baseline=F.scaled_dot_product_attention,
    test_shapes=list(_ATTN_TEST_SHAPES),
    bench_shapes=list(_ATTN_BENCH_SHAPES),
    dtypes=list(ALL_DTYPES),
    flops=lambda s: 4.0 * s[0] * s[1] * s[2] * s[2] * s[3],
    bytes_moved=lambda s, dt: 4.0 * s[0] * s[1] * s[2] * s[3] * element_size(dt),
    tolerance=_ATTN_TOL,
    shape_names=("B", "H", "S", "D"),
)


def _causal_useful_flops(s: Shape) -> float:
    # only the S*(S+1)/2 unmasked (query, key) pairs do work: QK^T and PV each
    # cost 2*D flops per pair
    B, H, S, D = s
    return 4.0 * B * H * (S * (S + 1) / 2.0) * D


ATTENTION_CAUSAL = KernelSpec(
    name="attention_causal",
    description="Causal scaled dot-product attention (query i attends to keys 0..i) for "
                "contiguous (B, H, S, D) tensors. Output has the input dtype.",
    signature="def kernel_fn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor)"
              " -> torch.Tensor  # (B, H, S, D)",
    make_inputs=_attention_inputs,
    reference=attention_causal_reference,
    baseline=lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True),
    test_shapes=list(_ATTN_TEST_SHAPES),
    bench_shapes=list(_ATTN_BENCH_SHAPES),
    dtypes=list(ALL_DTYPES),
    flops=_causal_useful_flops,
    bytes_moved=lambda s, dt: 4.0 * s[0] * s[1] * s[2] * s[3] * element_size(dt),
    tolerance=_ATTN_TOL,
    shape_names=("B", "H", "S", "D"),
)


# ------------------------------------------------------------------ layernorm

LAYERNORM_EPS = 1e-5


def layernorm_reference(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor
                        ) -> torch.Tensor:
    # eps = 1e-5, biased variance, normalized over the last dimension.
    return F.layer_norm(x.double(), (x.shape[-1],), weight.double(), bias.double(), 1e-5)


def _layernorm_inputs(shape, dtype, device, seed):
    M, N = shape
    g = generator(device, seed)
    x = randn((M, N), dtype, device, g, scale=2.0)
    w = (1.0 + 0.1 * torch.randn(N, generator=g, device=device)).to(dtype)
    b = (0.1 * torch.randn(N, generator=g, device=device)).to(dtype)
    return x, w, b


LAYERNORM = KernelSpec(
    name="layernorm",
    description="LayerNorm over the last dimension of a contiguous (M, N) tensor with "
                "elementwise affine weight and bias of shape (N,), eps=1e-5, biased variance. "
                "Output has the input dtype; compute statistics in float32.",
    signature="def kernel_fn(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor)"
              " -> torch.Tensor",
    make_inputs=_layernorm_inputs,
    reference=layernorm_reference,
    baseline=lambda x, w, b: F.layer_norm(x, (x.shape[-1],), w, b, LAYERNORM_EPS),
    test_shapes=[(1, 1), (1, 7), (3, 1000), (64, 1024), (17, 4097), (32, 12288), (2, 20000)],
    bench_shapes=[(4096, 1024), (4096, 4096), (8192, 8192)],
    dtypes=list(ALL_DTYPES),
    flops=lambda s: 8.0 * s[0] * s[1],
    bytes_moved=lambda s, dt: float((2 * s[0] * s[1] + 2 * s[1]) * element_size(dt)),
    tolerance=_half_or(Tolerance(1e-5, 1e-4), Tolerance(5e-3, 1e-2)),
    shape_names=("M", "N"),
)


SPECS: dict[str, KernelSpec] = {
    s.name: s for s in [VECTOR_ADD, REDUCE_SUM, SOFTMAX, MATMUL, LAYERNORM, ATTENTION,
                        ATTENTION_CAUSAL]
}


def get_spec(name: str) -> KernelSpec:
    if name not in SPECS:
        raise KeyError(f"unknown kernel {name!r}; choose from {sorted(SPECS)}")
    return SPECS[name]


# ------------------------------------------------------------------ headline workloads

def _uniform_pm1(shape, dtype, device, seed):
    g = generator(device, seed)
    x = torch.rand(shape, generator=g, device=device, dtype=torch.float32) * 2.0 - 1.0
    return (x.to(dtype),)


def _uniform_pm1_pair(shape, dtype, device, seed):
    g = generator(device, seed)
    return tuple((torch.rand(shape, generator=g, device=device, dtype=torch.float32) * 2.0 - 1.0)
                 .to(dtype) for _ in range(2))


def _matmul_scaled(shape, dtype, device, seed):
    M, N, K = shape
    g = generator(device, seed)
    s = 1.0 / math.sqrt(K)
    return randn((M, K), dtype, device, g, s), randn((K, N), dtype, device, g, s)


@dataclass(frozen=True)
class Workload:
    """One headline configuration: an op, one shape, one dtype and its generator."""
    key: str
    kernel: str
    shape: Shape
    dtype: torch.dtype
    make_inputs: Callable[[Shape, torch.dtype, torch.device, int], Inputs]
    bound: str          # "hbm" or "tensor"
    description: str

    @property
    def spec(self) -> KernelSpec:
        return get_spec(self.kernel)

    def inputs(self, device, seed: int = 0) -> Inputs:
        return self.make_inputs(self.shape, self.dtype, torch.device(device), seed)


CONFIGS: dict[str, Workload] = {w.key: w for w in [
    Workload("softmax_f32_4096x4097", "softmax", (4096, 4097), torch.float32,
             _softmax_inputs, "hbm", "row softmax fp32 [4096, 4097], N(0,1)*30"),
    Workload("reduce_f32_2p28p1", "reduce_sum", ((1 << 28) + 1,), torch.float32,
             _uniform_pm1, "hbm", "full sum fp32, n = 2^28+1, U(-1,1)"),
    Workload("softmax_bf16_65536x32768", "softmax", (65536, 32768), torch.bfloat16,
             _softmax_inputs, "hbm", "row softmax bf16 [65536, 32768], N(0,1)*30"),
    Workload("softmax_bf16_4096x131072", "softmax", (4096, 131072), torch.bfloat16,
             _softmax_inputs, "hbm",
             "long-row softmax bf16 [4096, 131072] (a cluster of CTAs per row), N(0,1)*30"),
    Workload("gemm_bf16_8192", "matmul", (8192, 8192, 8192), torch.bfloat16,
             _matmul_scaled, "tensor", "GEMM bf16 8192^3, N(0,1)/sqrt(K)"),
    Workload("gemm_bf16_4097x4097x4096", "matmul", (4097, 4097, 4096), torch.bfloat16,
             _matmul_scaled, "tensor", "GEMM bf16 M=N=4097 K=4096, N(0,1)/sqrt(K)"),
    Workload("vadd_f32_2p26", "vector_add", (1 << 26,), torch.float32,
             _uniform_pm1_pair, "hbm", "elementwise add fp32, n = 2^26, U(-1,1)"),
    Workload("layernorm_f32_8192x8192", "layernorm", (8192, 8192), torch.float32,
             _layernorm_inputs, "hbm", "LayerNorm fp32 [8192, 8192], x ~ N(0,1)*2, eps 1e-5"),
    Workload("layernorm_bf16_8192x8192", "layernorm", (8192, 8192), torch.bfloat16,
             _layernorm_inputs, "hbm", "LayerNorm bf16 [8192, 8192], x ~ N(0,1)*2, eps 1e-5"),
    Workload("attn_bf16_b8h32s4096d128", "attention", (8, 32, 4096, 128), torch.bfloat16,
             _attention_inputs, "tensor", "attention bf16 B8 H32 S4096 D128, non-causal"),
    Workload("attn_causal_bf16_b8h32s4096d128", "attention_causal", (8, 32, 4096, 128),
             torch.bfloat16, _attention_inputs, "tensor",
             "attention bf16 B8 H32 S4096 D128, causal"),
]}
