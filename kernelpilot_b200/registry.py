"""Every implementation of every op under one naming scheme:

    torch           PyTorch built-in (the baseline)
    cuda:<stage>    hand-written sm_100a kernel; stages ordered simple -> B200-tuned

Mirrors kernelpilot/registry.py (``HIP_STAGES`` :18-25, ``_hip_impl`` :41-48,
``get_impls`` :68-78). The stage index is the ``variant`` passed to the op, and the
counts match the reference (3 / 3 / 3 / 4 / 3 / 2), so a caller passing the reference's
"best" variant index gets the B200 kernel. LayerNorm's eps goes between the inputs and
the variant, as the reference's ``_HIP_EXTRA_ARGS`` (:28) passes it. Triton twins are not registered: the
product path has no Triton dispatch.
"""

from __future__ import annotations

from collections.abc import Callable

from . import ext
from .specs import LAYERNORM_EPS, get_spec

CUDA_STAGES: dict[str, list[str]] = {
    "vector_add": ["naive", "gridstride", "vectorized"],
    "reduce_sum": ["chunked", "gridstride", "persistent_vec"],
    "softmax": ["thread_row", "block_row", "staged_tma"],
    "matmul": ["naive", "smem_tiled", "reg_tiled", "tcgen05"],
    "layernorm": ["naive", "block_two_pass", "rows_in_registers"],
    "attention": ["naive", "tcgen05_flash"],
    "attention_causal": ["naive", "tcgen05_flash"],
}

BEST_VARIANT: dict[str, int] = {k: len(v) - 1 for k, v in CUDA_STAGES.items()}

# arguments an op takes between its tensors and the variant
EXTRA_ARGS: dict[str, tuple] = {"layernorm": (LAYERNORM_EPS,)}


def _cuda_impl(kernel: str, variant: int) -> Callable:
    extra = EXTRA_ARGS.get(kernel, ())

    def run(*inputs):
        return getattr(ext.ops(), kernel)(*inputs, *extra, variant)

    run.__name__ = f"cuda_{kernel}_{CUDA_STAGES[kernel][variant]}"
    return run


def cuda_impls(kernel: str) -> dict[str, Callable]:
    if not ext.load():
        return {}
    return {f"cuda:{stage}": _cuda_impl(kernel, i)
            for i, stage in enumerate(CUDA_STAGES.get(kernel, []))}


def best(kernel: str) -> Callable:
    """The B200-tuned implementation of ``kernel`` (raises if not built)."""
    ext.ops()
    return _cuda_impl(kernel, BEST_VARIANT[kernel])


def get_impls(kernel: str, include: tuple[str, ...] = ("torch", "cuda")
              ) -> dict[str, Callable]:
    spec = get_spec(kernel)
    impls: dict[str, Callable] = {}
    if "torch" in include:
        impls["torch"] = spec.baseline
    if "cuda" in include:
        impls.update(cuda_impls(kernel))
    return impls
