"""CPU oracle for the torch.ops.kp hot path: a float64 numpy restatement of the
reference's op semantics and of its correctness comparator.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this module: it is
used by tests/, by ``__graft_entry__.smoke()`` and by bench.py's ``cpu_baseline`` /
reference arm, and only ever as the reference results are compared against or as the
CPU baseline, never as the thing measured or shipped.

Pinned against the reference itself: tests/golden/make_golden.py imports the
reference package (kernelpilot/specs.py), generates seeded inputs with its own
generators and records its float64 outputs; tests/test_oracle.py checks every
function here against those fixtures, and the comparator against the reference's
own harness known-answer tests (kernelpilot tests/cpu/test_harness.py:12-41).

bf16 arrays travel as their raw uint16 bit patterns (numpy has no bf16 type);
``as_f64`` widens them exactly.
"""

from __future__ import annotations

import math

import numpy as np

DTYPES = ("float32", "float16", "bfloat16")


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns (uint16) to float32."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    out[nan] = np.uint16(0x7FC0)
    return out


def as_f64(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return bf16_bits_to_f32(a).astype(np.float64)
    return np.asarray(a).astype(np.float64)


# ------------------------------------------------------------------ op semantics

def vector_add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """a.double() + b.double() (kernelpilot/specs.py:77-78)."""
    return np.asarray(a, dtype=np.float64) + np.asarray(b, dtype=np.float64)


def layernorm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """F.layer_norm(x.double(), (N,), w, b, 1e-5) (kernelpilot/specs.py:217-220): per
    row, subtract the mean, divide by sqrt(biased variance + eps), then scale by w and
    shift by b."""
    x = np.asarray(x, dtype=np.float64)
    mean = np.mean(x, axis=-1, keepdims=True)
    var = np.mean((x - mean) ** 2, axis=-1, keepdims=True)
    return (x - mean) / np.sqrt(var + eps) * np.asarray(w, dtype=np.float64) + \
        np.asarray(b, dtype=np.float64)


def reduce_sum(x: np.ndarray) -> np.float64:
    """x.double().sum() (kernelpilot/specs.py:106-107), as a float64 scalar."""
    return np.float64(np.sum(np.asarray(x, dtype=np.float64)))


def softmax(x: np.ndarray) -> np.ndarray:
    """torch.softmax(x.double(), dim=-1) (kernelpilot/specs.py:141-142): subtract the
    row max, exponentiate, divide by the row sum."""
    x = np.asarray(x, dtype=np.float64)
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """a.double() @ b.double() (kernelpilot/specs.py:173-174)."""
    return np.asarray(a, dtype=np.float64) @ np.asarray(b, dtype=np.float64)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = False) -> np.ndarray:
    """softmax(q k^T / sqrt(D)) v in float64 (kernelpilot/specs.py:255-258); with
    ``causal`` the scores of keys j > query i are -inf before the softmax."""
    q, k, v = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    D = q.shape[-1]
    s = q @ np.swapaxes(k, -1, -2) / math.sqrt(D)
    if causal:
        S = q.shape[-2]
        s = np.where(np.triu(np.ones((S, S), dtype=bool), 1), -np.inf, s)
    return softmax(s) @ v


# ------------------------------------------------------------------ tolerances

def tolerance(op: str, shape: tuple[int, ...], dtype: str) -> tuple[float, float]:
    """(atol, rtol) per op and dtype (kernelpilot/specs.py:99-100, 114-117, 165-166,
    183-190, 246-247, 281-282); bf16 takes the non-fp32 branch like fp16."""
    fp32 = dtype == "float32"
    if op == "vector_add":  # bf16: one rounding of the sum is up to 2^-9 relative
        return (1e-6, 1e-6) if fp32 else ((1e-3, 4e-3) if dtype == "bfloat16" else (1e-3, 1e-3))
    if op == "layernorm":
        return (1e-5, 1e-4) if fp32 else (5e-3, 1e-2)
    if op == "reduce_sum":
        return 1e-5 * math.sqrt(shape[0]) + 1e-5, 1e-5
    if op == "softmax":
        return (1e-6, 1e-5) if fp32 else (1e-3, 1e-2)
    if op == "matmul":
        K = shape[2]
        return (2e-6 * K + 1e-5, 1e-4) if fp32 else (1e-3 * math.sqrt(K) + 1e-3, 1e-2)
    if op in ("attention", "attention_causal"):
        return (1e-5, 1e-4) if fp32 else (2e-3, 1e-2)
    raise KeyError(op)


# ------------------------------------------------------------------ comparator

def compare(out: np.ndarray, ref: np.ndarray, atol: float, rtol: float) -> dict:
    """|out - ref| <= atol + rtol*|ref| elementwise; a non-finite output only passes
    where the reference holds the same value (kernelpilot/correctness.py:52-78)."""
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    if o.shape != r.shape:
        raise ValueError(f"shape mismatch: got {o.shape}, expected {r.shape}")
    with np.errstate(invalid="ignore"):
        err = np.abs(o - r)
        agree = (~np.isfinite(r)) & (o == r)
        err = np.where(agree, 0.0, err)
        err = np.where(np.isnan(err), np.inf, err)
        bad = err > (atol + rtol * np.abs(r))
        rel = err / np.maximum(np.abs(r), 1e-12)
    info = {"max_abs_err": float(err.max()) if err.size else 0.0,
            "max_rel_err": float(rel.max()) if rel.size else 0.0,
            "num_mismatched": int(bad.sum()), "numel": int(err.size)}
    if info["num_mismatched"]:
        flat = int(np.argmax(np.where(bad, err, 0.0)))
        info["worst_index"] = tuple(int(i) for i in np.unravel_index(flat, err.shape)) \
            if err.ndim else ()
    return info


def run(op: str, inputs: list[np.ndarray], dtype: str) -> np.ndarray:
    """The float64 reference output of ``op`` on (possibly bf16-bit) inputs."""
    xs = [as_f64(a, dtype) for a in inputs]
    if op == "vector_add":
        return vector_add(*xs)
    if op == "layernorm":
        return layernorm(*xs)
    if op == "reduce_sum":
        return np.asarray(reduce_sum(xs[0]))
    if op == "softmax":
        return softmax(xs[0])
    if op == "matmul":
        return matmul(*xs)
    if op == "attention":
        return attention(*xs)
    if op == "attention_causal":
        return attention(*xs, causal=True)
    raise KeyError(op)
