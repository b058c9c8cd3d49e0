"""Correctness gate: a kernel's output against the float64 reference of its spec.

Same semantics as kernelpilot/correctness.py:
* ``compare`` (kernelpilot/correctness.py:52-78): elementwise
  ``|out - ref| <= atol + rtol*|ref|``; a NaN/Inf in the output is an error unless
  the reference holds the same non-finite value there; the worst offending element
  is reported by index;
* ``check_impl`` (kernelpilot/correctness.py:81-117): generate seeded inputs,
  snapshot them, run, synchronise, then fail on a crash, a wrong output dtype,
  in-place modification of an input, or a numeric mismatch. A crash is a failed
  result, never an exception.

``check_chunked`` adds one thing the reference does not need at its small sizes:
the same per-element test over row/head blocks, so that the headline workloads
(e.g. a 2^31-element softmax) are checked without materialising a float64 copy of
the whole output at once.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator
from dataclasses import asdict, dataclass

import torch

from .specs import KernelSpec, Shape


class KernelMismatch(AssertionError):
    pass


@dataclass
class CheckResult:
    kernel: str
    impl: str
    shape: Shape
    dtype: str
    ok: bool
    max_abs_err: float = 0.0
    max_rel_err: float = 0.0
    num_mismatched: int = 0
    numel: int = 0
    worst_index: tuple[int, ...] | None = None
    got: float | None = None
    expected: float | None = None
    atol: float = 0.0
    rtol: float = 0.0
    error: str | None = None

    def summary(self) -> str:
        head = f"{self.kernel}[{self.impl}] dtype={self.dtype} shape={self.shape}"
        if self.error:
            return f"{head}: {self.error}"
        status = "OK" if self.ok else "MISMATCH"
        msg = (f"{head}: {status} max_abs_err={self.max_abs_err:.3e} "
               f"max_rel_err={self.max_rel_err:.3e} (atol={self.atol:.1e}, rtol={self.rtol:.1e})")
        if not self.ok and self.worst_index is not None:
            msg += (f"; {self.num_mismatched}/{self.numel} elements out of tolerance, worst at "
                    f"index {self.worst_index}: got {self.got!r}, expected {self.expected!r}")
        return msg

    def to_dict(self) -> dict:
        return asdict(self)


def compare(out: torch.Tensor, ref: torch.Tensor, atol: float, rtol: float) -> dict:
    """Elementwise tolerance test; returns max errors, mismatch count and the worst
    offending element (by absolute error among the mismatches)."""
    if tuple(out.shape) != tuple(ref.shape):
        raise KernelMismatch(f"shape mismatch: got {tuple(out.shape)}, "
                             f"expected {tuple(ref.shape)}")
    o = out.detach().to(torch.float64)
    r = ref.detach().to(device=o.device, dtype=torch.float64)
    err = (o - r).abs()
    # a non-finite output is fine only where the reference is the same non-finite value
    agree_nonfinite = torch.logical_and(~torch.isfinite(r), o == r)
    err = err.masked_fill(agree_nonfinite, 0.0)
    err = err.masked_fill(torch.isnan(err), float("inf"))
    bad = err > (atol + rtol * r.abs())
    rel = err / r.abs().clamp_min(1e-12)
    n_bad = int(bad.sum())
    info = {
        "max_abs_err": float(err.max()) if err.numel() else 0.0,
        "max_rel_err": float(rel.max()) if rel.numel() else 0.0,
        "num_mismatched": n_bad,
        "numel": int(err.numel()),
    }
    if n_bad:
        flat = int(torch.argmax(err.masked_fill(~bad, 0.0)).item())
        if err.dim():
            idx = tuple(int(i) for i in torch.unravel_index(torch.tensor(flat), err.shape))
        else:
            idx = ()
        info.update(worst_index=idx, got=float(o.reshape(-1)[flat]),
                    expected=float(r.reshape(-1)[flat]))
    return info


def _dtype_name(dtype: torch.dtype) -> str:
    return str(dtype).replace("torch.", "")


def check_impl(spec: KernelSpec, impl_name: str, fn: Callable, shape: Shape,
               dtype: torch.dtype, device: str | torch.device = "cuda",
               seed: int = 0) -> CheckResult:
    device = torch.device(device)
    inputs = spec.make_inputs(shape, dtype, device, seed)
    return check_on_inputs(spec, impl_name, fn, inputs, shape, dtype)


def check_on_inputs(spec: KernelSpec, impl_name: str, fn: Callable, inputs: tuple,
                    shape: Shape, dtype: torch.dtype) -> CheckResult:
    """``check_impl`` on caller-made inputs (used for the headline generators)."""
    tol = spec.tolerance(shape, dtype)
    res = CheckResult(kernel=spec.name, impl=impl_name, shape=tuple(shape),
                      dtype=_dtype_name(dtype), ok=False, atol=tol.atol, rtol=tol.rtol)
    snapshot = [x.clone() for x in inputs]
    try:
        out = fn(*inputs)
        if inputs and inputs[0].is_cuda:
            torch.cuda.synchronize()
    except Exception as e:  # a crash is a failed check, reported, not raised
        res.error = f"{type(e).__name__}: {e}"
        return res
    if not isinstance(out, torch.Tensor):
        res.error = f"kernel returned {type(out).__name__}, expected torch.Tensor"
        return res
    want = spec.output_dtype(dtype)
    if out.dtype != want:
        res.error = f"kernel returned dtype {out.dtype}, expected {want}"
        return res
    if any(not torch.equal(a, b) for a, b in zip(inputs, snapshot, strict=True)):
        res.error = "kernel modified its inputs in place"
        return res
    del snapshot
    ref = spec.reference(*inputs)
    try:
        info = compare(out, ref, tol.atol, tol.rtol)
    except KernelMismatch as e:
        res.error = str(e)
        return res
    for k, v in info.items():
        setattr(res, k, v)
    res.ok = info["num_mismatched"] == 0
    return res


def assert_correct(spec: KernelSpec, impl_name: str, fn: Callable, shape: Shape,
                   dtype: torch.dtype, device: str | torch.device = "cuda") -> CheckResult:
    res = check_impl(spec, impl_name, fn, shape, dtype, device)
    if not res.ok:
        raise KernelMismatch(res.summary())
    return res


def check_all(spec: KernelSpec, impl_name: str, fn: Callable,
              shapes: list[Shape] | None = None, dtypes: list[torch.dtype] | None = None,
              device: str | torch.device = "cuda", stop_on_fail: bool = False
              ) -> list[CheckResult]:
    results = []
    for dtype in dtypes or spec.dtypes:
        for shape in shapes or spec.test_shapes:
            r = check_impl(spec, impl_name, fn, shape, dtype, device)
            results.append(r)
            if stop_on_fail and not r.ok:
                return results
    return results


# ------------------------------------------------------------------ chunked checks

def _row_blocks(n: int, block: int) -> Iterator[tuple[int, int]]:
    for s in range(0, n, block):
        yield s, min(n, s + block)


def _merge(acc: dict, info: dict, offset: tuple[int, ...]) -> None:
    acc["max_abs_err"] = max(acc["max_abs_err"], info["max_abs_err"])
    acc["max_rel_err"] = max(acc["max_rel_err"], info["max_rel_err"])
    acc["numel"] += info["numel"]
    if info["num_mismatched"]:
        if acc["num_mismatched"] == 0:
            idx = info["worst_index"]
            acc["worst_index"] = tuple(a + b for a, b in zip(offset, idx, strict=False)) \
                + tuple(idx[len(offset):])
            acc["got"], acc["expected"] = info["got"], info["expected"]
        acc["num_mismatched"] += info["num_mismatched"]


def check_chunked(spec: KernelSpec, impl_name: str, inputs: tuple, out: torch.Tensor,
                  shape: Shape, dtype: torch.dtype, elems_per_chunk: int = 1 << 25
                  ) -> CheckResult:
    """Per-element check of an already computed ``out`` against the float64
    reference, evaluated block by block along the leading axis the reference is
    independent over: rows for softmax, rows of C for matmul, (B, H) slices for
    attention, element blocks for vector_add. For reduce_sum the reference is one
    float64 sum of the input."""
    tol = spec.tolerance(shape, dtype)
    res = CheckResult(kernel=spec.name, impl=impl_name, shape=tuple(shape),
                      dtype=_dtype_name(dtype), ok=False, atol=tol.atol, rtol=tol.rtol)
    if out.dtype != spec.output_dtype(dtype):
        res.error = f"kernel returned dtype {out.dtype}, expected {spec.output_dtype(dtype)}"
        return res
    acc = {"max_abs_err": 0.0, "max_rel_err": 0.0, "num_mismatched": 0, "numel": 0}
    name = spec.name
    if name == "reduce_sum":
        (x,) = inputs
        ref = torch.zeros((), dtype=torch.float64, device=x.device)
        flat = x.reshape(-1)
        for s, e in _row_blocks(flat.numel(), elems_per_chunk):
            ref += flat[s:e].double().sum()
        _merge(acc, compare(out, ref, tol.atol, tol.rtol), ())
    elif name == "softmax":
        (x,) = inputs
        N = x.shape[-1]
        x2, o2 = x.reshape(-1, N), out.reshape(-1, N)
        rows = max(1, elems_per_chunk // max(N, 1))
        for s, e in _row_blocks(x2.shape[0], rows):
            info = compare(o2[s:e], spec.reference(x2[s:e]), tol.atol, tol.rtol)
            _merge(acc, info, (s,))
    elif name == "vector_add":
        a, b = (t.reshape(-1) for t in inputs)
        o1 = out.reshape(-1)
        for s, e in _row_blocks(a.numel(), elems_per_chunk):
            _merge(acc, compare(o1[s:e], spec.reference(a[s:e], b[s:e]), tol.atol, tol.rtol),
                   (s,))
    elif name == "layernorm":
        x, w, b = inputs
        N = x.shape[-1]
        x2, o2 = x.reshape(-1, N), out.reshape(-1, N)
        rows = max(1, elems_per_chunk // max(N, 1))
        for s, e in _row_blocks(x2.shape[0], rows):
            _merge(acc, compare(o2[s:e], spec.reference(x2[s:e], w, b), tol.atol, tol.rtol),
                   (s,))
    elif name == "matmul":
        a, b = inputs
        bd = b.double()
        rows = max(1, elems_per_chunk // max(b.shape[1], 1))
        for s, e in _row_blocks(a.shape[0], rows):
            info = compare(out[s:e], a[s:e].double() @ bd, tol.atol, tol.rtol)
            _merge(acc, info, (s, 0))
    elif name in ("attention", "attention_causal"):
        q, k, v = inputs
        B, H, S, D = q.shape
        qf, kf, vf, of = (t.reshape(B * H, S, D) for t in (q, k, v, out))
        # the float64 score block is S*S per head
        heads = max(1, elems_per_chunk // max(S * S, 1))
        for s, e in _row_blocks(B * H, heads):
            ref = spec.reference(qf[s:e], kf[s:e], vf[s:e])
            _merge(acc, compare(of[s:e], ref, tol.atol, tol.rtol), (s,))
    else:
        raise KeyError(f"no chunked check for {name}")
    for k2, v2 in acc.items():
        setattr(res, k2, v2)
    res.ok = acc["num_mismatched"] == 0
    return res
