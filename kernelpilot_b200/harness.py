"""kernelpilot's own correctness and benchmark harness, driving this library unchanged,
plus the few pieces B200 adds.

The reference harness (kernelpilot/correctness.py ``compare``/``check_impl``,
kernelpilot/benchmark.py ``time_fn``/``bench_one``/``bench_kernel``, kernelpilot/device.py
``GPUInfo``/``get_gpu_info``) is what checks and times the ``torch.ops.kp`` ops. It is
imported from its installed copy, not restated here: the directory named by
``KP_REF_HARNESS`` or, by default, ``baseline/_ref`` next to this package (made with
``pip install --no-index --no-deps --target baseline/_ref <kernelpilot source>``; it is
pure Python). This library's ``KernelSpec`` objects carry the reference's field names,
so the reference functions accept them as they are.

What this module adds, and why the reference does not have it:

* ``check_on_inputs``: ``check_impl`` on given tensors (the headline workloads draw
  U(-1,1) or N(0,1)/sqrt(K) inputs, not ``make_inputs``' N(0,1));
* ``check_chunked``: the same per-element test on an already computed output, block by
  block, so a 2^31-element softmax is checked without a float64 copy of all of it;
* ``flush_l2(clean=True)``: the reference's 256 MB flush followed by a read of the
  buffer, so the flush's dirty lines are not written back during the next timed call;
* ``gpu_info``: the reference's ``GPUInfo`` with a B200 row (the reference has none)
  and a bf16 peak (its ``peak_for`` gives every dtype but fp16 the fp32 CUDA-core
  peak, kernelpilot/device.py:42-44), taken from ``MEASURED_PEAKS.json`` when present.
"""

from __future__ import annotations

import dataclasses
import json
import os
import sys
import types
from collections.abc import Callable, Iterator
from functools import lru_cache
from pathlib import Path

import torch

REPO_ROOT = Path(__file__).resolve().parent.parent
DEFAULT_REF_ROOT = REPO_ROOT / "baseline" / "_ref"


def reference_root() -> Path:
    """Directory that holds the reference's ``kernelpilot`` package."""
    env = os.environ.get("KP_REF_HARNESS")
    return Path(env) if env else DEFAULT_REF_ROOT


@lru_cache(maxsize=1)
def reference() -> types.SimpleNamespace:
    """The reference harness modules: ``specs``, ``correctness``, ``benchmark``,
    ``device``, ``registry``, ``ext``. Raises with the install command when absent."""
    root = reference_root()
    if not (root / "kernelpilot" / "correctness.py").exists():
        raise RuntimeError(
            f"the kernelpilot harness is not installed under {root}: install it with "
            "`python -m pip install --no-index --no-build-isolation --no-deps --target "
            "baseline/_ref <path to the kernelpilot source>` or set KP_REF_HARNESS")
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    import importlib

    mods = {name: importlib.import_module(f"kernelpilot.{name}")
            for name in ("specs", "correctness", "benchmark", "device", "registry", "ext")}
    return types.SimpleNamespace(root=root, **mods)


def available() -> bool:
    try:
        reference()
    except RuntimeError:
        return False
    return True


# ------------------------------------------------------------------ the reference's API

def compare(out: torch.Tensor, ref: torch.Tensor, atol: float, rtol: float) -> dict:
    """kernelpilot/correctness.py:52-78, the per-element gate."""
    return reference().correctness.compare(out, ref, atol, rtol)


def check_impl(spec, impl_name: str, fn: Callable, shape, dtype: torch.dtype,
               device: str | torch.device = "cuda", seed: int = 0):
    """kernelpilot/correctness.py:81-117."""
    return reference().correctness.check_impl(spec, impl_name, fn, shape, dtype, device, seed)


def check_on_inputs(spec, impl_name: str, fn: Callable, inputs: tuple, shape,
                    dtype: torch.dtype):
    """The reference's ``check_impl`` run on the given input tensors: the spec's input
    generator is swapped for one that hands back exactly these tensors."""
    given = tuple(inputs)
    fixed = dataclasses.replace(spec, make_inputs=lambda *_a, **_k: given)
    device = given[0].device if given else torch.device("cuda")
    return check_impl(fixed, impl_name, fn, shape, dtype, device)


def new_result(spec, impl_name: str, shape, dtype: torch.dtype):
    tol = spec.tolerance(shape, dtype)
    return reference().correctness.CheckResult(
        kernel=spec.name, impl=impl_name, shape=tuple(shape),
        dtype=str(dtype).replace("torch.", ""), ok=False, atol=tol.atol, rtol=tol.rtol)


# ------------------------------------------------------------------ chunked checks

def _blocks(n: int, block: int) -> Iterator[tuple[int, int]]:
    for s in range(0, n, block):
        yield s, min(n, s + block)


def _fold(acc: dict, info: dict, offset: tuple[int, ...]) -> None:
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


def check_chunked(spec, impl_name: str, inputs: tuple, out: torch.Tensor, shape,
                  dtype: torch.dtype, elems_per_chunk: int = 1 << 25):
    """Per-element check of an already computed ``out`` against the float64
    reference, evaluated block by block along the axis the reference is independent
    over: rows (softmax, layernorm), rows of C (matmul), (B, H) slices (attention),
    element blocks (vector_add). For reduce_sum the reference is one float64 sum,
    accumulated over blocks. Same test and report as ``check_impl``."""
    res = new_result(spec, impl_name, shape, dtype)
    want = spec.output_dtype(dtype)
    if out.dtype != want:
        res.error = f"kernel returned dtype {out.dtype}, expected {want}"
        return res
    acc = {"max_abs_err": 0.0, "max_rel_err": 0.0, "num_mismatched": 0, "numel": 0}
    name = spec.name
    if name == "reduce_sum":
        (x,) = inputs
        ref = torch.zeros((), dtype=torch.float64, device=x.device)
        flat = x.reshape(-1)
        for s, e in _blocks(flat.numel(), elems_per_chunk):
            ref += flat[s:e].double().sum()
        _fold(acc, compare(out, ref, res.atol, res.rtol), ())
    elif name in ("softmax", "layernorm"):
        x = inputs[0]
        n = x.shape[-1]
        x2, o2 = x.reshape(-1, n), out.reshape(-1, n)
        rows = max(1, elems_per_chunk // max(n, 1))
        for s, e in _blocks(x2.shape[0], rows):
            ref = spec.reference(x2[s:e], *inputs[1:])
            _fold(acc, compare(o2[s:e], ref, res.atol, res.rtol), (s,))
    elif name == "vector_add":
        a, b = (t.reshape(-1) for t in inputs)
        o1 = out.reshape(-1)
        for s, e in _blocks(a.numel(), elems_per_chunk):
            _fold(acc, compare(o1[s:e], spec.reference(a[s:e], b[s:e]), res.atol, res.rtol),
                  (s,))
    elif name == "matmul":
        a, b = inputs
        bd = b.double()
        rows = max(1, elems_per_chunk // max(b.shape[1], 1))
        for s, e in _blocks(a.shape[0], rows):
            _fold(acc, compare(out[s:e], a[s:e].double() @ bd, res.atol, res.rtol), (s, 0))
    elif name in ("attention", "attention_causal"):
        q, k, v = inputs
        B, H, S, D = q.shape
        qf, kf, vf, of = (t.reshape(B * H, S, D) for t in (q, k, v, out))
        heads = max(1, elems_per_chunk // max(S * S, 1))  # the float64 scores are S*S
        for s, e in _blocks(B * H, heads):
            ref = spec.reference(qf[s:e], kf[s:e], vf[s:e])
            _fold(acc, compare(of[s:e], ref, res.atol, res.rtol), (s,))
        if "worst_index" in acc:  # (B*H, S, D) index -> (B, H, S, D)
            bh, i, d = acc["worst_index"]
            acc["worst_index"] = (bh // H, bh % H, i, d)
    else:
        raise KeyError(f"no chunked check for {name}")
    for key, val in acc.items():
        setattr(res, key, val)
    res.ok = acc["num_mismatched"] == 0
    return res


# ------------------------------------------------------------------ timing helpers

L2_FLUSH_BYTES = 256 << 20  # larger than the 126 MB L2 of a B200
_flush_buf: torch.Tensor | None = None


def flush_l2(clean: bool = True) -> None:
    """Evict L2 by writing a 256 MB buffer; with ``clean`` the buffer is then read, so
    the lines the write left dirty are written back now, not in the next timed call."""
    global _flush_buf
    if _flush_buf is None:
        _flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    _flush_buf.zero_()
    if clean:
        _flush_buf.sum()


# ------------------------------------------------------------------ peaks

# B200 datasheet figures (HGX): HBM3e GB/s, fp32 CUDA-core TFLOPS, dense fp16/bf16
# tensor TFLOPS.
B200_DATASHEET = (7700.0, 75.0, 2250.0)


def measured_peaks(path: str | Path | None = None) -> dict | None:
    """The copy bandwidth and bf16 GEMM rate measured on this pool's GPUs, or None."""
    p = Path(path) if path else REPO_ROOT / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return None


@lru_cache(maxsize=1)
def _b200_info_class():
    base = reference().device.GPUInfo

    @dataclasses.dataclass
    class B200GPUInfo(base):
        """The reference's ``GPUInfo`` whose ``peak_for`` also knows bf16."""

        def peak_for(self, dtype: torch.dtype) -> float | None:
            if dtype == torch.bfloat16:
                return self.peak_tflops.get("bfloat16", self.peak_tflops.get("float16"))
            return super().peak_for(dtype)

    return B200GPUInfo


def b200_info(name: str = "NVIDIA B200", measured_path: str | Path | None = None):
    """Peaks of a B200: measured (``MEASURED_PEAKS.json``) where available, else the
    datasheet; ``KP_PEAK_*`` environment overrides win as in the reference."""
    bw, fp32, fp16 = B200_DATASHEET
    info = _b200_info_class()(name=name, vendor="nvidia", peak_bw_gbs=bw,
                              peak_tflops={"float32": fp32, "float16": fp16,
                                           "bfloat16": fp16}, source="datasheet")
    meas = measured_peaks(measured_path)
    if meas and "hbm_gbs" in meas:
        info.peak_bw_gbs = float(meas["hbm_gbs"])
        if "bf16_tflops" in meas:
            info.peak_tflops["float16"] = info.peak_tflops["bfloat16"] = float(meas["bf16_tflops"])
        info.source = "measured (MEASURED_PEAKS.json: copy bandwidth, cuBLAS bf16 GEMM)"
    for env, key in (("KP_PEAK_FP32_TFLOPS", "float32"), ("KP_PEAK_FP16_TFLOPS", "float16"),
                     ("KP_PEAK_BF16_TFLOPS", "bfloat16")):
        if os.environ.get(env):
            info.peak_tflops[key], info.source = float(os.environ[env]), "env"
    if os.environ.get("KP_PEAK_BW_GBS"):
        info.peak_bw_gbs, info.source = float(os.environ["KP_PEAK_BW_GBS"]), "env"
    return info


def gpu_info():
    """This GPU's peaks: ``b200_info`` on a B200, else the reference's ``get_gpu_info``."""
    if torch.cuda.is_available() and "B200" in torch.cuda.get_device_name():
        return b200_info(torch.cuda.get_device_name())
    return reference().device.get_gpu_info()
