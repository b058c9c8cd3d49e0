"""GPU detection and the peaks that %-of-peak and roofline figures divide by.

Same API and lookup rules as kernelpilot/device.py (``GPUInfo``, ``lookup_peaks`` with
whole-word matching, ``KP_PEAK_*`` environment overrides, a measured copy bandwidth as
the last resort), with three additions:
* a B200 datasheet row and a ``bfloat16`` peak key (the reference maps every non-fp16
  dtype to the fp32 peak, kernelpilot/device.py:42-44, which would divide a bf16
  tensor-core kernel by the CUDA-core fp32 peak);
* ``MEASURED_PEAKS.json`` (a STREAM-style copy bandwidth and a cuBLAS bf16 GEMM rate
  measured on the very GPUs the benchmarks run on) takes precedence over the
  datasheet when present next to the package;
* ``KP_PEAK_BF16_TFLOPS`` next to the reference's three overrides.
"""

from __future__ import annotations

import json
import os
import re
from dataclasses import dataclass, field
from pathlib import Path

import torch

REPO_ROOT = Path(__file__).resolve().parent.parent

# Datasheet peaks: (memory GB/s, FP32 TFLOPS, FP16/BF16 dense tensor TFLOPS),
# matched as a whole word against the device name, first match wins.
KNOWN_GPUS: list[tuple[str, float, float, float]] = [
    ("B200", 7700.0, 75.0, 2250.0),
    ("T4", 320.0, 8.1, 65.0),
    ("V100", 900.0, 15.7, 125.0),
    ("A100-SXM4-80GB", 2039.0, 19.5, 312.0),
    ("A100 80GB", 1935.0, 19.5, 312.0),
    ("A100", 1555.0, 19.5, 312.0),
    ("L4", 300.0, 30.3, 121.0),
    ("H100 PCIe", 2000.0, 51.0, 756.0),
    ("H100", 3350.0, 67.0, 989.0),
    ("RTX 4090", 1008.0, 82.6, 165.2),
    ("MI300X", 5300.0, 163.4, 1307.4),
    ("MI250X", 1638.0, 47.9, 383.0),
    ("MI250", 1638.0, 45.3, 362.1),
    ("MI210", 1638.0, 22.6, 181.0),
    ("MI100", 1228.0, 23.1, 184.6),
    ("7900 XTX", 960.0, 61.4, 122.8),
]


@dataclass
class GPUInfo:
    name: str
    vendor: str  # "nvidia", "amd" or "none"
    peak_bw_gbs: float | None
    peak_tflops: dict[str, float] = field(default_factory=dict)
    source: str = "unknown"

    def peak_for(self, dtype: torch.dtype) -> float | None:
        if dtype == torch.float16:
            return self.peak_tflops.get("float16")
        if dtype == torch.bfloat16:
            return self.peak_tflops.get("bfloat16", self.peak_tflops.get("float16"))
        return self.peak_tflops.get("float32")

    def describe(self) -> str:
        bw = f"{self.peak_bw_gbs:.0f} GB/s" if self.peak_bw_gbs else "unknown BW"
        fl = ", ".join(f"{k} {v:.1f} TFLOPS" for k, v in self.peak_tflops.items()) or "unknown"
        return f"{self.name} ({self.vendor}): {bw}, {fl} [{self.source}]"


def gpu_available() -> bool:
    return torch.cuda.is_available()


def vendor() -> str:
    if not torch.cuda.is_available():
        return "none"
    return "amd" if torch.version.hip else "nvidia"


def lookup_peaks(name: str) -> tuple[float, float, float] | None:
    for key, bw, fp32, fp16 in KNOWN_GPUS:
        if re.search(rf"\b{re.escape(key)}\b", name, flags=re.IGNORECASE):
            return bw, fp32, fp16
    return None


def measured_peaks(path: str | Path | None = None) -> dict | None:
    """The measured copy bandwidth / bf16 GEMM rates, or None when absent."""
    p = Path(path) if path else REPO_ROOT / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return None


def measure_bandwidth_gbs(nbytes: int = 1 << 28, iters: int = 20) -> float:
    """Device-to-device copy bandwidth (read + write bytes), a stand-in peak."""
    src = torch.empty(nbytes // 4, dtype=torch.float32, device="cuda")
    dst = torch.empty_like(src)
    for _ in range(3):
        dst.copy_(src)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        dst.copy_(src)
    end.record()
    torch.cuda.synchronize()
    seconds = start.elapsed_time(end) / 1e3 / iters
    return 2 * nbytes / seconds / 1e9


def get_gpu_info(measured_path: str | Path | None = None) -> GPUInfo:
    if not torch.cuda.is_available():
        return GPUInfo(name="cpu", vendor="none", peak_bw_gbs=None, source="no GPU")
    name = torch.cuda.get_device_name()
    info = GPUInfo(name=name, vendor=vendor(), peak_bw_gbs=None)
    known = lookup_peaks(name)
    if known:
        bw, fp32, fp16 = known
        info.peak_bw_gbs = bw
        info.peak_tflops = {"float32": fp32, "float16": fp16, "bfloat16": fp16}
        info.source = "datasheet"
    meas = measured_peaks(measured_path)
    if meas and meas.get("gpu_name", "") and meas["gpu_name"] in name:
        info.peak_bw_gbs = float(meas["hbm_gbs"])
        if "bf16_tflops" in meas:
            info.peak_tflops["bfloat16"] = float(meas["bf16_tflops"])
            info.peak_tflops["float16"] = float(meas["bf16_tflops"])
        info.source = "measured (MEASURED_PEAKS.json)"
    for env, key in (("KP_PEAK_FP32_TFLOPS", "float32"), ("KP_PEAK_FP16_TFLOPS", "float16"),
                     ("KP_PEAK_BF16_TFLOPS", "bfloat16")):
        if os.environ.get(env):
            info.peak_tflops[key], info.source = float(os.environ[env]), "env"
    if os.environ.get("KP_PEAK_BW_GBS"):
        info.peak_bw_gbs, info.source = float(os.environ["KP_PEAK_BW_GBS"]), "env"
    if info.peak_bw_gbs is None:
        info.peak_bw_gbs = measure_bandwidth_gbs()
        info.source = "measured copy bandwidth (set KP_PEAK_* to override)"
    return info
