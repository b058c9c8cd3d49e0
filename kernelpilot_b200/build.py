"""Builds the two shared libraries in-tree under kernelpilot_b200/_lib/:

* ``libkp_b200.so``        the sm_100a kernels and the extern "C" ABI of
                           include/kp_b200.h (static cudart, no torch dependency);
* ``libkernelpilot_ops.so`` the ``torch.ops.kp`` operators (csrc/bindings.cpp),
                           linked against libkp_b200.so.

This replaces kernelpilot's CMakeLists.txt/Makefile (:15-52 there: ROCm or CUDA,
``.hip`` copied to ``.cu``, arch ``native`` or 75) with one CUDA-only recipe whose
only device target is ``sm_100a``. Objects are rebuilt when their source or any
header is newer; ``python -m kernelpilot_b200.build`` runs it.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
OBJ_DIR = REPO / "_build" / "obj"
INCLUDE = REPO / "include"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC", "-Xptxas", "-v", *ARCH]

CAPI_LIB = LIB_DIR / "libkp_b200.so"
OPS_LIB = LIB_DIR / "libkernelpilot_ops.so"


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], log: Path | None = None) -> str:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    out = proc.stdout + proc.stderr
    if log is not None:
        log.write_text(out)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{out}")
    return out


def _compile_cu(src: Path) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    if _stale(obj, [src, *_headers()]):
        _run([NVCC, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)],
             log=OBJ_DIR / (src.stem + ".ptxas.txt"))
    return obj


def build_capi(jobs: int = 8) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(_compile_cu, sources))
    if _stale(CAPI_LIB, objs):
        _run([NVCC, "-shared", *ARCH, "-o", str(CAPI_LIB), *map(str, objs),
              "-cudart", "static", "-Xlinker", "--no-undefined"])
    return CAPI_LIB


def build_ops() -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "bindings.cpp"
    if not _stale(OPS_LIB, [src, CAPI_LIB, *_headers()]):
        return OPS_LIB
    torch_lib = Path(torch.__file__).parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in cpp_extension.include_paths()]
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *incs, f"-I{INCLUDE}", str(src), "-o", str(OPS_LIB),
           f"-L{LIB_DIR}", "-lkp_b200", f"-L{torch_lib}", "-ltorch_cpu", "-lc10",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    _run(cmd)
    return OPS_LIB


def build(jobs: int = 8) -> tuple[Path, Path]:
    capi = build_capi(jobs)
    ops = build_ops()
    return capi, ops


def ptxas_report() -> str:
    """Registers / spills / shared memory per kernel from the last build."""
    return "\n".join(p.read_text() for p in sorted(OBJ_DIR.glob("*.ptxas.txt")))


if __name__ == "__main__":
    capi, ops = build()
    print(capi)
    print(ops)
    if "-v" in sys.argv:
        print(ptxas_report())
