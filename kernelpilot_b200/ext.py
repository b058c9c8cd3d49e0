"""Loads the in-tree libraries: ``torch.ops.kp`` (libkernelpilot_ops.so) and the
C ABI (libkp_b200.so, via ctypes).

Same contract as kernelpilot/ext.py: ``library_path()`` honours ``KP_EXT_PATH``,
``load()`` returns False instead of raising when the library is absent or no GPU is
present, and ``ops()`` raises with a build hint. There is no CPU fallback anywhere:
on a machine without the built library every op fails loudly.
"""

from __future__ import annotations

import ctypes
import os
from functools import lru_cache
from pathlib import Path

import torch

PKG_DIR = Path(__file__).resolve().parent
LIB_DIR = PKG_DIR / "_lib"
OPS_NAME = "libkernelpilot_ops.so"
CAPI_NAME = "libkp_b200.so"


def library_path() -> Path | None:
    env = os.environ.get("KP_EXT_PATH")
    if env:
        return Path(env)
    p = LIB_DIR / OPS_NAME
    return p if p.exists() else None


def capi_path() -> Path:
    return LIB_DIR / CAPI_NAME


@lru_cache(maxsize=1)
def load() -> bool:
    """Load the operator library once; False when it is missing or there is no GPU."""
    path = library_path()
    if path is None or not path.exists() or not torch.cuda.is_available():
        return False
    torch.ops.load_library(str(path))
    return True


def ops():
    if not load():
        raise RuntimeError(
            "kernelpilot_b200 extension not built or no GPU available; run "
            "`python -m kernelpilot_b200.build` (or set KP_EXT_PATH to the built library)."
        )
    return torch.ops.kp


# ------------------------------------------------------------------ C ABI (ctypes)

_i32, _i64, _sz, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p
_fp = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes); every function declared in include/kp_b200.h
CAPI_SIGNATURES: dict[str, tuple] = {
    "kpb_last_error": (ctypes.c_char_p, []),
    "kpb_version": (_i32, []),
    "kpb_num_variants": (_i32, [ctypes.c_char_p]),
    "kpb_device_errors": (_i32, [ctypes.POINTER(ctypes.c_uint)]),
    "kpb_vector_add": (_i32, [_i32, _i32, _vp, _vp, _vp, _i64, _vp]),
    "kpb_reduce_sum": (_i32, [_i32, _i32, _vp, _vp, _i64, _vp]),
    "kpb_reduce_sum_workspace_bytes": (_sz, [_i32, _i64]),
    "kpb_reduce_sum_ws": (_i32, [_i32, _i32, _vp, _vp, _i64, _vp, _sz, _vp]),
    "kpb_reduce_sum_noalloc": (_i32, [_i32, _vp, _vp, _i64, _vp]),
    "kpb_peer_sum_handle_bytes": (_sz, []),
    "kpb_peer_sum_create": (_i32, [_i32, _i32, _vp, ctypes.POINTER(_vp)]),
    "kpb_peer_sum_connect": (_i32, [_vp, _vp]),
    "kpb_peer_sum_workspace_bytes": (_sz, [_i64]),
    "kpb_peer_sum_run": (_i32, [_vp, _i32, _vp, _vp, _i64, _vp, _sz, _vp]),
    "kpb_peer_sum_status": (_i32, [_vp, ctypes.POINTER(_i32)]),
    "kpb_peer_sum_destroy": (_i32, [_vp]),
    "kpb_softmax": (_i32, [_i32, _i32, _vp, _vp, _i64, _i64, _vp]),
    "kpb_matmul": (_i32, [_i32, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "kpb_matmul_workspace_bytes": (_sz, [_i32, _i32, _i64, _i64, _i64]),
    "kpb_matmul_ws": (_i32, [_i32, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "kpb_layernorm": (_i32, [_i32, _i32, _vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp]),
    "kpb_attention": (_i32, [_i32, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "kpb_attention_causal": (_i32, [_i32, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
}

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


@lru_cache(maxsize=1)
def capi() -> ctypes.CDLL:
    """The C ABI library with argument types set. Loads without a GPU."""
    path = capi_path()
    if not path.exists():
        raise RuntimeError(f"{path} not built; run `python -m kernelpilot_b200.build`")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in CAPI_SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


def capi_check(rc: int) -> None:
    if rc != 0:
        msg = capi().kpb_last_error().decode()
        raise RuntimeError(f"kp_b200 call failed (status {rc}): {msg}")


def current_stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream
