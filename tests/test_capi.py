"""The C ABI library (include/kp_b200.h) without a GPU: it loads, exports every
function the header declares, and rejects bad arguments with status codes and a
message before touching the device."""

import ctypes
import re
from pathlib import Path

import pytest

from kernelpilot_b200 import ext

HEADER = Path(__file__).resolve().parent.parent / "include" / "kp_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(kpb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return ext.capi()


def test_header_declares_the_op_suite():
    names = declared_functions()
    for op in ["kpb_reduce_sum", "kpb_softmax", "kpb_matmul", "kpb_attention",
               "kpb_attention_causal", "kpb_last_error"]:
        assert op in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} missing from {ext.capi_path()}"
        assert name in ext.CAPI_SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_variant_counts(lib):
    assert lib.kpb_version() >= 100
    assert lib.kpb_num_variants(b"reduce_sum") == 3
    assert lib.kpb_num_variants(b"softmax") == 3
    assert lib.kpb_num_variants(b"matmul") == 4
    assert lib.kpb_num_variants(b"attention") == 2
    assert lib.kpb_num_variants(b"attention_causal") == 2
    assert lib.kpb_num_variants(b"vector_add") == 3
    assert lib.kpb_num_variants(b"layernorm") == 3
    assert lib.kpb_num_variants(b"rmsnorm") == -1


def test_variant_counts_match_registry(lib):
    from kernelpilot_b200.registry import CUDA_STAGES
    for op, stages in CUDA_STAGES.items():
        assert lib.kpb_num_variants(op.encode()) == len(stages)


@pytest.mark.parametrize("call,needle", [
    (lambda L: L.kpb_softmax(3, 0, None, None, 4, 4, None), "variant"),
    (lambda L: L.kpb_softmax(2, 9, None, None, 4, 4, None), "dtype"),
    (lambda L: L.kpb_softmax(2, 0, None, None, -1, 4, None), "M and N"),
    (lambda L: L.kpb_softmax(2, 0, None, None, 4, 4, None), "null"),
    (lambda L: L.kpb_reduce_sum(0, 0, None, None, 5, None), "null"),
    (lambda L: L.kpb_vector_add(3, 0, None, None, None, 5, None), "variant"),
    (lambda L: L.kpb_vector_add(2, 0, None, None, None, -1, None), "n must be"),
    (lambda L: L.kpb_vector_add(2, 0, None, None, None, 5, None), "null"),
    (lambda L: L.kpb_layernorm(3, 0, None, None, None, None, 4, 4, 1e-5, None), "variant"),
    (lambda L: L.kpb_layernorm(2, 5, None, None, None, None, 4, 4, 1e-5, None), "dtype"),
    (lambda L: L.kpb_layernorm(2, 0, None, None, None, None, 4, 1 << 31, 1e-5, None), "M and N"),
    (lambda L: L.kpb_layernorm(2, 0, None, None, None, None, 4, 4, 1e-5, None), "null"),
    (lambda L: L.kpb_matmul_ws(4, 2, None, None, None, 2, 2, 2, None, 0, None), "variant"),
    (lambda L: L.kpb_matmul_ws(3, 2, None, None, None, 1 << 31, 2, 2, None, 0, None), "2^31"),
    (lambda L: L.kpb_attention(1, 2, None, None, None, None, 1, 8, 300, None), "D <= 256"),
    (lambda L: L.kpb_attention_causal(1, 2, None, None, None, None, 70000, 8, 64, None),
     "B*H"),
])
def test_bad_arguments_are_rejected_without_a_device(lib, call, needle):
    rc = call(lib)
    assert rc == 1  # KPB_EINVAL
    assert needle in lib.kpb_last_error().decode()


def test_workspace_queries(lib):
    assert lib.kpb_reduce_sum_workspace_bytes(0, 0) == 0
    assert lib.kpb_reduce_sum_workspace_bytes(0, 4096) == 4 * 4
    assert lib.kpb_reduce_sum_workspace_bytes(2, (1 << 28) + 1) >= 148 * 4
    assert lib.kpb_matmul_workspace_bytes(3, 0, 64, 64, 64) == 0  # fp32 needs none


def test_ctypes_types_are_plain():
    # the boundary has no torch types: every argument is an int, a float, a size or a pointer
    allowed = {ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float,
               ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_void_p),
               ctypes.POINTER(ctypes.c_int)}
    for _name, (_res, args) in ext.CAPI_SIGNATURES.items():
        assert all(a in allowed for a in args)


def test_peer_sum_rejects_bad_arguments_without_a_gpu(lib):
    # argument checks come before any CUDA call
    handle = ctypes.create_string_buffer(lib.kpb_peer_sum_handle_bytes())
    ps = ctypes.c_void_p()
    assert lib.kpb_peer_sum_handle_bytes() == 64  # a cudaIpcMemHandle_t
    assert lib.kpb_peer_sum_create(0, 9, handle, ctypes.byref(ps)) == 1
    assert b"world" in lib.kpb_last_error()
    assert lib.kpb_peer_sum_create(2, 2, handle, ctypes.byref(ps)) == 1
    assert lib.kpb_peer_sum_create(0, 2, None, ctypes.byref(ps)) == 1
    assert lib.kpb_peer_sum_connect(None, handle) == 1
    assert lib.kpb_peer_sum_run(None, 0, None, None, 10, None, 0, None) == 1
    assert lib.kpb_peer_sum_destroy(None) == 0
    assert lib.kpb_peer_sum_workspace_bytes(0) == 0
    assert lib.kpb_peer_sum_workspace_bytes(1 << 20) >= 4


def test_peer_sum_status_rejects_null_without_a_gpu(lib):
    flag = ctypes.c_int(7)
    assert lib.kpb_peer_sum_status(None, ctypes.byref(flag)) == 1
    assert b"null" in lib.kpb_last_error()
