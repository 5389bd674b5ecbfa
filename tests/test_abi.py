"""CPU: the C-ABI library loads, exports every symbol include/chol_b200.h declares, and its
host-side argument checks behave (no compute call is made without a GPU)."""

import ctypes
import re
from pathlib import Path

import pytest

from linalg_kernels_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "chol_b200.h").read_text()
    return re.findall(r"^CHOL_API\s+[\w\s\*]+?\b(chol_\w+)\s*\(", text, flags=re.M)


def test_header_declares_expected_entry_points():
    names = header_functions()
    for required in ("chol_potrf_batched_f32", "chol_potrf_batched_ws_f32", "chol_prepare",
                     "chol_strerror", "chol_workspace_bytes", "chol_info_check"):
        assert required in names


def test_library_exports_every_header_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in header_functions():
        assert hasattr(lib, name), name
    # and the Python binding declares a signature for each
    assert set(header_functions()) == set(_lib.SIGNATURES)


def test_version_and_strerror():
    lib = _lib.load()
    assert lib.chol_version() >= 100
    for code in range(8):
        assert lib.chol_strerror(code)
    assert lib.chol_strerror(0) == b"success"
    assert b"unknown" in lib.chol_strerror(12345)


def test_workspace_bytes():
    lib = _lib.load()
    assert lib.chol_workspace_bytes(4096, 32) == 0  # register kernel needs none
    assert lib.chol_workspace_bytes(0, 512) == 0
    assert lib.chol_workspace_bytes(640, 512) >= 640 * 64 * 64 * 4


@pytest.mark.parametrize("batch,n", [(-1, 4), (2, -3)])
def test_invalid_shapes_rejected_before_device_work(batch, n):
    lib = _lib.load()
    assert lib.chol_potrf_batched_f32(None, None, batch, n, None, None) == _lib.CHOL_ERR_INVALID_ARG
    assert lib.chol_potrf_batched_ws_f32(None, None, batch, n, None, None, 0, None) == \
        _lib.CHOL_ERR_INVALID_ARG


def test_empty_problem_is_ok():
    lib = _lib.load()
    assert lib.chol_potrf_batched_f32(None, None, 0, 32, None, None) == _lib.CHOL_OK
    assert lib.chol_potrf_batched_f32(None, None, 5, 0, None, None) == _lib.CHOL_OK


def test_null_pointers_rejected():
    lib = _lib.load()
    assert lib.chol_potrf_batched_f32(None, None, 2, 8, None, None) == _lib.CHOL_ERR_INVALID_ARG


def test_partial_overlap_rejected():
    lib = _lib.load()
    buf = (ctypes.c_float * 1024)()
    base = ctypes.addressof(buf)
    # A and L overlap by all but 4 floats: rejected before any device call
    st = lib.chol_potrf_batched_f32(ctypes.c_void_p(base), ctypes.c_void_p(base + 16), 1, 8,
                                    None, None)
    assert st == _lib.CHOL_ERR_INVALID_ARG


def test_gemm_and_block_argument_checks():
    lib = _lib.load()
    assert lib.chol_block_potrf_f32(None, 1, 64, 64, 0, 65, None, None, None) == \
        _lib.CHOL_ERR_INVALID_ARG
    assert lib.chol_block_potrf_f32(None, 1, 64, 64, 0, 8, None, None, None) == \
        _lib.CHOL_ERR_INVALID_ARG
    buf = (ctypes.c_float * 64)()
    p = ctypes.c_void_p(ctypes.addressof(buf))
    # in-place only with beta == 0
    assert lib.chol_gemm_nt_f32(p, 1, 0, 8, 8, 8, 8, p, 0, 8, p, 0, 8, 1.0, 1.0, 0, 0, None) == \
        _lib.CHOL_ERR_INVALID_ARG
    # ldc smaller than ncols
    assert lib.chol_gemm_nt_f32(p, 1, 0, 4, 8, 8, 8, p, 0, 8, p, 0, 8, 1.0, 0.0, 0, 0, None) == \
        _lib.CHOL_ERR_INVALID_ARG
    assert lib.chol_gemm_nt_f32(p, 0, 0, 8, 8, 8, 8, p, 0, 8, p, 0, 8, 1.0, 0.0, 0, 0, None) == \
        _lib.CHOL_OK


def test_info_check_without_entries():
    lib = _lib.load()
    first = ctypes.c_int64(7)
    assert lib.chol_info_check(None, 0, None, ctypes.byref(first)) == _lib.CHOL_OK
    assert first.value == -1


def test_validate_argument_checks():
    """chol_validate_f32's host-side checks run before any device call."""
    lib = _lib.load()
    assert lib.chol_validate_work_bytes(3, 100) == 2 * 3 * 100 * 8
    assert lib.chol_validate_work_bytes(0, 100) == 0
    assert lib.chol_validate_f32(None, None, 0, 16, None, None, None) == _lib.CHOL_OK
    assert lib.chol_validate_f32(None, None, -1, 16, None, None, None) == \
        _lib.CHOL_ERR_INVALID_ARG
    assert lib.chol_validate_f32(None, None, 2, 16, None, None, None) == \
        _lib.CHOL_ERR_INVALID_ARG
    buf = (ctypes.c_double * 64)()
    p = ctypes.addressof(buf)
    # a misaligned output pointer is rejected
    assert lib.chol_validate_f32(ctypes.c_void_p(p), ctypes.c_void_p(p), 1, 4,
                                 ctypes.c_void_p(p + 4), ctypes.c_void_p(p), None) == \
        _lib.CHOL_ERR_INVALID_ARG


def test_check_implementation_contract_on_the_host():
    """The shape / dtype / device gates answer without a GPU; the residual gates need one
    (no CPU fallback)."""
    import torch

    from linalg_kernels_b200.validate import check_implementation, validate

    a = torch.eye(4).expand(2, 4, 4).contiguous()
    assert check_implementation(a, a[:1]) == (False, "output shape (1, 4, 4) != input shape "
                                                     "(2, 4, 4)")
    assert check_implementation(a, a.double())[0] is False
    assert check_implementation(a, None)[0] is False
    with pytest.raises(TypeError, match="GPU"):
        validate(a, a)
