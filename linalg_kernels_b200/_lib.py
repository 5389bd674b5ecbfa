"""ctypes binding of ``libchol_b200.so`` (the C ABI declared in include/chol_b200.h).

The library is loaded from the package directory. If it is missing, importing the
compute entry points raises: there is no CPU or torch fallback on the product path.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libchol_b200.so"

# status codes, as in include/chol_b200.h
CHOL_OK = 0
CHOL_ERR_INVALID_ARG = 1
CHOL_ERR_LAUNCH = 2
CHOL_ERR_NOT_SPD = 3
CHOL_ERR_WAIT_TIMEOUT = 4
CHOL_ERR_WORKSPACE = 5
CHOL_ERR_DEVICE = 6
CHOL_ERR_UNSUPPORTED = 7
CHOL_ERR_SCRATCH_LIMIT = 8
CHOL_PANEL_OUT_ONLY = 1

CHOL_OPT_GEMM_ENGINE = 1
CHOL_OPT_OUTER_WIDTH = 3
CHOL_OPT_LOOKAHEAD = 4
CHOL_OPT_CHAIN_SMS = 5
CHOL_OPT_PANEL_INVERSE = 6
CHOL_OPT_OVERLAP_CALLS = 7
CHOL_OPT_MID_KERNEL = 8
CHOL_OPT_WAIT_LIMIT_US = 9
CHOL_OPT_CHAIN_WIDTH = 10
CHOL_OPT_GEMM_CTAS = 11
ENGINE_AUTO, ENGINE_FMA, ENGINE_TENSOR = 0, 1, 2

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_int = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes); every function include/chol_b200.h declares
SIGNATURES: dict[str, tuple] = {
    "chol_version": (_int, []),
    "chol_strerror": (ctypes.c_char_p, [_int]),
    "chol_prepare": (_int, [_int]),
    "chol_workspace_bytes": (_sz, [_i64, _i64]),
    "chol_potrf_batched_f32": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "chol_potrf_batched_ws_f32": (_int, [_vp, _vp, _i64, _i64, _vp, _vp, _sz, _vp]),
    "chol_potrf_batched_noalloc_f32": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "chol_launch_count": (_i64, [_i64, _i64]),
    "chol_set_option": (_int, [_int, _int]),
    "chol_status_check": (_int, [_vp]),
    "chol_overlap_stats": (_int, [ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "chol_test_flag_wait": (_int, [_vp, _int, _vp]),
    "chol_info_check": (_int, [_vp, _i64, _vp, ctypes.POINTER(_i64)]),
    "chol_block_potrf_f32": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
    "chol_gemm_nt_f32": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64,
                                _vp, _i64, _i64, _f32, _f32, _i64, _int, _vp]),
    "chol_panel_potrf_f32": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "chol_panel_potrf_out_f32": (_int, [_vp, _i64, _i64, _i64, _vp, _int, _vp, _vp]),
    "chol_diag_potrf_inv_f32": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "chol_gemm_nt_cyclic_f32": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _f32,
                                       _f32, _i64, _int, _i64, _i64, _vp]),
    "chol_validate_work_bytes": (_sz, [_i64, _i64]),
    "chol_validate_f32": (_int, [_vp, _vp, _i64, _i64, _vp, _vp, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class CholeskyError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {strerror(status)} (status {status})")


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with every signature bound."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise ImportError(
                f"{p} is missing: build it with `python -m linalg_kernels_b200.build` "
                "(this package has no CPU fallback)")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


_pyext = None


def potrf_ws(a: int, l: int, batch: int, n: int, info: int, ws: int, ws_bytes: int,
             queue: int) -> int:
    """chol_potrf_batched_ws_f32 through the CPython fast-call binding (_cholpy), falling
    back to ctypes when the binding is not built. Integer arguments, 0 for NULL."""
    global _pyext
    if _pyext is None:
        load()
        try:
            from . import _cholpy  # type: ignore

            _pyext = _cholpy.potrf_ws
        except ImportError:
            lib = load()

            def _via_ctypes(*args):
                return lib.chol_potrf_batched_ws_f32(*[x if x else None for x in args[:2]],
                                                     args[2], args[3], args[4] or None,
                                                     args[5] or None, args[6], args[7] or None)

            _pyext = _via_ctypes
    return _pyext(a, l, batch, n, info, ws, ws_bytes, queue)


def strerror(status: int) -> str:
    try:
        return load().chol_strerror(int(status)).decode()
    except ImportError:
        return f"status {status}"


def check(status: int, where: str) -> None:
    if status != CHOL_OK:
        raise CholeskyError(status, where)


def fast_call():
    """(binding, queue getter) for the hot path: the chol_potrf_batched_ws_f32 binding (as
    potrf_ws takes it) and a function mapping a device index to the raw handle of torch's
    current queue there; None when torch has no raw getter."""
    import torch

    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is None:
        return None
    potrf_ws(0, 0, 0, 0, 0, 0, 0, 0)  # resolves the binding (an empty call does nothing)
    return _pyext, raw


def current_queue(device) -> int:
    """Raw handle of torch's current CUDA queue on ``device`` (0 = legacy default)."""
    import torch

    idx = device.index if isinstance(device, torch.device) else device
    if idx is None:
        idx = torch.cuda.current_device()
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:  # no Python queue object per call
        return int(raw(idx))
    return int(torch.cuda.current_stream(idx).cuda_stream)
