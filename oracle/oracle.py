"""CPU ORACLE for the batched Cholesky hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference
arm may import this module, and only as the checker or the CPU baseline. The product
path (``linalg_kernels_b200``) never calls it.

Contents:
* ``potrf``     — float32 LAPACK SPOTRF (lower) restated in plain C (``potrf_ref.c``),
                  the algorithm of the reference's path (torch.linalg.cholesky_ex ->
                  LAPACK, cholesky/cholesky.py:5850, submission.py:6-7).
* ``dpotrf``    — float64 factor of the same float32 input (diagnostics).
* ``reference_factor`` — the reference's own call, ``torch.linalg.cholesky_ex(A,
                  check_errors=False).L`` (submission.py:7) on CPU tensors (MKL 2024.2).
* property gates and the parity tolerance:
    - the reference harness gate (cholesky/b4096n32/cholesky_b4096n32_modal.py:307-334):
      finite, exact-zero strict upper, positive diagonal, scaled inf-norm residual
      max_row_sum|A - L L^T| / (eps * n * max_row_sum|A|) <= max(16, 8 * torch's own);
    - ||L L^T - A||_F / ||A||_F <= 1e-5 and
      max|L - L_ref| <= cond(A) * n * eps_fp32 * max|L_ref| per matrix.

Pinning: tests/test_oracle.py checks ``potrf`` against tests/golden/*.npz, which hold
outputs of the reference's own ``custom_kernel`` run in this container
(tests/golden/make_golden.py), and against known answers (diagonal, tridiagonal).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "potrf_ref.c"
LIB = HERE / "_build" / "liboracle.so"

EPS32 = float(np.finfo(np.float32).eps)
REL_RESIDUAL_TOL = 1e-5  # north star: ||L L^T - A||_F / ||A||_F

_lib = None


def build(force: bool = False) -> Path:
    """Compile potrf_ref.c with gcc (no FMA contraction, IEEE float32)."""
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".tmp.so")
    subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
                    "-o", str(tmp), str(SRC), "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        lib.oracle_spotrf_batched.restype = ctypes.c_int
        lib.oracle_spotrf_batched.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_long,
                                              ctypes.c_long, ctypes.c_int, ctypes.c_void_p]
        lib.oracle_dpotrf_batched.restype = ctypes.c_int
        lib.oracle_dpotrf_batched.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_long,
                                              ctypes.c_long, ctypes.c_void_p]
        _lib = lib
    return _lib


def _as_batch(a) -> tuple[np.ndarray, tuple]:
    a = np.asarray(a, dtype=np.float32)
    shape = a.shape
    if a.ndim < 2 or shape[-1] != shape[-2]:
        raise ValueError(f"expected (..., n, n), got {shape}")
    return np.ascontiguousarray(a.reshape(-1, shape[-1], shape[-1])), shape


def potrf(a, nb: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """float32 lower Cholesky (LAPACK SPOTRF restated). Returns (L, info)."""
    ab, shape = _as_batch(a)
    out = np.empty_like(ab)
    info = np.zeros(ab.shape[0], dtype=np.int32)
    _load().oracle_spotrf_batched(ab.ctypes.data, out.ctypes.data, ab.shape[0], ab.shape[1],
                                  int(nb), info.ctypes.data)
    return out.reshape(shape), info.reshape(shape[:-2])


def dpotrf(a) -> tuple[np.ndarray, np.ndarray]:
    """float64 factor of the float32 input (lower triangle). Returns (L64, info)."""
    ab, shape = _as_batch(a)
    out = np.zeros(ab.shape, dtype=np.float64)
    info = np.zeros(ab.shape[0], dtype=np.int32)
    _load().oracle_dpotrf_batched(ab.ctypes.data, out.ctypes.data, ab.shape[0], ab.shape[1],
                                  info.ctypes.data)
    return out.reshape(shape), info.reshape(shape[:-2])


def reference_factor(a_cpu_tensor):
    """The reference path itself on CPU: torch.linalg.cholesky_ex(A, check_errors=False).L
    (submission.py:7; cholesky/cholesky.py:5850)."""
    import torch

    return torch.linalg.cholesky_ex(a_cpu_tensor, check_errors=False).L


# ----------------------------------------------------------------------------------
# property gates and tolerances (float64 arithmetic on host arrays)
# ----------------------------------------------------------------------------------
def sym_from_lower(a: np.ndarray) -> np.ndarray:
    """The symmetric matrix the lower triangle of `a` defines (what uplo='L' factors)."""
    a = np.asarray(a, dtype=np.float64)
    low = np.tril(a)
    return low + np.swapaxes(np.tril(a, -1), -1, -2)


def rel_residual_fro(a, l) -> np.ndarray:
    """||L L^T - A||_F / ||A||_F per matrix (A taken from its lower triangle)."""
    s = sym_from_lower(a)
    l64 = np.asarray(l, dtype=np.float64)
    r = l64 @ np.swapaxes(l64, -1, -2) - s
    return np.linalg.norm(r, axis=(-2, -1)) / np.linalg.norm(s, axis=(-2, -1))


def scaled_inf_residual(a, l) -> np.ndarray:
    """max_row_sum|A - L L^T| / (eps32 * n * max_row_sum|A|) per matrix."""
    s = sym_from_lower(a)
    l64 = np.asarray(l, dtype=np.float64)
    r = np.abs(s - l64 @ np.swapaxes(l64, -1, -2)).sum(axis=-1).max(axis=-1)
    d = np.maximum(np.abs(s).sum(axis=-1).max(axis=-1), 1e-30)
    return r / (EPS32 * s.shape[-1] * d)


def factor_diff_bound(cond, n: int, l_ref) -> np.ndarray:
    """North-star elementwise bound: cond(A) * n * eps32 * max|L_ref| per matrix."""
    lr = np.abs(np.asarray(l_ref, dtype=np.float64)).reshape(-1, n * n).max(axis=1)
    return np.asarray(cond, dtype=np.float64).reshape(-1) * n * EPS32 * lr


def check_factor(a, l, l_ref=None, cond=None, ref_scaled=None) -> dict:
    """All gates for one batch. Returns a dict with 'ok' and the measured quantities."""
    a = np.asarray(a, dtype=np.float32)
    l = np.asarray(l, dtype=np.float32)
    n = a.shape[-1]
    lb = l.reshape(-1, n, n)
    ab = a.reshape(-1, n, n)
    out: dict = {}
    out["finite"] = bool(np.isfinite(lb).all())
    out["upper_max"] = float(np.abs(np.triu(lb, 1)).max()) if n > 1 else 0.0
    out["diag_min"] = float(np.diagonal(lb, axis1=1, axis2=2).min())
    rel = rel_residual_fro(ab, lb) if out["finite"] else np.array([np.inf])
    out["rel_residual_max"] = float(rel.max())
    scaled = scaled_inf_residual(ab, lb) if out["finite"] else np.array([np.inf])
    out["scaled_residual_max"] = float(scaled.max())
    gate = 16.0 if ref_scaled is None else max(16.0, 8.0 * float(ref_scaled))
    out["scaled_gate"] = gate
    ok = (out["finite"] and out["upper_max"] == 0.0 and out["diag_min"] > 0.0
          and out["rel_residual_max"] <= REL_RESIDUAL_TOL and out["scaled_residual_max"] <= gate)
    if l_ref is not None:
        lr = np.asarray(l_ref, dtype=np.float32).reshape(-1, n, n)
        diff = np.abs(lb.astype(np.float64) - lr.astype(np.float64)).reshape(-1, n * n).max(axis=1)
        out["max_abs_diff"] = float(diff.max())
        if cond is not None:
            bound = factor_diff_bound(cond, n, lr)
            out["diff_over_bound"] = float((diff / bound).max())
            ok = ok and bool((diff <= bound).all())
    out["ok"] = bool(ok)
    return out
