"""Device-side check of a Cholesky factor: the property gates of the reference's checker.

The reference's checker (its leaderboard's ``check_implementation``, called by the
evaluator at references/popcorn-eval/eval.py:133, 186-189, 207-211; the file itself is not
in the reference tree) validates shape, dtype, device, finiteness, lower-triangular
structure, positive diagonal and the reconstruction residual against the original FP32
input (AGENTS.md:47-50). Its Modal harness adds the scaled inf-norm gate
max_i sum_j |A - L L^T|_ij / (eps * n * max_i sum_j |A_ij|) <= max(16, 8 x torch's own)
(cholesky/b4096n32/cholesky_b4096n32_modal.py:307-334).

Here the residuals come from ``chol_validate_f32``, two kernels that form tril(L) tril(L)^T
with FP64 accumulation on the GPU, so a factor never leaves the device (at n = 32768 a
host check needs a 4 GiB copy and minutes of CPU time). The Frobenius gate is the north
star's ||L L^T - A||_F / ||A||_F <= 1e-5.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

REL_RESIDUAL_TOL = 1e-5
SCALED_GATE = 16.0
EPS32 = float(torch.finfo(torch.float32).eps)

_FIELDS = ("res2", "a2", "res_rowsum_max", "a_rowsum_max", "nonfinite", "upper_nonzero",
           "diag_not_positive")


def validate(a: torch.Tensor, l: torch.Tensor) -> dict[str, torch.Tensor]:
    """Per-matrix gate quantities (float64 host tensors of the leading batch shape) of the
    factor ``l`` of ``a`` (CUDA float32 tensors of the same shape (..., n, n)).

    rel_residual = ||tril(L) tril(L)^T - S||_F / ||S||_F, scaled_residual = the inf-norm
    gate's ratio, nonfinite / upper_nonzero / diag_not_positive = entry counts; S is the
    symmetric matrix the lower triangle of A defines."""
    if not (isinstance(a, torch.Tensor) and isinstance(l, torch.Tensor)):
        raise TypeError("validate expects tensors")
    if a.shape != l.shape or a.dim() < 2 or a.shape[-1] != a.shape[-2]:
        raise ValueError(f"expected two (..., n, n) tensors, got {tuple(a.shape)} and "
                         f"{tuple(l.shape)}")
    if not (a.is_cuda and l.is_cuda) or a.device != l.device:
        raise TypeError("validate runs on the GPU: both tensors on the same CUDA device")
    if a.dtype != torch.float32 or l.dtype != torch.float32:
        raise TypeError("validate expects float32 tensors")
    lead = a.shape[:-2]
    n = a.shape[-1]
    batch = 1
    for d in lead:
        batch *= int(d)
    a3 = a.reshape(batch, n, n).contiguous()
    l3 = l.reshape(batch, n, n).contiguous()
    out = torch.zeros(batch, 8, dtype=torch.float64, device=a.device)
    if batch == 0 or n == 0:
        stats = out.cpu()
    else:
        lib = _lib.load()
        work = torch.empty(int(lib.chol_validate_work_bytes(batch, n)), dtype=torch.uint8,
                           device=a.device)
        with torch.cuda.device(a.device):
            queue = _lib.current_queue(a.device)
            st = lib.chol_validate_f32(ctypes.c_void_p(a3.data_ptr()),
                                       ctypes.c_void_p(l3.data_ptr()), batch, n,
                                       ctypes.c_void_p(out.data_ptr()),
                                       ctypes.c_void_p(work.data_ptr()), ctypes.c_void_p(queue))
            _lib.check(st, "chol_validate_f32")
            stats = out.cpu()  # synchronises with the queue
    raw = {k: stats[:, i] for i, k in enumerate(_FIELDS)}
    rel = torch.sqrt(raw["res2"]) / torch.sqrt(raw["a2"]).clamp_min(1e-300)
    scaled = raw["res_rowsum_max"] / (EPS32 * max(n, 1) * raw["a_rowsum_max"].clamp_min(1e-30))
    res = {"rel_residual": rel, "scaled_residual": scaled, "nonfinite": raw["nonfinite"],
           "upper_nonzero": raw["upper_nonzero"],
           "diag_not_positive": raw["diag_not_positive"]}
    return {k: v.reshape(lead) for k, v in res.items()}


def check_implementation(data: torch.Tensor, output, rel_tol: float = REL_RESIDUAL_TOL,
                         scaled_gate: float = SCALED_GATE) -> tuple[bool, str]:
    """(good, message) for the factor ``output`` of ``data``, in the evaluator's calling
    convention. Fails on the first gate a matrix misses and names the matrix."""
    if not isinstance(output, torch.Tensor):
        return False, f"output is a {type(output).__name__}, not a tensor"
    if output.shape != data.shape:
        return False, f"output shape {tuple(output.shape)} != input shape {tuple(data.shape)}"
    if output.dtype != torch.float32:
        return False, f"output dtype {output.dtype}, expected torch.float32"
    if output.device != data.device:
        return False, f"output on {output.device}, input on {data.device}"
    v = validate(data, output)
    flat = {k: t.reshape(-1) for k, t in v.items()}
    gates = (
        ("nonfinite", lambda x: x == 0, "non-finite entries"),
        ("upper_nonzero", lambda x: x == 0, "non-zero entries above the diagonal"),
        ("diag_not_positive", lambda x: x == 0, "diagonal entries that are not positive"),
        ("rel_residual", lambda x: x <= rel_tol, f"relative residual above {rel_tol:g}"),
        ("scaled_residual", lambda x: x <= scaled_gate,
         f"scaled inf-norm residual above {scaled_gate:g}"),
    )
    for key, ok, what in gates:
        good = ok(flat[key])
        if not bool(good.all()):
            m = int((~good).nonzero()[0, 0])
            return False, f"matrix {m}: {what} ({flat[key][m].item():.6g})"
    return True, ""
