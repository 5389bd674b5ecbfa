"""GPU: the tcgen05 3xTF32 NT-GEMM (chol_gemm_nt_f32, tensor-core engine) against an FP64
reference, and against the FP32-FMA engine. Tolerance: 3xTF32 keeps every product to
~2^-21 relative, so |C - C64| <= 8 * K * 2^-22 * max|P| * max|Q| (+ FP32 rounding of C)."""

import ctypes

import pytest
import torch

from linalg_kernels_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _gemm(c, p, q, m, ncols, k, ldc, ldp, ldq, alpha, beta, lower, diag_offset, batch,
          cstride, pstride, qstride, engine):
    lib = _lib.load()
    lib.chol_set_option(_lib.CHOL_OPT_GEMM_ENGINE, engine)
    try:
        st = lib.chol_gemm_nt_f32(
            ctypes.c_void_p(c), batch, cstride, ldc, m, ncols, k, ctypes.c_void_p(p), pstride, ldp,
            ctypes.c_void_p(q), qstride, ldq, alpha, beta, diag_offset, lower,
            ctypes.c_void_p(_lib.current_queue(torch.device(DEV))))
        torch.cuda.synchronize()
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_GEMM_ENGINE, _lib.ENGINE_AUTO)
    return st


CASES = [
    # m, ncols, K, lower, batch, alpha, beta
    (128, 64, 64, 0, 1, 1.0, 0.0),
    (200, 64, 64, 0, 3, 1.0, 0.0),
    (256, 256, 128, 1, 2, -1.0, 1.0),
    (300, 180, 96, 1, 1, -1.0, 1.0),
    (512, 512, 512, 1, 1, -1.0, 1.0),
    (130, 257, 33, 0, 2, 0.5, -2.0),
    (1000, 600, 64, 1, 1, -1.0, 1.0),
    (64, 100, 160, 0, 5, 1.0, 1.0),
]


@pytest.mark.parametrize("m,ncols,K,lower,batch,alpha,beta", CASES)
@pytest.mark.parametrize("engine", [_lib.ENGINE_TENSOR, _lib.ENGINE_FMA])
def test_gemm_against_fp64(m, ncols, K, lower, batch, alpha, beta, engine):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + ncols * 13 + K)
    ld = ((K + 3) // 4) * 4 + 4
    ldc = ((ncols + 3) // 4) * 4 + 8
    p = torch.randn(batch, m, ld, device=DEV, generator=g)
    q = torch.randn(batch, ncols, ld, device=DEV, generator=g)
    c0 = torch.randn(batch, m, ldc, device=DEV, generator=g)
    c = c0.clone()
    diag_offset = 3 if lower else 0
    st = _gemm(c.data_ptr(), p.data_ptr(), q.data_ptr(), m, ncols, K, ldc, ld, ld, alpha, beta,
               lower, diag_offset, batch, m * ldc, m * ld, ncols * ld, engine)
    assert st == 0
    ref = alpha * (p[:, :, :K].double() @ q[:, :, :K].double().transpose(1, 2)) + \
        beta * c0[:, :, :ncols].double()
    got = c[:, :, :ncols].double()
    r = torch.arange(m, device=DEV).view(m, 1)
    cc = torch.arange(ncols, device=DEV).view(1, ncols)
    keep = (cc <= r + diag_offset) if lower else torch.ones(m, ncols, dtype=torch.bool, device=DEV)
    want = torch.where(keep, ref, c0[:, :, :ncols].double())
    tol = 8 * K * 2.0 ** -22 * p.abs().max().item() * q.abs().max().item() + \
        4 * 2.0 ** -24 * want.abs().max().item()
    err = (got - want).abs().max().item()
    assert err <= tol, (err, tol)
    # columns past ncols untouched
    assert torch.equal(c[:, :, ncols:], c0[:, :, ncols:])


def test_gemm_in_place_panel_solve():
    """C aliases P with beta == 0 and ncols == K == 64 (the panel solve X <- X T^T)."""
    m, k = 700, 64
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(2, m, 96, device=DEV, generator=g)
    t = torch.tril(torch.randn(2, 64, 64, device=DEV, generator=g))
    want = x[:, :, :k].double() @ t.double().transpose(1, 2)
    st = _gemm(x.data_ptr(), x.data_ptr(), t.data_ptr(), m, k, k, 96, 96, 64, 1.0, 0.0, 0, 0, 2,
               m * 96, m * 96, 64 * 64, _lib.ENGINE_TENSOR)
    assert st == 0
    err = (x[:, :, :k].double() - want).abs().max().item()
    assert err <= 8 * 64 * 2.0 ** -22 * 16.0, err


def test_tensor_engine_accuracy_vs_plain_tf32():
    """3xTF32 is two orders of magnitude more accurate than one TF32 pass. (The tensor
    core's FP32 accumulator truncates at every MMA step, so the error grows with K/8:
    measured ~8e-6 relative at K = 512 on random data; a single TF32 pass gives ~5e-4.)"""
    m = n = 256
    k = 512
    g = torch.Generator(device=DEV).manual_seed(9)
    p = torch.randn(1, m, k, device=DEV, generator=g)
    c = torch.zeros(1, m, n, device=DEV)
    assert _gemm(c.data_ptr(), p.data_ptr(), p.data_ptr(), m, n, k, n, k, k, 1.0, 0.0, 0, 0, 1,
                 m * n, m * k, m * k, _lib.ENGINE_TENSOR) == 0
    ref = p[0].double() @ p[0].double().t()
    rel = ((c[0].double() - ref).norm() / ref.norm()).item()
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        tf32 = (p[0] @ p[0].t()).double()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    rel_tf32 = ((tf32 - ref).norm() / ref.norm()).item()
    assert rel < 2e-5, rel
    assert rel < rel_tf32 / 20, (rel, rel_tf32)


def test_status_word_clear_after_normal_runs():
    lib = _lib.load()
    assert lib.chol_status_check(ctypes.c_void_p(_lib.current_queue(torch.device(DEV)))) == 0
