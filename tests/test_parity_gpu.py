"""GPU parity: the sm_100a kernels (through the C ABI) against the reference's outputs.

Small cases: elementwise against tests/golden (the reference's own custom_kernel output,
LAPACK SPOTRF) and against the CPU oracle, with the north-star tolerances
(||L L^T - A||_F / ||A||_F <= 1e-5, max|L - L_ref| <= cond(A) n eps32 max|L_ref|) plus the
reference harness's property gate. Benchmark sizes: the same bounds against the
reference path run on the GPU (torch.linalg.cholesky_ex, i.e. submission.py:7 on CUDA)
and size-independent properties (exact-zero upper, positive diagonal, residual,
determinism, input untouched).
"""

import ctypes

import numpy as np
import pytest
import torch

from linalg_kernels_b200 import _lib, inputs
from linalg_kernels_b200.cholesky import cholesky, cholesky_ex, custom_kernel
from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _names(golden):
    return [str(n) for n in golden["_names"]]


def _gpu_factor(a_np):
    a = torch.from_numpy(np.ascontiguousarray(a_np)).to(DEV)
    l = custom_kernel(a)
    torch.cuda.synchronize()
    return l.cpu().numpy()


def test_golden_cases_match_reference(golden):
    for name in _names(golden):
        a, l_ref, cond = golden[f"{name}/A"], golden[f"{name}/L"], golden[f"{name}/cond"]
        l = _gpu_factor(a)
        res = oracle.check_factor(a, l, l_ref=l_ref, cond=cond)
        assert res["ok"], (name, res)
        l_or, _ = oracle.potrf(a)
        res2 = oracle.check_factor(a, l, l_ref=l_or, cond=cond)
        assert res2["ok"], (name, "vs oracle", res2)


def test_not_spd_info_matches_reference(golden):
    for name in [str(n) for n in golden["_notspd"]]:
        a = torch.from_numpy(golden[f"{name}/A"]).to(DEV)
        _, info = cholesky_ex(a)
        np.testing.assert_array_equal(info.cpu().numpy(), golden[f"{name}/info"], err_msg=name)
        with pytest.raises(torch.linalg.LinAlgError):
            cholesky(a)


def test_lower_triangle_only(golden):
    a = golden["upper_garbage_b2n40/A"]
    np.testing.assert_array_equal(_gpu_factor(a), _gpu_factor(np.tril(a)))


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 8, 9, 15, 16, 17, 24, 31, 32, 33, 48, 63, 64, 65,
                               96, 100, 127, 128, 129, 191, 200, 255, 256, 257, 300])
@pytest.mark.parametrize("batch", [1, 7])
def test_sizes_against_oracle(n, batch):
    a, cond = inputs.spectral(batch, n, 100.0, 1000 * n + batch)
    a = a.numpy()
    l = _gpu_factor(a)
    l_or, info = oracle.potrf(a)
    assert (info == 0).all()
    res = oracle.check_factor(a, l, l_ref=l_or, cond=cond.numpy())
    assert res["ok"], (n, batch, res)


@pytest.mark.parametrize("name", ["dense", "diagonal", "tridiagonal", "lowrank", "spectrum",
                                  "rowscale"])
@pytest.mark.parametrize("n", [32, 64, 128, 256, 512])
def test_case_families(name, n):
    a = inputs.case(name, 2, n, 77 + n)
    ev = torch.linalg.eigvalsh(a.double())
    cond = (ev[:, -1] / ev[:, 0]).numpy()
    a = a.numpy()
    l = _gpu_factor(a)
    l_or, _ = oracle.potrf(a)
    res = oracle.check_factor(a, l, l_ref=l_or, cond=cond)
    assert res["ok"], (name, n, res)


def test_diagonal_known_answer():
    d = torch.logspace(-2, 2, 96)
    a = torch.diag_embed(d.expand(3, 96)).contiguous()
    l = custom_kernel(a.to(DEV)).cpu()
    want = torch.diag_embed(torch.sqrt(d).expand(3, 96))
    assert (l - want).abs().max().item() <= 2e-7 * 10.0


def _check_full_config(name, batch=None):
    cfg = inputs.GRID[name]
    a, cond = inputs.config_input(cfg, device=DEV, batch=batch)
    return _check_input(a, cond)


def _check_input(a, cond):
    a_before = a.clone()
    l = custom_kernel(a)
    l_ref = torch.linalg.cholesky_ex(a, check_errors=False).L  # the reference path on GPU
    torch.cuda.synchronize()
    assert torch.equal(a, a_before), "input was modified"
    n = a.shape[-1]
    assert torch.isfinite(l).all()
    assert (torch.triu(l, 1) == 0).all()
    assert (l.diagonal(dim1=-2, dim2=-1) > 0).all()
    # residual in float64 on the device, lower triangle of A
    a64 = torch.tril(a.double())
    a64 = a64 + torch.tril(a64, -1).transpose(-1, -2)
    l64 = l.double()
    rel = torch.linalg.matrix_norm(l64 @ l64.transpose(-1, -2) - a64) / torch.linalg.matrix_norm(a64)
    assert rel.max().item() <= oracle.REL_RESIDUAL_TOL, rel.max().item()
    diff = (l - l_ref).abs().reshape(l.shape[0], -1).amax(dim=1).double().cpu()
    bound = cond.reshape(-1).cpu() * n * oracle.EPS32 * l_ref.abs().reshape(l.shape[0], -1).amax(dim=1).double().cpu()
    assert (diff <= bound).all(), (diff.max().item(), bound.min().item())
    l2 = custom_kernel(a)
    assert torch.equal(l, l2), "not deterministic"
    return rel.max().item()


@pytest.mark.parametrize("name", ["b4096n32", "b1024n64", "b64n256", "b640n512", "b60n1024"])
def test_baseline_configs_full_size(name):
    _check_full_config(name)


def test_baseline_config_n16384():
    _check_full_config("b1n16384")


def test_baseline_config_n32768():
    """b1n32768 (4 GiB): the residual gates from the device checker (an FP64 product would
    need several 8 GiB buffers), and the elementwise bound against the reference path on
    the GPU (torch.linalg.cholesky_ex)."""
    from linalg_kernels_b200.validate import check_implementation, validate

    a, cond = inputs.config_input("b1n32768", device=DEV)
    a_before = a.clone()
    l = custom_kernel(a)
    torch.cuda.synchronize()
    assert torch.equal(a, a_before), "input was modified"
    del a_before
    good, msg = check_implementation(a, l)
    assert good, msg
    assert validate(a, l)["rel_residual"].item() <= oracle.REL_RESIDUAL_TOL
    l_ref = torch.linalg.cholesky_ex(a, check_errors=False).L
    diff = (l - l_ref).abs().max().item()
    bound = float(cond[0]) * a.shape[-1] * oracle.EPS32 * l_ref.abs().max().item()
    assert diff <= bound, (diff, bound)


# the rest of the reference's benchmark grid (AGENTS.md:66-81), full size
@pytest.mark.parametrize("name", [k for k in inputs.GRID if k not in inputs.CONFIGS])
def test_benchmark_grid_full_size(name):
    _check_full_config(name)


# the reference's 17 test shapes (AGENTS.md:83-100) with their seeds and structural cases;
# cond(A) from the FP64 eigenvalues
@pytest.mark.parametrize("spec", inputs.TEST_SHAPES,
                         ids=lambda s: f"b{s.batch}n{s.n}-{s.case or 'family'}-{s.seed}")
def test_reference_test_shapes(spec):
    a = inputs.spec_input(spec, device=DEV)
    ev = torch.linalg.eigvalsh(a.double())
    _check_input(a, ev[:, -1] / ev[:, 0])


def test_non_contiguous_input():
    a, _ = inputs.spectral(4, 48, 10.0, 3)
    big = torch.zeros(4, 48, 96, device=DEV)
    big[:, :, ::2] = a.to(DEV)
    x = big[:, :, ::2]
    assert not x.is_contiguous()
    l = custom_kernel(x).cpu().numpy()
    l_or, _ = oracle.potrf(a.numpy())
    assert oracle.check_factor(a.numpy(), l, l_ref=l_or, cond=np.full(4, 10.0))["ok"]


def test_leading_batch_dims_and_2d():
    a, _ = inputs.spectral(6, 40, 10.0, 4)
    l = custom_kernel(a.reshape(2, 3, 40, 40).to(DEV))
    assert l.shape == (2, 3, 40, 40)
    l2 = custom_kernel(a[0].to(DEV))
    assert l2.shape == (40, 40)
    assert torch.equal(l.reshape(6, 40, 40)[0], l2)


def _abi_call(a, l, batch, n):
    lib = _lib.load()
    return lib.chol_potrf_batched_f32(ctypes.c_void_p(a), ctypes.c_void_p(l), batch, n, None,
                                      ctypes.c_void_p(_lib.current_queue(torch.device(DEV))))


@pytest.mark.parametrize("n", [32, 64, 100, 200])
def test_abi_in_place_and_canaries(n):
    """Library-managed workspace entry point; A == L in place; canaries around L."""
    a, cond = inputs.spectral(3, n, 50.0, 11 + n)
    want = custom_kernel(a.to(DEV))
    pad = 64
    buf = torch.full((3 * n * n + 2 * pad,), 12345.0, device=DEV)
    buf[pad:pad + 3 * n * n] = a.reshape(-1).to(DEV)
    base = buf.data_ptr() + pad * 4
    assert _abi_call(base, base, 3, n) == _lib.CHOL_OK
    torch.cuda.synchronize()
    assert (buf[:pad] == 12345.0).all() and (buf[-pad:] == 12345.0).all()
    got = buf[pad:pad + 3 * n * n].reshape(3, n, n)
    assert torch.equal(got, want)


def test_building_blocks_against_torch():
    """chol_block_potrf_f32 + chol_gemm_nt_f32 reproduce one blocked step."""
    lib = _lib.load()
    n, kb = 160, 64
    a, _ = inputs.spectral(2, n, 20.0, 5)
    l = torch.tril(a).to(DEV).contiguous()
    tinv = torch.zeros(2, 64, 64, device=DEV)
    q = ctypes.c_void_p(_lib.current_queue(torch.device(DEV)))
    assert lib.chol_block_potrf_f32(ctypes.c_void_p(l.data_ptr()), 2, n * n, n, 0, kb,
                                    ctypes.c_void_p(tinv.data_ptr()), None, q) == 0
    l11 = l[:, :kb, :kb]
    ref11 = torch.linalg.cholesky(a[:, :kb, :kb].to(DEV).double()).float()
    assert (l11 - ref11).abs().max().item() < 1e-5
    eye = torch.eye(kb, device=DEV)
    assert (tinv @ l11 - eye).abs().max().item() < 1e-4
    # panel solve in place: X = A21 * T^T
    x = l[:, kb:, :kb]
    want_x = a[:, kb:, :kb].to(DEV) @ tinv.transpose(1, 2)
    st = lib.chol_gemm_nt_f32(ctypes.c_void_p(x.data_ptr()), 2, n * n, n, n - kb, kb, kb,
                              ctypes.c_void_p(x.data_ptr()), n * n, n,
                              ctypes.c_void_p(tinv.data_ptr()), 64 * 64, 64,
                              1.0, 0.0, 0, 0, q)
    assert st == 0
    torch.cuda.synchronize()
    assert (l[:, kb:, :kb] - want_x).abs().max().item() < 1e-4


def test_removed_fused_panel_option_is_rejected():
    assert _lib.load().chol_set_option(2, 1) == _lib.CHOL_ERR_INVALID_ARG


def test_row_chain_panel_solve_at_large_n():
    """n = 16384 with the panel solved by 64-wide steps over every row of the panel
    (CHOL_OPT_PANEL_INVERSE = 0) instead of one GEMM with the diagonal block's inverse."""
    lib = _lib.load()
    lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, 0)
    try:
        _check_full_config("b1n16384")
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, 1)


# n > 1024: several 512-wide outer panels. 1536/2048: whole panels; 2100: a 52-wide last
# panel; 1030, 2050: rows that are not 16-byte multiples (the schedule without the optional
# panel buffer). Spectral inputs up to cond 1e5 exercise the inverse-based panel solve.
@pytest.mark.parametrize("batch,n,lam", [(1, 1536, 1e3), (3, 2048, 1e4), (1, 2100, 1e5),
                                         (2, 1030, 1e3), (1, 2050, 1e4), (1, 4096, 1e5)])
@pytest.mark.parametrize("panel_inverse", [1, 2, 0])
def test_multi_panel_sizes(batch, n, lam, panel_inverse):
    lib = _lib.load()
    lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, panel_inverse)
    try:
        a, cond = inputs.spectral(batch, n, lam, 7000 + n, device=DEV)
        _check_input(a, cond)
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, 1)


# n <= 1024, n % 64 == 0, small batch: the whole matrix in one diagonal-block launch (FP32
# tile tasks); with the option at 0, the tensor-core chain for the same inputs.
@pytest.mark.parametrize("batch,n,lam", [(3, 512, 1e4), (2, 1024, 1e5), (5, 640, 1e3),
                                         (1, 128, 1e2)])
@pytest.mark.parametrize("panel_inverse", [1, 0])
def test_single_panel_sizes(batch, n, lam, panel_inverse):
    lib = _lib.load()
    lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, panel_inverse)
    try:
        a, cond = inputs.spectral(batch, n, lam, 8000 + n, device=DEV)
        _check_input(a, cond)
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, 1)


# 64 < n <= 128: the shared-memory kernel (one CTA per matrix), and ragged 128 < n <= 256:
# the wide kernel (one 512-thread CTA per matrix, the matrix in L), against the oracle, and
# the blocked schedule (CHOL_OPT_MID_KERNEL = 0, through the library-workspace C entry) for
# the same inputs within the same bounds
@pytest.mark.parametrize("batch,n", [(256, 128), (7, 65), (33, 100), (5, 127), (600, 96),
                                     (64, 129), (16, 255), (296, 200), (1024, 130), (3, 161),
                                     (9, 250)])
def test_mid_kernel_sizes(batch, n):
    lib = _lib.load()
    a, cond = inputs.spectral(batch, n, 1e3, 8500 + n)
    l_or, _ = oracle.potrf(a.numpy())
    a_dev = a.to(DEV)
    l_mid = custom_kernel(a_dev)
    lib.chol_set_option(_lib.CHOL_OPT_MID_KERNEL, 0)
    try:
        l_blk = torch.empty_like(a_dev)
        assert _abi_call(a_dev.data_ptr(), l_blk.data_ptr(), batch, n) == _lib.CHOL_OK
        torch.cuda.synchronize()
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_MID_KERNEL, 1)
    for name, l in (("mid", l_mid), ("blocked", l_blk)):
        res = oracle.check_factor(a.numpy(), l.cpu().numpy(), l_ref=l_or, cond=cond.numpy())
        assert res["ok"], (name, batch, n, res)


@pytest.mark.parametrize("n", [100, 200])
def test_mid_kernel_not_spd_info(n):
    """info from the shared-memory kernel (n = 100) and the wide kernel (n = 200): the first
    failing column, as LAPACK reports it (in the first panel, a later panel and the last
    column)."""
    a, _ = inputs.spectral(5, n, 10.0, 98, device=DEV)
    a = a.clone()
    a[1, 10, 10] = -1.0
    a[2, n - 30, n - 30] = -5.0
    a[4, n - 1, n - 1] = -3.0
    l, info = cholesky_ex(a)
    want = torch.linalg.cholesky_ex(a.cpu()).info
    assert torch.equal(info.cpu(), want), (info.cpu(), want)
    assert want.tolist()[0] == 0 and want.tolist()[3] == 0


# One panel, batches beyond the one-launch crossover: the left-looking chain, with 128-wide
# block columns (the default where n % 128 == 0: potrf_block128 factors and inverts each
# diagonal block) and with 64-wide ones (CHOL_OPT_CHAIN_WIDTH = 64), for the same inputs.
@pytest.mark.parametrize("batch,n,lam", [(256, 512, 1e4), (256, 1024, 1e5), (720, 256, 1e3),
                                         (256, 640, 1e3), (300, 768, 1e4), (96, 512, 1e3)])
@pytest.mark.parametrize("width", [128, 64])
def test_chain_widths(batch, n, lam, width):
    lib = _lib.load()
    assert batch * float(n) ** 3 > 1.2e10  # past the one-launch crossover
    assert lib.chol_set_option(_lib.CHOL_OPT_CHAIN_WIDTH, width) == _lib.CHOL_OK
    try:
        w = 128 if width == 128 and n % 128 == 0 and batch >= 256 else 64
        expect = 3 * (n // w) - 2 + (w == 64) if n % w == 0 else None
        if expect is not None:
            assert int(lib.chol_launch_count(batch, n)) == expect
        a, cond = inputs.spectral(batch, n, lam, 8200 + n, device=DEV)
        _check_input(a, cond)
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_CHAIN_WIDTH, 128)


def test_chain128_not_spd_info():
    """info from the 128-wide chain: the first failing column, in either 64-wide half of a
    diagonal block, in a later block and in the last column, as LAPACK reports it."""
    a, _ = inputs.spectral(256, 512, 10.0, 97, device=DEV)
    a = a.clone()
    a[1, 10, 10] = -1.0
    a[2, 100, 100] = -5.0
    a[4, 300, 300] = -2.0
    a[6, 511, 511] = -3.0
    assert int(_lib.load().chol_launch_count(256, 512)) == 10
    l, info = cholesky_ex(a)
    want = torch.linalg.cholesky_ex(a.cpu()).info
    assert torch.equal(info.cpu(), want), (info.cpu()[:8], want[:8])
    assert int(info.count_nonzero()) == 4


def test_single_panel_not_spd_info():
    """info from the one-launch path: the first failing column, as LAPACK reports it."""
    a, _ = inputs.spectral(4, 256, 10.0, 99, device=DEV)
    a = a.clone()
    a[1, 200, 200] = -5.0
    a[3, 10, 10] = -1.0
    l, info = cholesky_ex(a)
    want = torch.linalg.cholesky_ex(a.cpu()).info
    assert torch.equal(info.cpu(), want), (info.cpu(), want)


@pytest.mark.parametrize("n", [2048, 3072])
def test_lookahead_matches_in_order_schedule(n):
    """The side-queue look-ahead (CHOL_OPT_LOOKAHEAD) only reorders independent work:
    bitwise the same factor as the in-order schedule, with and without the panel inverse."""
    lib = _lib.load()
    a, _ = inputs.covariance(2, n, 0.5, 9000 + n, device=DEV)
    try:
        for inv in (1, 0):
            lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, inv)
            lib.chol_set_option(_lib.CHOL_OPT_LOOKAHEAD, 0)
            want = custom_kernel(a)
            lib.chol_set_option(_lib.CHOL_OPT_LOOKAHEAD, 1)
            got = custom_kernel(a)
            torch.cuda.synchronize()
            assert torch.equal(got, want), inv
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_LOOKAHEAD, -1)
        lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, 1)
