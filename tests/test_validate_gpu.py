"""GPU: the device-side checker (chol_validate_f32, linalg_kernels_b200.validate) against
the oracle's FP64 gate functions on the host, on factors from custom_kernel and on factors
with planted faults (a NaN, garbage above the diagonal, a negative pivot, a perturbation)."""

import numpy as np
import pytest
import torch

from linalg_kernels_b200 import inputs
from linalg_kernels_b200.cholesky import custom_kernel
from linalg_kernels_b200.validate import check_implementation, validate
from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _host_gates(a, l):
    """The oracle's gates on tril(L) (the device check reads only the lower triangle)."""
    a = a.cpu().numpy()
    lt = np.tril(l.cpu().numpy())
    lt = np.where(np.isfinite(lt), lt, np.nan)
    return oracle.rel_residual_fro(a, lt), oracle.scaled_inf_residual(a, lt)


@pytest.mark.parametrize("batch,n", [(3, 1), (5, 7), (64, 32), (16, 64), (4, 65), (3, 100),
                                     (2, 200), (1, 384)])
def test_matches_host_gates(batch, n):
    a, _ = inputs.spectral(batch, n, 100.0, 500 + n, device=DEV)
    l = custom_kernel(a)
    v = validate(a, l)
    rel, scaled = _host_gates(a, l)
    np.testing.assert_allclose(v["rel_residual"].numpy(), rel, rtol=1e-6, atol=1e-15)
    np.testing.assert_allclose(v["scaled_residual"].numpy(), scaled, rtol=1e-6, atol=1e-6)
    assert (v["nonfinite"] == 0).all() and (v["upper_nonzero"] == 0).all()
    assert (v["diag_not_positive"] == 0).all()
    assert check_implementation(a, l) == (True, "")


def test_reads_the_lower_triangle_of_a():
    a, _ = inputs.spectral(3, 96, 10.0, 61, device=DEV)
    l = custom_kernel(a)
    garbage = a + torch.triu(torch.full_like(a, 1e3), 1)
    v0, v1 = validate(a, l), validate(garbage, l)
    assert torch.equal(v0["rel_residual"], v1["rel_residual"])
    assert torch.equal(v0["scaled_residual"], v1["scaled_residual"])


def test_planted_faults_are_counted():
    n = 80
    a, _ = inputs.spectral(5, n, 10.0, 62, device=DEV)
    l = custom_kernel(a).clone()
    l[0, 40, 10] = float("nan")          # non-finite
    l[1, 3, 50] = 1.0                    # above the diagonal
    l[1, 4, 79] = -2.0
    l[2, 20, 20] = -l[2, 20, 20]         # negative diagonal entry
    l[3, 70, 30] += 1e-3                 # small perturbation below the diagonal
    v = validate(a, l)
    assert v["nonfinite"].tolist() == [1, 0, 0, 0, 0]
    assert v["upper_nonzero"].tolist() == [0, 2, 0, 0, 0]
    assert v["diag_not_positive"].tolist() == [0, 0, 1, 0, 0]
    assert np.isnan(v["rel_residual"][0].item())
    rel, scaled = _host_gates(a, l)
    np.testing.assert_allclose(v["rel_residual"][1:].numpy(), rel[1:], rtol=1e-6)
    np.testing.assert_allclose(v["scaled_residual"][1:].numpy(), scaled[1:], rtol=1e-6)
    assert v["rel_residual"][3].item() > 1e-5  # the perturbation fails the residual gate
    good, msg = check_implementation(a, l)
    assert not good and msg.startswith("matrix 0: non-finite")
    for m, start in ((1, "matrix 0: non-zero entries above"), (2, "matrix 0: diagonal"),
                     (3, "matrix 0: relative residual")):
        good, msg = check_implementation(a[m:m + 1], l[m:m + 1])
        assert not good and msg.startswith(start), msg
    assert check_implementation(a[4:], l[4:]) == (True, "")


def test_contract_checks():
    a, _ = inputs.spectral(2, 16, 10.0, 63, device=DEV)
    l = custom_kernel(a)
    assert check_implementation(a, l[:1])[0] is False
    assert check_implementation(a, l.double())[0] is False
    assert check_implementation(a, l.cpu())[0] is False
    assert check_implementation(a, [l])[0] is False


def test_full_size_against_torch_fp64():
    """b1n8192 from the benchmark grid: the device check against torch's FP64 product."""
    a, _ = inputs.config_input("b1n8192", device=DEV)
    l = custom_kernel(a)
    v = validate(a, l)
    a64 = torch.tril(a.double())
    a64 = a64 + torch.tril(a64, -1).transpose(-1, -2)
    l64 = l.double()
    r = l64 @ l64.transpose(-1, -2) - a64
    rel = (torch.linalg.matrix_norm(r) / torch.linalg.matrix_norm(a64)).cpu()
    scaled = (r.abs().sum(-1).amax(-1) / (oracle.EPS32 * a.shape[-1] *
                                          a64.abs().sum(-1).amax(-1))).cpu()
    np.testing.assert_allclose(v["rel_residual"].numpy(), rel.numpy(), rtol=1e-6)
    np.testing.assert_allclose(v["scaled_residual"].numpy(), scaled.numpy(), rtol=1e-6)
    assert check_implementation(a, l) == (True, "")
