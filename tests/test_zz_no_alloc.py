"""GPU: the no-allocation entry point chol_potrf_batched_noalloc_f32.

It exists for callers that cannot call cudaMalloc (a host that owns all device memory
through its own pool, or a path where cudaMalloc's implicit device synchronisation is not
allowed); its only scratch is a fixed 4 MiB device array inside the library. The test
calls it through the C ABI and checks it against the allocating entry point
chol_potrf_batched_f32, twice in a row (the shared array keeps the previous call's
contents), within the parity tolerance the other GPU tests use. It is kept in a file of its
own, collected last, and runs the same alone or after the rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

from linalg_kernels_b200 import _lib, inputs
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _queue():
    return ctypes.c_void_p(_lib.current_queue(torch.device(DEV)))


def _factor(entry, a, info):
    lib = _lib.load()
    out = torch.empty_like(a)
    st = getattr(lib, entry)(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                             a.shape[0], a.shape[-1], ctypes.c_void_p(info.data_ptr()), _queue())
    torch.cuda.synchronize()
    return st, out


@pytest.mark.parametrize("batch,n", [(96, 32), (7, 200), (16, 512), (256, 130), (1, 2048)])
def test_no_alloc_matches_allocating_entry_point(batch, n):
    for call in range(2):
        a, cond = inputs.spectral(batch, n, 100.0, 500 + 17 * n + call)
        a = a.to(DEV)
        info_ref = torch.full((batch,), -1, dtype=torch.int32, device=DEV)
        info_new = torch.full((batch,), -1, dtype=torch.int32, device=DEV)
        st_ref, l_ref = _factor("chol_potrf_batched_f32", a, info_ref)
        st_new, l_new = _factor("chol_potrf_batched_noalloc_f32", a, info_new)
        assert st_ref == _lib.CHOL_OK and st_new == _lib.CHOL_OK, (st_ref, st_new)
        assert (info_new == 0).all() and (info_ref == 0).all()
        res = oracle.check_factor(a.cpu().numpy(), l_new.cpu().numpy(),
                                  l_ref=l_ref.cpu().numpy(), cond=cond.cpu().numpy())
        assert res["ok"], (batch, n, call, res)


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    batch, n = 257, 192  # blocked path: 257 inverse blocks of 16 KiB > the fixed 4 MiB scratch
    a = torch.eye(n, device=DEV).expand(batch, n, n).contiguous()
    out = torch.empty_like(a)
    st = lib.chol_potrf_batched_noalloc_f32(ctypes.c_void_p(a.data_ptr()),
                                            ctypes.c_void_p(out.data_ptr()), batch, n, None,
                                            _queue())
    assert st == _lib.CHOL_ERR_SCRATCH_LIMIT
    assert "scratch" in lib.chol_strerror(st).decode()
    # the same batch of small matrices needs no scratch
    a = torch.eye(32, device=DEV).expand(batch, 32, 32).contiguous()
    out = torch.empty_like(a)
    st = lib.chol_potrf_batched_noalloc_f32(ctypes.c_void_p(a.data_ptr()),
                                            ctypes.c_void_p(out.data_ptr()), batch, 32, None,
                                            _queue())
    torch.cuda.synchronize()
    assert st == _lib.CHOL_OK
    assert torch.equal(out, a)


def test_no_alloc_reports_not_spd():
    a, _ = inputs.spectral(3, 96, 10.0, 77)
    a = a.clone()
    a[1, 70, 70] = -4.0
    a = a.to(DEV)
    info = torch.full((3,), -1, dtype=torch.int32, device=DEV)
    st, _ = _factor("chol_potrf_batched_noalloc_f32", a, info)
    assert st == _lib.CHOL_OK
    got = info.cpu().numpy()
    assert got[0] == 0 and got[2] == 0 and 0 < got[1] <= 71
    np.testing.assert_array_equal(got, torch.linalg.cholesky_ex(a.cpu()).info.numpy())
