"""GPU: the bounded device-side waits run out, are reported, and do not spoil later calls.

The diagonal-block kernel's CTAs wait for tiles that other CTAs publish; every such wait is
bounded (CHOL_OPT_WAIT_LIMIT_US, 2 s by default). chol_test_flag_wait runs the same bounded
wait on a flag that nothing sets, with the limit lowered to 1 ms: the wait gives up, records
CHOL_ERR_WAIT_TIMEOUT in the device status word and returns, and the GPU stays usable. Nothing
faults or hangs: the flag is a plain zeroed int and the wait ends by its time bound.
"""

import ctypes

import pytest
import torch

from linalg_kernels_b200 import _lib, inputs
from linalg_kernels_b200.cholesky import custom_kernel
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _q():
    return ctypes.c_void_p(_lib.current_queue(torch.device(DEV)))


@pytest.fixture
def short_waits():
    lib = _lib.load()
    assert lib.chol_status_check(_q()) in (_lib.CHOL_OK, _lib.CHOL_ERR_WAIT_TIMEOUT)
    assert lib.chol_set_option(_lib.CHOL_OPT_WAIT_LIMIT_US, 1000) == _lib.CHOL_OK
    yield lib
    assert lib.chol_set_option(_lib.CHOL_OPT_WAIT_LIMIT_US, 0) == _lib.CHOL_OK


def test_wait_limit_option_range():
    lib = _lib.load()
    assert lib.chol_set_option(_lib.CHOL_OPT_WAIT_LIMIT_US, -1) == _lib.CHOL_ERR_INVALID_ARG
    assert lib.chol_set_option(_lib.CHOL_OPT_WAIT_LIMIT_US, 0) == _lib.CHOL_OK


def test_published_flag_does_not_time_out(short_waits):
    lib = short_waits
    words = torch.tensor([7, 0], dtype=torch.int32, device=DEV)
    assert lib.chol_test_flag_wait(ctypes.c_void_p(words.data_ptr()), 7, _q()) == _lib.CHOL_OK
    assert lib.chol_status_check(_q()) == _lib.CHOL_OK
    assert words.tolist() == [7, 0]


def test_wait_runs_out_then_later_calls_are_correct(short_waits):
    lib = short_waits
    words = torch.zeros(2, dtype=torch.int32, device=DEV)
    assert lib.chol_test_flag_wait(ctypes.c_void_p(words.data_ptr()), 1, _q()) == _lib.CHOL_OK
    torch.cuda.synchronize()  # the wait ends by its 1 ms bound
    assert words.tolist() == [0, 1]  # the abort word holds the wait's value
    # the status word is still set: calls made now (one-launch diagonal-block path at
    # b64n256, several panels at n = 1536) must not drop their work because of it
    for batch, n in ((64, 256), (1, 1536)):
        a, cond = inputs.spectral(batch, n, 100.0, 4242 + n)
        l = custom_kernel(a.to(DEV)).cpu()
        l_or, info = oracle.potrf(a.numpy())
        res = oracle.check_factor(a.numpy(), l.numpy(), l_ref=l_or, cond=cond.numpy())
        assert res["ok"], (batch, n, res)
    # reported once, then clear
    assert lib.chol_status_check(_q()) == _lib.CHOL_ERR_WAIT_TIMEOUT
    assert lib.chol_status_check(_q()) == _lib.CHOL_OK
    # and the wait still works afterwards
    words.zero_()
    assert lib.chol_test_flag_wait(ctypes.c_void_p(words.data_ptr()), 1, _q()) == _lib.CHOL_OK
    assert lib.chol_status_check(_q()) == _lib.CHOL_ERR_WAIT_TIMEOUT
