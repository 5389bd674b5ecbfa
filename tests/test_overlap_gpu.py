"""GPU: back-to-back calls with n <= 64 on one queue (CHOL_OPT_OVERLAP_CALLS).

A call whose buffers are disjoint from those of the calls still possibly running starts
loading before they finish. These tests issue calls back to back without synchronising and
compare every result, bitwise, with the same calls made one at a time with the overlap off
(each followed by a device synchronise): independent buffers, a chain where each output is
the next input (read after write), a call that writes the previous call's input (write
after read) and output tensors whose memory the allocator hands from call to call (write
after write)."""

import ctypes

import pytest
import torch

from linalg_kernels_b200 import _lib, inputs
from linalg_kernels_b200.cholesky import cholesky_ex, custom_kernel

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _one_at_a_time(fn):
    lib = _lib.load()
    lib.chol_set_option(_lib.CHOL_OPT_OVERLAP_CALLS, 0)
    try:
        return fn(sync=True)
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_OVERLAP_CALLS, 1)


def _pool(n, batch, count, seed):
    return [inputs.spectral(batch, n, 100.0, seed + i, device=DEV)[0] for i in range(count)]


@pytest.mark.parametrize("n,batch", [(32, 4096), (64, 1024), (16, 333), (48, 257)])
def test_independent_calls(n, batch):
    pool = _pool(n, batch, 6, 100 + n)

    def run(sync=False):
        outs = []
        for i in range(30):
            outs.append(custom_kernel(pool[i % len(pool)]))
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return outs

    got = run()
    want = _one_at_a_time(run)
    for g, w in zip(got, want):
        assert torch.equal(g, w)


@pytest.mark.parametrize("n,batch", [(32, 2048), (64, 512)])
def test_chain_output_is_next_input(n, batch):
    # 4 I + small symmetric noise: the factor's lower triangle, read as a symmetric matrix,
    # is again SPD, so the chain stays finite
    g = torch.Generator(device=DEV).manual_seed(7)
    x = torch.randn(batch, n, n, device=DEV, generator=g) * 0.01
    a0 = x + x.transpose(1, 2) + 4.0 * torch.eye(n, device=DEV)

    def run(sync=False):
        seq = [a0]
        for _ in range(12):
            seq.append(custom_kernel(seq[-1]))
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return seq[1:]

    got = run()
    want = _one_at_a_time(run)
    for g_, w in zip(got, want):
        assert torch.isfinite(w).all()
        assert torch.equal(g_, w)


def test_call_writes_previous_input():
    n, batch = 64, 1024
    a1, a2, a3 = _pool(n, batch, 3, 300)
    lib = _lib.load()
    q = ctypes.c_void_p(_lib.current_queue(torch.device(DEV)))

    def run(sync=False):
        b1, b2, b3 = a1.clone(), a2.clone(), a3.clone()
        out1 = torch.empty_like(b1)
        torch.cuda.synchronize()
        st = [lib.chol_potrf_batched_f32(ctypes.c_void_p(b1.data_ptr()),
                                         ctypes.c_void_p(out1.data_ptr()), batch, n, None, q)]
        if sync:
            torch.cuda.synchronize()
        # the second call writes its factor over the first call's input
        st.append(lib.chol_potrf_batched_f32(ctypes.c_void_p(b2.data_ptr()),
                                             ctypes.c_void_p(b1.data_ptr()), batch, n, None, q))
        if sync:
            torch.cuda.synchronize()
        # the third reads the first call's output and writes over the second call's input
        st.append(lib.chol_potrf_batched_f32(ctypes.c_void_p(b3.data_ptr()),
                                             ctypes.c_void_p(b2.data_ptr()), batch, n, None, q))
        torch.cuda.synchronize()
        assert st == [0, 0, 0]
        return out1, b1, b2

    got = run()
    want = _one_at_a_time(run)
    for g_, w in zip(got, want):
        assert torch.equal(g_, w)


def test_reused_output_memory_and_shared_info():
    n, batch = 32, 4096
    pool = _pool(n, batch, 4, 500)
    info = torch.zeros(batch, dtype=torch.int32, device=DEV)
    lib = _lib.load()
    q = ctypes.c_void_p(_lib.current_queue(torch.device(DEV)))

    def run(sync=False):
        sums = []
        for i in range(40):
            if i % 2:
                # output tensor dropped at once: the next call gets the same block
                l = custom_kernel(pool[i % 4])
            else:
                l = torch.empty_like(pool[0])
                assert lib.chol_potrf_batched_f32(ctypes.c_void_p(pool[i % 4].data_ptr()),
                                                  ctypes.c_void_p(l.data_ptr()), batch, n,
                                                  ctypes.c_void_p(info.data_ptr()), q) == 0
            sums.append(l.double().sum(dim=(1, 2)))
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return sums + [info.clone()]

    got = run()
    want = _one_at_a_time(run)
    for g_, w in zip(got, want):
        assert torch.equal(g_, w)


def test_not_spd_info_with_overlap():
    a, _ = inputs.spectral(512, 32, 10.0, 901, device=DEV)
    bad = a.clone()
    bad[5, 20, 20] = -3.0
    outs = []
    for i in range(10):
        outs.append(cholesky_ex(bad if i % 2 else a))
    torch.cuda.synchronize()
    for i, (_, info) in enumerate(outs):
        if i % 2:
            assert int(info[5]) > 0 and int(info.count_nonzero()) == 1
        else:
            assert int(info.count_nonzero()) == 0
