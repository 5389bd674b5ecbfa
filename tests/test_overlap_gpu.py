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


# ---- work that is not the library's, enqueued on the same queue between two calls ----
def _stats():
    lib = _lib.load()
    early, withdrawn = ctypes.c_int64(), ctypes.c_int64()
    assert lib.chol_overlap_stats(ctypes.byref(early), ctypes.byref(withdrawn)) == _lib.CHOL_OK
    return early.value, withdrawn.value


@pytest.mark.parametrize("n,batch", [(64, 1024), (32, 4096)])
def test_evaluator_clone_between_calls(n, batch):
    # the reference's evaluator calls custom_kernel(clone(data)): a torch kernel writes the
    # next call's input immediately before the call
    pool = _pool(n, batch, 5, 700 + n)

    def run(sync=False):
        outs = []
        for i in range(25):
            outs.append(custom_kernel(pool[i % len(pool)].clone()))
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return outs

    got = run()
    want = _one_at_a_time(run)
    for g_, w in zip(got, want):
        assert torch.equal(g_, w)


def test_foreign_writes_of_next_input_and_output():
    # torch kernels write the next call's input (copy_, mul_) and fill the next call's
    # output buffer, each right before the call
    n, batch = 64, 1024
    src = _pool(n, batch, 4, 800)
    lib = _lib.load()
    q = ctypes.c_void_p(_lib.current_queue(torch.device(DEV)))

    def run(sync=False):
        ins = [torch.empty_like(src[0]) for _ in range(4)]
        outs = [torch.empty_like(src[0]) for _ in range(4)]
        res = []
        for i in range(16):
            k = i % 4
            ins[k].copy_(src[(i + 1) % 4])
            if i % 3 == 0:
                ins[k].mul_(1.5)
            outs[k].fill_(float("nan"))
            assert lib.chol_potrf_batched_f32(ctypes.c_void_p(ins[k].data_ptr()),
                                              ctypes.c_void_p(outs[k].data_ptr()), batch, n,
                                              None, q) == 0
            res.append(outs[k].double().sum(dim=(1, 2)))
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return res + outs

    got = run()
    want = _one_at_a_time(run)
    for g_, w in zip(got, want):
        assert torch.equal(g_, w)


def test_device_check_withdraws_early_start_after_foreign_kernel():
    # two calls on disjoint buffers (the host lets the second start early); a torch kernel
    # between them writes the second call's input. The second call's grid cannot start before
    # that kernel has completed, and so before the first call has; every one of its CTAs must
    # see that on the device and take the full wait
    n, batch = 64, 1024
    a1, a2, s2 = _pool(n, batch, 3, 900)
    o1, o2 = torch.empty_like(a1), torch.empty_like(a1)
    lib = _lib.load()
    q = ctypes.c_void_p(_lib.current_queue(torch.device(DEV)))
    ctas = (batch + 3) // 4  # 4 matrices per CTA at n = 64
    # start a fresh run on the queue: the first call below then waits as usual
    lib.chol_set_option(_lib.CHOL_OPT_OVERLAP_CALLS, 0)
    lib.chol_set_option(_lib.CHOL_OPT_OVERLAP_CALLS, 1)
    torch.cuda.synchronize()
    e0, w0 = _stats()
    assert lib.chol_potrf_batched_f32(ctypes.c_void_p(a1.data_ptr()),
                                      ctypes.c_void_p(o1.data_ptr()), batch, n, None, q) == 0
    a2.copy_(s2)
    assert lib.chol_potrf_batched_f32(ctypes.c_void_p(a2.data_ptr()),
                                      ctypes.c_void_p(o2.data_ptr()), batch, n, None, q) == 0
    torch.cuda.synchronize()
    e1, w1 = _stats()
    assert e1 - e0 == 0
    assert w1 - w0 == ctas
    assert torch.equal(o2, custom_kernel(s2))


def test_back_to_back_calls_still_start_early():
    # without foreign work between them, consecutive calls keep overlapping
    n, batch = 64, 1024
    pool = _pool(n, batch, 4, 950)
    torch.cuda.synchronize()
    e0, _ = _stats()
    for i in range(40):
        custom_kernel(pool[i % 4])
    torch.cuda.synchronize()
    e1, _ = _stats()
    assert e1 > e0
