"""GPU: the block-column-cyclic driver with the CUDA ops on one rank (no process group):
the same schedule the multi-GPU path runs, checked against the oracle's bounds."""

import ctypes

import numpy as np
import pytest
import torch

from linalg_kernels_b200 import inputs
from linalg_kernels_b200.distributed import (CyclicLayout, factor_block_cyclic,
                                             gather_block_cyclic, scatter_block_cyclic)
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("n,bs", [(1024, 256), (700, 256), (640, 128)])
def test_cyclic_single_rank_matches_oracle(n, bs):
    a, cond = inputs.covariance(1, n, 0.5, 900 + n)
    lay = CyclicLayout(n, 1, 0, bs)
    local = scatter_block_cyclic(a[0].to(DEV), lay)
    factor_block_cyclic(local, lay, pg=None)
    torch.cuda.synchronize()
    l = gather_block_cyclic([local], n, 1, bs).cpu().numpy()[None]
    l_or, _ = oracle.potrf(a.numpy())
    res = oracle.check_factor(a.numpy(), l, l_ref=l_or, cond=cond.numpy())
    assert res["ok"], res


@pytest.mark.parametrize("queues", [(32, 100), (148, 148), (8, 8)])
@pytest.mark.parametrize("paired", [True, False])
def test_cyclic_queue_pair_matches_one_queue(queues, paired):
    """The chain/bulk queue pair (any GEMM CTA caps) computes bitwise what the same schedule
    computes in order on one queue: the events order every block's updates the same way, and a
    cap changes which CTA computes a tile, not its arithmetic."""
    from linalg_kernels_b200 import _lib

    n, bs = 2560, 256
    a, cond = inputs.covariance(1, n, 0.5, 4100)
    lay = CyclicLayout(n, 1, 0, bs)
    base = scatter_block_cyclic(a[0].to(DEV), lay)
    one = factor_block_cyclic(base.clone(), lay, pg=None, paired=paired, queues=None)
    two = factor_block_cyclic(base.clone(), lay, pg=None, paired=paired, queues=queues)
    torch.cuda.synchronize()
    assert torch.equal(one, two)
    lib = _lib.load()
    assert lib.chol_set_option(_lib.CHOL_OPT_GEMM_CTAS, -1) == _lib.CHOL_ERR_INVALID_ARG
    l = gather_block_cyclic([two], n, 1, bs).cpu().numpy()[None]
    l_or, _ = oracle.potrf(a.numpy())
    assert oracle.check_factor(a.numpy(), l, l_ref=l_or, cond=cond.numpy())["ok"]


@pytest.mark.parametrize("n", [2560, 700])
def test_cyclic_split_send_matches_unsplit(n):
    """split_send (each block sent unfactored, then [L11 | inv(L11)], every rank solving the
    rows below itself) computes bitwise what the owner-factors-the-panel schedule computes:
    the same diagonal-block kernel and the same solve GEMM, on contiguous copies. n = 700
    ends with a 188-wide block (factored whole by its owner)."""
    bs = 256
    a, cond = inputs.covariance(1, n, 0.5, 4300 + n)
    lay = CyclicLayout(n, 1, 0, bs)
    base = scatter_block_cyclic(a[0].to(DEV), lay)
    one = factor_block_cyclic(base.clone(), lay, pg=None, split_send=False)
    two = factor_block_cyclic(base.clone(), lay, pg=None, split_send=True)
    three = factor_block_cyclic(base.clone(), lay, pg=None, split_send=True, queues=(56, 76))
    torch.cuda.synchronize()
    assert torch.equal(one, two)
    assert torch.equal(one, three)
    l = gather_block_cyclic([two], n, 1, bs).cpu().numpy()[None]
    l_or, _ = oracle.potrf(a.numpy())
    assert oracle.check_factor(a.numpy(), l, l_ref=l_or, cond=cond.numpy())["ok"]


@pytest.mark.parametrize("w", [256, 512, 64])
def test_diag_potrf_inv(w):
    """chol_diag_potrf_inv_f32: the block factored in place equals the top block of the
    one-launch panel factor (bitwise), and V = inv(L11) to FP32 accuracy."""
    from linalg_kernels_b200 import _lib
    from linalg_kernels_b200.distributed import CudaOps

    ops = CudaOps(torch.device(DEV))
    m = w + 300
    a, _ = inputs.covariance(1, m, 0.5, 900 + w)
    base = torch.tril(a[0]).to(DEV).contiguous()
    ref = base.clone()
    out = torch.empty(m, w, device=DEV)
    assert ops.panel_potrf_out(ref[:, :w], out, None)
    blk = base[:w, :w].clone()
    v = torch.full((w, w), float("nan"), device=DEV)
    info = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    assert ops.diag_potrf_inv(blk, v, info)
    torch.cuda.synchronize()
    assert int(info.item()) == 0
    assert torch.equal(torch.tril(blk), torch.tril(ref[:w, :w]))
    assert torch.equal(torch.triu(v, 1), torch.zeros_like(v))
    eye = torch.tril(blk).double() @ v.double()
    assert (eye - torch.eye(w, device=DEV, dtype=torch.float64)).abs().max().item() < 1e-3
    lib = _lib.load()
    assert lib.chol_diag_potrf_inv_f32(ctypes.c_void_p(blk.data_ptr()), w, w - 32,
                                       ctypes.c_void_p(v.data_ptr()), None, None) \
        == _lib.CHOL_ERR_UNSUPPORTED  # w not a multiple of 64
    assert lib.chol_diag_potrf_inv_f32(ctypes.c_void_p(blk.data_ptr()), w, w,
                                       ctypes.c_void_p(blk.data_ptr()), None, None) \
        == _lib.CHOL_ERR_INVALID_ARG  # V overlaps L


@pytest.mark.parametrize("world", [2, 4])
def test_cyclic_emulated_ranks_on_one_gpu(world):
    """Each emulated rank's columns factored by the same schedule must equal the
    single-layout factor (the broadcast is replaced by reading the owner's panel)."""
    n, bs = 768, 128
    a, cond = inputs.covariance(1, n, 0.5, 77)
    full = torch.tril(a[0]).to(DEV)
    lay1 = CyclicLayout(n, 1, 0, bs)
    one = scatter_block_cyclic(full, lay1)
    factor_block_cyclic(one, lay1, pg=None)
    torch.cuda.synchronize()
    want = gather_block_cyclic([one], n, 1, bs)
    l = want.cpu().numpy()[None]
    l_or, _ = oracle.potrf(a.numpy())
    assert oracle.check_factor(a.numpy(), l, l_ref=l_or, cond=cond.numpy())["ok"]
    # layouts for `world` ranks partition the columns exactly
    parts = [scatter_block_cyclic(want, CyclicLayout(n, world, r, bs)) for r in range(world)]
    assert torch.equal(gather_block_cyclic(parts, n, world, bs), want)


def _nccl_worker(rank, world, port, n, bs, seed, out_dir, split=False):
    import os

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        a, _ = inputs.covariance(1, n, 0.5, seed)
        lay = CyclicLayout(n, world, rank, bs)
        local = scatter_block_cyclic(a[0].to(f"cuda:{rank}"), lay)
        factor_block_cyclic(local, lay, pg=dist, split_send=split)
        torch.cuda.synchronize()
        torch.save(local.cpu(), os.path.join(out_dir, f"part{rank}.pt"))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("split", [False, True])
def test_cyclic_two_ranks_nccl(tmp_path, split):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    n, bs = 1536, 256
    mp.spawn(_nccl_worker, args=(2, port, n, bs, 4242, str(tmp_path), split), nprocs=2,
             join=True)
    parts = [torch.load(tmp_path / f"part{r}.pt") for r in range(2)]
    l = gather_block_cyclic(parts, n, 2, bs).numpy()[None]
    a, cond = inputs.covariance(1, n, 0.5, 4242)
    l_or, _ = oracle.potrf(a.numpy())
    res = oracle.check_factor(a.numpy(), l, l_ref=l_or, cond=cond.numpy())
    assert res["ok"], res


def _sharded_nccl_worker(rank, world, port, batch, n, out_dir):
    import datetime
    import os

    import torch.distributed as dist

    from linalg_kernels_b200.distributed import factor_batch_sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        a = None
        if rank == 0:
            a, _ = inputs.spectral(batch, n, 100.0, 4343, device="cuda:0")
        l = factor_batch_sharded(a, batch, n, dist, root=0)
        torch.cuda.synchronize()
        if rank == 0:
            torch.save(l.cpu(), os.path.join(out_dir, "l.pt"))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_batch_sharded_two_ranks_nccl(tmp_path):
    """A batch on cuda:0 factored by two ranks (slices out and factors back over NCCL)
    equals the one-GPU factor bitwise: the same kernel on the same matrices."""
    import socket

    import torch.multiprocessing as mp

    from linalg_kernels_b200.cholesky import custom_kernel

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    batch, n = 9, 48
    mp.spawn(_sharded_nccl_worker, args=(2, port, batch, n, str(tmp_path)), nprocs=2,
             join=True)
    l = torch.load(tmp_path / "l.pt")
    a, _ = inputs.spectral(batch, n, 100.0, 4343, device=DEV)
    want = torch.cat([custom_kernel(a[:5]), custom_kernel(a[5:])]).cpu()
    assert torch.equal(l, want)


@pytest.mark.parametrize("world,nblk", [(1, 3), (2, 3), (3, 2)])
def test_cyclic_gemm_matches_per_block(world, nblk):
    """chol_gemm_nt_cyclic_f32 (one launch over cyclically stored blocks) equals the same
    update done block by block in FP64."""
    from linalg_kernels_b200.distributed import CudaOps

    bs, k = 256, 256
    stride = bs * world
    m = (nblk - 1) * stride + bs + 100  # rows below the first block's diagonal
    g = torch.Generator(device=DEV).manual_seed(world * 10 + nblk)
    p = torch.randn(m, k, device=DEV, generator=g)
    c0 = torch.randn(m, nblk * bs - 40, device=DEV, generator=g)
    c = c0.clone()
    CudaOps(torch.device(DEV)).cyclic_update(c, p, bs, stride)
    torch.cuda.synchronize()
    want = c0.double().clone()
    for b in range(nblk):
        w = min(bs, c0.shape[1] - b * bs)
        r = b * stride
        upd = want[r:, b * bs:b * bs + w] - p[r:].double() @ p[r:r + w].double().T
        keep = torch.ones_like(upd, dtype=torch.bool).tril()
        want[r:, b * bs:b * bs + w] = torch.where(keep, upd, want[r:, b * bs:b * bs + w])
    err = (c.double() - want).abs().max().item()
    assert err < 8 * k * 2.0 ** -22 * 25.0, err


@pytest.mark.parametrize("m,w", [(3000, 256), (1500, 128), (256, 256), (900, 100)])
@pytest.mark.parametrize("panel_inverse", [1, 0])
def test_panel_potrf_building_block(m, w, panel_inverse):
    """chol_panel_potrf_f32: the first w columns of an m-row panel factored in place equal
    the first w columns of an FP64 Cholesky of the m x m matrix (the panel's rows), with
    the one-launch block + inverse solve (option 1, w % 64 == 0) and the 64-wide steps."""
    from linalg_kernels_b200 import _lib
    from linalg_kernels_b200.distributed import CudaOps

    lib = _lib.load()
    a, _ = inputs.covariance(1, m, 0.5, 31 * m + w)
    full = a[0].to(DEV)
    panel = torch.tril(full).contiguous()  # the panel is the first w columns of these rows
    tinv = torch.empty(64, 64, device=DEV)
    info = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, panel_inverse)
    try:
        CudaOps(torch.device(DEV)).panel_potrf(panel[:, :w], tinv, info)
        torch.cuda.synchronize()
    finally:
        lib.chol_set_option(_lib.CHOL_OPT_PANEL_INVERSE, 1)
    want = torch.linalg.cholesky(full.double())[:, :w]
    got = torch.tril(panel[:, :w].double())
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert int(info.item()) == 0
    assert err < 2e-5, err


def test_panel_potrf_reports_not_spd():
    from linalg_kernels_b200.distributed import CudaOps

    m, w = 1024, 256
    a, _ = inputs.covariance(1, m, 0.5, 5)
    full = a[0].clone()
    full[130, 130] = -50.0
    panel = torch.tril(full).to(DEV).contiguous()
    tinv = torch.empty(64, 64, device=DEV)
    info = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    CudaOps(torch.device(DEV)).panel_potrf(panel[:, :w], tinv, info)
    torch.cuda.synchronize()
    assert int(info.item()) == 131


@pytest.mark.parametrize("m,w", [(3000, 256), (512, 256), (1500, 128)])
def test_panel_potrf_out_flags(m, w):
    """chol_panel_potrf_out_f32: the factored panel in the contiguous send buffer equals the
    panel factored in place by chol_panel_potrf_f32 (the same kernels, bitwise); with
    CHOL_PANEL_OUT_ONLY, L receives the top block only and the rows below stay as they were
    (the multi-GPU driver copies them back beside the send)."""
    from linalg_kernels_b200 import _lib
    from linalg_kernels_b200.distributed import CudaOps

    lib = _lib.load()
    ops = CudaOps(torch.device(DEV))
    a, _ = inputs.covariance(1, m, 0.5, 77 * m + w)
    base = torch.tril(a[0]).to(DEV).contiguous()
    ref = base.clone()
    ops.panel_potrf(ref[:, :w], torch.empty(64, 64, device=DEV), None)
    for out_only in (False, True):
        panel = base.clone()
        out = torch.full((m, w), float("nan"), device=DEV)
        assert ops.panel_potrf_out(panel[:, :w], out, None, out_only=out_only)
        torch.cuda.synchronize()
        assert torch.equal(out, ref[:, :w])
        assert torch.equal(panel[:w, :w], ref[:w, :w])
        if out_only:
            assert torch.equal(panel[w:, :w], base[w:, :w])
        else:
            assert torch.equal(panel[:, :w], ref[:, :w])
    st = lib.chol_panel_potrf_out_f32(ctypes.c_void_p(base.data_ptr()), m, m, w,
                                      ctypes.c_void_p(out.data_ptr()), 2, None, None)
    assert st == _lib.CHOL_ERR_INVALID_ARG
