"""CPU: the block-column-cyclic multi-rank schedule (linalg_kernels_b200.distributed) with
gloo ranks. The GPU arithmetic is replaced by a torch-CPU stand-in defined here, so this
checks the host logic: ownership, panel packing, broadcast order and look-ahead, update
ranges, and the reassembled factor against a float64 Cholesky."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from linalg_kernels_b200.distributed import (CyclicLayout, factor_block_cyclic,
                                             gather_block_cyclic, scatter_block_cyclic)


class CpuOps:
    def potrf_block(self, diag, tinv, info):
        kb = diag.shape[0]
        l = torch.linalg.cholesky(torch.tril(diag) + torch.tril(diag, -1).T)
        diag.copy_(l)
        tinv.zero_()
        tinv.fill_diagonal_(1.0)
        tinv[:kb, :kb] = torch.linalg.inv(l)

    def panel_potrf(self, panel, tinv, info):
        w = panel.shape[1]
        d = panel[:w]
        l = torch.linalg.cholesky(torch.tril(d) + torch.tril(d, -1).T)
        d.copy_(l)
        if panel.shape[0] > w:
            panel[w:] = torch.linalg.solve_triangular(l, panel[w:].T, upper=False).T

    def diag_potrf_inv(self, block, v, info):
        l = torch.linalg.cholesky(torch.tril(block) + torch.tril(block, -1).T)
        block.copy_(l)
        v.copy_(torch.linalg.inv(l))
        return True

    def cyclic_update(self, c, p, block, stride):
        nc = c.shape[1]
        for b in range(0, nc, block):
            w = min(block, nc - b)
            r = (b // block) * stride
            self.gemm_nt(c[r:, b:b + w], p[r:], p[r:r + w], -1.0, 1.0, True)

    def gemm_nt(self, c, p, q, alpha, beta, lower_only):
        new = alpha * (p @ q.T) + (beta * c if beta != 0.0 else 0.0)
        if lower_only:
            keep = torch.ones_like(c, dtype=torch.bool).tril()
            c.copy_(torch.where(keep, new, c))
        else:
            c.copy_(new)


def _matrix(n, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, n, generator=g, dtype=torch.float64)
    return (x @ x.T / n + torch.eye(n, dtype=torch.float64) * 0.5).float()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, bs, seed, out_dir, paired=True, split=None):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a = _matrix(n, seed)
        lay = CyclicLayout(n, world, rank, bs)
        local = scatter_block_cyclic(a, lay)
        factor_block_cyclic(local, lay, pg=dist, ops=CpuOps(), paired=paired, split_send=split)
        torch.save(local, os.path.join(out_dir, f"part{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,bs,paired,split", [(2, 300, 64, True, None),
                                                     (3, 260, 32, True, None),
                                                     (2, 128, 64, True, None),
                                                     (3, 260, 32, False, None),
                                                     (4, 520, 32, True, None),
                                                     (3, 260, 32, True, True),
                                                     (2, 300, 64, False, True),
                                                     (4, 520, 32, True, True),
                                                     (8, 680, 32, True, None)])
def test_block_cyclic_gloo_matches_cholesky(tmp_path, world, n, bs, paired, split):
    # paired: every other update of the blocks right of the look-ahead block is deferred
    # and applied for two panels at once; split (split_send, off by default): each block is
    # sent unfactored, then [L11 | inv(L11)], and every rank solves the rows below itself
    port = _free_port()
    mp.spawn(_worker, args=(world, port, n, bs, 11 + n, str(tmp_path), paired, split),
             nprocs=world, join=True)
    parts = [torch.load(tmp_path / f"part{r}.pt") for r in range(world)]
    l = gather_block_cyclic(parts, n, world, bs).double()
    a = _matrix(n, 11 + n).double()
    ref = torch.linalg.cholesky(a)
    assert (l.triu(1) == 0).all()
    assert (l - ref).abs().max().item() < 1e-4
    rel = ((l @ l.T - a).norm() / a.norm()).item()
    assert rel < 1e-5, rel


@pytest.mark.parametrize("split", [False, True])
def test_single_rank_without_process_group(split):
    n, bs = 200, 64
    a = _matrix(n, 5)
    lay = CyclicLayout(n, 1, 0, bs)
    local = scatter_block_cyclic(a, lay)
    factor_block_cyclic(local, lay, pg=None, ops=CpuOps(), split_send=split)
    ref = torch.linalg.cholesky(a.double())
    assert (local.double() - ref).abs().max().item() < 1e-4


def test_layout_ownership_and_local_columns():
    lay = CyclicLayout(n=1000, world=3, rank=1, bs=256)
    assert lay.nblocks == 4
    assert lay.owned() == [1]
    assert lay.n_local == 256
    lay2 = CyclicLayout(n=1000, world=3, rank=0, bs=256)
    assert lay2.owned() == [0, 3]
    assert lay2.width(3) == 1000 - 768
    assert lay2.local_col(3) == 256
    assert lay2.n_local == 256 + 232
    assert [lay2.owner(t) for t in range(4)] == [0, 1, 2, 0]


def test_scatter_gather_roundtrip():
    n, world, bs = 333, 2, 64
    a = torch.tril(_matrix(n, 3))
    parts = [scatter_block_cyclic(a, CyclicLayout(n, world, r, bs)) for r in range(world)]
    assert torch.equal(gather_block_cyclic(parts, n, world, bs), a)


# --------------------------------------------------------------------------------------
# batches of independent matrices from one root (factor_batch_sharded)
# --------------------------------------------------------------------------------------
def _cpu_factor(x):
    return torch.linalg.cholesky_ex(x).L  # stand-in for custom_kernel (test only)


def _batch(batch, n, seed):
    return torch.stack([_matrix(n, seed + i) for i in range(batch)])


def _sharded_worker(rank, world, port, batch, n, root, out_dir):
    import torch.distributed as dist

    from linalg_kernels_b200.distributed import factor_batch_sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a = _batch(batch, n, 40) if rank == root else None
        seen = []

        def factor(x):
            seen.append(x.shape[0])
            return _cpu_factor(x)

        l = factor_batch_sharded(a, batch, n, dist, factor=factor, root=root,
                                 device=torch.device("cpu"))
        torch.save({"l": l, "seen": seen}, os.path.join(out_dir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_batch_slices():
    from linalg_kernels_b200.distributed import batch_slices

    assert batch_slices(10, 4) == [(0, 3), (3, 3), (6, 2), (8, 2)]
    assert batch_slices(8, 2) == [(0, 4), (4, 4)]
    assert sum(c for _, c in batch_slices(1024, 8)) == 1024


@pytest.mark.parametrize("world,batch,root", [(2, 5, 0), (3, 7, 1), (2, 2, 0)])
def test_batch_sharded_gloo_matches_one_rank(tmp_path, world, batch, root):
    """Every rank factors its own contiguous slice; the root gets back the whole factor,
    equal to the stand-in over the whole batch, and the other ranks get None."""
    from linalg_kernels_b200.distributed import batch_slices

    n = 24
    port = _free_port()
    mp.spawn(_sharded_worker, args=(world, port, batch, n, root, str(tmp_path)), nprocs=world,
             join=True)
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    want = _cpu_factor(_batch(batch, n, 40))
    assert torch.equal(res[root]["l"], want)
    for r in range(world):
        assert res[r]["seen"] == [batch_slices(batch, world)[r][1]]
        if r != root:
            assert res[r]["l"] is None


def test_batch_sharded_single_rank_and_argument_checks():
    from linalg_kernels_b200.distributed import factor_batch_sharded

    class OneRank:
        def get_world_size(self):
            return 1

        def get_rank(self):
            return 0

    a = _batch(3, 16, 7)
    assert torch.equal(factor_batch_sharded(a, 3, 16, OneRank(), factor=_cpu_factor),
                       _cpu_factor(a))
    with pytest.raises(ValueError):
        factor_batch_sharded(None, 3, 16, OneRank(), factor=_cpu_factor)

    class TwoRanks(OneRank):
        def get_world_size(self):
            return 2

    with pytest.raises(ValueError, match="every rank"):
        factor_batch_sharded(a[:1], 1, 16, TwoRanks(), factor=_cpu_factor)


def test_auto_queue_caps_follow_the_rank_count():
    """One rank runs in order; over several ranks the chain's share of the SMs grows with the
    rank count (each rank's bulk work shrinks as 1/ranks), and 16 SMs stay free for NCCL."""
    from linalg_kernels_b200.distributed import auto_queues

    assert auto_queues(1) is None
    caps = [auto_queues(w) for w in (2, 4, 8)]
    assert [c[0] for c in caps] == sorted(c[0] for c in caps)
    assert all(c[0] + c[1] == 132 for c in caps)
