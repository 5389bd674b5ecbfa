"""Multi-GPU Cholesky of one large matrix: 1-D block-column-cyclic over ranks, NCCL panels.

The reference has no multi-GPU path (its n = 32768 kernel runs on one B200,
cholesky/cholesky.py:5692-5802). Here one process per GPU holds the column blocks
``t = rank, rank + P, rank + 2P, ...`` (block width ``bs``, default 256) of the matrix,
row-major in a local ``(n, n_local)`` tensor. For every block column ``j``:

1. its owner factors the panel ``L[j*bs:, j*bs:(j+1)*bs]`` in place with one
   ``chol_panel_potrf_out_f32`` call (one diagonal-block launch that factors the ``bs x bs``
   top block and writes its inverse ``V``, then one tensor-core GEMM ``X = A21 V^T`` that
   solves every row below), which also leaves the factored panel (rows ``j*bs .. n``, ``bs``
   columns, at most 32 MiB at n = 32768) packed contiguously in the send buffer;
2. NCCL broadcasts it from the owner into every rank's receive buffer (local memory; no
   kernel reads another GPU's memory);
3. every rank applies ``C -= P P^T`` (lower tiles) to its blocks right of the look-ahead
   block with ``chol_gemm_nt_cyclic_f32`` (the GEMM maps local column blocks to their
   global columns, so masking and Q's rows follow the cyclic layout).

Look-ahead of depth 2 on two queues of each GPU: when panel ``j`` has arrived, the
high-priority "chain" queue updates blocks ``j+1`` and ``j+2`` with it (on their owners),
and the owner of ``j+1`` factors it and starts its broadcast; the low-priority "bulk" queue
updates every block right of ``j+2``. A block leaves the bulk set one step before the chain
needs it, so each bulk update has two chain steps to finish in, and the chain never waits
behind a bulk update in queue order. Events order the two queues (the chain's update of
block ``j+2`` waits for the bulk's previous work, the bulk waits for panel ``j``, a receive
buffer is rewritten only after the bulk has read it). Both queues' GEMMs run with capped
grids (``CHOL_OPT_GEMM_CTAS``), so that the persistent kernels of one queue never hold SMs
the other needs, and some SMs stay free for NCCL.

Paired updates: the bulk update is deferred every other step and then applied for two
panels at once, ``P = [panel j-1 | panel j]`` (K = 2 bs = 512), copied side by side into one
buffer (by the bulk queue; the chain's update of block ``j+2`` takes the same K = 512
product). A K = 256 update spends as long in its epilogue (the read-modify-write of C) as
in its tensor-core main loop; at K = 512 the main loop hides it, and the trailing matrix is
read and written half as often. Receive buffers rotate over four panels. Every rank issues
the same collectives in the same order.

The arithmetic goes through an ``ops`` object: ``CudaOps`` (the C ABI of libchol_b200.so,
the product path). Tests substitute a CPU implementation to check the schedule with
``gloo`` ranks on machines without GPUs.
"""

from __future__ import annotations

import contextlib
import ctypes
from dataclasses import dataclass

import torch

from . import _lib

__all__ = ["CyclicLayout", "CudaOps", "factor_block_cyclic", "scatter_block_cyclic",
           "gather_block_cyclic", "batch_slices", "factor_batch_sharded"]


@dataclass(frozen=True)
class CyclicLayout:
    n: int
    world: int
    rank: int
    bs: int = 256

    @property
    def nblocks(self) -> int:
        return (self.n + self.bs - 1) // self.bs

    def owner(self, t: int) -> int:
        return t % self.world

    def owned(self) -> list[int]:
        return list(range(self.rank, self.nblocks, self.world))

    def width(self, t: int) -> int:
        return min(self.bs, self.n - t * self.bs)

    def local_col(self, t: int) -> int:
        """First local column of block t (t must be owned by this rank)."""
        return (t // self.world) * self.bs

    @property
    def n_local(self) -> int:
        blocks = self.owned()
        return sum(self.width(t) for t in blocks)


def scatter_block_cyclic(a: torch.Tensor, lay: CyclicLayout) -> torch.Tensor:
    """This rank's columns of the full matrix ``a`` (lower triangle kept, zeros above)."""
    n = lay.n
    out = torch.zeros(n, lay.n_local, dtype=a.dtype, device=a.device)
    for t in lay.owned():
        c0, w, lc = t * lay.bs, lay.width(t), lay.local_col(t)
        out[c0:, lc:lc + w] = torch.tril(a[c0:, c0:c0 + w])
    return out


def gather_block_cyclic(parts: list[torch.Tensor], n: int, world: int, bs: int = 256):
    """Reassemble the full matrix from every rank's local tensor (tests, e2e output)."""
    full = torch.zeros(n, n, dtype=parts[0].dtype, device=parts[0].device)
    for r in range(world):
        lay = CyclicLayout(n, world, r, bs)
        for t in lay.owned():
            c0, w, lc = t * bs, lay.width(t), lay.local_col(t)
            full[:, c0:c0 + w] = parts[r][:, lc:lc + w]
    return full


def _rowmajor(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("expected a row-major 2-D view")
    return t.stride(0)


class CudaOps:
    """Product backend: the sm_100a kernels through the C ABI, on torch's current queue."""

    def __init__(self, device: torch.device):
        self.lib = _lib.load()
        self.device = device

    def _q(self):
        return ctypes.c_void_p(_lib.current_queue(self.device))

    def queues(self, chain_ctas: int, bulk_ctas: int) -> "QueuePair":
        return QueuePair(self, chain_ctas, bulk_ctas)

    def diag_potrf_inv(self, block: torch.Tensor, v: torch.Tensor,
                       info: torch.Tensor | None) -> bool:
        """Factor the w x w block view in place and write v = inv(L11) (w x w, contiguous).
        False when the one-launch form does not take the shape (nothing done)."""
        w = block.shape[0]
        st = self.lib.chol_diag_potrf_inv_f32(
            ctypes.c_void_p(block.data_ptr()), _rowmajor(block), w, ctypes.c_void_p(v.data_ptr()),
            ctypes.c_void_p(info.data_ptr()) if info is not None else None, self._q())
        if st == _lib.CHOL_ERR_UNSUPPORTED:
            return False
        _lib.check(st, "chol_diag_potrf_inv_f32")
        return True

    def potrf_block(self, diag: torch.Tensor, tinv: torch.Tensor, info: torch.Tensor | None):
        """Factor diag (kb x kb view, kb <= 64) in place; tinv (64 x 64) <- inv(L)."""
        ld = _rowmajor(diag)
        st = self.lib.chol_block_potrf_f32(
            ctypes.c_void_p(diag.data_ptr()), 1, 0, ld, 0, diag.shape[0],
            ctypes.c_void_p(tinv.data_ptr()),
            ctypes.c_void_p(info.data_ptr()) if info is not None else None, self._q())
        _lib.check(st, "chol_block_potrf_f32")

    def panel_potrf_out(self, panel: torch.Tensor, out: torch.Tensor,
                        info: torch.Tensor | None, out_only: bool = False) -> bool:
        """Factor a tall panel view in place and write it to ``out`` (m x w, contiguous) as
        well; with ``out_only`` the rows below the w x w top block stay in ``out`` only (the
        caller copies them into ``panel``). False when the one-launch form does not take the
        shape (nothing done)."""
        m, w = panel.shape
        st = self.lib.chol_panel_potrf_out_f32(
            ctypes.c_void_p(panel.data_ptr()), _rowmajor(panel), m, w,
            ctypes.c_void_p(out.data_ptr()), _lib.CHOL_PANEL_OUT_ONLY if out_only else 0,
            ctypes.c_void_p(info.data_ptr()) if info is not None else None, self._q())
        if st == _lib.CHOL_ERR_UNSUPPORTED:
            return False
        _lib.check(st, "chol_panel_potrf_out_f32")
        return True

    def panel_potrf(self, panel: torch.Tensor, tinv: torch.Tensor, info: torch.Tensor | None):
        """Factor a tall panel view (m x w, element (0,0) on the diagonal) in place."""
        m, w = panel.shape
        st = self.lib.chol_panel_potrf_f32(
            ctypes.c_void_p(panel.data_ptr()), _rowmajor(panel), m, w,
            ctypes.c_void_p(tinv.data_ptr()),
            ctypes.c_void_p(info.data_ptr()) if info is not None else None, self._q())
        _lib.check(st, "chol_panel_potrf_f32")

    def cyclic_update(self, c: torch.Tensor, p: torch.Tensor, block: int, stride: int):
        """c -= p q^T over cyclically stored column blocks (q = rows of p at the mapped
        global columns), lower part only; element (0,0) of c is on the diagonal."""
        m, nc = c.shape
        k = p.shape[1]
        if block == 256:
            st = self.lib.chol_gemm_nt_cyclic_f32(
                ctypes.c_void_p(c.data_ptr()), _rowmajor(c), m, nc, k,
                ctypes.c_void_p(p.data_ptr()), _rowmajor(p),
                ctypes.c_void_p(p.data_ptr()), _rowmajor(p), -1.0, 1.0, 0, 1, block, stride,
                self._q())
            if st != _lib.CHOL_ERR_UNSUPPORTED:
                _lib.check(st, "chol_gemm_nt_cyclic_f32")
                return
        for b in range(0, nc, block):  # one launch per block
            w = min(block, nc - b)
            r = (b // block) * stride
            self.gemm_nt(c[r:, b:b + w], p[r:], p[r:r + w], -1.0, 1.0, True)

    def gemm_nt(self, c: torch.Tensor, p: torch.Tensor, q: torch.Tensor, alpha: float,
                beta: float, lower_only: bool):
        """c = alpha * p q^T + beta * c; lower_only keeps elements with col <= row."""
        m, nc = c.shape
        k = p.shape[1]
        st = self.lib.chol_gemm_nt_f32(
            ctypes.c_void_p(c.data_ptr()), 1, 0, _rowmajor(c), m, nc, k,
            ctypes.c_void_p(p.data_ptr()), 0, _rowmajor(p),
            ctypes.c_void_p(q.data_ptr()), 0, _rowmajor(q),
            float(alpha), float(beta), 0, 1 if lower_only else 0, self._q())
        _lib.check(st, "chol_gemm_nt_f32")


def _factor_panel(local: torch.Tensor, lay: CyclicLayout, t: int, ops, tinv, info, out=None,
                  defer_copy: bool = False):
    """Owner: factor block column t in place (rows t*bs..n of its local columns); with
    ``out`` (rows x width, contiguous) the factored panel is also left there. With
    ``defer_copy`` the rows below the top block may be left in ``out`` only: the return value
    is then the (destination, source) pair still to copy, else None."""
    c0, w, lc = t * lay.bs, lay.width(t), lay.local_col(t)
    view = local[c0:, lc:lc + w]
    fused = getattr(ops, "panel_potrf_out", None)
    if out is not None and fused is not None:
        if defer_copy and view.shape[0] > w and fused(view, out, info, out_only=True):
            return view[w:], out[w:]
        if fused(view, out, info):
            return None
    ops.panel_potrf(view, tinv, info)
    if out is not None:
        out.copy_(view)
    return None


def _update_blocks(local: torch.Tensor, lay: CyclicLayout, blocks: list[int], first_row: int,
                   panel, ops):
    """Owned blocks `blocks` (consecutive in this rank's storage) -= P P^T, lower part, in one
    call, where P = panel's rows from the blocks' first row (panel row 0 is global row
    first_row): local column block b stands for global block blocks[0] + b*world."""
    bs = lay.bs
    t0 = blocks[0]
    c0, lc0 = t0 * bs, lay.local_col(t0)
    width = sum(lay.width(t) for t in blocks)
    p = panel[c0 - first_row:]
    ops.cyclic_update(local[c0:, lc0:lc0 + width], p, bs, bs * lay.world)


class _OneQueue:
    """Stand-in for a queue pair where ops has none (CPU ops): one queue, no events."""

    def on(self, name):
        return contextlib.nullcontext()

    def record(self):
        return None

    def wait(self, ev):
        pass

    def join(self):
        pass


class QueuePair:
    """Two torch queues of one device for the column-cyclic schedule: "chain" (high priority:
    the look-ahead updates, the panel factor and its broadcast) and "bulk" (low priority: the
    update of every block right of the look-ahead blocks), each with its own cap on the
    library's tensor-core GEMM grids (``CHOL_OPT_GEMM_CTAS``, set per call from this thread)
    so that the persistent GEMMs of the two queues hold disjoint SMs and leave some free for
    NCCL. Both queues start after the caller's queue and the caller's queue waits for both
    at ``join``."""

    def __init__(self, ops: "CudaOps", chain_ctas: int, bulk_ctas: int):
        self.ops = ops
        dev = ops.device
        self.caller = torch.cuda.current_stream(dev)
        self.streams = {"chain": torch.cuda.Stream(dev, priority=-1),
                        "bulk": torch.cuda.Stream(dev, priority=0)}
        self.caps = {"chain": int(chain_ctas), "bulk": int(bulk_ctas)}
        start = self.caller.record_event()
        for q in self.streams.values():
            q.wait_event(start)

    @contextlib.contextmanager
    def on(self, name):
        with torch.cuda.stream(self.streams[name]):
            _lib.check(self.ops.lib.chol_set_option(_lib.CHOL_OPT_GEMM_CTAS, self.caps[name]),
                       "chol_set_option")
            try:
                yield
            finally:
                self.ops.lib.chol_set_option(_lib.CHOL_OPT_GEMM_CTAS, 0)

    def record(self):
        return torch.cuda.current_stream(self.ops.device).record_event()

    def wait(self, ev):
        if ev is not None:
            torch.cuda.current_stream(self.ops.device).wait_event(ev)

    def join(self):
        for q in self.streams.values():
            self.caller.wait_stream(q)


# (chain, bulk) GEMM CTA caps of the two queues by rank count; 148 - 132 = 16 SMs stay free
# for NCCL's kernels. Each rank's bulk work shrinks as 1/ranks while the chain's does not,
# so the chain's share grows with the rank count. n = 32768: at 2 GPUs 54.7 ms in order,
# 51.3 at (40, 92), 51.9 at (32, 100), 52.1 at (48, 84), 56.2 at (24, 108), 60.4 at
# (64, 64), 54.0 uncapped; at 4 GPUs 43.0 in order, 40.9 at (40, 92), 38.1 at (56, 76),
# 39.8 at (72, 60); at 8 GPUs 34.3 at (88, 44) and 35.9 at (56, 76), steady over repeats,
# while (72, 60) varied from 34 to 42 ms between repeats.
def auto_queues(world: int) -> tuple[int, int] | None:
    if world <= 1:
        return None
    if world == 2:
        return (40, 92)
    if world <= 4:
        return (56, 76)
    return (88, 44)


def factor_block_cyclic(local: torch.Tensor, lay: CyclicLayout, pg=None, group=None, ops=None,
                        info: torch.Tensor | None = None, paired: bool = True,
                        queues: tuple[int, int] | None | str = "auto",
                        split_send: bool | None = None) -> torch.Tensor:
    """Factor in place the block-column-cyclic matrix whose local columns are ``local``.

    ``pg`` is ``torch.distributed`` (or None for a single rank); ``ops`` defaults to
    ``CudaOps`` on ``local``'s device. Look-ahead of depth 2: at step ``j`` (panel ``j``
    received) the chain queue updates blocks ``j+1`` and ``j+2`` with it and factors and
    broadcasts block ``j+1``; the bulk queue updates the blocks right of ``j+2``. A block
    leaves the bulk set one step before the chain needs it, so each bulk update has two
    steps of the chain to finish in. ``paired`` defers every other bulk update and applies
    two panels at once (K = 2 bs). ``queues`` = (chain, bulk) GEMM CTA caps of the two
    queues (``QueuePair``); None runs everything in order on the caller's queue; "auto" =
    ``auto_queues(world)``: None on one rank (there the bulk is the whole trailing update
    and every SM it gives up costs more than the overlap wins: n = 32768 on one GPU 86.1 ms
    in order, 90.0 ms at (32, 100)).

    ``split_send`` (off by default): the
    owner broadcasts block ``j+1`` as soon as its look-ahead update is done, unfactored, and
    factors only its diagonal block meanwhile (``chol_diag_potrf_inv_f32``: L11 and
    V = inv(L11)); a second, small broadcast sends L11 and V, and every rank solves the rows
    below itself (X = A21 V^T). The large send then overlaps the diagonal factor instead of
    following the whole panel factor. The owner keeps the block it sends in a contiguous
    buffer (copied out of its columns after the block's last update before the look-ahead),
    so the send needs no packing. Every rank computes the same products as the owner would,
    so the factor is bitwise that of the unsplit schedule. It measured no faster (n = 32768:
    2 GPUs 52.6 against 50.8 ms, 4 GPUs 38.0-41.2 against 38.5-40.1, 8 GPUs 33.3-37.0
    against 34.3-36.1): the solve moves onto every rank's chain, and at 2-4 GPUs the bulk,
    not the chain, sets the time. Returns ``local`` (now this rank's columns of L).
    """
    if isinstance(queues, str):
        if queues != "auto":
            raise ValueError(f"queues: {queues!r}")
        queues = auto_queues(lay.world)
    if ops is None:
        ops = CudaOps(local.device)
    if split_send is None:
        split_send = False
    n, bs = lay.n, lay.bs
    nb = lay.nblocks
    dev = local.device
    tinv = torch.zeros(64, 64, dtype=local.dtype, device=dev)
    paired = paired and nb > 3
    nbuf = 4  # panel j's buffer is rewritten by panel j + 4 (its readers end at step j + 1)
    bufs = [torch.empty(n * bs, dtype=local.dtype, device=dev) for _ in range(nbuf)]
    combs = [torch.empty(n * 2 * bs, dtype=local.dtype, device=dev) for _ in range(2 if paired else 0)]
    # split_send: the sent (unfactored) block columns and [L11 | V] of the last two blocks
    raws = [torch.empty(n * bs, dtype=local.dtype, device=dev) for _ in range(2 if split_send else 0)]
    svs = [torch.empty(2 * bs * bs, dtype=local.dtype, device=dev) for _ in range(2 if split_send else 0)]
    make = getattr(ops, "queues", None)
    qs = make(*queues) if (queues is not None and make is not None) else _OneQueue()
    owned = lay.owned()
    multi = pg is not None and lay.world > 1

    def mine(t):
        return t < nb and lay.owner(t) == lay.rank

    def panel_view(j):
        rows = n - j * bs
        return bufs[j % nbuf][: rows * lay.width(j)].view(rows, lay.width(j))

    def raw_view(t):
        rows = n - t * bs
        return raws[t % 2][: rows * lay.width(t)].view(rows, lay.width(t))

    def sv_view(t):
        w = lay.width(t)
        return svs[t % 2][: 2 * w * w].view(2, w, w)

    def local_block(t):
        lc = lay.local_col(t)
        return local[t * bs:, lc:lc + lay.width(t)]

    def bcast(x, t):
        return pg.broadcast(x, src=_global_rank(pg, group, lay.owner(t)), group=group,
                            async_op=True)

    bulk_done = {}  # step -> event after the bulk queue's work of that step

    def publish(j):
        """Chain queue: the owner factors block j (fully updated) into its send buffer; every
        rank joins the broadcast. The owner copies the solved rows back into its own columns
        after the broadcast is issued, so that copy runs beside the send. Returns the work
        handles."""
        qs.wait(bulk_done.get(j - nbuf + 1))  # the buffer's previous panel is read out
        pv = panel_view(j)
        back = None
        if mine(j):
            back = _factor_panel(local, lay, j, ops, tinv, info, out=pv, defer_copy=True)
        handles = [bcast(pv, j)] if multi else []
        if back is not None:
            back[0].copy_(back[1])
        return handles

    def publish_split(t):
        """Chain queue, split_send: send block t unfactored, factor its diagonal block beside
        the send, then send [L11 | V]. The last block (no rows below) is factored whole by
        its owner and sent once."""
        r = raw_view(t)
        handles = []
        if t == nb - 1:
            if mine(t):
                ops.panel_potrf(r, tinv, info)
            return [bcast(r, t)] if multi else []
        if multi:
            handles.append(bcast(r, t))
        sv = sv_view(t)
        if mine(t):
            sv[0].copy_(r[: lay.width(t)])
            if not ops.diag_potrf_inv(sv[0], sv[1], info):
                raise RuntimeError("chol_diag_potrf_inv_f32 does not take this block")
        if multi:
            handles.append(bcast(sv, t))
        return handles

    def finish_split(t):
        """Chain queue, split_send, once block t's sends have arrived: panel t = [L11; A21 V^T]
        into its buffer (the owner copies it into its own columns later in the step, after
        the next block's sends are issued)."""
        qs.wait(bulk_done.get(t - nbuf + 1))  # the buffer's previous panel is read out
        pv, r, w = panel_view(t), raw_view(t), lay.width(t)
        if t == nb - 1:
            pv.copy_(r)
        else:
            sv = sv_view(t)
            pv[:w].copy_(sv[0])
            ops.gemm_nt(pv[w:], r[w:], sv[1], 1.0, 0.0, False)

    def stage(t):
        """Owner, split_send: block t (all updates before the look-ahead applied) into its
        contiguous send buffer, where the look-ahead update then applies."""
        if mine(t):
            raw_view(t).copy_(local_block(t))

    with qs.on("chain"):
        if split_send:
            stage(0)
            stage(1)
            work = publish_split(0)
        else:
            work = publish(0)
    pending = None  # step whose bulk update is deferred to the next step (paired)
    ncomb = 0  # combined buffers alternate: one is read while the next is written
    for j in range(nb):
        l1, l2 = j + 1, j + 2
        with qs.on("chain"):
            for h in work:
                h.wait()
            if split_send:
                finish_split(j)
            ready = qs.record()
        rest = [t for t in owned if t > l2]
        defer = paired and pending is None and l2 + 1 < nb
        comb = None
        with qs.on("bulk"):
            qs.wait(ready)
            if pending is not None and (rest or mine(l2)):
                # P = [panel pending | panel j] from block l2's first row down, side by side
                rows = n - l2 * bs
                comb = combs[ncomb % 2][: rows * 2 * bs].view(rows, 2 * bs)
                ncomb += 1
                comb[:, :bs].copy_(panel_view(pending)[l2 * bs - pending * bs:])
                comb[:, bs:].copy_(panel_view(j)[l2 * bs - j * bs:])
            pre = qs.record()  # the bulk's earlier updates and this step's P are in place
            if rest and not defer:
                if comb is not None:
                    _update_blocks(local, lay, rest, l2 * bs, comb, ops)
                else:
                    _update_blocks(local, lay, rest, j * bs, panel_view(j), ops)
            bulk_done[j] = qs.record()
        with qs.on("chain"):
            if mine(l1):
                if split_send:
                    p = panel_view(j)[bs:]  # rows from block l1's first row
                    ops.gemm_nt(raw_view(l1), p, p[: lay.width(l1)], -1.0, 1.0, True)
                else:
                    _update_blocks(local, lay, [l1], j * bs, panel_view(j), ops)
            if l1 < nb:
                work = publish_split(l1) if split_send else publish(l1)
            else:
                work = []
            if split_send and mine(j):
                local_block(j).copy_(panel_view(j))  # panel j into the owner's columns
            if mine(l2):
                qs.wait(pre)  # block l2 left the bulk set at this step
                if comb is not None:
                    _update_blocks(local, lay, [l2], l2 * bs, comb, ops)
                else:
                    _update_blocks(local, lay, [l2], j * bs, panel_view(j), ops)
                if split_send:
                    stage(l2)
        bulk_done.pop(j - nbuf, None)
        pending = j if defer else None
    qs.join()
    return local


def _global_rank(pg, group, r):
    if group is None:
        return r
    return pg.get_global_rank(group, r)


# --------------------------------------------------------------------------------------
# batches of independent matrices (M1) from one GPU
# --------------------------------------------------------------------------------------
def batch_slices(batch: int, world: int) -> list[tuple[int, int]]:
    """(offset, count) of each rank's contiguous slice of the batch; the first
    ``batch % world`` ranks take one matrix more."""
    base, extra = divmod(batch, world)
    out, off = [], 0
    for r in range(world):
        c = base + (1 if r < extra else 0)
        out.append((off, c))
        off += c
    return out


def _p2p(pg, ops):
    """Start a group of point-to-point transfers (none for an empty list)."""
    return pg.batch_isend_irecv(ops) if ops else []


def factor_batch_sharded(a: torch.Tensor | None, batch: int, n: int, pg, factor=None,
                         root: int = 0, device=None) -> torch.Tensor | None:
    """Batched factorisation spread over the ranks when the whole batch lives on one GPU.

    ``a`` is the contiguous ``(batch, n, n)`` input on the root rank's device, and None on
    the other ranks. The root sends each rank its contiguous slice of matrices by
    point-to-point transfers (NCCL over NVLink on GPUs). Every rank factors its slice with
    ``factor`` (``custom_kernel`` by default) and sends the factor back. The root returns
    the ``(batch, n, n)`` factor and the other ranks return None. The matrices are
    independent, so the two transfers are the only communication, and the root's own slice
    never moves. Every rank calls this with the same ``batch``, ``n`` and ``root``. Each
    rank needs at least one matrix: with NCCL, the first point-to-point call of a group
    must include every rank. ``device`` is where the non-root ranks receive (default: the
    current CUDA device)."""
    world, rank = pg.get_world_size(), pg.get_rank()
    if batch < world:
        raise ValueError(f"batch {batch} < {world} ranks: every rank needs a matrix")
    if factor is None:
        from .cholesky import custom_kernel as factor
    sl = batch_slices(batch, world)
    off, cnt = sl[rank]
    if rank == root:
        if a is None or tuple(a.shape) != (batch, n, n) or not a.is_contiguous():
            raise ValueError("the root needs the contiguous (batch, n, n) input")
        sends = [pg.P2POp(pg.isend, a[o:o + c], r) for r, (o, c) in enumerate(sl) if r != root]
        sent = _p2p(pg, sends)
        # the root's own slice is disjoint from what it sends: it is factored while the
        # sends are in flight (NCCL runs them on its own queue)
        mine = a[off:off + cnt]
        l_mine = factor(mine)
        for w in sent:
            w.wait()
        out = torch.empty(batch, n, n, dtype=a.dtype, device=a.device)
        recvs = [pg.P2POp(pg.irecv, out[o:o + c], r) for r, (o, c) in enumerate(sl)
                 if r != root]
        reqs = _p2p(pg, recvs)
        out[off:off + cnt].copy_(l_mine)
        for w in reqs:
            w.wait()
        return out
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    mine = torch.empty(cnt, n, n, dtype=torch.float32, device=dev)
    for w in _p2p(pg, [pg.P2POp(pg.irecv, mine, root)]):
        w.wait()
    l_mine = factor(mine).contiguous()
    for w in _p2p(pg, [pg.P2POp(pg.isend, l_mine, root)]):
        w.wait()
    return None
