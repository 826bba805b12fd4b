"""Row-sharded multi-GPU SpMM (one process per GPU, torch.distributed).

The reference has no multi-device code; this is the B200 scale-out of the
same operator.  A is cut into contiguous row ranges balanced by nonzeros at
16-row window boundaries (so window layouts built per shard keep whole
windows), B is replicated on every GPU, and each rank computes its own rows
with the single-GPU operators - there is no communication in the SpMM
itself.  For the mixed (window + CSR) operator each rank runs the
reference's task mapping on its own row slice (``ShardedMixed``), so the
window/CSR decisions stay local to the shard.  C stays row-sharded; when a caller asks for the full C on every
rank, ``MulticastRows`` fuses the gather into the SpMM (each finished row is
stored once through an NVLink multicast address and the NVSwitch writes it
into every GPU's copy while the kernel runs), and ``allgather_rows``
assembles it over NCCL where multicast is not available (one all-gather for
equal shards, one broadcast per rank otherwise).

Failure handling (no GPU fault is involved in any of it): ``Membership``
keeps the ranks' presence in the process group's store, so a rank that
leaves between steps is seen by the others on the host before their next
launch (``RankDeparted``); ``wait_bounded`` gives a collective a deadline
and aborts the process group when it passes (``CollectiveTimeout``);
``nccl_options`` makes the NCCL communicator non-blocking, so such an abort
never waits behind a blocked NCCL call.
"""

from __future__ import annotations

import time

import torch

WINDOW = 16


# --------------------------------------------------------------------------
# failure handling: departed ranks and bounded collectives
# --------------------------------------------------------------------------

class RankDeparted(RuntimeError):
    """Another rank left the job between steps (or stopped answering)."""

    def __init__(self, ranks, step):
        self.ranks = sorted(ranks)
        self.step = step
        super().__init__(f"rank(s) {self.ranks} left before step {step}; no collective was entered")


class CollectiveTimeout(RuntimeError):
    """A collective did not complete within its deadline; the process group
    was aborted."""


def nccl_options(nonblocking: bool = True):
    """Process-group options for the row-sharded job over NCCL.  With
    ``nonblocking`` the communicator is created non-blocking (ncclConfig_t
    blocking = 0): NCCL calls return at once, their progress and errors are
    read through ncclCommGetAsyncError by the process group, and a
    communicator whose peer is gone can be aborted from the host instead of
    blocking the calling thread."""
    import torch.distributed as dist

    opts = dist.ProcessGroupNCCL.Options()
    opts.config.blocking = 0 if nonblocking else 1
    return opts


def abort_group(group=None) -> bool:
    """Aborts a process group (NCCL: ncclCommAbort on its communicators,
    which also ends their device work).  Returns False when the backend
    offers no abort (then the group's own timeout ends its operations)."""
    import torch.distributed as dist

    try:
        dist.distributed_c10d._abort_process_group(group if group is not None else dist.group.WORLD)
        return True
    except Exception:   # backend without abort support (e.g. gloo builds)
        return False


def wait_bounded(works, timeout_s: float, group=None, what: str = "collective"):
    """Waits for async collective handles with a deadline, polling
    ``is_completed`` (for NCCL a query of the collective's CUDA event, so
    the host thread never blocks inside NCCL).  On expiry the group is
    aborted and CollectiveTimeout raised."""
    works = [w for w in (works if isinstance(works, (list, tuple)) else [works]) if w is not None]
    deadline = time.monotonic() + timeout_s
    for w in works:
        while not w.is_completed():
            if time.monotonic() > deadline:
                aborted = abort_group(group)
                raise CollectiveTimeout(f"{what} did not complete within {timeout_s:.1f} s"
                                        f"{'; process group aborted' if aborted else ''}")
            time.sleep(0.0005)
        w.wait()


class Membership:
    """Which ranks of a row-sharded job are still in it, kept in the process
    group's key-value store (the TCPStore of torch.distributed), so that no
    rank enters a collective that a departed peer can never join.

    Each step every rank calls ``enter(step)`` before its first launch: it
    publishes ``ready/<step>/<rank>`` and waits (bounded, on the host) until
    every other rank has published the same key or ``left/<rank>``.  A rank
    that leaves between steps calls ``leave()``; the others then raise
    RankDeparted at their next ``enter`` instead of hanging in a
    collective.  A rank that neither arrives nor leaves within ``timeout_s``
    is reported as departed too."""

    def __init__(self, store, rank: int, world: int, prefix: str = "spmm_dist/", timeout_s: float = 30.0):
        self.store, self.rank, self.world = store, rank, world
        self.prefix, self.timeout_s = prefix, timeout_s

    @classmethod
    def for_default_group(cls, timeout_s: float = 30.0, prefix: str = "spmm_dist/"):
        import torch.distributed as dist

        return cls(dist.distributed_c10d._get_default_store(), dist.get_rank(), dist.get_world_size(), prefix,
                   timeout_s)

    def _key(self, *parts) -> str:
        return self.prefix + "/".join(str(p) for p in parts)

    def _has(self, key: str) -> bool:
        return bool(self.store.check([key]))

    def leave(self, reason: str = "left") -> None:
        self.store.set(self._key("left", self.rank), reason)

    def departed(self) -> list:
        return [r for r in range(self.world) if r != self.rank and self._has(self._key("left", r))]

    def enter(self, step: int) -> None:
        self.store.set(self._key("ready", step, self.rank), "1")
        if step >= 2:   # every rank passed step - 1, so nobody reads step - 2's keys any more
            try:
                self.store.delete_key(self._key("ready", step - 2, self.rank))
            except Exception:   # stores without deletion keep the key
                pass
        pending = {r for r in range(self.world) if r != self.rank}
        deadline = time.monotonic() + self.timeout_s
        while pending:
            gone = {r for r in pending if self._has(self._key("left", r))}
            if gone:
                raise RankDeparted(gone, step)
            pending = {r for r in pending if not self._has(self._key("ready", step, r))}
            if not pending:
                return
            if time.monotonic() > deadline:
                raise RankDeparted(pending, step)
            time.sleep(0.001)


def shard_bounds(rowptr: torch.Tensor, world: int) -> list[tuple[int, int]]:
    """Row ranges [r0, r1) for each of ``world`` ranks.

    Cut points fall on 16-row window boundaries and split the nonzeros as
    evenly as that allows (target k * nnz / world for cut k).
    """
    M = rowptr.numel() - 1
    if world <= 1 or M == 0:
        return [(0, M)] + [(M, M)] * max(0, world - 1)
    rp = rowptr.detach().to(torch.int64).cpu()
    win = rp[::WINDOW].contiguous()
    if int(win[-1]) != int(rp[-1]):
        win = torch.cat([win, rp[-1:]])
    nnz = int(rp[-1])
    targets = torch.tensor([k * nnz // world for k in range(world + 1)], dtype=torch.int64)
    cut = torch.searchsorted(win, targets).clamp(max=win.numel() - 1) * WINDOW
    cut = cut.clamp(max=M)
    cut[0], cut[-1] = 0, M
    cut = torch.cummax(cut, 0).values
    return [(int(cut[k]), int(cut[k + 1])) for k in range(world)]


def shard_csr(rowptr, col, val, r0: int, r1: int):
    """CSR of rows [r0, r1) with a rebased row pointer (same index dtype)."""
    p0, p1 = int(rowptr[r0]), int(rowptr[r1])
    rp = rowptr[r0:r1 + 1].to(torch.int64) - p0
    return rp.to(rowptr.dtype).contiguous(), col[p0:p1].contiguous(), val[p0:p1].contiguous()


def allgather_rows(local: torch.Tensor, bounds: list[tuple[int, int]], group=None, out=None,
                   timeout_s: float | None = None) -> torch.Tensor:
    """Full C on every rank from row shards ``local`` ([r1 - r0, N] per rank).

    Equal shards: one all_gather_into_tensor straight into the result.
    Uneven shards: the local shard is copied into its rows of the result and
    every rank's rows are broadcast from their owner (NCCL over NVLink on
    GPUs, gloo on CPU), so no padded copies are made: the result (or ``out``)
    is the only extra buffer.  With ``timeout_s`` the collectives are issued
    asynchronously and waited for with that deadline (``wait_bounded``).
    """
    import torch.distributed as dist

    asy = timeout_s is not None

    world = len(bounds)
    rows = [r1 - r0 for r0, r1 in bounds]
    tail = tuple(local.shape[1:])
    total = sum(rows)
    full = out if out is not None else local.new_empty((total, *tail))
    works = []
    if all(r == rows[0] for r in rows):
        works.append(dist.all_gather_into_tensor(full, local.contiguous(), group=group, async_op=asy))
    else:
        me = dist.get_rank(group) if group is not None else dist.get_rank()
        offs = [sum(rows[:k]) for k in range(world)]
        full[offs[me]: offs[me] + rows[me]].copy_(local)
        for k in range(world):
            if rows[k]:
                src = dist.get_global_rank(group, k) if group is not None else k
                works.append(dist.broadcast(full[offs[k]: offs[k] + rows[k]], src=src, group=group, async_op=asy))
    if asy:
        wait_bounded(works, timeout_s, group, "row all-gather")
    return full


def group_barrier(group=None, timeout_s: float | None = None, device=None) -> None:
    """Stream-ordered barrier: a one-element all-reduce on the current stream
    (it completes on a rank only after every rank's earlier work on its own
    stream), waited for with ``timeout_s`` when given."""
    import torch.distributed as dist

    flag = torch.zeros(1, device=device)
    work = dist.all_reduce(flag, group=group, async_op=timeout_s is not None)
    if timeout_s is not None:
        wait_bounded([work], timeout_s, group, "barrier")


class MulticastRows:
    """The full C ([rows, N]) replicated on every rank of ``group`` in NVLink
    multicast memory: one buffer per GPU from torch's symmetric memory, bound
    by the CUDA driver into one multicast object (NVLS through the NVSwitch).

    ``spmm_csr_sharded(..., gather=True, replica=this)`` runs the CSR kernels
    with this rank's rows stored through the multicast address
    (``custom_ops_lib.spmm_csr_multicast``): each finished row goes out once
    and the switch writes it into every GPU's copy while the kernel runs, so
    no separate all-gather pass follows.  Each call is bracketed by
    stream-ordered barriers: the one before keeps a rank from overwriting
    copies that another rank still reads from the previous call, the one
    after completes every copy.  Raises ``RuntimeError`` where the group has
    no multicast support (use ``allgather_rows`` there).
    """

    def __init__(self, rows: int, N: int, dtype, device, group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        grp = group if group is not None else dist.group.WORLD
        self.group = group
        try:
            self.buf = symm.empty((rows, N), dtype=dtype, device=device)
            self.handle = symm.rendezvous(self.buf, grp)
            mc_base = int(self.handle.multicast_ptr)
        except Exception as e:   # allocation or rendezvous refused by the runtime
            raise RuntimeError(f"symmetric-memory replica unavailable: {e}") from e
        if not mc_base:
            raise RuntimeError("NVLink multicast (NVLS) is not available to this group")
        # the multicast object binds each rank's buffer from its first byte;
        # the replica must lie inside that buffer
        base = int(self.handle.buffer_ptrs[self.handle.rank])
        off = self.buf.data_ptr() - base
        if off < 0 or off + self.buf.numel() * self.buf.element_size() > int(self.handle.buffer_size):
            raise RuntimeError("replica lies outside its symmetric-memory buffer")
        self.mc = mc_base + off
        if self.mc % 16:
            raise RuntimeError("multicast address of the replica is not 16-byte aligned")

    def close(self) -> None:
        """Drops the replica; call on every rank at the same point, after the
        last step and before the process group is destroyed, so no rank's
        copy leaves the multicast object while another still writes it."""
        self.handle = None
        self.buf = None

    def rows_mc(self, r0: int) -> int:
        """Multicast address of row ``r0`` of the replica."""
        return self.mc + r0 * self.buf.shape[1] * self.buf.element_size()


def spmm_csr_sharded(rowptr, col, val, dense, rank: int, world: int, gather: bool = False, group=None,
                     members: Membership | None = None, step: int = 0, timeout_s: float | None = None,
                     replica: MulticastRows | None = None):
    """This rank's rows of A @ B with the engine's CSR operator; with
    ``gather=True`` the full C on every rank: with ``replica`` (a
    ``MulticastRows`` of C's shape) the rows are multicast by the SpMM
    kernels themselves and ``replica.buf`` is returned, otherwise they are
    all-gathered over NCCL afterwards.  With ``members`` the step first
    checks (on the host, before any launch) that every other rank is still
    in the job; ``timeout_s`` bounds the collectives."""
    import spmm_npu

    if members is not None:
        members.enter(step)
    bounds = shard_bounds(rowptr, world)
    r0, r1 = bounds[rank]
    rp, c, v = shard_csr(rowptr, col, val, r0, r1)
    M = rowptr.numel() - 1
    if gather and replica is not None:
        import custom_ops_lib

        if tuple(replica.buf.shape) != (M, dense.shape[1]) or replica.buf.dtype != dense.dtype:
            raise ValueError("replica must be a [rows, N] buffer of the dense operand's dtype")
        group_barrier(group, timeout_s, dense.device)
        custom_ops_lib.spmm_csr_multicast(rp, c, v, dense, replica.buf[r0:r1], replica.rows_mc(r0))
        group_barrier(group, timeout_s, dense.device)
        return replica.buf, (0, M)
    start = torch.zeros(40, dtype=torch.int32, device=dense.device)
    local = spmm_npu.spmm_csr(rp, c, v, dense, start)
    if not gather:
        return local, (r0, r1)
    return allgather_rows(local, bounds, group, timeout_s=timeout_s), (0, M)


class ShardedMixed:
    """This rank's rows of ``A @ B`` through the mixed (window + CSR)
    operator ``spmm_ascend_cube``, with the layout built per shard.

    The rows of A are cut by ``shard_bounds`` (nonzero-balanced, on 16-row
    window boundaries) and the rank runs ``preprocess`` - the reference's task
    mapping (extension/custom_op.cpp:765-1137) - on its own row slice only,
    so every window and every AIC/AIV decision is local to the shard and no
    rank ever holds another rank's layout.  The layout is built once, at
    construction; each call runs the operator on the given dense operand,
    restores the shard's rows to original order (the layout's
    ``inv_permutation``) and, with ``gather=True``, assembles the full C on
    every rank with ``allgather_rows`` (NCCL; bounded by ``timeout_s``).

    ``A`` (``rowptr``, ``col``, ``val``) may live on the CPU or the GPU; the
    layout is built on the current CUDA device.  An empty shard (more ranks
    than windows) computes nothing and contributes no rows.
    """

    KEYS = ("crow_window_ptr", "unique_col_ids", "value", "vrow_window_ptr", "vcol_indices", "vvalue")

    def __init__(self, rowptr, col, val, ncols: int, rank: int, world: int, device=None):
        import spmm_npu

        self.bounds = shard_bounds(rowptr, world)
        self.r0, self.r1 = self.bounds[rank]
        self.rows = rowptr.numel() - 1
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.layout = None
        if self.r1 > self.r0:
            rp, c, v = shard_csr(rowptr, col, val, self.r0, self.r1)
            m = spmm_npu.preprocess(rp.to(self.device), c.to(self.device), v.to(self.device), self.r1 - self.r0,
                                    int(ncols), WINDOW, False)
            self.layout = [m[k] for k in self.KEYS]
            self.inv_permutation = m["inv_permutation"]
            self.packed_rows = int(m["packed_rows"].item())
        self._cstart = torch.zeros(20, dtype=torch.int32, device=self.device)
        self._vstart = torch.zeros(40, dtype=torch.int32, device=self.device)

    def packed(self, dense: torch.Tensor) -> torch.Tensor:
        """The shard's rows in the layout's packed order (the operator's own output)."""
        import spmm_npu

        if self.layout is None:
            return dense.new_empty((0, dense.shape[1]))
        return spmm_npu.spmm_ascend_cube(*self.layout, dense, self._cstart, self._vstart)

    def __call__(self, dense: torch.Tensor, gather: bool = False, group=None, timeout_s: float | None = None):
        """``(rows, (r0, r1))``: the shard's rows of C in original order, or
        with ``gather=True`` the full C on every rank and ``(0, rows)``."""
        import spmm_npu

        if self.layout is None:
            local = dense.new_empty((0, dense.shape[1]))
        else:
            local = spmm_npu.restore_node_tensor(self.packed(dense), self.inv_permutation)
        if not gather:
            return local, (self.r0, self.r1)
        return allgather_rows(local, self.bounds, group, timeout_s=timeout_s), (0, self.rows)
