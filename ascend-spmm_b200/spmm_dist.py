"""Row-sharded multi-GPU SpMM (one process per GPU, torch.distributed).

The reference has no multi-device code; this is the B200 scale-out of the
same operator.  A is cut into contiguous row ranges balanced by nonzeros at
16-row window boundaries (so window layouts built per shard keep whole
windows), B is replicated on every GPU, and each rank computes its own rows
with the single-GPU operators - there is no communication in the SpMM
itself.  C stays row-sharded; ``allgather_rows`` assembles the full C over
NCCL (one all-gather for equal shards, one broadcast per rank otherwise) only
when a caller asks for it.
"""

from __future__ import annotations

import torch

WINDOW = 16


def shard_bounds(rowptr: torch.Tensor, world: int) -> list[tuple[int, int]]:
    """Row ranges [r0, r1) for each of ``world`` ranks.

    Cut points fall on 16-row window boundaries and split the nonzeros as
    evenly as that allows (target k * nnz / world for cut k).
    """
    M = rowptr.numel() - 1
    if world <= 1 or M == 0:
        return [(0, M)] + [(M, M)] * max(0, world - 1)
    rp = rowptr.detach().to(torch.int64).cpu()
    win = rp[::WINDOW]
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


def allgather_rows(local: torch.Tensor, bounds: list[tuple[int, int]], group=None, out=None) -> torch.Tensor:
    """Full C on every rank from row shards ``local`` ([r1 - r0, N] per rank).

    Equal shards: one all_gather_into_tensor straight into the result.
    Uneven shards: the local shard is copied into its rows of the result and
    every rank's rows are broadcast from their owner (NCCL over NVLink on
    GPUs, gloo on CPU), so no padded copies are made: the result (or ``out``)
    is the only extra buffer.
    """
    import torch.distributed as dist

    world = len(bounds)
    rows = [r1 - r0 for r0, r1 in bounds]
    tail = tuple(local.shape[1:])
    total = sum(rows)
    full = out if out is not None else local.new_empty((total, *tail))
    if all(r == rows[0] for r in rows):
        dist.all_gather_into_tensor(full, local.contiguous(), group=group)
        return full
    me = dist.get_rank(group) if group is not None else dist.get_rank()
    offs = [sum(rows[:k]) for k in range(world)]
    full[offs[me]: offs[me] + rows[me]].copy_(local)
    for k in range(world):
        if rows[k]:
            src = dist.get_global_rank(group, k) if group is not None else k
            dist.broadcast(full[offs[k]: offs[k] + rows[k]], src=src, group=group)
    return full


def spmm_csr_sharded(rowptr, col, val, dense, rank: int, world: int, gather: bool = False, group=None):
    """This rank's rows of A @ B with the engine's CSR operator; with
    ``gather=True`` the full C assembled on every rank."""
    import spmm_npu

    bounds = shard_bounds(rowptr, world)
    r0, r1 = bounds[rank]
    rp, c, v = shard_csr(rowptr, col, val, r0, r1)
    start = torch.zeros(40, dtype=torch.int32, device=dense.device)
    local = spmm_npu.spmm_csr(rp, c, v, dense, start)
    if not gather:
        return local, (r0, r1)
    return allgather_rows(local, bounds, group), (0, rowptr.numel() - 1)
