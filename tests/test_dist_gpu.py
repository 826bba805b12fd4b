"""Row-sharded SpMM on 2 GPUs (NCCL): every rank computes its shard with the
engine's CSR operator, the all-gather assembles C, and the result matches the
float64 oracle.  Runs as child processes; skipped with fewer than 2 GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import sys
    from datetime import timedelta
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for p in (root / "ascend-spmm_b200", root, root / "oracle", root / "tests"):
        sys.path.insert(0, str(p))
    import torch.distributed as dist

    import workloads
    from spmm_dist import spmm_csr_sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = workloads.make(2, scale=0.02, device=f"cuda:{rank}")
        full, _ = spmm_csr_sharded(w.rowptr, w.col, w.val, w.B, rank, world, gather=True)
        torch.cuda.synchronize()
        if rank == 0:
            q.put(full.cpu())
    finally:
        dist.destroy_process_group()


def test_two_gpu_row_sharded_spmm():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import oracle
    import workloads
    from helpers import assert_close

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    full = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = workloads.make(2, scale=0.02, device="cuda:0")
    ref = oracle.spmm_csr_f64(w.rowptr.cpu(), w.col.cpu(), w.val.cpu(), w.B.cpu())
    assert_close(full, ref, torch.float16, "2-GPU sharded")


def _leaving_rank(rank, world, port, q):
    """Two NCCL ranks on a non-blocking communicator: a bounded all-gather at
    step 0, then rank 1 leaves between steps (no kernel or collective in
    flight) and rank 0 learns it from the store before step 1's launch."""
    import sys
    from datetime import timedelta
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for p in (root / "ascend-spmm_b200", root, root / "oracle", root / "tests"):
        sys.path.insert(0, str(p))
    import torch.distributed as dist

    import workloads
    from spmm_dist import Membership, RankDeparted, nccl_options, spmm_csr_sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=30),
                            device_id=torch.device("cuda", rank), pg_options=nccl_options(nonblocking=True))
    members = Membership.for_default_group(timeout_s=30.0)
    try:
        w = workloads.make(2, scale=0.02, device=f"cuda:{rank}")
        full, _ = spmm_csr_sharded(w.rowptr, w.col, w.val, w.B, rank, world, gather=True, members=members,
                                   step=0, timeout_s=30.0)
        torch.cuda.synchronize()
        if rank == 1:
            members.leave("test")
            return
        try:
            spmm_csr_sharded(w.rowptr, w.col, w.val, w.B, rank, world, gather=True, members=members, step=1,
                             timeout_s=30.0)
            q.put("entered")
        except RankDeparted as exc:
            q.put(exc.ranks)
    finally:
        dist.destroy_process_group()


def test_two_gpu_departed_rank_is_seen_on_the_host():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_leaving_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got == [1]
