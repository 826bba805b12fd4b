"""Row-sharded SpMM on 2 GPUs (NCCL): every rank computes its shard with the
engine's CSR operator, and with the mixed operator on a layout built from
its own rows (ShardedMixed), the all-gather assembles C, and both results
match the float64 oracle.  Runs as child processes; skipped with fewer than
2 GPUs."""

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
    from spmm_dist import ShardedMixed, spmm_csr_sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = workloads.make(2, scale=0.02, device=f"cuda:{rank}")
        full, _ = spmm_csr_sharded(w.rowptr, w.col, w.val, w.B, rank, world, gather=True)
        mixed, rows = ShardedMixed(w.rowptr, w.col, w.val, w.K, rank, world)(w.B, gather=True, timeout_s=60.0)
        torch.cuda.synchronize()
        assert rows == (0, w.M)
        if rank == 0:
            q.put((full.cpu(), mixed.cpu()))
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
    full, mixed = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = workloads.make(2, scale=0.02, device="cuda:0")
    ref = oracle.spmm_csr_f64(w.rowptr.cpu(), w.col.cpu(), w.val.cpu(), w.B.cpu())
    assert_close(full, ref, torch.float16, "2-GPU sharded")
    assert_close(mixed, ref, torch.float16, "2-GPU sharded mixed (per-shard task mapping)")


def _multicast_rank(rank, world, port, q):
    """The fused path: rows stored through the NVLink multicast address of a
    symmetric-memory replica of C; every rank's copy must equal the NCCL
    all-gather of the same shards, bit for bit, over two steps."""
    import sys
    from datetime import timedelta
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for p in (root / "ascend-spmm_b200", root, root / "oracle", root / "tests"):
        sys.path.insert(0, str(p))
    import torch.distributed as dist

    import workloads
    from spmm_dist import MulticastRows, spmm_csr_sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = workloads.make(2, scale=0.02, device=f"cuda:{rank}")
        M = w.rowptr.numel() - 1
        try:
            rep = MulticastRows(M, w.B.shape[1], w.B.dtype, torch.device("cuda", rank))
        except RuntimeError as e:
            q.put(("skip", rank, str(e)))
            return
        ref, _ = spmm_csr_sharded(w.rowptr, w.col, w.val, w.B, rank, world, gather=True)
        outs = []
        for step in range(2):
            B = w.B if step == 0 else (w.B * 0.5)
            full, rows = spmm_csr_sharded(w.rowptr, w.col, w.val, B, rank, world, gather=True, replica=rep,
                                          timeout_s=60.0)
            torch.cuda.synchronize()
            assert rows == (0, M)
            outs.append(full.clone())
        ref2, _ = spmm_csr_sharded(w.rowptr, w.col, w.val, w.B * 0.5, rank, world, gather=True)
        torch.cuda.synchronize()
        q.put(("ok", rank, bool(torch.equal(outs[0], ref)), bool(torch.equal(outs[1], ref2)), outs[0].cpu()))
        torch.cuda.synchronize()
        dist.barrier()          # no rank writes the replicas any more
        rep.close()
        del outs
        torch.cuda.synchronize()
        dist.barrier()          # every rank has dropped its copy
    finally:
        dist.destroy_process_group()


def test_two_gpu_multicast_rows_fused_gather():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import oracle
    import workloads
    from helpers import assert_close

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_multicast_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    if any(g[0] == "skip" for g in got):
        pytest.skip(next(g for g in got if g[0] == "skip")[2])
    for g in got:
        assert g[2] and g[3], f"rank {g[1]}: multicast rows differ from the NCCL all-gather"
    assert torch.equal(got[0][4], got[1][4]), "the two GPUs' copies differ"
    w = workloads.make(2, scale=0.02, device="cuda:0")
    ref = oracle.spmm_csr_f64(w.rowptr.cpu(), w.col.cpu(), w.val.cpu(), w.B.cpu())
    assert_close(got[0][4], ref, torch.float16, "2-GPU multicast rows")


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
