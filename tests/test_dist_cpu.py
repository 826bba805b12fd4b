"""Multi-rank host logic on CPU (gloo, world_size 2): row partition, shard
slicing, the all-gather of row-sharded C and the sharded mixed operator.  The per-rank product is the
float64 oracle here (no GPU); the GPU path is the same code with
spmm_npu.spmm_csr as the local operator."""

import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
import workloads
from spmm_dist import allgather_rows, shard_bounds, shard_csr


def test_shard_bounds_balanced_and_window_aligned():
    w = workloads.make(2, scale=0.02)
    for world in (1, 2, 3, 4, 8):
        b = shard_bounds(w.rowptr, world)
        assert len(b) == world and b[0][0] == 0 and b[-1][1] == w.M
        for (a0, a1), (c0, c1) in zip(b, b[1:]):
            assert a1 == c0
        for r0, r1 in b:
            assert r0 % 16 == 0 and r0 <= r1
        nz = [int(w.rowptr[r1]) - int(w.rowptr[r0]) for r0, r1 in b]
        assert sum(nz) == w.nnz
        # balance within one window's worth of nonzeros plus the largest row
        deg = (w.rowptr[1:] - w.rowptr[:-1]).to(torch.int64)
        slack = int(deg.max()) * 16
        assert max(nz) - w.nnz / world <= slack


def test_shard_bounds_degenerate():
    rp = torch.tensor([0, 2, 2, 5], dtype=torch.int32)
    assert shard_bounds(rp, 4) == [(0, 3), (3, 3), (3, 3), (3, 3)]
    assert shard_bounds(torch.zeros(1, dtype=torch.int32), 2) == [(0, 0), (0, 0)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = workloads.make(3, scale=0.01)
        bounds = shard_bounds(w.rowptr, world)
        r0, r1 = bounds[rank]
        rp, c, v = shard_csr(w.rowptr, w.col, w.val, r0, r1)
        local = torch.from_numpy(oracle.spmm_csr_f64(rp, c, v, w.B))
        results[rank] = allgather_rows(local, bounds).numpy()           # uneven shards: broadcasts
        half = w.M // 2 // 16 * 16
        even = [(0, half), (half, 2 * half)]
        rp, c, v = shard_csr(w.rowptr, w.col, w.val, *even[rank])
        local = torch.from_numpy(oracle.spmm_csr_f64(rp, c, v, w.B))
        results[("even", rank)] = allgather_rows(local, even).numpy()   # equal shards: all-gather
    finally:
        dist.destroy_process_group()


def test_allgather_reassembles_full_product():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        w = workloads.make(3, scale=0.01)
        ref = oracle.spmm_csr_f64(w.rowptr, w.col, w.val, w.B)
        half = w.M // 2 // 16 * 16
        assert shard_bounds(w.rowptr, world)[0][1] != half   # the first case really is uneven
        for r in range(world):
            np.testing.assert_allclose(results[r], ref, rtol=0, atol=0)
            np.testing.assert_allclose(results[("even", r)], ref[: 2 * half], rtol=0, atol=0)


def _mixed_worker(rank, world, port, results):
    """ShardedMixed's host logic on gloo: the device operators are replaced
    by the CPU oracle (layout builder, mixed product) and an index gather
    (row restore), so sharding, per-shard layouts, the restore to original
    order and the all-gather are what runs."""
    import torch.distributed as dist

    import spmm_npu
    from spmm_dist import ShardedMixed

    spmm_npu.preprocess = oracle.preprocess
    spmm_npu.spmm_ascend_cube = lambda *a: torch.from_numpy(oracle.spmm_mixed_f64(*a[:7]))
    spmm_npu.restore_node_tensor = lambda packed, inv: packed[inv.to(torch.long)]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = workloads.make(3, scale=0.01)
        op = ShardedMixed(w.rowptr, w.col, w.val, w.K, rank, world, device="cpu")
        local, rows = op(w.B)
        results[("local", rank)] = (rows, local.numpy())
        full, rows = op(w.B, gather=True)
        results[("full", rank)] = (rows, full.numpy())
        results[("windows", rank)] = int(op.layout[0].numel() - 1)
    finally:
        dist.destroy_process_group()


def test_sharded_mixed_host_logic_two_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_mixed_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=180)
            assert p.exitcode == 0
        w = workloads.make(3, scale=0.01)
        ref = oracle.spmm_csr_f64(w.rowptr, w.col, w.val, w.B)
        bounds = shard_bounds(w.rowptr, world)
        for r in range(world):
            rows, local = results[("local", r)]
            assert rows == bounds[r] and local.shape == (rows[1] - rows[0], w.N)
            np.testing.assert_allclose(local, ref[rows[0]:rows[1]], rtol=1e-12, atol=1e-12)
            rows, full = results[("full", r)]
            assert rows == (0, w.M)
            np.testing.assert_allclose(full, ref, rtol=1e-12, atol=1e-12)
            assert results[("windows", r)] > 0   # each shard has its own window layout


# ---------------------------------------------------------------- failure handling

def _leaver(rank, world, port, results):
    """Step 0 with both ranks; then rank 1 leaves the job and rank 0 must
    learn it on the host before entering step 1's collective."""
    import torch.distributed as dist

    from spmm_dist import Membership, RankDeparted, spmm_csr_sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    members = Membership.for_default_group(timeout_s=20.0)
    w = workloads.make(3, scale=0.01)
    try:
        members.enter(0)
        bounds = shard_bounds(w.rowptr, world)
        rp, c, v = shard_csr(w.rowptr, w.col, w.val, *bounds[rank])
        full = allgather_rows(torch.from_numpy(oracle.spmm_csr_f64(rp, c, v, w.B)), bounds, timeout_s=20.0)
        results[("step0", rank)] = full.shape[0]
        if rank == 1:
            members.leave("test: leaving between steps")
            results[("left", rank)] = True
            return
        t0 = time.monotonic()
        try:
            members.enter(1)
            results[("step1", rank)] = "entered"
        except RankDeparted as exc:
            results[("step1", rank)] = (exc.ranks, exc.step, time.monotonic() - t0)
    finally:
        dist.destroy_process_group()


def _silent(rank, world, port, results):
    """Rank 1 passes the membership check of step 1 and then never joins the
    collective (it stops between steps without telling anyone); rank 0's
    all-gather must end at its deadline with CollectiveTimeout."""
    from datetime import timedelta

    import torch.distributed as dist

    from spmm_dist import CollectiveTimeout, Membership

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    members = Membership.for_default_group(timeout_s=20.0)
    local = torch.full((16, 8), float(rank))
    bounds = [(0, 16), (16, 32)]
    members.enter(0)
    allgather_rows(local, bounds, timeout_s=20.0)
    members.enter(1)
    if rank == 1:
        results["silent"] = True
        time.sleep(4.0)           # gone quiet: no collective
        os._exit(0)               # leaves without destroying the group
    t0 = time.monotonic()
    try:
        allgather_rows(local, bounds, timeout_s=1.5)
        results["timeout"] = "completed"
    except CollectiveTimeout as exc:
        results["timeout"] = (str(exc), time.monotonic() - t0)
    os._exit(0)


def _run(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=target, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=timeout)
            assert p.exitcode == 0, p.exitcode
        return dict(results)


def test_departed_rank_is_seen_before_the_next_collective():
    res = _run(_leaver)
    assert res[("step0", 0)] == res[("step0", 1)] > 0 and res[("left", 1)]
    ranks, step, waited = res[("step1", 0)]
    assert ranks == [1] and step == 1 and waited < 10.0


def test_collective_wait_is_bounded():
    res = _run(_silent)
    assert res["silent"]
    msg, waited = res["timeout"]
    assert "did not complete within 1.5 s" in msg and 1.4 <= waited < 6.0


def test_membership_keys_do_not_accumulate():
    """Each rank removes its step key two steps later (single-process store)."""
    from datetime import timedelta

    import torch.distributed as dist

    from spmm_dist import Membership

    store = dist.HashStore()
    store.set_timeout(timedelta(seconds=5))
    m = Membership(store, rank=0, world=1, timeout_s=1.0)
    for step in range(6):
        m.enter(step)
    assert store.check(["spmm_dist/ready/5/0"]) and store.check(["spmm_dist/ready/4/0"])
    assert not store.check(["spmm_dist/ready/3/0"]) and not store.check(["spmm_dist/ready/0/0"])


def test_multicast_replica_refuses_cleanly_where_unavailable(tmp_path):
    """Where the group cannot hold an NVLink multicast replica (here: CPU
    tensors on a gloo group) MulticastRows raises RuntimeError, the signal
    for callers to take the NCCL all-gather instead; nothing is left bound."""
    import torch.distributed as dist

    from spmm_dist import MulticastRows

    dist.init_process_group("gloo", init_method=f"file://{tmp_path / 'store'}", rank=0, world_size=1)
    try:
        with pytest.raises(RuntimeError, match="replica unavailable|multicast"):
            MulticastRows(32, 16, torch.float16, torch.device("cpu"))
    finally:
        dist.destroy_process_group()
