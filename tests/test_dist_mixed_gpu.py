"""The row-sharded mixed operator (spmm_dist.ShardedMixed) on one GPU: each
rank's object is built as that rank would build it (task mapping on its own
row slice only) and run here one after another, so the shards of every rank
of a 1-, 2- and 3-rank job are checked against the float64 oracle, and
together they must give the whole product.  The collective path (gather=True)
runs on 2 GPUs in test_dist_gpu.py."""

import pytest
import torch

import oracle
import workloads
from helpers import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg,scale", [(2, 0.02), (3, 0.02), (4, 0.004)])
@pytest.mark.parametrize("world", [1, 2, 3])
def test_sharded_mixed_matches_oracle(cfg, scale, world):
    from spmm_dist import ShardedMixed

    w = workloads.make(cfg, scale=scale, device="cpu")
    ref = oracle.spmm_csr_f64(w.rowptr, w.col, w.val, w.B)
    B = w.B.cuda()
    pieces = []
    for rank in range(world):
        sm = ShardedMixed(w.rowptr, w.col, w.val, w.K, rank, world)
        rows, (r0, r1) = sm(B)
        assert rows.shape == (r1 - r0, w.N) and rows.dtype == w.dtype
        if r1 > r0:
            # the layout covers this shard only
            assert sm.inv_permutation.numel() == r1 - r0
        assert_close(rows.cpu(), ref[r0:r1], w.dtype, f"cfg{cfg} rank {rank}/{world}")
        pieces.append((r0, rows.cpu()))
    bounds = [p[0] for p in pieces]
    assert bounds == sorted(bounds) and bounds[0] == 0
    full = torch.cat([p[1] for p in pieces])
    assert full.shape[0] == w.M
    assert_close(full, ref, w.dtype, f"cfg{cfg} world {world} assembled")


def test_sharded_mixed_more_ranks_than_windows():
    from spmm_dist import ShardedMixed

    w = workloads.make(1, scale=0.002, device="cpu")   # 32 rows: 2 windows
    ref = oracle.spmm_csr_f64(w.rowptr, w.col, w.val, w.B)
    B = w.B.cuda()
    got = []
    for rank in range(4):
        rows, (r0, r1) = ShardedMixed(w.rowptr, w.col, w.val, w.K, rank, 4)(B)
        assert rows.shape[0] == r1 - r0
        got.append(rows.cpu())
    assert sum(g.shape[0] for g in got) == w.M
    assert_close(torch.cat(got), ref, w.dtype, "more ranks than windows")
