"""Host side of the Table 6 task-mapping helpers (ascend-spmm_b200/task_mapping.py):
partitioners against the NumPy restatement of the reference
(tests/task_mapping/common.py:146-283), payload files, dataset discovery.
The partitioners are device-agnostic tensor code; here they run on CPU
tensors."""

import numpy as np
import pytest
import torch

import oracle
import task_mapping as tm
import workloads
from helpers import rand_csr


@pytest.mark.parametrize("rows,cols,nnz,expect", [
    (0, 10, 0, 32),
    (1000, 1000, 100, 4),              # sparsity 1e-4 < 2e-4, alpha 1.0, avg 0.1 -> 4
    (2_000_000, 2_000_000, 64_000_000, int(32 * 1.8)),
    (100, 100, 500, max(4, int(5 * 0.25))),   # sparsity 0.05 > 0.01
    (1000, 1000, 5000, max(4, int(5 * 0.55))),
    (1000, 1000, 50_000, int(50 * 0.25)),      # sparsity 0.05
    (10_000, 10_000, 500_000, int(50 * 0.55)),  # sparsity 0.005
])
def test_neutronsparse_threshold(rows, cols, nnz, expect):
    assert tm.compute_neutronsparse_threshold(rows, cols, nnz) == expect


def _cases():
    w = workloads.make(2, scale=0.004)
    yield "powerlaw", w.M, w.K, w.rowptr.to(torch.int64), w.col.to(torch.int64)
    w = workloads.make(4, scale=0.003)
    yield "cluster", w.M, w.K, w.rowptr, w.col
    crow, col = rand_csr(600, 500, 0.05, seed=4, long_rows={3: 400, 77: 450}, empty_every=9)
    yield "random", 600, 500, crow, col


@pytest.mark.parametrize("sym", [False, True])
def test_neutronsparse_matches_reference_restatement(sym):
    for name, rows, cols, crow, col in _cases():
        vals = torch.arange(col.numel(), dtype=torch.float32)
        cube, vec, meta = tm.neutronsparse_parts(crow, col, vals, rows, cols, sym)
        thr = tm.compute_neutronsparse_threshold(rows, cols, col.numel())
        mask, cc, vc, drows, dcols = oracle.neutronsparse_parts_np(crow, col, rows, cols, sym, thr)
        assert meta["threshold"] == thr and meta["dense_rows"] == drows and meta["dense_columns"] == dcols, name
        assert meta["aic_nnz"] == int(mask.sum()) and meta["aiv_nnz"] == int((~mask).sum())
        ptr = lambda c: np.concatenate([[0], np.cumsum(c)])  # noqa: E731
        assert np.array_equal(cube[0].numpy(), ptr(cc)) and np.array_equal(vec[0].numpy(), ptr(vc)), name
        assert cube[0].dtype == crow.dtype
        assert np.array_equal(cube[1].numpy(), col.numpy()[mask]) and np.array_equal(vec[1].numpy(), col.numpy()[~mask])
        assert np.array_equal(cube[2].numpy(), vals.numpy()[mask]) and np.array_equal(vec[2].numpy(), vals.numpy()[~mask])
        if name == "powerlaw":
            assert meta["aic_nnz"] > 0 and meta["aiv_nnz"] > 0


@pytest.mark.parametrize("fraction", [1.0 / 3.0, 0.0, 1.0, 0.37])
def test_naive_parts(fraction):
    crow, col = rand_csr(300, 200, 0.05, seed=5, empty_every=7)
    vals = torch.arange(col.numel(), dtype=torch.float32)
    cube, vec, meta = tm.naive_parts(crow, col, vals, 300, fraction)
    nnz = col.numel()
    pivot = nnz // 3 if fraction == 1.0 / 3.0 else int(nnz * fraction)
    assert meta["pivot_nnz"] == pivot and meta["aic_nnz"] + meta["aiv_nnz"] == nnz
    assert torch.equal(cube[0], crow.clamp_max(pivot)) and torch.equal(vec[0], (crow - pivot).clamp_min(0))
    assert torch.equal(torch.cat([cube[1], vec[1]]), col) and torch.equal(torch.cat([cube[2], vec[2]]), vals)


def test_prepare_partition_argument_errors():
    crow, col = rand_csr(20, 20, 0.2, seed=1)
    vals = torch.ones(col.numel())
    with pytest.raises(ValueError, match="unknown partition method"):
        tm.prepare_partition("x", 20, 20, crow, col, vals)
    with pytest.raises(ValueError, match="block_ratio must be positive"):
        tm.prepare_partition("naive", 20, 20, crow, col, vals, block_ratio=0)
    with pytest.raises(ValueError, match="naive_fraction must be in"):
        tm.prepare_partition("naive", 20, 20, crow, col, vals, naive_fraction=1.5)


def test_payload_roundtrip_and_checks(tmp_path):
    crow, col = rand_csr(50, 40, 0.1, seed=2)
    p = tmp_path / "sub" / "mat_csr.pt"
    tm.save_payload(p, "", 50, 40, crow, col)
    name, rows, cols, c2, k2 = tm.load_payload(p)
    assert (name, rows, cols) == ("mat", 50, 40)
    assert c2.dtype == torch.int64 and torch.equal(c2, crow.to(torch.int64)) and torch.equal(k2, col.to(torch.int64))

    def bad(payload, msg):
        q = tmp_path / "bad.pt"
        torch.save(payload, q)
        with pytest.raises(ValueError, match=msg):
            tm.load_payload(q)

    ok = {"shape": (50, 40), "crow_indices": crow.to(torch.int64), "col_indices": col.to(torch.int64)}
    bad({"shape": (50, 40)}, r"payload lacks field\(s\): col_indices, crow_indices")
    bad({**ok, "shape": (0, 40)}, "matrix shape must be positive")
    bad({**ok, "crow_indices": crow[:-1].to(torch.int64)}, "crow_indices needs rows \\+ 1")
    bad({**ok, "col_indices": col[:-1].to(torch.int64)}, "crow_indices must run from 0")
    c3 = crow.to(torch.int64).clone()
    a10, a11 = int(c3[10]), int(c3[11])
    c3[10], c3[11] = a11 + 1, a10
    bad({**ok, "crow_indices": c3}, "decreases|must run from 0")
    k3 = col.to(torch.int64).clone()
    k3[0] = 40
    bad({**ok, "col_indices": k3}, "col_indices must lie in")
    bad({**ok, "nnz": col.numel() + 1}, "declares nnz")
    bad({"shape": (3, 3), "crow_indices": torch.zeros(4, dtype=torch.int64),
         "col_indices": torch.zeros(0, dtype=torch.int64)}, "no stored entries")


def test_convert_matrix_market(tmp_path):
    import scipy.io
    import scipy.sparse as sp

    rows = np.array([0, 0, 2, 1, 0, 2])
    cols = np.array([3, 1, 0, 2, 3, 2])
    vals = np.array([1.0, 2.0, 0.0, 4.0, 5.0, 6.0])        # (0,3) twice: summed; (2,0) = 0: dropped
    src = tmp_path / "m" / "m.mtx"
    src.parent.mkdir()
    scipy.io.mmwrite(str(src), sp.coo_matrix((vals, (rows, cols)), shape=(3, 4)))
    r, c, nnz = tm.convert_matrix(src, tmp_path / "out" / "m_csr.pt")
    assert (r, c, nnz) == (3, 4, 4)
    name, rows_, cols_, crow, col = tm.load_payload(tmp_path / "out" / "m_csr.pt")
    assert name == "m" and crow.tolist() == [0, 2, 3, 4] and col.tolist() == [1, 3, 2, 2]


def test_discover_and_seed(tmp_path):
    crow, col = rand_csr(10, 10, 0.3, seed=3)
    for rel in ("b/b.pt", "a/a.pt", "a/other.pt"):
        tm.save_payload(tmp_path / rel, rel, 10, 10, crow, col)
    names = [p.relative_to(tmp_path).as_posix() for p in tm.discover_datasets(tmp_path)]
    assert names == ["a/a.pt", "a/other.pt", "b/b.pt"]
    assert [p.name for p in tm.discover_datasets(tmp_path, name="a")] == ["a.pt", "other.pt"]
    assert tm.discover_datasets(tmp_path, index=2)[0].name == "b.pt"
    assert len(tm.discover_datasets(tmp_path, start=1, limit=1)) == 1
    with pytest.raises(ValueError, match="is not among"):
        tm.discover_datasets(tmp_path, index=3)
    with pytest.raises(ValueError, match="no .pt datasets selected"):
        tm.discover_datasets(tmp_path, name="zzz")
    assert tm.stable_seed(2027, "a/a.pt") == tm.stable_seed(2027, "a/a.pt") != tm.stable_seed(2027, "b/b.pt")
    import hashlib

    salt = int.from_bytes(hashlib.sha256(b"a/a.pt").digest()[:8], "little")
    assert tm.stable_seed(2027, "a/a.pt") == (2027 + salt) % (2**63 - 1)
    for kw, msg in (({"start": -1}, "start must be"), ({"start": 2, "stop": 1}, "must not be below"),
                    ({"limit": 0}, "limit must be positive")):
        with pytest.raises(ValueError, match=msg):
            tm.discover_datasets(tmp_path, **kw)
    assert [p.name for p in tm.discover_datasets(tmp_path, start=1, stop=3)] == ["other.pt", "b.pt"]
    s = tm.make_start(torch.tensor([0, 5, 5, 9, 20]), 4)
    assert s.dtype == torch.int32 and s.tolist() == oracle.make_start(torch.tensor([0, 5, 5, 9, 20]), 4).tolist()
