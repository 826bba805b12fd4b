"""CPU oracle vs the committed golden fixtures (produced by the reference's
own compiled preprocessing; see tests/golden/make_golden.py)."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from golden.make_golden import CASES, FUNCS, run_funcs

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_case(name):
    z = np.load(GOLDEN / f"{name}.npz")
    idt = torch.int32 if z["crow"].dtype == np.int32 else torch.int64
    crow = torch.from_numpy(z["crow"]).to(idt)
    col = torch.from_numpy(z["col"]).to(idt)
    values = torch.from_numpy(z["values"])
    dense = torch.from_numpy(z["dense"])
    return z, int(z["nrows"]), int(z["ncols"]), crow, col, values, dense


def as_bytes(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy() if t.numel() else np.zeros(0, np.uint8)


def expect_equal(golden: np.ndarray, got: torch.Tensor, key):
    g = torch.from_numpy(np.ascontiguousarray(golden))
    assert got.dtype == g.dtype, (key, got.dtype, g.dtype)
    assert tuple(got.shape) == tuple(g.shape), (key, got.shape, g.shape)
    assert np.array_equal(as_bytes(got), as_bytes(g)), key


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_oracle_layouts_match_golden(name):
    z, nrows, ncols, crow, col, values, _ = load_case(name)
    outs = run_funcs(oracle, nrows, ncols, crow, col, values)
    for fn in FUNCS:
        keys = {k.split("/", 1)[1] for k in z.files if k.startswith(fn + "/")}
        assert keys == set(outs[fn].keys()), (fn, keys ^ set(outs[fn].keys()))
        for k in keys:
            expect_equal(z[f"{fn}/{k}"], outs[fn][k], f"{name}:{fn}/{k}")


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_oracle_spmm_matches_golden(name):
    z, _, _, crow, col, values, dense = load_case(name)
    y = oracle.spmm_csr_f64(crow, col, values, dense)
    np.testing.assert_allclose(y, z["spmm_f64"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_oracle_mixed_semantics_reproduce_product(name):
    """Every layout, fed to the mixed-operator semantics, reproduces A @ B
    (preprocess in packed row order)."""
    z, nrows, ncols, crow, col, values, dense = load_case(name)
    ref = z["spmm_f64"]
    for fn in ("block_level_split", "preprocess", "preprocess_graph"):
        m = {k.split("/", 1)[1]: torch.from_numpy(np.ascontiguousarray(z[k]))
             for k in z.files if k.startswith(fn + "/")}
        y = oracle.spmm_mixed_f64(m["crow_window_ptr"], m["unique_col_ids"], m["value"],
                                  m["vrow_window_ptr"], m["vcol_indices"], m["vvalue"], dense)
        if fn.startswith("preprocess"):
            perm = m["permutation"].numpy()
            keep = perm >= 0
            np.testing.assert_allclose(y[: perm.size][keep], ref[perm[keep]], rtol=1e-9, atol=1e-9)
        else:
            np.testing.assert_allclose(y[:nrows], ref, rtol=1e-9, atol=1e-9)
    bc = {k.split("/", 1)[1]: torch.from_numpy(np.ascontiguousarray(z[k]))
          for k in z.files if k.startswith("csr_to_bcsr/")}
    empty_i = torch.zeros(1, dtype=torch.int64)
    y = oracle.spmm_mixed_f64(bc["crow_window_ptr"], bc["unique_col_ids"], bc["value"],
                              empty_i, torch.zeros(0, dtype=torch.int64),
                              torch.zeros(0, dtype=values.dtype), dense)
    np.testing.assert_allclose(y[:nrows], ref, rtol=1e-9, atol=1e-9)


def test_oracle_graph_layout_identity():
    """(P A P^T)(P B) = P (A B) for the relabelled forward layout, and the
    fixed-layout transpose reproduces P A^T P^T."""
    z, nrows, ncols, crow, col, values, dense = load_case("graph_i32_f16")
    m = {k.split("/", 1)[1]: torch.from_numpy(np.ascontiguousarray(z[k]))
         for k in z.files if k.startswith("preprocess_graph/")}
    prow = int(m["packed_rows"][0])
    inv = m["inv_permutation"].numpy()
    perm = m["permutation"].numpy()
    Bp = np.zeros((prow, dense.shape[1]))
    Bp[inv] = dense.double().numpy()
    y = oracle.spmm_mixed_f64(m["crow_window_ptr"], m["renumbered_unique_col_ids"], m["value"],
                              m["vrow_window_ptr"], m["renumbered_vcol_indices"], m["vvalue"], Bp)
    ref = z["spmm_f64"]
    keep = perm >= 0
    np.testing.assert_allclose(y[:prow][keep], ref[perm[keep]], rtol=1e-9, atol=1e-9)
    # transpose: (P A^T P^T)(P B) = P (A^T B)
    import scipy.sparse as sp
    A = sp.csr_matrix((values.double().numpy(), col.numpy(), crow.numpy()), shape=(nrows, ncols))
    refT = A.T @ dense.double().numpy()
    yt = oracle.spmm_mixed_f64(m["transpose_crow_window_ptr"], m["transpose_unique_col_ids"],
                               m["transpose_value"], m["transpose_vrow_window_ptr"],
                               m["transpose_vcol_indices"], m["transpose_vvalue"], Bp)
    np.testing.assert_allclose(yt[:prow][keep], refT[perm[keep]], rtol=1e-9, atol=1e-9)


def test_oracle_empty_and_edge_inputs():
    crow = torch.zeros(6, dtype=torch.int32)
    col = torch.zeros(0, dtype=torch.int32)
    val = torch.zeros(0, dtype=torch.float16)
    d = oracle.csr_to_bcsr(crow, col, val, 5, 7, 16)
    assert d["crow_window_ptr"].tolist() == [0, 0] and d["unique_col_ids"].numel() == 0
    p = oracle.preprocess(crow, col, val, 5, 7, 16, False)
    assert int(p["packed_rows"][0]) == 5 and p["vrow_window_ptr"].tolist() == [0] * 6
    b = oracle.block_level_split(crow, col, val, 5, 7, 0.5, 16)
    assert b["vrow_window_ptr"].numel() == 17
    with pytest.raises(ValueError):
        oracle.preprocess(crow, col, val, 5, 7, 8, False)
    with pytest.raises(ValueError):
        oracle.csr_to_bcsr(torch.tensor([0, 1], dtype=torch.int32), torch.tensor([9], dtype=torch.int32),
                           torch.ones(1, dtype=torch.float16), 1, 7, 16)
    # a column occupied more than 16 times in the marginal window (duplicate
    # coordinates) makes the bucket sort throw, as in the reference
    crow = torch.tensor([0, 17], dtype=torch.int32)
    col = torch.full((17,), 3, dtype=torch.int32)
    with pytest.raises(ValueError, match="coalesce"):
        oracle.preprocess(crow, col, torch.ones(17, dtype=torch.float16), 1, 5, 16, False)


def test_make_start_matches_reference_rule():
    ptr = torch.tensor([0, 3, 3, 10, 11, 20], dtype=torch.int64)
    s = oracle.make_start(ptr, 4)
    # chunk = 5 -> targets 0,5,10,15 -> rows 0,2,3,4 (searchsorted right - 1)
    assert s.tolist() == [0, 2, 3, 4]
    assert oracle.make_start(torch.zeros(3, dtype=torch.int64), 4).tolist() == [0, 0, 0, 0]


def cube_to_bcsr(rowptr, col, value):
    """(16 x 1)-block layout implied by a spmm_cube window encoding: runs of
    equal column are blocks, the last entry of a row in a run wins."""
    rp, c = rowptr.to(torch.int64).numpy(), col.to(torch.int64).numpy()
    v = value.numpy()
    cptr, ucol, vals = [0], [], []
    for w in range(rp.size - 1):
        last = None
        for p in range(rp[w], rp[w + 1]):
            cc, r = int(c[p]) >> 4, int(c[p]) & 15
            if cc != last:
                ucol.append(cc)
                vals.append(np.zeros(16, v.dtype))
                last = cc
            vals[-1][r] = v[p]
        cptr.append(len(ucol))
    val = np.concatenate(vals) if vals else np.zeros(0, v.dtype)
    return np.array(cptr, np.int64), np.array(ucol, np.int64), val


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_oracle_cube_producer_matches_reference_bcsr(name):
    """Runs of the producer's window encoding are exactly the reference's
    csr_to_bcsr blocks (golden, bit-exact), and the encoding keeps every
    entry."""
    z, nrows, ncols, crow, col, values, _ = load_case(name)
    cube = oracle.csr_to_spmm_cube(crow, col, values, nrows, ncols, 16)
    assert cube["rowptr"].dtype == crow.dtype and cube["col"].dtype == crow.dtype
    assert cube["value"].dtype == values.dtype
    assert cube["col"].numel() == col.numel()
    nwin = (nrows + 15) // 16
    assert torch.equal(cube["rowptr"].to(torch.int64),
                       crow.to(torch.int64)[torch.clamp(torch.arange(nwin + 1) * 16, max=nrows)])
    cptr, ucol, val = cube_to_bcsr(cube["rowptr"], cube["col"], cube["value"])
    assert np.array_equal(cptr, z["csr_to_bcsr/crow_window_ptr"].astype(np.int64))
    assert np.array_equal(ucol, z["csr_to_bcsr/unique_col_ids"].astype(np.int64))
    assert np.array_equal(val.view(np.uint8), np.ascontiguousarray(z["csr_to_bcsr/value"]).view(np.uint8))


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_oracle_cube_semantics_reproduce_product(name):
    z, nrows, ncols, crow, col, values, dense = load_case(name)
    cube = oracle.csr_to_spmm_cube(crow, col, values, nrows, ncols, 16)
    y = oracle.spmm_cube_f64(cube["rowptr"], cube["col"], cube["value"], dense)
    assert y.shape == (16 * ((nrows + 15) // 16), dense.shape[1])
    np.testing.assert_allclose(y[:nrows], z["spmm_f64"], rtol=1e-9, atol=1e-9)
    assert not y[nrows:].any()


def test_oracle_cube_runs_and_last_write():
    """Hand-made window: a column that reappears after another column opens
    a second block; a repeated row inside one run keeps the last value."""
    B = torch.arange(4 * 16, dtype=torch.float64).reshape(4, 16) + 1
    enc = lambda c, r: (c << 4) | r
    rowptr = torch.tensor([0, 5, 5, 6])
    col = torch.tensor([enc(1, 0), enc(1, 3), enc(1, 0), enc(2, 0), enc(1, 0), enc(3, 15)])
    val = torch.tensor([5.0, 2.0, 7.0, 1.0, 3.0, 4.0])
    y = oracle.spmm_cube_f64(rowptr, col, val, B)
    want = np.zeros((48, 16))
    want[0] = 7.0 * B[1] + 1.0 * B[2] + 3.0 * B[1]   # 5.0 overwritten by 7.0
    want[3] = 2.0 * B[1]
    want[32 + 15] = 4.0 * B[3]
    np.testing.assert_array_equal(y, want)


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_oracle_tile_semantics_reproduce_product(name):
    """The reference's own csr_to_ascend_cube tiles (golden fixtures), read
    as value[256 t + 16 r + k] x B[unique_col_ids[16 t + k]], give A @ B:
    the semantics the tile consumer implements."""
    z, nrows, _, _, _, _, dense = load_case(name)
    t = {k.split("/", 1)[1]: torch.from_numpy(np.ascontiguousarray(z[k]))
         for k in z.files if k.startswith("csr_to_ascend_cube/")}
    y = oracle.spmm_ascend_cube_tiles_f64(t["crow_window_ptr"], t["unique_col_ids"], t["value"], dense)
    assert y.shape == (16 * ((nrows + 15) // 16), dense.shape[1])
    np.testing.assert_allclose(y[:nrows], z["spmm_f64"], rtol=1e-9, atol=1e-9)
    assert not y[nrows:].any()
