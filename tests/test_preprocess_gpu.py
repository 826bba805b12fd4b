"""GPU layout builders are bit-exact with the reference.

* against the golden fixtures (outputs of the reference's own compiled
  preprocessing, tests/golden/make_golden.py);
* against the CPU oracle (pinned to the reference by tests/test_oracle_pin.py)
  on random and BASELINE-config-shaped matrices, including the full-size
  config 2 matrix;
* error behaviour of the reference (column range, occupancy, window size)
  plus this engine's sortedness check for the merge-order builders.
"""

import numpy as np
import pytest
import torch

import oracle
import workloads
from golden.make_golden import CASES, FUNCS
from helpers import assert_close, load_golden, rand_csr

pytestmark = pytest.mark.gpu
DEV = "cuda"
BLOCK_RATIO = (222.0 / 190.0) * 0.5


@pytest.fixture(scope="module")
def npu():
    import build

    build.build()
    import spmm_npu

    return spmm_npu


def as_bytes(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    return t.view(torch.uint8).numpy() if t.numel() else np.zeros(0, np.uint8)


def same_dict(got: dict, exp: dict, what=""):
    assert set(got) == set(exp), (what, set(got) ^ set(exp))
    for k in exp:
        g, e = got[k], exp[k]
        if not isinstance(e, torch.Tensor):
            e = torch.from_numpy(np.ascontiguousarray(e))
        assert g.is_cuda, (what, k)
        assert g.dtype == e.dtype, (what, k, g.dtype, e.dtype)
        assert tuple(g.shape) == tuple(e.shape), (what, k, tuple(g.shape), tuple(e.shape))
        assert np.array_equal(as_bytes(g), as_bytes(e)), (what, k)


def gpu_funcs(npu, nrows, ncols, crow, col, values):
    c, k, v = crow.to(DEV), col.to(DEV), values.to(DEV)
    return {
        "csr_to_bcsr": npu.csr_to_bcsr(c, k, v, nrows, ncols, 16),
        "csr_to_ascend_cube": npu.csr_to_ascend_cube(c, k, v, nrows, ncols, 16),
        "block_level_split": npu.block_level_split(c, k, v, nrows, ncols, BLOCK_RATIO, 16),
        "preprocess": npu.preprocess(c, k, v, nrows, ncols, 16, False),
        "preprocess_graph": npu.preprocess(c, k, v, nrows, ncols, 16, True),
    }


def oracle_funcs(nrows, ncols, crow, col, values, sorted_rows=True):
    out = {
        "block_level_split": oracle.block_level_split(crow, col, values, nrows, ncols, BLOCK_RATIO, 16),
        "preprocess": oracle.preprocess(crow, col, values, nrows, ncols, 16, False),
        "preprocess_graph": oracle.preprocess(crow, col, values, nrows, ncols, 16, True),
    }
    if sorted_rows:
        out["csr_to_bcsr"] = oracle.csr_to_bcsr(crow, col, values, nrows, ncols, 16)
        out["csr_to_ascend_cube"] = oracle.csr_to_ascend_cube(crow, col, values, nrows, ncols, 16)
    return out


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_layouts_match_reference_golden(npu, name):
    c = load_golden(name)
    got = gpu_funcs(npu, c["nrows"], c["ncols"], c["crow"], c["col"], c["values"])
    z = c["z"]
    for fn in FUNCS:
        exp = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(fn + "/")}
        same_dict(got[fn], exp, f"{name}:{fn}")


@pytest.mark.parametrize("seed", range(10))
def test_layouts_match_oracle_random(npu, seed):
    g = np.random.default_rng(seed)
    nrows = int(g.integers(1, 300))
    ncols = nrows if seed % 2 == 0 else int(g.integers(1, 300))
    idt = torch.int32 if seed % 3 else torch.int64
    vdt = (torch.float16, torch.float32, torch.float64)[seed % 3]
    long_rows = {int(g.integers(0, nrows)): int(g.integers(0, ncols + 1))}
    crow, col = rand_csr(nrows, ncols, float(g.uniform(0, 0.2)), seed=seed, long_rows=long_rows,
                         empty_every=int(g.integers(0, 6)), idt=idt)
    vals = (torch.rand(col.numel(), generator=torch.Generator().manual_seed(seed)) * 2 - 1).to(vdt)
    got = gpu_funcs(npu, nrows, ncols, crow, col, vals)
    exp = oracle_funcs(nrows, ncols, crow, col, vals)
    for fn in exp:
        same_dict(got[fn], exp[fn], f"seed{seed}:{fn}")


@pytest.mark.parametrize("cfg,scale", [(1, 0.25), (2, 0.05), (3, 0.03), (4, 0.01), (5, 0.002)])
def test_layouts_match_oracle_configs(npu, cfg, scale):
    w = workloads.make(cfg, scale=scale)
    got = gpu_funcs(npu, w.M, w.K, w.rowptr, w.col, w.val)
    exp = oracle_funcs(w.M, w.K, w.rowptr, w.col, w.val)
    for fn in exp:
        same_dict(got[fn], exp[fn], f"cfg{cfg}:{fn}")


def test_preprocess_full_config2_bit_exact(npu):
    """Full-size config 2 (1M rows, ~16M nonzeros): GPU preprocess equals the
    oracle on every key; the mixed SpMM on that layout matches A @ B on a
    row sample."""
    w = workloads.make(2, device=DEV)
    crow, col, val = w.rowptr.cpu(), w.col.cpu(), w.val.cpu()
    got = npu.preprocess(w.rowptr, w.col, w.val, w.M, w.K, 16, False)
    exp = oracle.preprocess(crow, col, val, w.M, w.K, 16, False)
    same_dict(got, exp, "cfg2 full")
    start = torch.zeros(40, dtype=torch.int32, device=DEV)
    y = npu.spmm_ascend_cube(got["crow_window_ptr"], got["unique_col_ids"], got["value"], got["vrow_window_ptr"],
                             got["vcol_indices"], got["vvalue"], w.B, start[:20], start)
    rows = torch.randperm(w.M, generator=torch.Generator().manual_seed(0))[:512]
    packed = got["inv_permutation"].cpu()[rows]
    rp, cc, vv = [], [], []
    for r in rows.tolist():
        a, b = int(crow[r]), int(crow[r + 1])
        rp.append(b - a)
        cc.append(col[a:b])
        vv.append(val[a:b])
    sub_ptr = torch.zeros(len(rp) + 1, dtype=torch.int64)
    sub_ptr[1:] = torch.cumsum(torch.tensor(rp), 0)
    ref = oracle.spmm_csr_f64(sub_ptr, torch.cat(cc), torch.cat(vv), w.B.cpu())
    assert_close(y[packed.to(DEV)], ref, torch.float16, "cfg2 mixed sample")


def test_unsorted_rows(npu):
    """block_level_split and preprocess accept unsorted rows (the graph
    transpose feeds them unsorted rows too); the merge-order builders reject
    them instead of reproducing a merge of unsorted lists."""
    g = np.random.default_rng(7)
    nrows = ncols = 120
    crow, col = rand_csr(nrows, ncols, 0.1, seed=7)
    perm_col = col.clone()
    for r in range(nrows):
        a, b = int(crow[r]), int(crow[r + 1])
        perm_col[a:b] = col[a:b][torch.from_numpy(g.permutation(b - a))]
    vals = torch.rand(col.numel()).half()
    got_b = npu.block_level_split(crow.to(DEV), perm_col.to(DEV), vals.to(DEV), nrows, ncols, 0.6, 16)
    same_dict(got_b, oracle.block_level_split(crow, perm_col, vals, nrows, ncols, 0.6, 16), "bls unsorted")
    for gl in (False, True):
        got_p = npu.preprocess(crow.to(DEV), perm_col.to(DEV), vals.to(DEV), nrows, ncols, 16, gl)
        same_dict(got_p, oracle.preprocess(crow, perm_col, vals, nrows, ncols, 16, gl), "pre unsorted")
    with pytest.raises(RuntimeError, match="sorted in ascending order"):
        npu.csr_to_bcsr(crow.to(DEV), perm_col.to(DEV), vals.to(DEV), nrows, ncols, 16)


def test_edge_inputs(npu):
    # empty matrix (the reference dereferences an empty column array here)
    crow = torch.zeros(6, dtype=torch.int32)
    col = torch.zeros(0, dtype=torch.int32)
    val = torch.zeros(0, dtype=torch.float16)
    got = gpu_funcs(npu, 5, 7, crow, col, val)
    exp = oracle_funcs(5, 7, crow, col, val)
    for fn in exp:
        same_dict(got[fn], exp[fn], f"empty:{fn}")
    # CPU inputs are accepted and produce CUDA outputs
    c = load_golden("ragged_i32_f32")
    d = npu.preprocess(c["crow"], c["col"], c["values"], c["nrows"], c["ncols"])
    assert d["permutation"].is_cuda


def test_error_behaviour(npu):
    crow = torch.tensor([0, 2, 3], dtype=torch.int32, device=DEV)
    col = torch.tensor([1, 9, 0], dtype=torch.int32, device=DEV)
    val = torch.ones(3, dtype=torch.float16, device=DEV)
    with pytest.raises(RuntimeError, match="column index out of range"):
        npu.preprocess(crow, col, val, 2, 5, 16, False)
    with pytest.raises(RuntimeError, match="requires a 16-row window"):
        npu.preprocess(crow, col.clamp(max=4), val, 2, 5, 8, False)
    # a column occupied 17 times in the marginal window -> ValueError, as the
    # reference's bucket sort throws std::invalid_argument
    crow = torch.tensor([0, 17], dtype=torch.int32, device=DEV)
    col = torch.full((17,), 3, dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError, match="coalesce duplicate CSR entries"):
        npu.preprocess(crow, col, torch.ones(17, dtype=torch.float16, device=DEV), 1, 5, 16, False)
    with pytest.raises(RuntimeError, match="int32 or int64"):
        npu.csr_to_bcsr(crow.short(), col.short(), torch.ones(17, dtype=torch.float16, device=DEV), 1, 5, 16)


def test_gpu_layouts_drive_spmm(npu):
    """End to end on the device: GPU preprocess -> spmm_ascend_cube ->
    restore_node_tensor reproduces A @ B; block_level_split and csr_to_bcsr
    layouts likewise."""
    w = workloads.make(3, scale=0.02, device=DEV)
    ref = oracle.spmm_csr_f64(w.rowptr, w.col, w.val, w.B)
    s = torch.zeros(40, dtype=torch.int32, device=DEV)
    m = npu.preprocess(w.rowptr, w.col, w.val, w.M, w.K)
    y = npu.spmm_ascend_cube(m["crow_window_ptr"], m["unique_col_ids"], m["value"], m["vrow_window_ptr"],
                             m["vcol_indices"], m["vvalue"], w.B, s[:20], s)
    assert_close(npu.restore_node_tensor(y, m["inv_permutation"]), ref, torch.float16, "preprocess")
    b = npu.block_level_split(w.rowptr, w.col, w.val, w.M, w.K, BLOCK_RATIO)
    y = npu.spmm_ascend_cube(b["crow_window_ptr"], b["unique_col_ids"], b["value"], b["vrow_window_ptr"],
                             b["vcol_indices"], b["vvalue"], w.B, s[:20], s)
    assert_close(y[: w.M], ref, torch.float16, "block_level_split")
    bc = npu.csr_to_bcsr(w.rowptr, w.col, w.val, w.M, w.K)
    z = torch.zeros(1, dtype=torch.int32, device=DEV)
    y = npu.spmm_ascend_cube(bc["crow_window_ptr"], bc["unique_col_ids"], bc["value"], z, z[:0], w.val[:0], w.B,
                             s[:20], s)
    assert_close(y[: w.M], ref, torch.float16, "csr_to_bcsr")
    code, detail = npu.device_status(True)
    assert code == 0, (code, detail)


@pytest.mark.parametrize("cfg,scale", [(1, 1.0), (2, 0.05), (3, 0.05), (4, 0.02)])
def test_layouts_match_compiled_reference(npu, cfg, scale):
    """GPU layouts against the reference's own compiled CPU preprocessing
    (oracle/_ref, built from the reference tree) on config 1 at full size,
    config 2 at scale 0.05, config 3 at scale 0.05 and config 4 (fp32) at
    scale 0.02, graph layout included."""
    import contextlib
    import io

    import build_ref

    ref = build_ref.load()
    if ref is None:
        pytest.skip("the compiled reference preprocessing (oracle/_ref) is not on this machine")
    w = workloads.make(cfg, scale=scale)
    got = gpu_funcs(npu, w.M, w.K, w.rowptr, w.col, w.val)
    with contextlib.redirect_stdout(io.StringIO()):
        exp = {
            "csr_to_bcsr": ref.csr_to_bcsr(w.rowptr, w.col, w.val, w.M, w.K, 16),
            "csr_to_ascend_cube": ref.csr_to_ascend_cube(w.rowptr, w.col, w.val, w.M, w.K, 16),
            "block_level_split": ref.block_level_split(w.rowptr, w.col, w.val, w.M, w.K, BLOCK_RATIO, 16),
            "preprocess": ref.preprocess(w.rowptr, w.col, w.val, w.M, w.K, 16, False),
            "preprocess_graph": ref.preprocess(w.rowptr, w.col, w.val, w.M, w.K, 16, True),
        }
    for fn in exp:
        same_dict(got[fn], exp[fn], f"cfg{cfg}:{fn} vs compiled reference")
