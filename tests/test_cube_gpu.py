"""GPU parity of ``spmm_cube`` and of its producer ``csr_to_spmm_cube``.

``spmm_cube`` consumes 16-row windows whose entries are encoded as
``(column << 4) | row`` (reference op custom_op.cpp:91-113, kernel
op_kernel/spmm_cube.cpp:51-147): a run of equal columns inside a window is
one (16 x 1) block and the last entry of a row in a run wins.  The oracle
restates that walk in float64 (oracle.spmm_cube_f64); the producer's
encoding must match the oracle's bit for bit (its runs are pinned to the
reference's csr_to_bcsr blocks in tests/test_oracle_golden.py).
"""

import numpy as np
import pytest
import torch

import oracle
import workloads
from golden.make_golden import CASES
from helpers import assert_close, load_golden, rand_csr

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def npu():
    import build

    build.build()
    import spmm_npu

    assert torch.cuda.is_available()
    return spmm_npu


def start_of(ptr, cores=20):
    return oracle.make_start(ptr.cpu().to(torch.int64), cores).to(DEV)


def cube_call(npu, rowptr, col, val, B):
    return npu.spmm_cube(rowptr.to(DEV), col.to(DEV), val.to(DEV), B.to(DEV), start_of(rowptr))


def check_status(npu):
    code, detail = npu.device_status(True)
    assert code == 0, f"device status {code} at {detail}"


def same_bytes(a: torch.Tensor, b: torch.Tensor, what):
    a, b = a.cpu().contiguous(), b.cpu().contiguous()
    assert a.dtype == b.dtype and a.shape == b.shape, (what, a.dtype, b.dtype, a.shape, b.shape)
    assert torch.equal(a.view(torch.uint8) if a.numel() else a, b.view(torch.uint8) if b.numel() else b), what


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_producer_bit_exact_and_product(npu, name):
    c = load_golden(name)
    nrows, ncols = c["nrows"], c["ncols"]
    got = npu.csr_to_spmm_cube(c["crow"].to(DEV), c["col"].to(DEV), c["values"].to(DEV), nrows, ncols, 16)
    want = oracle.csr_to_spmm_cube(c["crow"], c["col"], c["values"], nrows, ncols, 16)
    assert set(got) == {"rowptr", "col", "value"}
    for k in want:
        assert got[k].device.type == "cuda"
        same_bytes(got[k], want[k], f"{name}:{k}")
    y = cube_call(npu, got["rowptr"], got["col"], got["value"], c["dense"])
    torch.cuda.synchronize()
    assert y.shape == (16 * ((nrows + 15) // 16), c["dense"].shape[1]) and y.dtype == c["values"].dtype
    assert_close(y[:nrows], c["z"]["spmm_f64"], y.dtype, name)
    assert not bool(y[nrows:].any())
    check_status(npu)


@pytest.mark.parametrize("dtype,N", [(torch.float16, 16), (torch.float16, 128), (torch.float16, 1024),
                                     (torch.float32, 16), (torch.float32, 256), (torch.float32, 512)])
@pytest.mark.parametrize("idt", [torch.int32, torch.int64])
def test_spmm_cube_random_widths(npu, dtype, N, idt):
    M, K = 517, 389
    crow, col = rand_csr(M, K, 0.04, seed=N + 7, long_rows={3: 300, 250: 389}, empty_every=11, idt=idt)
    g = torch.Generator().manual_seed(N)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
    B = torch.randn(K, N, generator=g).to(dtype)
    enc = npu.csr_to_spmm_cube(crow.to(DEV), col.to(DEV), val.to(DEV), M, K, 16)
    y = cube_call(npu, enc["rowptr"], enc["col"], enc["value"], B)
    assert_close(y[:M], oracle.spmm_csr_f64(crow, col, val, B), dtype, f"{dtype} N={N}")
    check_status(npu)


def test_spmm_cube_runs_duplicates_and_chunks(npu):
    """Arbitrary entry order: columns that reappear open new blocks, repeated
    rows inside one run keep the last value, runs longer than one 128-entry
    chunk, empty windows, and a window whose single run spans three chunks."""
    g = np.random.default_rng(5)
    K, N = 40, 32
    windows = []
    for w in range(9):
        if w % 4 == 1:
            windows.append([])
            continue
        ents = []
        for _ in range(int(g.integers(1, 30))):
            c = int(g.integers(0, K))
            for _ in range(int(g.integers(1, 12))):
                ents.append((c, int(g.integers(0, 16))))
        windows.append(ents)
    windows.append([(7, i % 16) for i in range(300)])          # one long run, many duplicates
    windows.append([(c % 3, (c * 5) % 16) for c in range(200)])  # runs of length 1, reappearing columns
    rowptr = np.zeros(len(windows) + 1, np.int64)
    rowptr[1:] = np.cumsum([len(e) for e in windows])
    col = np.array([(c << 4) | r for e in windows for (c, r) in e], np.int64)
    val = torch.from_numpy(g.uniform(-1, 1, col.size)).to(torch.float16)
    B = torch.randn(K, N, generator=torch.Generator().manual_seed(1)).to(torch.float16)
    for idt in (torch.int32, torch.int64):
        rp, cc = torch.from_numpy(rowptr).to(idt), torch.from_numpy(col).to(idt)
        y = cube_call(npu, rp, cc, val, B)
        assert_close(y, oracle.spmm_cube_f64(rp, cc, val, B), torch.float16, str(idt))
    check_status(npu)


def test_spmm_cube_fp32_tight(npu):
    crow, col = rand_csr(300, 300, 0.1, seed=3)
    val = torch.rand(col.numel(), generator=torch.Generator().manual_seed(3)) * 2 - 1
    B = torch.randn(300, 64, generator=torch.Generator().manual_seed(4))
    enc = npu.csr_to_spmm_cube(crow.to(DEV), col.to(DEV), val.to(DEV), 300, 300)
    y = cube_call(npu, enc["rowptr"], enc["col"], enc["value"], B)
    ref = oracle.spmm_cube_f64(enc["rowptr"], enc["col"], enc["value"], B)
    assert_close(y, ref, torch.float32)
    np.testing.assert_allclose(y.cpu().double().numpy()[:300], oracle.spmm_csr_f64(crow, col, val, B),
                               rtol=1e-4, atol=1e-4)


def test_spmm_cube_config3_sample(npu):
    w = workloads.make(3, scale=0.02)
    enc = npu.csr_to_spmm_cube(w.rowptr.to(DEV), w.col.to(DEV), w.val.to(DEV), w.M, w.K, 16)
    y = cube_call(npu, enc["rowptr"], enc["col"], enc["value"], w.B.to(DEV))
    assert_close(y[: w.M], oracle.spmm_csr_f64(w.rowptr, w.col, w.val, w.B), torch.float16, "cfg3")
    check_status(npu)


def test_spmm_cube_edges(npu):
    B = torch.randn(10, 16).half()
    # no windows
    y = cube_call(npu, torch.zeros(1, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                  torch.zeros(0).half(), B)
    assert y.shape == (0, 16)
    # windows without entries
    y = cube_call(npu, torch.zeros(4, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                  torch.zeros(0).half(), B)
    assert y.shape == (48, 16) and not bool(y.any())
    # producer on an empty matrix and on a matrix with empty rows only
    enc = npu.csr_to_spmm_cube(torch.zeros(21, dtype=torch.int32, device=DEV),
                               torch.zeros(0, dtype=torch.int32, device=DEV), torch.zeros(0, device=DEV).half(),
                               20, 10)
    assert enc["rowptr"].tolist() == [0, 0, 0] and enc["col"].numel() == 0
    check_status(npu)


def test_spmm_cube_contract_errors(npu):
    rp = torch.tensor([0, 1], dtype=torch.int32)
    c = torch.tensor([3 << 4], dtype=torch.int32)
    with pytest.raises(RuntimeError, match="spmm_cube requires feature width divisible by 16, but got 8"):
        cube_call(npu, rp, c, torch.ones(1), torch.randn(5, 8))
    with pytest.raises(RuntimeError, match="col and value must be same size, but got different: -1"):
        cube_call(npu, rp, c, torch.ones(2).half(), torch.randn(5, 16).half())
    with pytest.raises(RuntimeError, match="value must have the same dtype as dense"):
        cube_call(npu, rp, c, torch.ones(1), torch.randn(5, 16).half())
    with pytest.raises(RuntimeError, match="requires 0 < feature width <= 512 for FP32"):
        cube_call(npu, rp, c, torch.ones(1), torch.randn(5, 528))
    with pytest.raises(RuntimeError, match="must be CUDA tensor"):
        npu.spmm_cube(rp, c.to(DEV), torch.ones(1, device=DEV).half(), torch.randn(5, 16, device=DEV).half(),
                      start_of(rp))


def test_spmm_cube_invalid_column_is_reported(npu):
    rp = torch.tensor([0, 2], dtype=torch.int32)
    c = torch.tensor([(1 << 4) | 2, (9 << 4) | 3], dtype=torch.int32)   # column 9 >= K = 5
    B = torch.randn(5, 16).half()
    y = cube_call(npu, rp, c, torch.ones(2).half(), B)
    torch.cuda.synchronize()
    code, _ = npu.device_status(True)
    assert code == 1   # SPMM_DEV_BAD_COLUMN
    assert torch.allclose(y[2].float().cpu(), B[1].float(), atol=1e-3)
    assert not bool(y[3].any())


# ---- spmm_ascend_cube_tiles: consumer of csr_to_ascend_cube's 16 x 16 tiles ----

def tiles_call(npu, t, B):
    return npu.spmm_ascend_cube_tiles(t["crow_window_ptr"].to(DEV), t["unique_col_ids"].to(DEV),
                                      t["value"].to(DEV), B.to(DEV))


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_tiles_on_golden_layouts(npu, name):
    """GPU producer (bit-exact with the golden csr_to_ascend_cube) feeding the
    tile consumer reproduces A @ B and the literal tile semantics."""
    c = load_golden(name)
    nrows, ncols = c["nrows"], c["ncols"]
    t = npu.csr_to_ascend_cube(c["crow"].to(DEV), c["col"].to(DEV), c["values"].to(DEV), nrows, ncols, 16)
    y = tiles_call(npu, t, c["dense"])
    torch.cuda.synchronize()
    assert y.shape == (16 * ((nrows + 15) // 16), c["dense"].shape[1]) and y.dtype == c["values"].dtype
    assert_close(y[:nrows], c["z"]["spmm_f64"], y.dtype, name)
    assert not bool(y[nrows:].any())
    ref = oracle.spmm_ascend_cube_tiles_f64(t["crow_window_ptr"].cpu(), t["unique_col_ids"].cpu(),
                                            t["value"].cpu(), c["dense"])
    assert_close(y, ref, y.dtype, name + " tiles")
    check_status(npu)


@pytest.mark.parametrize("dtype,N", [(torch.float16, 16), (torch.float16, 128), (torch.float16, 1024),
                                     (torch.float32, 16), (torch.float32, 128), (torch.float32, 512)])
@pytest.mark.parametrize("idt", [torch.int32, torch.int64])
def test_tiles_random_widths(npu, dtype, N, idt):
    M, K = 533, 401
    crow, col = rand_csr(M, K, 0.05, seed=N + 11, long_rows={7: 390, 530: 200}, empty_every=13, idt=idt)
    g = torch.Generator().manual_seed(N + 1)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
    B = torch.randn(K, N, generator=g).to(dtype)
    t = npu.csr_to_ascend_cube(crow.to(DEV), col.to(DEV), val.to(DEV), M, K, 16)
    y = tiles_call(npu, t, B)
    assert_close(y[:M], oracle.spmm_csr_f64(crow, col, val, B), dtype, f"{dtype} N={N} {idt}")
    if dtype == torch.float32:
        np.testing.assert_allclose(y.cpu().double().numpy()[:M], oracle.spmm_csr_f64(crow, col, val, B),
                                   rtol=1e-4, atol=1e-4)
    check_status(npu)


def test_tiles_hand_made_layout(npu):
    """Tiles written by hand, not by the producer: repeated columns across
    tiles, a window with no tiles, and entries in the padding positions."""
    g = torch.Generator().manual_seed(21)
    K, N = 50, 32
    tptr = torch.tensor([0, 2, 2, 5], dtype=torch.int64)
    ucol = torch.randint(0, K, (16 * 5,), generator=g, dtype=torch.int64)
    val = (torch.rand(256 * 5, generator=g) * 2 - 1).half()
    B = torch.randn(K, N, generator=g).half()
    for idt in (torch.int32, torch.int64):
        t = {"crow_window_ptr": tptr.to(idt), "unique_col_ids": ucol.to(idt), "value": val}
        y = tiles_call(npu, t, B)
        assert_close(y, oracle.spmm_ascend_cube_tiles_f64(tptr, ucol, val, B), torch.float16, str(idt))
        assert not bool(y[16:32].any())
    check_status(npu)


def test_tiles_config3_sample(npu):
    w = workloads.make(3, scale=0.02)
    t = npu.csr_to_ascend_cube(w.rowptr.to(DEV), w.col.to(DEV), w.val.to(DEV), w.M, w.K, 16)
    y = tiles_call(npu, t, w.B)
    assert_close(y[: w.M], oracle.spmm_csr_f64(w.rowptr, w.col, w.val, w.B), torch.float16, "cfg3 tiles")
    check_status(npu)


def test_tiles_edges_and_contract(npu):
    B = torch.randn(10, 16).half()
    empty = {"crow_window_ptr": torch.zeros(1, dtype=torch.int32), "unique_col_ids": torch.zeros(0, dtype=torch.int32),
             "value": torch.zeros(0).half()}
    assert tiles_call(npu, empty, B).shape == (0, 16)
    no_tiles = dict(empty, crow_window_ptr=torch.zeros(3, dtype=torch.int32))
    y = tiles_call(npu, no_tiles, B)
    assert y.shape == (32, 16) and not bool(y.any())
    one = {"crow_window_ptr": torch.tensor([0, 1], dtype=torch.int32),
           "unique_col_ids": torch.zeros(16, dtype=torch.int32), "value": torch.zeros(256).half()}
    with pytest.raises(RuntimeError, match="requires feature width divisible by 16, but got 8"):
        tiles_call(npu, one, torch.randn(5, 8).half())
    with pytest.raises(RuntimeError, match="value must hold 256 entries per tile"):
        tiles_call(npu, dict(one, value=torch.zeros(255).half()), B)
    with pytest.raises(RuntimeError, match="unique_col_ids must hold 16 columns per tile"):
        tiles_call(npu, dict(one, unique_col_ids=torch.zeros(15, dtype=torch.int32)), B)
    with pytest.raises(RuntimeError, match="value must have the same dtype as dense"):
        tiles_call(npu, dict(one, value=torch.zeros(256)), B)
    check_status(npu)


def test_tiles_bad_window_pointer_is_reported(npu):
    t = {"crow_window_ptr": torch.tensor([0, 3], dtype=torch.int32),    # 3 > 1 tile
         "unique_col_ids": torch.zeros(16, dtype=torch.int32), "value": torch.ones(256).half()}
    tiles_call(npu, t, torch.randn(4, 16).half())
    torch.cuda.synchronize()
    code, _ = npu.device_status(True)
    assert code == 2   # SPMM_DEV_BAD_ROWPTR
