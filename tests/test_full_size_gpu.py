"""Parity at the benchmarked sizes.

* Config 5 at full size (16.8M x 16.8M, ~469M nonzeros, N = 1024, B = 34 GB):
  the configuration the bench headline runs.  Its B offsets cross 2^32
  elements (column * N > 2^32 for columns above 4,194,304), the limit of
  the reference's 32-bit offsets (kernels/op_kernel/spmm_csr.cpp:6).
* Config 2 at full size through ``spmm_csr``.
* Config 4 (fp32, N = 512, tolerance 1e-4) at scale 0.1 through ``spmm_csr``
  and ``spmm_ascend_cube`` on its GPU ``preprocess`` layout, every row.
* Matrices whose B has more rows than the benchmark's, so that byte and
  element offsets of gathered rows exceed 2^32 (and 16-byte-vector offsets
  exceed 2^31), for each kernel family: the CUDA-core ring kernel (fp16
  N = 1024, fp32 N = 512), the tensor-core gather (fp16 N = 128) and the
  window kernels (mixed operator), with int32 and int64 indices.

Each full-size case compares a row sample (random rows plus rows that reach
the highest columns) with the float64 oracle at the reference's tolerance
(tests/task_mapping/correctness.py:140-143) and probes every row with the
linearity check of ``helpers.assert_linear``.
"""

import pytest
import torch

import oracle
import workloads
from helpers import assert_close, assert_linear, sample_oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def npu():
    import build

    build.build()
    import spmm_npu

    assert torch.cuda.is_available()
    yield spmm_npu
    torch.cuda.empty_cache()


@pytest.fixture(autouse=True)
def _release():
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def status_ok(npu):
    code, detail = npu.device_status(True)
    assert code == 0, f"device status {code} at {detail}"


def sample_rows(rowptr, col, N, n=1024, seed=0):
    """n/2 random rows and n/2 rows holding a column whose B offset
    (column * N elements) is at or beyond 2^32, when there are such."""
    M = rowptr.numel() - 1
    g = torch.Generator().manual_seed(seed)
    rand = torch.randperm(M, generator=g)[: n // 2]
    far = torch.nonzero(col.to(torch.int64) * N >= 2**32).flatten()
    if far.numel():
        pick = far[torch.randperm(far.numel(), generator=g)[: n // 2].to(far.device)]
        owner = torch.searchsorted(rowptr.to(torch.int64), pick, right=True) - 1
        rand = torch.cat([rand, owner.cpu()])
    return torch.unique(rand)


def check_sample(y, rowptr, col, val, B, what, dtype):
    rows = sample_rows(rowptr, col, B.shape[1])
    ref = sample_oracle(rowptr, col, val, B, rows)
    assert_close(y[rows.to(y.device)], ref, dtype, what)
    return rows


def test_config5_full_spmm_csr(npu):
    w = workloads.make(5, device=DEV)
    assert int(w.col.max()) * w.N >= 2**32
    start = torch.zeros(40, dtype=torch.int32, device=DEV)
    y = npu.spmm_csr(w.rowptr, w.col, w.val, w.B, start)
    torch.cuda.synchronize()
    status_ok(npu)
    rows = check_sample(y, w.rowptr, w.col, w.val, w.B, "cfg5 sample", torch.float16)
    assert rows.numel() > 600
    assert_linear(y, w.rowptr, w.col, w.val, w.B, "cfg5 all rows")


def test_config2_full_spmm_csr(npu):
    w = workloads.make(2, device=DEV)
    start = torch.zeros(40, dtype=torch.int32, device=DEV)
    y = npu.spmm_csr(w.rowptr, w.col, w.val, w.B, start)
    torch.cuda.synchronize()
    status_ok(npu)
    check_sample(y, w.rowptr, w.col, w.val, w.B, "cfg2 sample", torch.float16)
    assert_linear(y, w.rowptr, w.col, w.val, w.B, "cfg2 all rows")


def test_config4_scale_01_both_operators(npu):
    w = workloads.make(4, device=DEV, scale=0.1)
    assert w.dtype == torch.float32 and w.N == 512
    crow, col, val, B = (t.cpu() for t in (w.rowptr, w.col, w.val, w.B))
    ref = oracle.spmm_csr_f64(crow, col, val, B)
    start = torch.zeros(40, dtype=torch.int32, device=DEV)
    y = npu.spmm_csr(w.rowptr, w.col, w.val, w.B, start)
    assert_close(y, ref, torch.float32, "cfg4/0.1 spmm_csr")
    m = npu.preprocess(w.rowptr, w.col, w.val, w.M, w.K, 16, False)
    assert m["unique_col_ids"].numel() > 0 and m["vcol_indices"].numel() > 0   # both parts in use
    ym = npu.spmm_ascend_cube(m["crow_window_ptr"], m["unique_col_ids"], m["value"], m["vrow_window_ptr"],
                              m["vcol_indices"], m["vvalue"], w.B, start[:20], start)
    got = npu.restore_node_tensor(ym, m["inv_permutation"])
    assert_close(got, ref, torch.float32, "cfg4/0.1 spmm_ascend_cube")
    status_ok(npu)


def far_matrix(M, K, N, idt, seed):
    """M rows over K columns, ~40 nonzeros per row: half drawn from the last
    2^22 columns (B offsets beyond 2^32 elements), half anywhere, a few
    empty rows and two long rows; every fourth 16-row window also shares 24
    far columns across all its rows, so ``preprocess`` sends it to the
    window kernel."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    deg = torch.randint(0, 80, (M,), generator=g, device=DEV)
    deg[::97] = 0
    deg[5], deg[M - 3] = 3000, 1500
    rows = torch.repeat_interleave(torch.arange(M, device=DEV), deg)
    far = torch.randint(K - (1 << 22), K, (rows.numel(),), generator=g, device=DEV)
    any_ = torch.randint(0, K, (rows.numel(),), generator=g, device=DEV)
    cols = torch.where(torch.rand(rows.numel(), generator=g, device=DEV) < 0.5, far, any_)
    dense_win = torch.arange(0, M // 16, 4, device=DEV)
    shared = torch.randint(K - (1 << 22), K, (dense_win.numel(), 24), generator=g, device=DEV)
    wr = (dense_win[:, None, None] * 16 + torch.arange(16, device=DEV)[None, :, None]).expand(-1, 16, 24)
    wc = shared[:, None, :].expand(-1, 16, 24)
    rows = torch.cat([rows, wr.reshape(-1)])
    cols = torch.cat([cols, wc.reshape(-1)])
    key = torch.unique(rows * K + cols)
    r, c = key // K, key % K
    rowptr = torch.zeros(M + 1, dtype=torch.int64, device=DEV)
    rowptr[1:] = torch.cumsum(torch.bincount(r, minlength=M), 0)
    return rowptr.to(idt), c.to(idt)


@pytest.mark.parametrize("dtype,N,K,idt", [
    (torch.float16, 1024, 17_000_000, torch.int32),   # 34.8 GB B: vector offsets beyond 2^31
    (torch.float16, 1024, 4_500_000, torch.int64),
    (torch.float16, 128, 34_000_000, torch.int32),    # tensor-core gather
    (torch.float32, 512, 8_500_000, torch.int32),
])
def test_b_offsets_beyond_32_bits(npu, dtype, N, K, idt):
    M = 2048
    assert (K - 1) * N >= 2**32
    rowptr, col = far_matrix(M, K, N, idt, seed=N)
    g = torch.Generator(device=DEV).manual_seed(1)
    val = (torch.rand(col.numel(), generator=g, device=DEV) * 2 - 1).to(dtype)
    B = torch.empty((K, N), dtype=dtype, device=DEV).normal_(generator=g)
    start = torch.zeros(40, dtype=torch.int32, device=DEV)
    ref = sample_oracle(rowptr, col, val, B, torch.arange(M))
    y = npu.spmm_csr(rowptr, col, val, B, start)
    assert_close(y, ref, dtype, f"spmm_csr N={N} K={K}")
    # the mixed operator on the preprocess layout (window kernels + CSR rows)
    m = npu.preprocess(rowptr, col, val, M, K, 16, False)
    assert m["unique_col_ids"].numel() > 0 and m["vcol_indices"].numel() > 0   # both parts in use
    ym = npu.spmm_ascend_cube(m["crow_window_ptr"], m["unique_col_ids"], m["value"], m["vrow_window_ptr"],
                              m["vcol_indices"], m["vvalue"], B, start[:20], start)
    assert_close(npu.restore_node_tensor(ym, m["inv_permutation"]), ref, dtype, f"mixed N={N} K={K}")
    status_ok(npu)
