"""GPU parity of the SpMM operators against the float64 CPU oracle.

Tolerances are the reference's (fp16 2e-2, fp32 1e-4,
tests/task_mapping/correctness.py:140-143); CUDA-core variants must agree
bitwise (tests/aic_aiv_ablation/bitwise_correctness.py:238-239).  All calls
go through ``spmm_npu`` -> ``custom_ops_lib`` -> the C ABI of
libspmm_b200.so.
"""

import numpy as np
import pytest
import torch

import oracle
from golden.make_golden import CASES
from helpers import assert_close, golden_layout, load_golden, rand_csr

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def npu():
    import build

    build.build()
    import spmm_npu

    assert torch.cuda.is_available()
    return spmm_npu


def start_of(ptr, cores):
    return oracle.make_start(ptr.cpu().to(torch.int64), cores).to(DEV)


def csr_call(npu, crow, col, val, B, op="spmm_csr"):
    return getattr(npu, op)(crow.to(DEV), col.to(DEV), val.to(DEV), B.to(DEV), start_of(crow, 40))


def mixed_call(npu, m, B, op="spmm_ascend_cube", cols_key="unique_col_ids", vcols_key="vcol_indices"):
    args = [m["crow_window_ptr"], m[cols_key], m["value"], m["vrow_window_ptr"], m[vcols_key], m["vvalue"]]
    args = [a.to(DEV) for a in args]
    return getattr(npu, op)(*args, B.to(DEV), start_of(m["crow_window_ptr"], 20),
                            start_of(m["vrow_window_ptr"], 40))


def check_status(npu):
    code, detail = npu.device_status(True)
    assert code == 0, f"device status {code} at {detail}"


# ---------------------------------------------------------------- spmm_csr

@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_spmm_csr_golden(npu, name):
    c = load_golden(name)
    y = csr_call(npu, c["crow"], c["col"], c["values"], c["dense"])
    torch.cuda.synchronize()
    assert y.dtype == c["values"].dtype and y.shape == (c["nrows"], c["dense"].shape[1])
    assert_close(y, c["z"]["spmm_f64"], y.dtype, name)
    check_status(npu)


@pytest.mark.parametrize("dtype,N", [(torch.float16, w) for w in (16, 32, 48, 64, 128, 256, 512, 1024)]
                         + [(torch.float32, w) for w in (8, 24, 64, 256, 512)])
def test_spmm_csr_widths(npu, dtype, N):
    M, K = 700, 523
    crow, col = rand_csr(M, K, 0.03, seed=N, long_rows={5: 400, 333: 520}, empty_every=7)
    g = torch.Generator().manual_seed(N)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
    B = torch.randn(K, N, generator=g).to(dtype)
    y = csr_call(npu, crow, col, val, B)
    assert_close(y, oracle.spmm_csr_f64(crow, col, val, B), dtype, f"N={N}")
    check_status(npu)


@pytest.mark.parametrize("idt", [torch.int32, torch.int64])
def test_spmm_csr_long_rows_cross_many_units(npu, idt):
    """Rows much longer than a unit are split across units and re-summed by
    the fix-up pass; includes a row spanning > 20 units and empty rows at
    unit boundaries."""
    M, K = 64, 9000
    crow, col = rand_csr(M, K, 0.01, seed=3, long_rows={0: 6000, 10: 300, 63: 8000}, empty_every=5, idt=idt)
    g = torch.Generator().manual_seed(1)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).half()
    B = torch.randn(K, 64, generator=g).half()
    y = csr_call(npu, crow, col, val, B)
    assert_close(y, oracle.spmm_csr_f64(crow, col, val, B), torch.float16)
    check_status(npu)


def test_spmm_csr_edge_shapes(npu):
    # no nonzeros at all: every row is zero
    crow = torch.zeros(33, dtype=torch.int32)
    y = csr_call(npu, crow, torch.zeros(0, dtype=torch.int32), torch.zeros(0, dtype=torch.float16),
                 torch.randn(8, 16).half())
    assert y.shape == (32, 16) and not bool(y.any())
    # zero rows
    y = csr_call(npu, torch.zeros(1, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                 torch.zeros(0, dtype=torch.float16), torch.randn(8, 16).half())
    assert y.shape == (0, 16)
    # single nonzero
    y = csr_call(npu, torch.tensor([0, 1], dtype=torch.int32), torch.tensor([3], dtype=torch.int32),
                 torch.tensor([0.5], dtype=torch.float16), torch.arange(64).reshape(4, 16).half())
    assert torch.equal(y.cpu(), (0.5 * torch.arange(48, 64)).half().reshape(1, 16))
    check_status(npu)


def test_variants_bitwise_identical(npu):
    """All CUDA-core variants share one nnz split and one per-element fma
    order: spmm_csr == spmm_csr_aiv_mb_batch == pure-CSR spmm_ascend_cube ==
    spmm_ascend_cube_aiv_mb, for every width."""
    M, K = 2000, 1500
    crow, col = rand_csr(M, K, 0.01, seed=11, long_rows={7: 1200, 1999: 900}, empty_every=13)
    g = torch.Generator().manual_seed(5)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).half()
    empty = {"crow_window_ptr": torch.zeros(1, dtype=torch.int32),
             "unique_col_ids": torch.zeros(0, dtype=torch.int32),
             "value": torch.zeros(0, dtype=torch.float16),
             "vrow_window_ptr": crow, "vcol_indices": col, "vvalue": val}
    for N in (16, 32, 64, 128, 256):
        B = torch.randn(K, N, generator=g).half()
        ref = csr_call(npu, crow, col, val, B)
        for other in (csr_call(npu, crow, col, val, B, "spmm_csr_aiv_mb_batch"),
                      mixed_call(npu, empty, B)[:M],
                      mixed_call(npu, empty, B, "spmm_ascend_cube_aiv_mb")[:M]):
            assert torch.equal(other, ref), N
    check_status(npu)


# --------------------------------------------------------- mixed operator

@pytest.mark.parametrize("name", [c[0] for c in CASES])
@pytest.mark.parametrize("layout", ["block_level_split", "preprocess", "preprocess_graph", "csr_to_bcsr"])
def test_mixed_golden_layouts(npu, name, layout):
    """The reference's own layouts (golden fixtures) fed to spmm_ascend_cube
    reproduce A @ B; preprocess layouts in packed row order."""
    c = load_golden(name)
    m = golden_layout(c, layout)
    dtype = c["values"].dtype
    if layout == "csr_to_bcsr":
        m.update(vrow_window_ptr=torch.zeros(1, dtype=m["crow_window_ptr"].dtype),
                 vcol_indices=torch.zeros(0, dtype=m["crow_window_ptr"].dtype),
                 vvalue=torch.zeros(0, dtype=dtype))
    B = c["dense"]
    ref = c["z"]["spmm_f64"]
    for op in ("spmm_ascend_cube", "spmm_ascend_cube_aic_without_pipeline", "spmm_ascend_cube_aiv_mb"):
        y = mixed_call(npu, m, B, op)
        nwin = m["crow_window_ptr"].numel() - 1
        assert y.shape[0] == max(16 * nwin, m["vrow_window_ptr"].numel() - 1)
        if layout.startswith("preprocess"):
            perm = m["permutation"].numpy()
            keep = perm >= 0
            assert_close(y[: perm.size].cpu()[torch.from_numpy(keep)], ref[perm[keep]], dtype, f"{name}/{layout}/{op}")
        else:
            assert_close(y[: c["nrows"]], ref, dtype, f"{name}/{layout}/{op}")
    check_status(npu)


def test_mixed_graph_layout_relabelled(npu):
    """(P A P^T)(P B) = P (A B) through the renumbered forward layout, and the
    fixed-layout transpose gives P (A^T B)."""
    c = load_golden("graph_i32_f16")
    m = golden_layout(c, "preprocess_graph")
    inv = m["inv_permutation"]
    prow = int(m["packed_rows"][0])
    Bp = npu.pack_node_tensor(c["dense"].to(DEV), inv.to(DEV), prow)
    y = mixed_call(npu, m, Bp, cols_key="renumbered_unique_col_ids", vcols_key="renumbered_vcol_indices")
    restored = npu.restore_node_tensor(y, inv.to(DEV))
    assert_close(restored, c["z"]["spmm_f64"], torch.float16, "forward")
    t = {k[len("transpose_"):]: v for k, v in m.items() if k.startswith("transpose_")}
    yt = mixed_call(npu, t, Bp)
    import scipy.sparse as sp
    A = sp.csr_matrix((c["values"].double().numpy(), c["col"].numpy(), c["crow"].numpy()),
                      shape=(c["nrows"], c["ncols"]))
    refT = A.T @ c["dense"].double().numpy()
    assert_close(npu.restore_node_tensor(yt, inv.to(DEV)), refT, torch.float16, "transpose")
    check_status(npu)


@pytest.mark.parametrize("dtype,N", [(torch.float16, 16), (torch.float16, 272), (torch.float16, 1024),
                                     (torch.float16, 64), (torch.float32, 16), (torch.float32, 128),
                                     (torch.float32, 384), (torch.float32, 512)])
def test_mixed_random_windows(npu, dtype, N):
    """Windows with many blocks (several pipeline chunks), CSR rows fused into
    every window, and CSR rows beyond the window region."""
    g = np.random.default_rng(N)
    nwin, K = 9, 700
    nb = g.integers(0, 80, nwin)
    nb[3] = 0
    cptr = torch.from_numpy(np.concatenate([[0], np.cumsum(nb)])).to(torch.int32)
    ccol = torch.from_numpy(np.concatenate([np.sort(g.choice(K, int(n), replace=False)) for n in nb])).to(torch.int32)
    gen = torch.Generator().manual_seed(N)
    cval = (torch.rand(16 * int(nb.sum()), generator=gen) * 2 - 1).to(dtype)
    cval[torch.rand(cval.numel(), generator=gen) < 0.4] = 0
    vrows = 16 * nwin + 37
    vcrow, vcol = rand_csr(vrows, K, 0.02, seed=N, long_rows={20: 300, 16 * nwin + 3: 500}, empty_every=4)
    vval = (torch.rand(vcol.numel(), generator=gen) * 2 - 1).to(dtype)
    B = torch.randn(K, N, generator=gen).to(dtype)
    m = {"crow_window_ptr": cptr, "unique_col_ids": ccol, "value": cval,
         "vrow_window_ptr": vcrow, "vcol_indices": vcol, "vvalue": vval}
    ref = oracle.spmm_mixed_f64(cptr, ccol, cval, vcrow, vcol, vval, B)
    for op in ("spmm_ascend_cube", "spmm_ascend_cube_aic_without_pipeline", "spmm_ascend_cube_aiv_mb"):
        assert_close(mixed_call(npu, m, B, op), ref, dtype, op)
    check_status(npu)


def test_mixed_op_graph_capture_and_threads(npu):
    """The mixed operator forks its CSR rows onto an internal side stream: a
    CUDA graph capture records the fork and replays to the eager bits, and
    host threads calling it on their own streams get the same bits."""
    import threading

    crow, col = rand_csr(900, 700, 0.03, seed=5, long_rows={3: 600, 880: 500}, empty_every=9)
    g = torch.Generator().manual_seed(5)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).half()
    B = torch.randn(700, 128, generator=g).half().to(DEV)
    m = npu.preprocess(crow.to(DEV), col.to(DEV), val.to(DEV), 900, 700, 16, False)
    assert m["crow_window_ptr"].numel() > 1 and m["vrow_window_ptr"].numel() - 1 > 16 * (m["crow_window_ptr"].numel() - 1)

    args = [m[k] for k in ("crow_window_ptr", "unique_col_ids", "value", "vrow_window_ptr", "vcol_indices",
                           "vvalue")]
    cstart, vstart = start_of(m["crow_window_ptr"], 20), start_of(m["vrow_window_ptr"], 40)

    def call():   # device tensors only, so it can be captured
        return npu.spmm_ascend_cube(*args, B, cstart, vstart)

    eager = call()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            call()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = call()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, eager)

    outs = [None] * 4
    errors = []

    def work(i):
        try:
            st = torch.cuda.Stream()
            with torch.cuda.stream(st):
                for _ in range(5):
                    outs[i] = call()
            st.synchronize()
        except Exception as exc:   # surfaced below
            errors.append(exc)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for o in outs:
        assert torch.equal(o, eager)
    check_status(npu)


# ------------------------------------------------------ failure handling

def test_invalid_columns_are_reported_not_faulted(npu):
    npu.device_status(True)
    crow = torch.tensor([0, 2, 3], dtype=torch.int32)
    col = torch.tensor([1, 99, 0], dtype=torch.int32)   # 99 >= K
    val = torch.ones(3, dtype=torch.float16)
    B = torch.ones(4, 16, dtype=torch.float16)
    y = csr_call(npu, crow, col, val, B)
    code, detail = npu.device_status(True)
    assert code == 1 and detail == 1
    assert torch.equal(y.cpu(), torch.ones(2, 16, dtype=torch.float16))
    # a row pointer past nnz is clamped and reported
    crow = torch.tensor([0, 2, 9], dtype=torch.int32)
    y = csr_call(npu, crow, col, val, B)
    code, _ = npu.device_status(True)
    assert code == 2


def test_contract_errors(npu):
    crow = torch.tensor([0, 1], dtype=torch.int32, device=DEV)
    col = torch.tensor([0], dtype=torch.int32, device=DEV)
    v = torch.ones(1, dtype=torch.float16, device=DEV)
    s = torch.zeros(40, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="feature width divisible by 16"):
        npu.spmm_csr(crow, col, v, torch.ones(2, 24, dtype=torch.float16, device=DEV), s)
    with pytest.raises(RuntimeError, match="0 < feature width <= 512 for FP32"):
        npu.spmm_csr(crow, col, v.float(), torch.ones(2, 520, device=DEV), s)
    with pytest.raises(RuntimeError, match="value must have the same dtype as dense"):
        npu.spmm_csr(crow, col, v, torch.ones(2, 16, device=DEV), s)
    with pytest.raises(RuntimeError, match="col and value must be same size"):
        npu.spmm_csr(crow, col, torch.ones(2, dtype=torch.float16, device=DEV),
                     torch.ones(2, 16, dtype=torch.float16, device=DEV), s)
    with pytest.raises(RuntimeError, match="requires a contiguous dense tensor"):
        npu.spmm_csr(crow, col, v, torch.ones(16, 2, dtype=torch.float16, device=DEV).t(), s)
    z = torch.zeros(1, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="spmm_ascend_cube requires feature width divisible by 16"):
        npu.spmm_ascend_cube(z, z[:0], v[:0], crow, col, v.float(), torch.ones(2, 8, device=DEV), s, s)


# ------------------------------------------------------ pack / restore

def test_pack_restore_roundtrip(npu):
    n = 37
    inv = torch.randperm(48, generator=torch.Generator().manual_seed(0))[:n]
    for x in (torch.randn(n, 5), torch.randn(n, 16).half(), torch.arange(n, dtype=torch.int64)):
        xp = npu.pack_node_tensor(x.to(DEV), inv.to(DEV), 48)
        assert xp.shape[0] == 48
        ref = torch.zeros((48, *x.shape[1:]), dtype=x.dtype)
        ref.index_copy_(0, inv, x)
        assert torch.equal(xp.cpu(), ref)
        assert torch.equal(npu.restore_node_tensor(xp, inv.to(DEV)).cpu(), x)
    with pytest.raises(ValueError, match="smaller than the permutation extent"):
        npu.pack_node_tensor(torch.zeros(n, 2, device=DEV), inv.to(DEV), 10)
    with pytest.raises(ValueError, match="one entry per original node"):
        npu.pack_node_tensor(torch.zeros(n + 1, 2, device=DEV), inv.to(DEV))


_ROW_KERNEL_SNIPPET = r"""
import sys, torch
sys.path[:0] = sys.argv[3].split(":")
import spmm_npu
d = torch.load(sys.argv[1])
outs = []
for case in d:
    crow, col, val, B = (t.cuda() for t in case)
    s = torch.zeros(40, dtype=torch.int32, device="cuda")
    outs.append(spmm_npu.spmm_csr(crow, col, val, B, s).cpu())
torch.save(outs, sys.argv[2])
"""


def row_window_csr(K, seed, idt, unit=256):
    """Row structure aimed at the ring kernel's row-end window: leading and
    trailing empty rows, runs of 33-100 empty rows between short rows (more
    row ends in one 8-position batch than one 32-row window holds), empty
    runs that start exactly at a unit boundary (owned by the next unit),
    one-nonzero rows (a row end at every position) and a few long rows."""
    g = np.random.default_rng(seed)
    deg = [0] * 40
    nnz = 0
    while nnz < 24 * unit:
        d = int(g.choice([1, 1, 2, 3, 5, 9, 17, 40, 300]))
        deg.append(d)
        nnz += d
        if nnz % unit and unit - nnz % unit <= 12:    # land exactly on a unit boundary
            while nnz % unit:
                deg.append(1)
                nnz += 1
        if nnz % unit == 0:
            deg += [0] * 45
        if g.random() < 0.05:
            deg += [0] * int(g.integers(33, 101))
    deg += [0] * 70
    rows = [np.sort(g.choice(K, size=d, replace=False)) for d in deg]
    crow = np.zeros(len(rows) + 1, np.int64)
    crow[1:] = np.cumsum([len(r) for r in rows])
    return torch.from_numpy(crow).to(idt), torch.from_numpy(np.concatenate(rows)).to(idt)


@pytest.mark.parametrize("dtype,N,idt", [(torch.float16, 256, torch.int32), (torch.float16, 1024, torch.int64),
                                         (torch.float32, 128, torch.int32), (torch.float32, 512, torch.int64)])
def test_ring_row_window_structure(npu, dtype, N, idt):
    crow, col = row_window_csr(700, N, idt)
    g = torch.Generator().manual_seed(N)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
    B = torch.randn(700, N, generator=g).to(dtype)
    y = csr_call(npu, crow, col, val, B)
    assert_close(y, oracle.spmm_csr_f64(crow, col, val, B), dtype, f"{dtype} N={N}")
    y2 = csr_call(npu, crow, col, val, B, "spmm_csr_aiv_mb_batch")
    assert torch.equal(y, y2)
    check_status(npu)


def test_ring_malformed_row_pointers_are_reported(npu):
    """Whole-warp rows (ring kernel): a decreasing row pointer and one past
    nnz are reported through the device status; nothing faults."""
    K, N = 64, 256
    B = torch.randn(K, N).half()
    for crow in ([0, 5, 3, 8], [0, 2, 4, 6, 9, 8], [0, 3, 30]):
        crow = torch.tensor(crow, dtype=torch.int32)
        nnz = 8
        col = torch.arange(nnz, dtype=torch.int32) % K
        val = torch.ones(nnz).half()
        npu.device_status(True)
        csr_call(npu, crow, col, val, B)
        torch.cuda.synchronize()
        code, _ = npu.device_status(True)
        assert code == 2, crow.tolist()


def test_cuda_core_kernels_bitwise_identical(npu, tmp_path):
    """The CUDA-core kernels - ring (cp.async ring, mixed-precision
    fma.rn.f32.f16 / packed f32x2 fma), flat stream and row (convert + fmaf) -
    produce the same bits for every width and index type.  Each runs in a
    child process selected by SPMM_B200_GATHER (the choice is read once per
    process)."""
    import os
    import subprocess
    import sys

    cases = []
    for N, dtype, idt in [(128, torch.float16, torch.int32), (256, torch.float16, torch.int64),
                          (512, torch.float16, torch.int32), (1024, torch.float16, torch.int32),
                          (64, torch.float32, torch.int32), (512, torch.float32, torch.int64)]:
        crow, col = rand_csr(1500, 900, 0.02, seed=N, long_rows={3: 700, 1499: 880}, empty_every=11, idt=idt)
        g = torch.Generator().manual_seed(N)
        val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
        B = torch.randn(900, N, generator=g).to(dtype)
        cases.append((crow, col, val, B))
        crow, col = row_window_csr(900, N + 1, idt)
        val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
        cases.append((crow, col, val, B))
    src = tmp_path / "in.pt"
    torch.save(cases, src)
    here = os.path.dirname(os.path.abspath(__file__))
    paths = ":".join([os.path.join(here, "..", "ascend-spmm_b200"), here])
    results = {}
    for kern in ("ring", "stream", "row"):
        dst = tmp_path / f"out_{kern}.pt"
        env = dict(os.environ, SPMM_B200_GATHER=kern)
        subprocess.run([sys.executable, "-c", _ROW_KERNEL_SNIPPET, str(src), str(dst), paths], env=env, check=True,
                       timeout=300)
        results[kern] = torch.load(dst)
    for kern in ("stream", "row"):
        for (c, a, b) in zip(cases, results["ring"], results[kern]):
            assert torch.equal(a, b), (kern, c[3].shape, c[3].dtype)
    # the default (tensor-core kernel for fp16 widths that are multiples of
    # 64) agrees with them within the reference tolerance
    for c, r in zip(cases, results["ring"]):
        y = csr_call(npu, *c).cpu()
        assert_close(y, oracle.spmm_csr_f64(*c), c[3].dtype)
        assert_close(r, oracle.spmm_csr_f64(*c), c[3].dtype)
