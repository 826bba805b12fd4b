"""The L2 residency plan of spmm_csr (hot B rows gathered with an evict_last
L2 policy, the rest with evict_first), called through the C ABI.

SPMM_B200_L2PLAN=on makes these test-sized problems plan (by default only
dense operands of at least 16x L2 do).  Checked: the plan's header after a
launch (a power-law matrix enables it, a uniform one does not), outputs
bitwise equal to the launch without a plan (only cache priorities differ),
and sampled rows against the float64 oracle."""

import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
import workloads
from helpers import assert_close

pytestmark = pytest.mark.gpu

V, I64, INT, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t


class Header(ctypes.Structure):
    _fields_ = [("threshold", ctypes.c_uint32), ("hot_bins", ctypes.c_uint32), ("budget", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32), ("samples", ctypes.c_uint64), ("hot_samples", ctypes.c_uint64)]


@pytest.fixture(scope="module")
def lib():
    import build

    build.build()
    L = ctypes.CDLL(str(build.LIB))
    L.spmm_last_error.restype = ctypes.c_char_p
    L.spmm_csr_workspace_bytes.restype = SZ
    L.spmm_csr_workspace_bytes.argtypes = [I64, I64, I64, INT]
    L.spmm_csr_l2_plan_offset.restype = SZ
    L.spmm_csr_l2_plan_offset.argtypes = [I64, I64, I64, INT]
    L.spmm_csr_launch.restype = INT
    L.spmm_csr_launch.argtypes = [V, V, V, V, V, I64, V, I64, I64, I64, I64, INT, INT, V, SZ, V]
    L.spmm_csr_aiv_mb_batch_launch.restype = INT
    L.spmm_csr_aiv_mb_batch_launch.argtypes = L.spmm_csr_launch.argtypes
    return L


def run(L, rp, col, val, B, mode, entry="spmm_csr_launch"):
    """spmm_csr (or another entry point with its signature) through the C
    ABI under SPMM_B200_L2PLAN=mode; the output and the plan header (None
    when the problem reserves no plan)."""
    old = os.environ.get("SPMM_B200_L2PLAN")
    os.environ["SPMM_B200_L2PLAN"] = mode
    try:
        M, K, N, nnz = rp.numel() - 1, B.shape[0], B.shape[1], col.numel()
        dt = 0 if B.dtype == torch.float16 else 1
        it = 0 if rp.dtype == torch.int32 else 1
        wb = L.spmm_csr_workspace_bytes(M, N, nnz, dt)
        off = L.spmm_csr_l2_plan_offset(M, N, nnz, dt)
        ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
        out = torch.empty(M, N, dtype=B.dtype, device="cuda")
        rc = getattr(L, entry)(rp.data_ptr(), col.data_ptr(), val.data_ptr(), B.data_ptr(), None, 0,
                               out.data_ptr(), M, K, N, nnz, it, dt, ws.data_ptr(), wb,
                               torch.cuda.current_stream().cuda_stream)
        assert rc == 0, L.spmm_last_error()
        torch.cuda.synchronize()
        hdr = None
        if off != ctypes.c_size_t(-1).value:
            raw = ws[off: off + ctypes.sizeof(Header)].cpu().numpy().tobytes()
            hdr = Header.from_buffer_copy(raw)
        return out, hdr
    finally:
        if old is None:
            os.environ.pop("SPMM_B200_L2PLAN", None)
        else:
            os.environ["SPMM_B200_L2PLAN"] = old


def enabled(h):
    return h.threshold > 0 and h.samples > 0 and 4 * h.hot_samples >= h.samples


def check_rows(y, rp, col, val, B, n=384, seed=0):
    rows = np.sort(np.random.default_rng(seed).choice(rp.numel() - 1, n, replace=False))
    rpc, colc, valc = rp.cpu().to(torch.int64), col.cpu(), val.cpu()
    starts, ends = rpc[rows], rpc[rows + 1]
    idx = torch.cat([torch.arange(int(s), int(e)) for s, e in zip(starts, ends)])
    sub = torch.zeros(n + 1, dtype=torch.int64)
    sub[1:] = torch.cumsum(ends - starts, 0)
    ref = oracle.spmm_csr_f64(sub, colc[idx].to(torch.int64), valc[idx], B.cpu())
    assert_close(y[torch.from_numpy(rows).cuda()].cpu(), ref, B.dtype, "sampled rows vs float64 oracle")


@pytest.mark.parametrize("dtype,N,idt", [(torch.float16, 512, torch.int32), (torch.float32, 256, torch.int64),
                                         (torch.float16, 1024, torch.int32)])
def test_power_law_plan_enables_and_keeps_results(lib, dtype, N, idt):
    w = workloads.make(5, scale=0.01, device="cuda", N=N)
    rp, col = w.rowptr.to(idt), w.col.to(idt)
    val, B = w.val.to(dtype), w.B.to(dtype)
    y_plan, h = run(lib, rp, col, val, B, "on")
    y_off, h_off = run(lib, rp, col, val, B, "off")
    assert h is not None and h_off is None
    assert h.samples == min(col.numel(), 1 << 22)
    assert 2 <= h.threshold and 0 < h.hot_bins <= h.budget
    assert enabled(h), (h.threshold, h.hot_bins, h.samples, h.hot_samples)
    assert torch.equal(y_plan, y_off), "cache priorities changed the result"
    y_again, _ = run(lib, rp, col, val, B, "on")   # the plan region is rebuilt on every call
    assert torch.equal(y_again, y_off)
    # the deep-batch ablation variant under the plan: same sums, bit for bit
    y_deep, h_deep = run(lib, rp, col, val, B, "on", "spmm_csr_aiv_mb_batch_launch")
    assert h_deep is not None and enabled(h_deep)
    assert torch.equal(y_deep, y_off)
    check_rows(y_plan, rp, col, val, B)


def test_uniform_columns_leave_the_plan_disabled(lib):
    g = torch.Generator(device="cuda").manual_seed(5)
    M, K, per = 200_000, 1 << 20, 10
    rows = torch.arange(M, device="cuda").repeat_interleave(per)
    cols = torch.randint(0, K, (M * per,), generator=g, device="cuda")
    key = torch.unique(rows * K + cols)
    r, c = key // K, key % K
    rp = torch.zeros(M + 1, dtype=torch.int64, device="cuda")
    rp[1:] = torch.cumsum(torch.bincount(r, minlength=M), 0)
    rp, col = rp.int(), c.int()
    val = (torch.rand(col.numel(), generator=g, device="cuda") * 2 - 1).half()
    B = torch.randn(K, 512, generator=g, device="cuda").half()
    y_plan, h = run(lib, rp, col, val, B, "on")
    y_off, _ = run(lib, rp, col, val, B, "off")
    assert h is not None and not enabled(h), (h.threshold, h.hot_bins, h.samples, h.hot_samples)
    assert torch.equal(y_plan, y_off)
    check_rows(y_plan, rp, col, val, B, n=256, seed=1)

