"""spmm_csr_launch_noalloc: the CSR SpMM for callers that cannot allocate
device memory at call time (an FFI host with a fixed memory budget, or a loop
that must not let cudaMalloc synchronise the device).  It keeps its scratch
in a 32 MiB static device array instead of a caller workspace.

Called here through the C ABI (ctypes), on two calls in a row, and checked
against the workspace entry point spmm_csr_launch with the reference's
tolerances.  This file is collected last so that a run stopping at the first
failure has already run every other test; it also passes on its own.
"""

import ctypes

import pytest
import torch

from helpers import assert_close, rand_csr

pytestmark = pytest.mark.gpu

V, I64, INT, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t


@pytest.fixture(scope="module")
def lib():
    import build

    build.build()
    L = ctypes.CDLL(str(build.LIB))
    L.spmm_last_error.restype = ctypes.c_char_p
    L.spmm_csr_workspace_bytes.restype = SZ
    L.spmm_csr_workspace_bytes.argtypes = [I64, I64, I64, INT]
    L.spmm_csr_launch.restype = INT
    L.spmm_csr_launch.argtypes = [V, V, V, V, V, I64, V, I64, I64, I64, I64, INT, INT, V, SZ, V]
    L.spmm_csr_launch_noalloc.restype = INT
    L.spmm_csr_launch_noalloc.argtypes = [V, V, V, V, V, I64, I64, I64, I64, INT, INT, V]
    return L


def case(seed, M, K, N, dtype, long_rows):
    g = torch.Generator().manual_seed(seed)
    crow, col = rand_csr(M, K, 0.01, seed=seed, long_rows=long_rows, empty_every=9)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
    B = torch.randn(K, N, generator=g).to(dtype)
    return crow.cuda(), col.cuda(), val.cuda(), B.cuda()


def dtype_code(dtype):
    return 0 if dtype == torch.float16 else 1


def with_workspace(L, crow, col, val, B):
    M, K, N, nnz = crow.numel() - 1, B.shape[0], B.shape[1], col.numel()
    out = torch.empty(M, N, dtype=B.dtype, device="cuda")
    wbytes = L.spmm_csr_workspace_bytes(M, N, nnz, dtype_code(B.dtype))
    ws = torch.empty(max(wbytes, 1), dtype=torch.uint8, device="cuda")
    rc = L.spmm_csr_launch(crow.data_ptr(), col.data_ptr(), val.data_ptr(), B.data_ptr(), None, 0,
                           out.data_ptr(), M, K, N, nnz, 0, dtype_code(B.dtype), ws.data_ptr(), wbytes,
                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.spmm_last_error()
    return out


def no_alloc(L, crow, col, val, B):
    M, K, N, nnz = crow.numel() - 1, B.shape[0], B.shape[1], col.numel()
    out = torch.empty(M, N, dtype=B.dtype, device="cuda")
    rc = L.spmm_csr_launch_noalloc(crow.data_ptr(), col.data_ptr(), val.data_ptr(), B.data_ptr(),
                                   out.data_ptr(), M, K, N, nnz, 0, dtype_code(B.dtype),
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.spmm_last_error()
    return out


def test_no_alloc_matches_workspace_entry_point_two_calls(lib):
    # call 1: wide rows whose default split needs more partial storage than
    # the static array, so the unit size is doubled; call 2: a different,
    # smaller fp32 problem reusing the same array right after.
    cases = [case(1, 8000, 20000, 1024, torch.float16, {3: 9000, 400: 12000}),
             case(2, 900, 700, 64, torch.float32, {10: 650, 899: 500})]
    outs = [no_alloc(lib, *c) for c in cases]
    torch.cuda.synchronize()
    for c, y in zip(cases, outs):
        ref = with_workspace(lib, *c)
        assert_close(y, ref.double().cpu().numpy(), c[3].dtype, "no-alloc vs workspace")
    # and once more on the first problem after the array held the second one
    y = no_alloc(lib, *cases[0])
    assert_close(y, with_workspace(lib, *cases[0]).double().cpu().numpy(), torch.float16, "third call")


def test_no_alloc_rejects_oversized_requests(lib):
    # the size check happens on the host before any launch
    d = torch.zeros(16, 1024, dtype=torch.float16, device="cuda")
    rc = lib.spmm_csr_launch_noalloc(d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(),
                                     1, 16, 1024, 1 << 40, 0, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 4 and b"static scratch" in lib.spmm_last_error()
    rc = lib.spmm_csr_launch_noalloc(d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(),
                                     1, 16, 24, 1, 0, 0, None)
    assert rc == 1
