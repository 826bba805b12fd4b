"""spmm_csr_launch_noalloc: the CSR SpMM for callers that cannot allocate
device memory at call time (an FFI host with a fixed memory budget, or a loop
that must not let cudaMalloc synchronise the device).  It keeps its scratch
in a 32 MiB static device array instead of a caller workspace.

Called here through the C ABI (ctypes), on calls in a row, and checked
against the workspace entry point spmm_csr_launch and the float64 oracle with
the reference's tolerances.  The cases cover every kernel family the entry
point can reach: the CUDA-core ring kernel (fp16, 1024 features), the
tensor-core gather (fp16, 128 features) and the stream kernel (fp32, 64
features, int64 indices); the first two need more partial storage than the
static array under the default split, so their units are coarsened.  This
file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own.
"""

import ctypes

import pytest
import torch

import oracle
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


STATIC_SCRATCH = 32 << 20   # bytes of the library's static scratch array


def case(seed, M, K, N, dtype, long_rows, idt=torch.int32):
    g = torch.Generator().manual_seed(seed)
    crow, col = rand_csr(M, K, 0.01, seed=seed, long_rows=long_rows, empty_every=9, idt=idt)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
    B = torch.randn(K, N, generator=g).to(dtype)
    return crow.cuda(), col.cuda(), val.cuda(), B.cuda()


def exact_nnz_case(seed, M, K, N, nnz):
    """fp16 CSR with exactly nnz nonzeros (distinct sorted columns per row,
    a few empty rows), built on the device."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    deg = torch.full((M,), nnz // M, dtype=torch.int64, device="cuda")
    deg[: nnz % M] += 1
    deg[::101] = 0
    live = torch.nonzero(deg).flatten()
    deg[live[: nnz - int(deg.sum())]] += 1   # hand the empty rows' share to the first nonempty ones
    assert int(deg.sum()) == nnz and int(deg.max()) <= K
    rows = torch.repeat_interleave(torch.arange(M, device="cuda"), deg)
    start = torch.cumsum(deg, 0) - deg
    # row r takes the deg[r] columns (off + k * stride) % K, distinct because stride is odd and K a power of two
    k = torch.arange(rows.numel(), device="cuda") - start[rows]
    off = torch.randint(0, K, (M,), generator=g, device="cuda")
    cols = (off[rows] + k * 2 * (rows % 7) + k) % K
    key = rows * K + cols
    key, _ = torch.sort(key)
    crow = torch.zeros(M + 1, dtype=torch.int64, device="cuda")
    crow[1:] = torch.cumsum(deg, 0)
    val = (torch.rand(nnz, generator=g, device="cuda") * 2 - 1).half()
    B = torch.randn(K, N, generator=g, device="cuda").half()
    return crow.int(), (key % K).int(), val, B


def dtype_code(dtype):
    return 0 if dtype == torch.float16 else 1


def itype_code(idt):
    return 0 if idt == torch.int32 else 1


def with_workspace(L, crow, col, val, B):
    M, K, N, nnz = crow.numel() - 1, B.shape[0], B.shape[1], col.numel()
    out = torch.empty(M, N, dtype=B.dtype, device="cuda")
    wbytes = L.spmm_csr_workspace_bytes(M, N, nnz, dtype_code(B.dtype))
    ws = torch.empty(max(wbytes, 1), dtype=torch.uint8, device="cuda")
    rc = L.spmm_csr_launch(crow.data_ptr(), col.data_ptr(), val.data_ptr(), B.data_ptr(), None, 0,
                           out.data_ptr(), M, K, N, nnz, itype_code(crow.dtype), dtype_code(B.dtype),
                           ws.data_ptr(), wbytes, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.spmm_last_error()
    return out


def no_alloc(L, crow, col, val, B):
    M, K, N, nnz = crow.numel() - 1, B.shape[0], B.shape[1], col.numel()
    out = torch.empty(M, N, dtype=B.dtype, device="cuda")
    rc = L.spmm_csr_launch_noalloc(crow.data_ptr(), col.data_ptr(), val.data_ptr(), B.data_ptr(),
                                   out.data_ptr(), M, K, N, nnz, itype_code(crow.dtype), dtype_code(B.dtype),
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.spmm_last_error()
    return out


def needs_coarser_units(L, c):
    crow, col, _, B = c
    return L.spmm_csr_workspace_bytes(crow.numel() - 1, B.shape[1], col.numel(), dtype_code(B.dtype)) > STATIC_SCRATCH


def test_no_alloc_matches_workspace_entry_point_and_oracle(lib):
    # call 1: ring kernel (fp16, 1024 features) whose default split needs
    # more partial storage than the static array; call 2: tensor-core gather
    # (fp16, 128 features) at ~2^23 nonzeros, likewise coarsened (and
    # coarsened again by that kernel); call 3: a small fp32 problem with int64
    # indices (stream kernel) reusing the same array right after.
    cases = [case(1, 8000, 20000, 1024, torch.float16, {3: 9000, 400: 12000}),
             exact_nnz_case(2, 100_000, 1 << 16, 128, 8_380_000),
             case(3, 900, 700, 64, torch.float32, {10: 650, 899: 500}, idt=torch.int64)]
    assert needs_coarser_units(lib, cases[0]) and needs_coarser_units(lib, cases[1])
    assert not needs_coarser_units(lib, cases[2])
    outs = [no_alloc(lib, *c) for c in cases]
    torch.cuda.synchronize()
    for i, (c, y) in enumerate(zip(cases, outs)):
        crow, col, val, B = c
        assert_close(y, with_workspace(lib, *c).double().cpu().numpy(), B.dtype, f"case {i}: vs workspace")
        assert_close(y, oracle.spmm_csr_f64(crow.cpu(), col.cpu(), val.cpu(), B.cpu()), B.dtype,
                     f"case {i}: vs float64 oracle")
    # and once more on the first two problems after the array held the others
    for i in (0, 1):
        y = no_alloc(lib, *cases[i])
        assert_close(y, with_workspace(lib, *cases[i]).double().cpu().numpy(), torch.float16, f"repeat {i}")


def test_no_alloc_rejects_oversized_requests(lib):
    # the size check happens on the host before any launch
    d = torch.zeros(16, 1024, dtype=torch.float16, device="cuda")
    rc = lib.spmm_csr_launch_noalloc(d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(),
                                     1, 16, 1024, 1 << 40, 0, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 4 and b"static scratch" in lib.spmm_last_error()
    rc = lib.spmm_csr_launch_noalloc(d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(),
                                     1, 16, 24, 1, 0, 0, None)
    assert rc == 1
