// spmm_csr_launch_noalloc: the CSR SpMM with its scratch in a fixed,
// library-owned device array, for callers that cannot allocate device
// memory at call time.
//
// Who needs it: hosts that bind the C ABI directly and own no device
// allocator they can hand us (a Go/Java/Rust service calling through
// cgo/JNI/FFI with a fixed memory budget reserved at start-up, or a
// real-time loop where cudaMalloc/cudaFree would synchronise the device and
// stall other streams).  spmm_csr_launch needs a caller-provided workspace
// of spmm_csr_workspace_bytes(); this variant needs none.
//
// How: the fp32 partial rows of the nnz-unit split (see gather.cu) and the
// per-unit first rows live in
// g_noalloc_scratch below, a static __device__ array of kNoallocScratchBytes
// (32 MiB) that every GPU loading this library holds until the process
// exits.  Host code cannot use the array's name as a device address, so the
// first call on each device resolves it with cudaGetSymbolAddress (with that
// device current) and caches the pointer; make that first call before any
// stream capture.  When the default split would need more partial storage
// than the array holds, the unit size is doubled until it fits (results then
// differ from spmm_csr_launch only by fp32 rounding order); calls needing
// units above kNoallocMaxUnit are rejected with SPMM_ERR_UNSUPPORTED.
//
// Every call shares the one array.  Nothing in it has to start at zero (each
// partial slot is written before the fix-up reads it), but two calls whose
// kernels overlap on the GPU - on different streams, or from different host
// threads - race on it: serialise them on one stream.
#include <algorithm>
#include <cstdint>
#include <mutex>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

constexpr size_t kNoallocScratchBytes = size_t(32) << 20;  // 32 MiB per device
constexpr int64_t kNoallocMaxUnit = int64_t(1) << 20;        // nonzeros per unit

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
float *g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of the static scratch array on the current device.
float *noalloc_scratch(cudaError_t *err)
{
    int dev = 0;
    *err = cudaGetDevice(&dev);
    if (*err != cudaSuccess) return nullptr;
    if (dev < 0 || dev >= kMaxDevices) {
        *err = cudaErrorInvalidDevice;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (*err != cudaSuccess) return nullptr;
        g_scratch_ptr[dev] = static_cast<float *>(p);
    }
    return g_scratch_ptr[dev];
}

}  // namespace

}  // namespace spmmb

extern "C" int spmm_csr_launch_noalloc(const void *rowptr, const void *col, const void *value, const void *dense,
                                       void *out, int64_t M, int64_t K, int64_t N, int64_t nnz, int itype,
                                       int dtype, void *stream)
{
    using namespace spmmb;
    const char *op = "spmm_csr_launch_noalloc";
    // The same argument contract as spmm_csr_launch (one shared check).
    const int rc = check_csr_args(rowptr, col, value, dense, out, M, K, N, nnz, itype, dtype, op);
    if (rc || M == 0) return rc;

    GatherPlan plan = plan_gather(nnz, N, dtype);
    while (plan.workspace_bytes() > kNoallocScratchBytes && plan.unit < kNoallocMaxUnit) {
        plan.unit *= 2;
        plan.unit_end = units_for(nnz, plan.unit);
    }
    if (plan.workspace_bytes() > kNoallocScratchBytes)
        return capi_error(SPMM_ERR_UNSUPPORTED,
                          "%s: %lld nonzeros at width %lld need more than the %zu-byte static scratch", op,
                          (long long)nnz, (long long)N, kNoallocScratchBytes);
    cudaError_t e;
    float *scratch = noalloc_scratch(&e);
    if (!scratch) return capi_error(SPMM_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", op, cudaGetErrorString(e));
    DevStatus *st = device_status_ptr(&e);
    if (!st) return capi_error(SPMM_ERR_CUDA, "%s: %s", op, cudaGetErrorString(e));
    GatherArgs a{};
    a.rowptr = rowptr; a.col = col; a.val = value; a.B = dense; a.out = out;
    a.M = M; a.K = K; a.N = N; a.nnz = nnz; a.row_begin = 0;
    a.unit = plan.unit; a.unit_begin = plan.unit_begin; a.unit_end = plan.unit_end;
    set_workspace(a, plan, scratch);
    a.status = st;
    e = launch_gather(a, itype, dtype, 0, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return capi_error(SPMM_ERR_CUDA, "%s: %s", op, cudaGetErrorString(e));
    return SPMM_OK;
}
