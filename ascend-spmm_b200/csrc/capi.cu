// extern "C" entry points of libspmm_b200.so (declared in include/spmm_b200.h).
//
// Each SpMM entry point mirrors one operator of the reference's torch
// extension (extension/custom_op.cpp:25-264): the same dimension and width
// contract (check_dense_contract, custom_op.cpp:39-57), the same output row
// count, and an asynchronous launch on the caller's stream.  Argument errors
// return SPMM_ERR_ARG with the reference's message text.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace {

thread_local std::string g_last_error;

int set_error(int code, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_error(cudaError_t e, const char *where)
{
    return set_error(SPMM_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

// check_dense_contract (custom_op.cpp:39-57).
int check_dense(int dtype, int64_t N, int64_t alignment, const char *op)
{
    if (dtype != SPMM_F16 && dtype != SPMM_F32)
        return set_error(SPMM_ERR_ARG, "%s supports only FP16 and FP32 dense tensors", op);
    const bool half = dtype == SPMM_F16;
    const int64_t max_width = half ? 1024 : 512;
    if (N <= 0 || N > max_width)
        return set_error(SPMM_ERR_ARG, "%s requires 0 < feature width <= %lld for %s, but got %lld", op,
                         (long long)max_width, half ? "FP16" : "FP32", (long long)N);
    if (N % alignment != 0)
        return set_error(SPMM_ERR_ARG,
                         "%s requires feature width divisible by %lld, but got %lld. Pad and crop the dense "
                         "tensor or use a safe PyTorch fallback.",
                         op, (long long)alignment, (long long)N);
    return SPMM_OK;
}

// 16-byte vector loads/stores and cp.async need 16-byte aligned bases.
bool misaligned(const void *p) { return ((uintptr_t)p & 15u) != 0; }

int check_itype(int itype, const char *op)
{
    if (itype != SPMM_I32 && itype != SPMM_I64)
        return set_error(SPMM_ERR_ARG, "%s: index arrays must be int32 or int64", op);
    return SPMM_OK;
}

}  // namespace

namespace spmmb {
int check_csr_args(const void *rowptr, const void *col, const void *value, const void *dense, const void *out,
                   int64_t M, int64_t K, int64_t N, int64_t nnz, int itype, int dtype, const char *op)
{
    int rc = check_dense(dtype, N, dtype == SPMM_F16 ? 16 : 8, op);
    if (rc) return rc;
    if ((rc = check_itype(itype, op))) return rc;
    if (M < 0 || K < 0 || nnz < 0) return set_error(SPMM_ERR_ARG, "%s: negative size", op);
    if (M == 0) return SPMM_OK;
    if (!rowptr || !dense || !out || (nnz > 0 && (!col || !value)))
        return set_error(SPMM_ERR_ARG, "%s: null array", op);
    if (misaligned(dense) || misaligned(out))
        return set_error(SPMM_ERR_ARG, "%s: dense and out must be 16-byte aligned", op);
    return SPMM_OK;
}
}  // namespace spmmb

namespace {

int csr_impl(const void *rowptr, const void *col, const void *value, const void *dense, void *out,
             int64_t M, int64_t K, int64_t N, int64_t nnz, int itype, int dtype, void *workspace,
             size_t workspace_bytes, void *stream, int batch_depth, const char *op, void *out_mc = nullptr)
{
    int rc = spmmb::check_csr_args(rowptr, col, value, dense, out, M, K, N, nnz, itype, dtype, op);
    if (rc || M == 0) return rc;
    if (misaligned(workspace))
        return set_error(SPMM_ERR_ARG, "%s: workspace must be 16-byte aligned", op);
    if (misaligned(out_mc))
        return set_error(SPMM_ERR_ARG, "%s: the multicast address must be 16-byte aligned", op);
    const spmmb::GatherPlan plan = spmmb::plan_gather(nnz, N, dtype, true);
    if (workspace_bytes < plan.workspace_bytes() || !workspace)
        return set_error(SPMM_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the %zu required", op,
                         workspace_bytes, plan.workspace_bytes());
    cudaError_t e;
    spmmb::DevStatus *st = spmmb::device_status_ptr(&e);
    if (!st) return cuda_error(e, op);
    spmmb::GatherArgs a{};
    a.rowptr = rowptr; a.col = col; a.val = value; a.B = dense; a.out = out;
    a.M = M; a.K = K; a.N = N; a.nnz = nnz; a.row_begin = 0;
    a.unit = plan.unit; a.unit_begin = plan.unit_begin; a.unit_end = plan.unit_end;
    spmmb::set_workspace(a, plan, workspace);
    a.out_mc = out_mc;
    a.status = st;
    if (plan.l2) {   // hot B rows kept in L2 for the ring kernel (cache priorities only)
        e = spmmb::launch_l2_plan(a, itype, dtype, static_cast<char *>(workspace) + plan.l2_offset(),
                                  static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_error(e, op);
    }
    e = spmmb::launch_gather(a, itype, dtype, batch_depth, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, op);
    return SPMM_OK;
}

// Side stream of each (host thread, device) for the mixed operator: its CSR
// rows beyond the windows run there concurrently with the window kernel
// (disjoint output rows; the window kernel uses no workspace), forked from
// and joined back to the caller's stream by events.  Per host thread, so
// callers on different threads (and a stream capture on one of them) never
// share one; created on first use and destroyed when the thread exits (a
// thread pool that retires threads gives the streams and events back).
struct SideStream {
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
constexpr int kMaxSideDevices = 128;
struct ThreadSideStreams {
    SideStream dev[kMaxSideDevices];
    ~ThreadSideStreams()
    {
        // Work already queued on a stream completes before its resources are
        // released; errors (a runtime already unloading at process exit) are
        // ignored.
        for (int d = 0; d < kMaxSideDevices; ++d) {
            SideStream &x = dev[d];
            if (!x.stream) continue;
            cudaSetDevice(d);
            cudaEventDestroy(x.join);
            cudaEventDestroy(x.fork);
            cudaStreamDestroy(x.stream);
            x = SideStream{};
        }
    }
};
thread_local ThreadSideStreams g_side;

cudaError_t side_stream(SideStream **out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxSideDevices) return cudaErrorInvalidDevice;
    SideStream &x = g_side.dev[dev];
    if (!x.stream) {   // all three or none are kept
        SideStream y;
        e = cudaStreamCreateWithFlags(&y.stream, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&y.fork, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&y.join, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            if (y.fork) cudaEventDestroy(y.fork);
            if (y.stream) cudaStreamDestroy(y.stream);
            return e;
        }
        x = y;
    }
    *out = &x;
    return cudaSuccess;
}

// Workspace of the mixed operator: the window kernel's item schedule
// (window_sched_bytes, when there are windows), then the CSR kernels'
// scratch for the rows beyond the windows.
size_t mixed_sched_bytes(int64_t n_windows, int64_t N)
{
    return n_windows > 0 ? spmmb::window_sched_bytes(n_windows, N) : 0;
}
size_t mixed_workspace(int64_t n_windows, int64_t v_rows, int64_t v_nnz, int64_t N, int dtype)
{
    const size_t csr = v_rows > 16 * n_windows ? spmmb::plan_gather(v_nnz, N, dtype).workspace_bytes() : 0;
    return mixed_sched_bytes(n_windows, N) + csr;
}

int mixed_impl(const void *Crowptr, const void *Ccol, const void *Cvalue, const void *Vrowptr,
               const void *Vcol, const void *Vvalue, const void *dense, void *out, int64_t n_windows,
               int64_t n_blocks, int64_t v_rows, int64_t v_nnz, int64_t K, int64_t N, int itype, int dtype,
               void *workspace, size_t workspace_bytes, void *stream, int pipelined, int batch_depth,
               const char *op)
{
    int rc = check_dense(dtype, N, 16, op);
    if (rc) return rc;
    if ((rc = check_itype(itype, op))) return rc;
    if (n_windows < 0 || n_blocks < 0 || v_rows < 0 || v_nnz < 0 || K < 0)
        return set_error(SPMM_ERR_ARG, "%s: negative size", op);
    const int64_t rows = n_windows * 16 > v_rows ? n_windows * 16 : v_rows;
    if (rows == 0) return SPMM_OK;
    if (!dense || !out || (n_windows > 0 && !Crowptr) || (v_rows > 0 && !Vrowptr))
        return set_error(SPMM_ERR_ARG, "%s: null array", op);
    if (misaligned(dense) || misaligned(out) || misaligned(Cvalue) || misaligned(workspace))
        return set_error(SPMM_ERR_ARG, "%s: dense, Cvalue, out and workspace must be 16-byte aligned", op);
    const size_t sched = mixed_sched_bytes(n_windows, N);
    const size_t need = mixed_workspace(n_windows, v_rows, v_nnz, N, dtype);
    if (workspace_bytes < need || (need && !workspace))
        return set_error(SPMM_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the %zu required", op,
                         workspace_bytes, need);
    cudaError_t e;
    spmmb::DevStatus *st = spmmb::device_status_ptr(&e);
    if (!st) return cuda_error(e, op);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool both = n_windows > 0 && v_rows > 16 * n_windows;
    SideStream *side = nullptr;
    cudaStream_t sg = s;   // stream of the CSR rows
    if (both) {
        if ((e = side_stream(&side)) != cudaSuccess) return cuda_error(e, op);
        if ((e = cudaEventRecord(side->fork, s)) != cudaSuccess) return cuda_error(e, op);
        if ((e = cudaStreamWaitEvent(side->stream, side->fork, 0)) != cudaSuccess) return cuda_error(e, op);
        sg = side->stream;
    }
    if (n_windows > 0) {
        spmmb::WindowArgs w{};
        w.cptr = Crowptr; w.ccol = Ccol; w.cval = Cvalue;
        w.vptr = Vrowptr; w.vcol = Vcol; w.vval = Vvalue;
        w.B = dense; w.out = out;
        w.nwin = n_windows; w.nblocks = n_blocks; w.vrows = v_rows; w.vnnz = v_nnz;
        w.K = K; w.N = N; w.status = st;
        w.sched = sched ? workspace : nullptr;
        e = spmmb::launch_window(w, itype, dtype, pipelined, s);
        if (e != cudaSuccess) return cuda_error(e, op);
    }
    if (v_rows > 16 * n_windows) {
        const spmmb::GatherPlan plan = spmmb::plan_gather(v_nnz, N, dtype);
        spmmb::GatherArgs a{};
        a.rowptr = Vrowptr; a.col = Vcol; a.val = Vvalue; a.B = dense; a.out = out;
        a.M = v_rows; a.K = K; a.N = N; a.nnz = v_nnz; a.row_begin = 16 * n_windows;
        a.unit = plan.unit; a.unit_begin = plan.unit_begin; a.unit_end = plan.unit_end;
        spmmb::set_workspace(a, plan, static_cast<char *>(workspace) + sched);
        a.status = st;
        e = spmmb::launch_gather(a, itype, dtype, batch_depth, sg);
        if (both) {   // join even after a launch error, so s never races the side stream
            const cudaError_t e1 = cudaEventRecord(side->join, sg);
            const cudaError_t e2 = e1 == cudaSuccess ? cudaStreamWaitEvent(s, side->join, 0) : e1;
            if (e == cudaSuccess) e = e2;
        }
        if (e != cudaSuccess) return cuda_error(e, op);
    }
    return SPMM_OK;
}

}  // namespace

namespace spmmb {
int capi_error(int code, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}
}  // namespace spmmb

extern "C" {

const char *spmm_last_error(void) { return g_last_error.c_str(); }

int spmm_abi_version(void) { return 1; }

int spmm_device_status(int *code, int64_t *detail, int reset, void *stream)
{
    cudaError_t e;
    spmmb::DevStatus *st = spmmb::device_status_ptr(&e);
    if (!st) return cuda_error(e, "spmm_device_status");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    spmmb::DevStatus h{};
    e = cudaMemcpyAsync(&h, st, sizeof h, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && reset) {
        const spmmb::DevStatus z{};
        e = cudaMemcpyAsync(st, &z, sizeof z, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    if (e != cudaSuccess) return cuda_error(e, "spmm_device_status");
    if (code) *code = h.code;
    if (detail) *detail = h.detail;
    return SPMM_OK;
}

size_t spmm_csr_workspace_bytes(int64_t M, int64_t N, int64_t nnz, int dtype)
{
    (void)M;
    return spmmb::plan_gather(nnz, N, dtype, true).workspace_bytes();
}

size_t spmm_csr_l2_plan_offset(int64_t M, int64_t N, int64_t nnz, int dtype)
{
    (void)M;
    const spmmb::GatherPlan plan = spmmb::plan_gather(nnz, N, dtype, true);
    return plan.l2 ? plan.l2_offset() : SIZE_MAX;
}

int spmm_csr_launch(const void *rowptr, const void *col, const void *value, const void *dense,
                    const int32_t *start, int64_t n_start, void *out, int64_t M, int64_t K, int64_t N,
                    int64_t nnz, int itype, int dtype, void *workspace, size_t workspace_bytes, void *stream)
{
    (void)start;
    (void)n_start;
    return csr_impl(rowptr, col, value, dense, out, M, K, N, nnz, itype, dtype, workspace, workspace_bytes,
                    stream, 0, "spmm_csr");
}

int spmm_csr_launch_multicast(const void *rowptr, const void *col, const void *value, const void *dense,
                              void *out, void *out_multicast, int64_t M, int64_t K, int64_t N, int64_t nnz,
                              int itype, int dtype, void *workspace, size_t workspace_bytes, void *stream)
{
    if (!out_multicast) return set_error(SPMM_ERR_ARG, "spmm_csr_multicast: null multicast address");
    return csr_impl(rowptr, col, value, dense, out, M, K, N, nnz, itype, dtype, workspace, workspace_bytes,
                    stream, 0, "spmm_csr_multicast", out_multicast);
}

int spmm_csr_aiv_mb_batch_launch(const void *rowptr, const void *col, const void *value, const void *dense,
                                 const int32_t *start, int64_t n_start, void *out, int64_t M, int64_t K,
                                 int64_t N, int64_t nnz, int itype, int dtype, void *workspace,
                                 size_t workspace_bytes, void *stream)
{
    (void)start;
    (void)n_start;
    return csr_impl(rowptr, col, value, dense, out, M, K, N, nnz, itype, dtype, workspace, workspace_bytes,
                    stream, 1, "spmm_csr_aiv_mb_batch");
}

size_t spmm_ascend_cube_workspace_bytes(int64_t n_windows, int64_t n_blocks, int64_t v_rows, int64_t v_nnz,
                                        int64_t N, int dtype)
{
    (void)n_blocks;
    return mixed_workspace(n_windows, v_rows, v_nnz, N, dtype);
}

#define SPMM_MIXED_ARGS                                                                                      \
    const void *Crowptr, const void *Ccol_ids, const void *Cvalue, const void *Vrowptr, const void *Vcol_ids, \
        const void *Vvalue, const void *dense, const int32_t *Cstart, int64_t n_cstart,                        \
        const int32_t *Vstart, int64_t n_vstart, void *out, int64_t n_windows, int64_t n_blocks,              \
        int64_t v_rows, int64_t v_nnz, int64_t K, int64_t N, int itype, int dtype, void *workspace,           \
        size_t workspace_bytes, void *stream

#define SPMM_MIXED_FORWARD                                                                             \
    Crowptr, Ccol_ids, Cvalue, Vrowptr, Vcol_ids, Vvalue, dense, out, n_windows, n_blocks, v_rows, v_nnz, \
        K, N, itype, dtype, workspace, workspace_bytes, stream

int spmm_ascend_cube_launch(SPMM_MIXED_ARGS)
{
    (void)Cstart; (void)n_cstart; (void)Vstart; (void)n_vstart;
    return mixed_impl(SPMM_MIXED_FORWARD, 1, 0, "spmm_ascend_cube");
}

int spmm_ascend_cube_aic_without_pipeline_launch(SPMM_MIXED_ARGS)
{
    (void)Cstart; (void)n_cstart; (void)Vstart; (void)n_vstart;
    return mixed_impl(SPMM_MIXED_FORWARD, 0, 0, "spmm_ascend_cube_aic_without_pipeline");
}

int spmm_ascend_cube_aiv_mb_launch(SPMM_MIXED_ARGS)
{
    (void)Cstart; (void)n_cstart; (void)Vstart; (void)n_vstart;
    return mixed_impl(SPMM_MIXED_FORWARD, 1, 1, "spmm_ascend_cube_aiv_mb");
}

size_t spmm_cube_workspace_bytes(int64_t n_windows, int64_t nnz, int64_t N, int itype, int dtype)
{
    (void)N;
    if (n_windows <= 0) return 0;
    return spmmb::cube_workspace_bytes(n_windows, nnz, itype, dtype);
}

int spmm_cube_launch(const void *rowptr, const void *col, const void *value, const void *dense,
                     const int32_t *start, int64_t n_start, void *out, int64_t n_windows, int64_t K, int64_t N,
                     int64_t nnz, int itype, int dtype, void *workspace, size_t workspace_bytes, void *stream)
{
    (void)start;
    (void)n_start;
    const char *op = "spmm_cube";
    int rc = check_dense(dtype, N, 16, op);   // custom_op.cpp:102
    if (rc) return rc;
    if ((rc = check_itype(itype, op))) return rc;
    if (n_windows < 0 || K < 0 || nnz < 0) return set_error(SPMM_ERR_ARG, "%s: negative size", op);
    if (n_windows == 0) return SPMM_OK;
    if (!rowptr || !dense || !out || (nnz > 0 && (!col || !value)))
        return set_error(SPMM_ERR_ARG, "%s: null array", op);
    if (misaligned(dense) || misaligned(out) || misaligned(workspace))
        return set_error(SPMM_ERR_ARG, "%s: dense, out and workspace must be 16-byte aligned", op);
    const size_t need = spmmb::cube_workspace_bytes(n_windows, nnz, itype, dtype);
    if (workspace_bytes < need || !workspace)
        return set_error(SPMM_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the %zu required", op,
                         workspace_bytes, need);
    cudaError_t e;
    spmmb::DevStatus *st = spmmb::device_status_ptr(&e);
    if (!st) return cuda_error(e, op);
    spmmb::CubeArgs a{};
    a.rowptr = rowptr; a.col = col; a.val = value; a.B = dense; a.out = out;
    a.nwin = n_windows; a.K = K; a.N = N; a.nnz = nnz; a.status = st;
    e = spmmb::launch_cube(a, itype, dtype, workspace, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, op);
    return SPMM_OK;
}

size_t spmm_ascend_cube_tiles_workspace_bytes(int64_t n_windows, int64_t n_tiles, int64_t N, int itype, int dtype)
{
    (void)N;
    if (n_windows <= 0) return 0;
    return spmmb::tiles_workspace_bytes(n_windows, n_tiles, itype, dtype);
}

int spmm_ascend_cube_tiles_launch(const void *crow_window_ptr, const void *unique_col_ids, const void *value,
                                  const void *dense, void *out, int64_t n_windows, int64_t n_tiles, int64_t K,
                                  int64_t N, int itype, int dtype, void *workspace, size_t workspace_bytes,
                                  void *stream)
{
    const char *op = "spmm_ascend_cube_tiles";
    int rc = check_dense(dtype, N, 16, op);
    if (rc) return rc;
    if ((rc = check_itype(itype, op))) return rc;
    if (n_windows < 0 || n_tiles < 0 || K < 0) return set_error(SPMM_ERR_ARG, "%s: negative size", op);
    if (itype == SPMM_I32 && 16 * n_tiles > INT32_MAX)
        return set_error(SPMM_ERR_ARG, "%s: 16 * %lld tiles do not fit int32 block offsets", op, (long long)n_tiles);
    if (n_windows == 0) return SPMM_OK;
    if (!crow_window_ptr || !dense || !out || (n_tiles > 0 && (!unique_col_ids || !value)))
        return set_error(SPMM_ERR_ARG, "%s: null array", op);
    if (misaligned(dense) || misaligned(out) || misaligned(workspace))
        return set_error(SPMM_ERR_ARG, "%s: dense, out and workspace must be 16-byte aligned", op);
    const size_t need = spmmb::tiles_workspace_bytes(n_windows, n_tiles, itype, dtype);
    if (workspace_bytes < need || !workspace)
        return set_error(SPMM_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the %zu required", op,
                         workspace_bytes, need);
    cudaError_t e;
    spmmb::DevStatus *st = spmmb::device_status_ptr(&e);
    if (!st) return cuda_error(e, op);
    spmmb::TileArgs a{};
    a.tptr = crow_window_ptr; a.col = unique_col_ids; a.val = value; a.B = dense; a.out = out;
    a.nwin = n_windows; a.ntiles = n_tiles; a.K = K; a.N = N; a.status = st;
    e = spmmb::launch_tiles(a, itype, dtype, workspace, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, op);
    return SPMM_OK;
}

int spmm_csr_to_spmm_cube_run(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                              int64_t nnz, int64_t window_size, int itype, int vbytes, const spmm_allocator *alloc,
                              spmm_layout *out, void *stream)
{
    return spmmb::pre_csr_to_spmm_cube(crow, col, val, nrows, ncols, nnz, window_size, itype, vbytes, alloc, out,
                                       stream);
}

int spmm_csr_to_bcsr_run(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                         int64_t nnz, int64_t window_size, int itype, int vbytes, const spmm_allocator *alloc,
                         spmm_layout *out, void *stream)
{
    return spmmb::pre_csr_to_bcsr(crow, col, val, nrows, ncols, nnz, window_size, itype, vbytes, alloc, out, stream,
                                  false);
}

int spmm_csr_to_ascend_cube_run(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                                int64_t nnz, int64_t window_size, int itype, int vbytes,
                                const spmm_allocator *alloc, spmm_layout *out, void *stream)
{
    return spmmb::pre_csr_to_bcsr(crow, col, val, nrows, ncols, nnz, window_size, itype, vbytes, alloc, out, stream,
                                  true);
}

int spmm_block_level_split_run(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                               int64_t nnz, double a, int64_t window_size, int itype, int vbytes,
                               const spmm_allocator *alloc, spmm_layout *out, void *stream)
{
    return spmmb::pre_block_level_split(crow, col, val, nrows, ncols, nnz, a, window_size, itype, vbytes, alloc,
                                        out, stream);
}

int spmm_preprocess_run(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                        int64_t nnz, int64_t window_size, int graph_layout, int itype, int vbytes,
                        const spmm_allocator *alloc, spmm_preprocess_result *out, void *stream)
{
    return spmmb::pre_preprocess(crow, col, val, nrows, ncols, nnz, window_size, graph_layout, itype, vbytes,
                                 alloc, out, stream);
}

int spmm_pack_rows_launch(const void *src, const int64_t *inv, int64_t n, int64_t row_bytes, void *dst,
                          int64_t packed_rows, void *stream)
{
    if (n < 0 || row_bytes < 0 || packed_rows < 0) return set_error(SPMM_ERR_ARG, "pack_rows: negative size");
    if (packed_rows == 0 || row_bytes == 0) return SPMM_OK;
    if (!dst || (n > 0 && (!src || !inv))) return set_error(SPMM_ERR_ARG, "pack_rows: null array");
    cudaError_t e;
    spmmb::DevStatus *st = spmmb::device_status_ptr(&e);
    if (!st) return cuda_error(e, "pack_rows");
    e = spmmb::launch_pack_rows(src, inv, n, row_bytes, dst, packed_rows, st, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SPMM_OK : cuda_error(e, "pack_rows");
}

int spmm_restore_rows_launch(const void *src, int64_t src_rows, const int64_t *inv, int64_t n,
                             int64_t row_bytes, void *dst, void *stream)
{
    if (n < 0 || row_bytes < 0 || src_rows < 0) return set_error(SPMM_ERR_ARG, "restore_rows: negative size");
    if (n == 0 || row_bytes == 0) return SPMM_OK;
    if (!dst || !src || !inv) return set_error(SPMM_ERR_ARG, "restore_rows: null array");
    cudaError_t e;
    spmmb::DevStatus *st = spmmb::device_status_ptr(&e);
    if (!st) return cuda_error(e, "restore_rows");
    e = spmmb::launch_restore_rows(src, src_rows, inv, n, row_bytes, dst, st, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SPMM_OK : cuda_error(e, "restore_rows");
}

}  // extern "C"
