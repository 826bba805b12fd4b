// custom_ops_lib: the torch-facing operator module of the B200 SpMM engine.
//
// Mirrors the reference's pybind module of the same name
// (extension/custom_op.cpp:1413-1492): same function names, positional
// arguments, output shapes and TORCH_CHECK messages.  Tensors must live on a
// CUDA device (the reference requires NPU tensors, custom_op.cpp:25-33);
// there is no CPU path.  All compute goes through the C ABI of
// libspmm_b200.so (include/spmm_b200.h) on the current CUDA stream.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAFunctions.h>

#include <map>
#include <stdexcept>
#include <unordered_map>

#include "spmm_b200.h"

namespace {

#define TORCH_CHECK_CUDA(tensor) TORCH_CHECK((tensor).is_cuda(), #tensor " must be CUDA tensor")

constexpr int64_t kHalfMaxWidth = 1024;   // custom_op.cpp:35
constexpr int64_t kFloatMaxWidth = 512;   // custom_op.cpp:36

// check_dense_contract, custom_op.cpp:39-57 (same messages).
void check_dense_contract(const at::Tensor &dense, int64_t alignment, const char *op_name)
{
    TORCH_CHECK(dense.scalar_type() == at::kHalf || dense.scalar_type() == at::kFloat, op_name,
                " supports only FP16 and FP32 dense tensors");
    TORCH_CHECK(dense.is_contiguous(), op_name, " requires a contiguous dense tensor");
    const int64_t width = dense.size(1);
    const bool is_half = dense.scalar_type() == at::kHalf;
    const int64_t max_width = is_half ? kHalfMaxWidth : kFloatMaxWidth;
    TORCH_CHECK(width > 0 && width <= max_width, op_name, " requires 0 < feature width <= ", max_width,
                " for ", is_half ? "FP16" : "FP32", ", but got ", width);
    TORCH_CHECK(width % alignment == 0, op_name, " requires feature width divisible by ", alignment,
                ", but got ", width, ". Pad and crop the dense tensor or use a safe PyTorch fallback.");
}

// check_value_contract, custom_op.cpp:59-64.
void check_value_contract(const at::Tensor &value, const at::Tensor &dense, const char *name)
{
    TORCH_CHECK(value.scalar_type() == dense.scalar_type(), name, " must have the same dtype as dense");
    TORCH_CHECK(value.is_contiguous(), name, " must be contiguous");
}

// The kernels use 16-byte vector accesses; views with an odd storage offset
// are copied to a fresh (aligned) allocation.
at::Tensor aligned16(const at::Tensor &t)
{
    return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) ? t.clone() : t;
}

int dtype_code(const at::Tensor &t) { return t.scalar_type() == at::kHalf ? SPMM_F16 : SPMM_F32; }

// Index tensors: int32 or int64, one dtype per operator call, contiguous.
int index_code(std::initializer_list<const at::Tensor *> ts, const char *op)
{
    const at::ScalarType st = (*ts.begin())->scalar_type();
    TORCH_CHECK(st == at::kInt || st == at::kLong, op, ": index tensors must be int32 or int64");
    for (const at::Tensor *t : ts) {
        TORCH_CHECK(t->scalar_type() == st, op, ": index tensors must share one dtype");
        TORCH_CHECK(t->is_contiguous(), op, ": index tensors must be contiguous");
    }
    return st == at::kInt ? SPMM_I32 : SPMM_I64;
}

void same_device(std::initializer_list<const at::Tensor *> ts, const at::Tensor &ref, const char *op)
{
    for (const at::Tensor *t : ts)
        TORCH_CHECK(t->device() == ref.device(), op, ": all tensors must be on ", ref.device());
}

void check_rc(int rc) { TORCH_CHECK(rc == SPMM_OK, spmm_last_error()); }

void *stream_of(const at::Tensor &t)
{
    return static_cast<void *>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

at::Tensor workspace(size_t bytes, const at::Tensor &like)
{
    return at::empty({(int64_t)std::max<size_t>(bytes, 1)}, like.options().dtype(at::kByte));
}

// ---------------------------------------------------------------------------
// CSR operators: spmm_csr (custom_op.cpp:67-88) and its batching ablation
// spmm_csr_aiv_mb_batch (custom_op.cpp:154-187).
// ---------------------------------------------------------------------------
using CsrLaunch = int (*)(const void *, const void *, const void *, const void *, const int32_t *, int64_t,
                          void *, int64_t, int64_t, int64_t, int64_t, int, int, void *, size_t, void *);

at::Tensor csr_op(const at::Tensor &rowptr, const at::Tensor &col, const at::Tensor &value,
                  const at::Tensor &dense, const at::Tensor &start, const char *op, bool ablation_messages,
                  CsrLaunch launch)
{
    TORCH_CHECK_CUDA(rowptr);
    TORCH_CHECK_CUDA(col);
    TORCH_CHECK_CUDA(value);
    TORCH_CHECK_CUDA(dense);
    TORCH_CHECK_CUDA(start);
    if (ablation_messages) {
        TORCH_CHECK(rowptr.dim() == 1, op, ": rowptr must be one-dimensional");
        TORCH_CHECK(col.dim() == 1, op, ": col must be one-dimensional");
        TORCH_CHECK(value.dim() == 1, op, ": value must be one-dimensional");
        TORCH_CHECK(dense.dim() == 2, op, ": dense must be two-dimensional");
        TORCH_CHECK(start.dim() == 1, op, ": start must be one-dimensional");
    } else {
        TORCH_CHECK(rowptr.dim() == 1, "row must be a 1D Tensor, but got: ", rowptr.dim());
        TORCH_CHECK(col.dim() == 1, "col must be a 1D Tensor, but got: ", col.dim());
        TORCH_CHECK(value.dim() == 1, "value must be a 1D Tensor, but got: ", value.dim());
        TORCH_CHECK(dense.dim() == 2, "dense must be a 2D Tensor, but got: ", dense.dim());
        TORCH_CHECK(start.dim() == 1, "start must be a 1D Tensor, but got: ", start.dim());
    }
    check_dense_contract(dense, dense.scalar_type() == at::kHalf ? 16 : 8, op);
    check_value_contract(value, dense, "value");
    if (ablation_messages) {
        TORCH_CHECK(col.size(0) == value.size(0), op, ": col and value must have equal length");
    } else {
        TORCH_CHECK(col.size(0) == value.size(0), "col and value must be same size, but got different: ",
                    col.size(0) - value.size(0));
    }
    TORCH_CHECK(rowptr.size(0) >= 1, op, ": rowptr must hold rows + 1 entries");
    same_device({&rowptr, &col, &value, &start}, dense, op);
    const int itype = index_code({&rowptr, &col}, op);
    c10::cuda::CUDAGuard guard(dense.device());

    const int64_t rows = rowptr.size(0) - 1, D = dense.size(1), nnz = col.size(0);
    at::Tensor result = at::empty({rows, D}, dense.options());
    const int dt = dtype_code(dense);
    const size_t wbytes = spmm_csr_workspace_bytes(rows, D, nnz, dt);
    at::Tensor ws = workspace(wbytes, dense);
    at::Tensor start_i = start.scalar_type() == at::kInt ? start.contiguous() : start.to(at::kInt).contiguous();
    const at::Tensor B = aligned16(dense);
    check_rc(launch(rowptr.data_ptr(), col.data_ptr(), value.data_ptr(), B.data_ptr(),
                    start_i.data_ptr<int32_t>(), start_i.numel(), result.data_ptr(), rows, dense.size(0), D,
                    nnz, itype, dt, ws.data_ptr(), wbytes, stream_of(dense)));
    return result;
}

at::Tensor spmm_csr_impl(const at::Tensor &rowptr, const at::Tensor &col, const at::Tensor &value,
                         const at::Tensor &dense, const at::Tensor &start)
{
    return csr_op(rowptr, col, value, dense, start, "spmm_csr", false, &spmm_csr_launch);
}

// This rank's row shard of C written through an NVLink multicast address of
// `out` (spmm_csr_launch_multicast): every GPU whose copy is bound to the
// multicast object receives the rows.  `out` is this rank's rows of the
// replicated C; `out_multicast` the multicast address of out's first byte.
at::Tensor spmm_csr_multicast_impl(const at::Tensor &rowptr, const at::Tensor &col, const at::Tensor &value,
                                   const at::Tensor &dense, const at::Tensor &out, int64_t out_multicast)
{
    const char *op = "spmm_csr_multicast";
    TORCH_CHECK_CUDA(rowptr);
    TORCH_CHECK_CUDA(col);
    TORCH_CHECK_CUDA(value);
    TORCH_CHECK_CUDA(dense);
    TORCH_CHECK_CUDA(out);
    TORCH_CHECK(rowptr.dim() == 1 && col.dim() == 1 && value.dim() == 1, op, ": rowptr, col and value must be 1-D");
    TORCH_CHECK(dense.dim() == 2, op, ": dense must be two-dimensional");
    check_dense_contract(dense, dense.scalar_type() == at::kHalf ? 16 : 8, op);
    check_value_contract(value, dense, "value");
    TORCH_CHECK(col.size(0) == value.size(0), op, ": col and value must have equal length");
    TORCH_CHECK(rowptr.size(0) >= 1, op, ": rowptr must hold rows + 1 entries");
    same_device({&rowptr, &col, &value, &out}, dense, op);
    const int itype = index_code({&rowptr, &col}, op);
    const int64_t rows = rowptr.size(0) - 1, D = dense.size(1), nnz = col.size(0);
    TORCH_CHECK(out.scalar_type() == dense.scalar_type(), op, ": out must have the dtype of dense");
    TORCH_CHECK(out.dim() == 2 && out.size(0) == rows && out.size(1) == D && out.is_contiguous(), op,
                ": out must be a contiguous [rows, N] tensor");
    TORCH_CHECK(out_multicast != 0 && out_multicast % 16 == 0, op, ": multicast address must be 16-byte aligned");
    c10::cuda::CUDAGuard guard(dense.device());
    const int dt = dtype_code(dense);
    const size_t wbytes = spmm_csr_workspace_bytes(rows, D, nnz, dt);
    at::Tensor ws = workspace(wbytes, dense);
    const at::Tensor B = aligned16(dense);
    check_rc(spmm_csr_launch_multicast(rowptr.data_ptr(), col.data_ptr(), value.data_ptr(), B.data_ptr(),
                                       out.data_ptr(), reinterpret_cast<void *>(out_multicast), rows, dense.size(0),
                                       D, nnz, itype, dt, ws.data_ptr(), wbytes, stream_of(dense)));
    return out;
}

at::Tensor spmm_csr_aiv_mb_batch_impl(const at::Tensor &rowptr, const at::Tensor &col, const at::Tensor &value,
                                      const at::Tensor &dense, const at::Tensor &start)
{
    return csr_op(rowptr, col, value, dense, start, "spmm_csr_aiv_mb_batch", true,
                  &spmm_csr_aiv_mb_batch_launch);
}

// ---------------------------------------------------------------------------
// Mixed operators: spmm_ascend_cube (custom_op.cpp:115-152) and its two
// ablations (custom_op.cpp:189-264).
// ---------------------------------------------------------------------------
using MixedLaunch = int (*)(const void *, const void *, const void *, const void *, const void *, const void *,
                            const void *, const int32_t *, int64_t, const int32_t *, int64_t, void *, int64_t,
                            int64_t, int64_t, int64_t, int64_t, int64_t, int, int, void *, size_t, void *);

at::Tensor mixed_op(const at::Tensor &Crowptr, const at::Tensor &Ccol_ids, const at::Tensor &Cvalue,
                    const at::Tensor &Vrowptr, const at::Tensor &Vcol_ids, const at::Tensor &Vvalue,
                    const at::Tensor &dense, const at::Tensor &Cstart, const at::Tensor &Vstart, const char *op,
                    bool ablation_messages, MixedLaunch launch)
{
    TORCH_CHECK_CUDA(Crowptr);
    TORCH_CHECK_CUDA(Ccol_ids);
    TORCH_CHECK_CUDA(Cvalue);
    TORCH_CHECK_CUDA(Vrowptr);
    TORCH_CHECK_CUDA(Vcol_ids);
    TORCH_CHECK_CUDA(Vvalue);
    TORCH_CHECK_CUDA(dense);
    TORCH_CHECK_CUDA(Cstart);
    TORCH_CHECK_CUDA(Vstart);
    if (ablation_messages) {
        TORCH_CHECK(Crowptr.dim() == 1, op, ": Crowptr must be one-dimensional");
        TORCH_CHECK(Ccol_ids.dim() == 1, op, ": Ccol_ids must be one-dimensional");
        TORCH_CHECK(Cvalue.dim() == 1, op, ": Cvalue must be one-dimensional");
        TORCH_CHECK(Vrowptr.dim() == 1, op, ": Vrowptr must be one-dimensional");
        TORCH_CHECK(Vcol_ids.dim() == 1, op, ": Vcol_ids must be one-dimensional");
        TORCH_CHECK(Vvalue.dim() == 1, op, ": Vvalue must be one-dimensional");
        TORCH_CHECK(dense.dim() == 2, op, ": dense must be two-dimensional");
        TORCH_CHECK(Cstart.dim() == 1, op, ": Cstart must be one-dimensional");
        TORCH_CHECK(Vstart.dim() == 1, op, ": Vstart must be one-dimensional");
    } else {
        TORCH_CHECK(Crowptr.dim() == 1, "Crow must be a 1D Tensor, but got: ", Crowptr.dim());
        TORCH_CHECK(Ccol_ids.dim() == 1, "Ccol_ids must be a 1D Tensor, but got: ", Ccol_ids.dim());
        TORCH_CHECK(Cvalue.dim() == 1, "Cvalue must be a 1D Tensor, but got: ", Cvalue.dim());
        TORCH_CHECK(Vrowptr.dim() == 1, "Vrow must be a 1D Tensor, but got: ", Vrowptr.dim());
        TORCH_CHECK(Vcol_ids.dim() == 1, "Vcol_ids must be a 1D Tensor, but got: ", Vcol_ids.dim());
        TORCH_CHECK(Vvalue.dim() == 1, "Vvalue must be a 1D Tensor, but got: ", Vvalue.dim());
        TORCH_CHECK(dense.dim() == 2, "dense must be a 2D Tensor, but got: ", dense.dim());
        TORCH_CHECK(Cstart.dim() == 1, "Cstart must be a 1D Tensor, but got: ", Cstart.dim());
        TORCH_CHECK(Vstart.dim() == 1, "Vstart must be a 1D Tensor, but got: ", Vstart.dim());
    }
    check_dense_contract(dense, 16, op);
    check_value_contract(Cvalue, dense, "Cvalue");
    check_value_contract(Vvalue, dense, "Vvalue");
    TORCH_CHECK(Crowptr.size(0) >= 1 && Vrowptr.size(0) >= 1, op, ": row pointers must hold rows + 1 entries");
    TORCH_CHECK(Cvalue.size(0) == 16 * Ccol_ids.size(0), op, ": Cvalue must hold 16 values per block");
    TORCH_CHECK(Vcol_ids.size(0) == Vvalue.size(0), op, ": Vcol_ids and Vvalue must have equal length");
    same_device({&Crowptr, &Ccol_ids, &Cvalue, &Vrowptr, &Vcol_ids, &Vvalue, &Cstart, &Vstart}, dense, op);
    const int itype = index_code({&Crowptr, &Ccol_ids, &Vrowptr, &Vcol_ids}, op);
    c10::cuda::CUDAGuard guard(dense.device());

    const int64_t nwin = Crowptr.size(0) - 1, vrows = Vrowptr.size(0) - 1;
    const int64_t rows = std::max(nwin * 16, vrows), D = dense.size(1);
    at::Tensor result = at::empty({rows, D}, dense.options());
    const int dt = dtype_code(dense);
    const size_t wbytes = spmm_ascend_cube_workspace_bytes(nwin, Ccol_ids.size(0), vrows, Vcol_ids.size(0), D, dt);
    at::Tensor ws = workspace(wbytes, dense);
    at::Tensor cs = Cstart.to(at::kInt).contiguous(), vs = Vstart.to(at::kInt).contiguous();
    const at::Tensor B = aligned16(dense), Cv = aligned16(Cvalue);
    check_rc(launch(Crowptr.data_ptr(), Ccol_ids.data_ptr(), Cv.data_ptr(), Vrowptr.data_ptr(),
                    Vcol_ids.data_ptr(), Vvalue.data_ptr(), B.data_ptr(), cs.data_ptr<int32_t>(), cs.numel(),
                    vs.data_ptr<int32_t>(), vs.numel(), result.data_ptr(), nwin, Ccol_ids.size(0), vrows,
                    Vcol_ids.size(0), dense.size(0), D, itype, dt, ws.data_ptr(), wbytes, stream_of(dense)));
    return result;
}

#define MIXED_SIG                                                                                              \
    const at::Tensor &Crowptr, const at::Tensor &Ccol_ids, const at::Tensor &Cvalue, const at::Tensor &Vrowptr, \
        const at::Tensor &Vcol_ids, const at::Tensor &Vvalue, const at::Tensor &dense, const at::Tensor &Cstart,  \
        const at::Tensor &Vstart
#define MIXED_ARGS Crowptr, Ccol_ids, Cvalue, Vrowptr, Vcol_ids, Vvalue, dense, Cstart, Vstart

at::Tensor spmm_ascend_cube_impl(MIXED_SIG)
{
    return mixed_op(MIXED_ARGS, "spmm_ascend_cube", false, &spmm_ascend_cube_launch);
}

at::Tensor spmm_ascend_cube_aic_without_pipeline_impl(MIXED_SIG)
{
    return mixed_op(MIXED_ARGS, "spmm_ascend_cube_aic_without_pipeline", true,
                    &spmm_ascend_cube_aic_without_pipeline_launch);
}

at::Tensor spmm_ascend_cube_aiv_mb_impl(MIXED_SIG)
{
    return mixed_op(MIXED_ARGS, "spmm_ascend_cube_aiv_mb", true, &spmm_ascend_cube_aiv_mb_launch);
}

// ---------------------------------------------------------------------------
// spmm_cube (custom_op.cpp:91-113): windows of (column << 4 | row) entries.
// ---------------------------------------------------------------------------
at::Tensor spmm_cube_impl(const at::Tensor &rowptr, const at::Tensor &col, const at::Tensor &value,
                          const at::Tensor &dense, const at::Tensor &start)
{
    TORCH_CHECK_CUDA(rowptr);
    TORCH_CHECK_CUDA(col);
    TORCH_CHECK_CUDA(value);
    TORCH_CHECK_CUDA(dense);
    TORCH_CHECK_CUDA(start);
    TORCH_CHECK(rowptr.dim() == 1, "row must be a 1D Tensor, but got: ", rowptr.dim());
    TORCH_CHECK(col.dim() == 1, "col must be a 1D Tensor, but got: ", col.dim());
    TORCH_CHECK(value.dim() == 1, "value must be a 1D Tensor, but got: ", value.dim());
    TORCH_CHECK(dense.dim() == 2, "dense must be a 2D Tensor, but got: ", dense.dim());
    TORCH_CHECK(start.dim() == 1, "start must be a 1D Tensor, but got: ", start.dim());
    check_dense_contract(dense, 16, "spmm_cube");
    check_value_contract(value, dense, "value");
    TORCH_CHECK(col.size(0) == value.size(0), "col and value must be same size, but got different: ",
                col.size(0) - value.size(0));
    TORCH_CHECK(rowptr.size(0) >= 1, "spmm_cube: rowptr must hold windows + 1 entries");
    same_device({&rowptr, &col, &value, &start}, dense, "spmm_cube");
    const int itype = index_code({&rowptr, &col}, "spmm_cube");
    c10::cuda::CUDAGuard guard(dense.device());

    const int64_t nwin = rowptr.size(0) - 1, D = dense.size(1), nnz = col.size(0);
    at::Tensor result = at::empty({nwin * 16, D}, dense.options());
    const int dt = dtype_code(dense);
    const size_t wbytes = spmm_cube_workspace_bytes(nwin, nnz, D, itype, dt);
    at::Tensor ws = workspace(wbytes, dense);
    at::Tensor start_i = start.to(at::kInt).contiguous();
    const at::Tensor B = aligned16(dense);
    check_rc(spmm_cube_launch(rowptr.data_ptr(), col.data_ptr(), value.data_ptr(), B.data_ptr(),
                              start_i.data_ptr<int32_t>(), start_i.numel(), result.data_ptr(), nwin, dense.size(0), D,
                              nnz, itype, dt, ws.data_ptr(), wbytes, stream_of(dense)));
    return result;
}

// ---------------------------------------------------------------------------
// spmm_ascend_cube_tiles: consumer of csr_to_ascend_cube's 16 x 16 tiles
// (custom_op.cpp:429-592 is the producer; the reference has no consumer).
// Same checks and messages as spmm_cube; output [16 * windows, N].
// ---------------------------------------------------------------------------
at::Tensor spmm_ascend_cube_tiles_impl(const at::Tensor &crow_window_ptr, const at::Tensor &unique_col_ids,
                                       const at::Tensor &value, const at::Tensor &dense)
{
    const char *op = "spmm_ascend_cube_tiles";
    TORCH_CHECK_CUDA(crow_window_ptr);
    TORCH_CHECK_CUDA(unique_col_ids);
    TORCH_CHECK_CUDA(value);
    TORCH_CHECK_CUDA(dense);
    TORCH_CHECK(crow_window_ptr.dim() == 1, "row must be a 1D Tensor, but got: ", crow_window_ptr.dim());
    TORCH_CHECK(unique_col_ids.dim() == 1, "col must be a 1D Tensor, but got: ", unique_col_ids.dim());
    TORCH_CHECK(value.dim() == 1, "value must be a 1D Tensor, but got: ", value.dim());
    TORCH_CHECK(dense.dim() == 2, "dense must be a 2D Tensor, but got: ", dense.dim());
    check_dense_contract(dense, 16, op);
    check_value_contract(value, dense, "value");
    TORCH_CHECK(unique_col_ids.size(0) % 16 == 0, op, ": unique_col_ids must hold 16 columns per tile, but got ",
                unique_col_ids.size(0));
    TORCH_CHECK(value.size(0) == 16 * unique_col_ids.size(0), op,
                ": value must hold 256 entries per tile, but got ", value.size(0), " for ",
                unique_col_ids.size(0) / 16, " tiles");
    TORCH_CHECK(crow_window_ptr.size(0) >= 1, op, ": crow_window_ptr must hold windows + 1 entries");
    same_device({&crow_window_ptr, &unique_col_ids, &value}, dense, op);
    const int itype = index_code({&crow_window_ptr, &unique_col_ids}, op);
    c10::cuda::CUDAGuard guard(dense.device());

    const int64_t nwin = crow_window_ptr.size(0) - 1, D = dense.size(1), ntiles = unique_col_ids.size(0) / 16;
    at::Tensor result = at::empty({nwin * 16, D}, dense.options());
    const int dt = dtype_code(dense);
    const size_t wbytes = spmm_ascend_cube_tiles_workspace_bytes(nwin, ntiles, D, itype, dt);
    at::Tensor ws = workspace(wbytes, dense);
    const at::Tensor B = aligned16(dense);
    check_rc(spmm_ascend_cube_tiles_launch(crow_window_ptr.data_ptr(), unique_col_ids.data_ptr(), value.data_ptr(),
                                           B.data_ptr(), result.data_ptr(), nwin, ntiles, dense.size(0), D, itype, dt,
                                           ws.data_ptr(), wbytes, stream_of(dense)));
    return result;
}

// ---------------------------------------------------------------------------
// Layout builders: csr_to_bcsr, csr_to_ascend_cube, block_level_split,
// preprocess (custom_op.cpp:429-1412).  Same argument order and dict keys as
// the reference; inputs may be CPU or CUDA tensors (CPU inputs are copied to
// the current CUDA device - no CPU compute) and every output lives on that
// device.  Index outputs keep the input index dtype; permutations and audit
// counters are int64, costs float64 (custom_op.cpp:1037-1109).
// ---------------------------------------------------------------------------

// spmm_allocator backed by the torch caching allocator: every block is a
// uint8 tensor kept alive in `live` until handed out as an output or
// released as a temporary.
struct TorchAllocator {
    at::TensorOptions opts;
    std::unordered_map<void *, at::Tensor> live;
    spmm_allocator handle;

    explicit TorchAllocator(const at::Device &dev) : opts(at::TensorOptions().device(dev).dtype(at::kByte))
    {
        handle.ctx = this;
        handle.alloc = &TorchAllocator::alloc;
        handle.release = &TorchAllocator::release;
    }
    static void *alloc(void *ctx, size_t bytes)
    {
        auto *self = static_cast<TorchAllocator *>(ctx);
        try {
            at::Tensor t = at::empty({(int64_t)bytes}, self->opts);
            void *p = t.data_ptr();
            self->live.emplace(p, std::move(t));
            return p;
        } catch (...) {
            return nullptr;
        }
    }
    static void release(void *ctx, void *p) { static_cast<TorchAllocator *>(ctx)->live.erase(p); }
    at::Tensor take(const spmm_array &a, at::ScalarType st)
    {
        if (a.len == 0 || a.data == nullptr) return at::empty({0}, opts.dtype(st));
        auto it = live.find(a.data);
        TORCH_CHECK(it != live.end(), "internal: output array not owned by the allocator");
        at::Tensor raw = it->second;
        live.erase(it);
        return raw.narrow(0, 0, a.len * (int64_t)c10::elementSize(st)).view(st);
    }
};

struct CsrInput {
    at::Tensor crow, col, val;
    int itype;
    int vbytes;
};

CsrInput prepare_csr(const at::Tensor &crow_ptr, const at::Tensor &col_indices, const at::Tensor &values,
                     const char *op)
{
    TORCH_CHECK(crow_ptr.dim() == 1 && col_indices.dim() == 1 && values.dim() == 1, op,
                ": crow_ptr, col_indices and values must be one-dimensional");
    TORCH_CHECK(crow_ptr.scalar_type() == at::kInt || crow_ptr.scalar_type() == at::kLong, op,
                ": index tensors must be int32 or int64");
    TORCH_CHECK(col_indices.scalar_type() == crow_ptr.scalar_type(), op,
                ": crow_ptr and col_indices must have the same dtype");
    const at::ScalarType vt = values.scalar_type();
    TORCH_CHECK(vt == at::kHalf || vt == at::kFloat || vt == at::kDouble, op,
                ": values must be float16, float32 or float64");
    TORCH_CHECK(values.size(0) == col_indices.size(0), op, ": col_indices and values must have equal length");
    TORCH_CHECK(crow_ptr.size(0) >= 1, op, ": crow_ptr must hold nrows + 1 entries");
    at::Device dev = crow_ptr.is_cuda() ? crow_ptr.device()
                                        : at::Device(at::kCUDA, c10::cuda::current_device());
    auto to_dev = [&](const at::Tensor &t) { return t.to(dev).contiguous(); };
    CsrInput in{to_dev(crow_ptr), to_dev(col_indices), aligned16(to_dev(values)),
                crow_ptr.scalar_type() == at::kInt ? SPMM_I32 : SPMM_I64, (int)values.element_size()};
    return in;
}

void check_rows(const CsrInput &in, int64_t nrows, const char *op)
{
    TORCH_CHECK(nrows >= 0 && in.crow.size(0) == nrows + 1, op, ": crow_ptr must hold nrows + 1 = ", nrows + 1,
                " entries, but has ", in.crow.size(0));
}

// Layout dict keys of a (window, CSR) pair.
void put_layout(std::map<std::string, at::Tensor> &d, TorchAllocator &A, const spmm_layout &L, at::ScalarType it,
                at::ScalarType vt, const std::string &prefix, bool with_v)
{
    d[prefix + "crow_window_ptr"] = A.take(L.crow_window_ptr, it);
    d[prefix + "unique_col_ids"] = A.take(L.unique_col_ids, it);
    d[prefix + "value"] = A.take(L.value, vt);
    if (with_v) {
        d[prefix + "vrow_window_ptr"] = A.take(L.vrow_window_ptr, it);
        d[prefix + "vcol_indices"] = A.take(L.vcol_indices, it);
        d[prefix + "vvalue"] = A.take(L.vvalue, vt);
    }
}

// Preprocessing errors: occupancy violations raise ValueError like the
// reference's std::invalid_argument (extension/boundary_bucket_sort.h:34).
void check_pre(int rc)
{
    if (rc == SPMM_OK) return;
    const std::string msg = spmm_last_error();
    if (msg.find("block occupancy") != std::string::npos) throw std::invalid_argument(msg);
    TORCH_CHECK(false, msg);
}

std::map<std::string, at::Tensor> csr_to_bcsr(at::Tensor crow_ptr, at::Tensor col_indices, at::Tensor values,
                                              int64_t nrows, int64_t ncols, int64_t window_size)
{
    CsrInput in = prepare_csr(crow_ptr, col_indices, values, "csr_to_bcsr");
    check_rows(in, nrows, "csr_to_bcsr");
    c10::cuda::CUDAGuard guard(in.crow.device());
    TorchAllocator A(in.crow.device());
    spmm_layout L{};
    check_pre(spmm_csr_to_bcsr_run(in.crow.data_ptr(), in.col.data_ptr(), in.val.data_ptr(), nrows, ncols,
                                   in.col.size(0), window_size, in.itype, in.vbytes, &A.handle, &L, stream_of(in.crow)));
    std::map<std::string, at::Tensor> d;
    put_layout(d, A, L, crow_ptr.scalar_type(), values.scalar_type(), "", false);
    return d;
}

std::map<std::string, at::Tensor> csr_to_ascend_cube(at::Tensor crow_ptr, at::Tensor col_indices, at::Tensor values,
                                                     int64_t nrows, int64_t ncols, int64_t window_size)
{
    CsrInput in = prepare_csr(crow_ptr, col_indices, values, "csr_to_ascend_cube");
    check_rows(in, nrows, "csr_to_ascend_cube");
    c10::cuda::CUDAGuard guard(in.crow.device());
    TorchAllocator A(in.crow.device());
    spmm_layout L{};
    check_pre(spmm_csr_to_ascend_cube_run(in.crow.data_ptr(), in.col.data_ptr(), in.val.data_ptr(), nrows, ncols,
                                          in.col.size(0), window_size, in.itype, in.vbytes, &A.handle, &L,
                                          stream_of(in.crow)));
    std::map<std::string, at::Tensor> d;
    put_layout(d, A, L, crow_ptr.scalar_type(), values.scalar_type(), "", false);
    return d;
}

// Producer of spmm_cube's input: {"rowptr", "col", "value"}.
std::map<std::string, at::Tensor> csr_to_spmm_cube(at::Tensor crow_ptr, at::Tensor col_indices, at::Tensor values,
                                                   int64_t nrows, int64_t ncols, int64_t window_size)
{
    CsrInput in = prepare_csr(crow_ptr, col_indices, values, "csr_to_spmm_cube");
    check_rows(in, nrows, "csr_to_spmm_cube");
    c10::cuda::CUDAGuard guard(in.crow.device());
    TorchAllocator A(in.crow.device());
    spmm_layout L{};
    check_pre(spmm_csr_to_spmm_cube_run(in.crow.data_ptr(), in.col.data_ptr(), in.val.data_ptr(), nrows, ncols,
                                        in.col.size(0), window_size, in.itype, in.vbytes, &A.handle, &L,
                                        stream_of(in.crow)));
    std::map<std::string, at::Tensor> d;
    d["rowptr"] = A.take(L.crow_window_ptr, crow_ptr.scalar_type());
    d["col"] = A.take(L.unique_col_ids, crow_ptr.scalar_type());
    d["value"] = A.take(L.value, values.scalar_type());
    return d;
}

std::map<std::string, at::Tensor> block_level_split(at::Tensor crow_ptr, at::Tensor col_indices, at::Tensor values,
                                                    int64_t nrows, int64_t ncols, double a, int64_t window_size)
{
    CsrInput in = prepare_csr(crow_ptr, col_indices, values, "block_level_split");
    check_rows(in, nrows, "block_level_split");
    c10::cuda::CUDAGuard guard(in.crow.device());
    TorchAllocator A(in.crow.device());
    spmm_layout L{};
    check_pre(spmm_block_level_split_run(in.crow.data_ptr(), in.col.data_ptr(), in.val.data_ptr(), nrows, ncols,
                                         in.col.size(0), a, window_size, in.itype, in.vbytes, &A.handle, &L,
                                         stream_of(in.crow)));
    std::map<std::string, at::Tensor> d;
    put_layout(d, A, L, crow_ptr.scalar_type(), values.scalar_type(), "", true);
    return d;
}

std::map<std::string, at::Tensor> preprocess(at::Tensor crow_ptr, at::Tensor col_indices, at::Tensor values,
                                             int64_t nrows, int64_t ncols, int64_t window_size, bool graph_layout)
{
    CsrInput in = prepare_csr(crow_ptr, col_indices, values, "preprocess");
    check_rows(in, nrows, "preprocess");
    c10::cuda::CUDAGuard guard(in.crow.device());
    TorchAllocator A(in.crow.device());
    spmm_preprocess_result R{};
    check_pre(spmm_preprocess_run(in.crow.data_ptr(), in.col.data_ptr(), in.val.data_ptr(), nrows, ncols,
                                  in.col.size(0), window_size, graph_layout ? 1 : 0, in.itype, in.vbytes, &A.handle,
                                  &R, stream_of(in.crow)));
    const at::ScalarType it = crow_ptr.scalar_type(), vt = values.scalar_type();
    std::map<std::string, at::Tensor> d;
    put_layout(d, A, R.fwd, it, vt, "", true);
    d["renumbered_unique_col_ids"] = A.take(R.renumbered_unique_col_ids, it);
    d["renumbered_vcol_indices"] = A.take(R.renumbered_vcol_indices, it);
    put_layout(d, A, R.transpose, it, vt, "transpose_", true);
    d["permutation"] = A.take(R.permutation, at::kLong);
    d["inv_permutation"] = A.take(R.inv_permutation, at::kLong);
    auto dev = in.crow.device();
    auto i64 = [&](int64_t v) { return at::full({1}, v, at::TensorOptions().dtype(at::kLong).device(dev)); };
    auto f64 = [&](double v) { return at::full({1}, v, at::TensorOptions().dtype(at::kDouble).device(dev)); };
    d["packed_rows"] = i64(R.packed_rows);
    d["packed_layout_supported"] = i64(R.packed_layout_supported);
    d["marginal_window"] = i64(R.marginal_window);
    d["marginal_aic_blocks"] = i64(R.marginal_aic_blocks);
    d["marginal_total_blocks"] = i64(R.marginal_total_blocks);
    d["shared_windows"] = i64(R.shared_windows);
    d["estimated_aic_cost"] = f64(R.estimated_aic_cost);
    d["estimated_aiv_cost"] = f64(R.estimated_aiv_cost);
    d["estimated_max_cost"] = f64(R.estimated_max_cost);
    return d;
}

// Row permutation helpers behind pack_node_tensor / restore_node_tensor
// (spmm_npu.py:22-61); argument checks with the reference's messages stay in
// the Python wrappers.
at::Tensor pack_rows(const at::Tensor &tensor, const at::Tensor &index, int64_t packed_rows)
{
    TORCH_CHECK_CUDA(tensor);
    TORCH_CHECK_CUDA(index);
    TORCH_CHECK(index.scalar_type() == at::kLong && index.is_contiguous(), "pack_rows: index must be contiguous int64");
    TORCH_CHECK(tensor.is_contiguous() && tensor.dim() >= 1, "pack_rows: tensor must be contiguous, dim >= 1");
    TORCH_CHECK(index.numel() == tensor.size(0), "pack_rows: one index per row");
    c10::cuda::CUDAGuard guard(tensor.device());
    std::vector<int64_t> shape(tensor.sizes().begin(), tensor.sizes().end());
    shape[0] = packed_rows;
    at::Tensor out = at::empty(shape, tensor.options());
    const int64_t row_bytes = tensor.size(0) ? tensor.nbytes() / tensor.size(0) : 0;
    check_rc(spmm_pack_rows_launch(tensor.data_ptr(), index.data_ptr<int64_t>(), tensor.size(0), row_bytes,
                                   out.data_ptr(), packed_rows, stream_of(tensor)));
    return out;
}

at::Tensor restore_rows(const at::Tensor &packed, const at::Tensor &index)
{
    TORCH_CHECK_CUDA(packed);
    TORCH_CHECK_CUDA(index);
    TORCH_CHECK(index.scalar_type() == at::kLong && index.is_contiguous(), "restore_rows: index must be contiguous int64");
    TORCH_CHECK(packed.is_contiguous() && packed.dim() >= 1, "restore_rows: tensor must be contiguous, dim >= 1");
    c10::cuda::CUDAGuard guard(packed.device());
    std::vector<int64_t> shape(packed.sizes().begin(), packed.sizes().end());
    shape[0] = index.numel();
    at::Tensor out = at::empty(shape, packed.options());
    int64_t row_bytes = 1;
    for (size_t d = 1; d < shape.size(); ++d) row_bytes *= shape[d];
    row_bytes *= packed.element_size();
    check_rc(spmm_restore_rows_launch(packed.data_ptr(), packed.size(0), index.data_ptr<int64_t>(), index.numel(),
                                      row_bytes, out.data_ptr(), stream_of(packed)));
    return out;
}

// Sticky device status (code, detail), optionally cleared.  Synchronises.
std::tuple<int64_t, int64_t> device_status(bool reset)
{
    int code = 0;
    int64_t detail = 0;
    check_rc(spmm_device_status(&code, &detail, reset ? 1 : 0,
                                static_cast<void *>(at::cuda::getCurrentCUDAStream().stream())));
    return {code, detail};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m)
{
    m.def("spmm_csr", &spmm_csr_impl,
          "CUDA CSR SpMM; FP16 width divisible by 16 with MAXD=1024, FP32 width divisible by 8 with MAXD=512");
    m.def("spmm_csr_multicast", &spmm_csr_multicast_impl,
          "this rank's rows of A @ B stored through an NVLink multicast address of out (every bound copy)");
    m.def("spmm_cube", &spmm_cube_impl,
          "CUDA window SpMM over (column << 4 | row) entries; width divisible by 16, MAXD=1024 for FP16 and 512 "
          "for FP32");
    m.def("spmm_ascend_cube_tiles", &spmm_ascend_cube_tiles_impl,
          "CUDA SpMM over csr_to_ascend_cube's 16 x 16 tiles (crow_window_ptr, unique_col_ids, value, dense); "
          "width divisible by 16, MAXD=1024 for FP16 and 512 for FP32");
    m.def("spmm_ascend_cube", &spmm_ascend_cube_impl,
          "CUDA mixed window/CSR SpMM; width divisible by 16, MAXD=1024 for FP16 and 512 for FP32");
    m.def("spmm_ascend_cube_aic_without_pipeline", &spmm_ascend_cube_aic_without_pipeline_impl,
          "Window-path ablation: single-stage block stream instead of the multi-stage ring");
    m.def("spmm_ascend_cube_aiv_mb", &spmm_ascend_cube_aiv_mb_impl,
          "CSR-path ablation: deeper gather batches (bitwise-identical CSR results)");
    m.def("spmm_csr_aiv_mb_batch", &spmm_csr_aiv_mb_batch_impl,
          "CSR ablation: deeper gather batches (bitwise-identical results)");
    m.def("csr_to_ascend_cube", &csr_to_ascend_cube,
          "Convert CSR to the 16 x 16 tile format on the GPU (rows must be sorted). Returns dict with keys "
          "crow_window_ptr [nwindows + 1], unique_col_ids [total_blocks * 16], value [total_blocks * 256]",
          pybind11::arg("crow_ptr"), pybind11::arg("col_indices"), pybind11::arg("values"), pybind11::arg("nrows"),
          pybind11::arg("ncols"), pybind11::arg("window_size") = 16);
    m.def("csr_to_bcsr", &csr_to_bcsr,
          "Convert CSR to BCSR(16 x 1) on the GPU (rows must be sorted). Returns dict with keys "
          "crow_window_ptr [nwindows + 1], unique_col_ids [total_blocks], value [total_blocks * 16]",
          pybind11::arg("crow_ptr"), pybind11::arg("col_indices"), pybind11::arg("values"), pybind11::arg("nrows"),
          pybind11::arg("ncols"), pybind11::arg("window_size") = 16);
    m.def("preprocess", &preprocess,
          "Partition coalesced CSR by the calibrated 295/505 GB/s window/CSR bandwidths on the GPU; returns the "
          "packed window/CSR tensors, row permutations and audit fields (and with graph_layout=True on a square "
          "graph the P*A*P^T relabel and its fixed-layout transpose), bit-exact with the reference.",
          pybind11::arg("crow_ptr"), pybind11::arg("col_indices"), pybind11::arg("values"), pybind11::arg("nrows"),
          pybind11::arg("ncols"), pybind11::arg("window_size") = 16, pybind11::arg("graph_layout") = false);
    m.def("csr_to_spmm_cube", &csr_to_spmm_cube,
          "Encode CSR for spmm_cube on the GPU: dict with rowptr [nwindows + 1] (entry offsets per 16-row window), "
          "col [nnz] = (column << 4) | row in (column, row) order per window, value [nnz]",
          pybind11::arg("crow_ptr"), pybind11::arg("col_indices"), pybind11::arg("values"), pybind11::arg("nrows"),
          pybind11::arg("ncols"), pybind11::arg("window_size") = 16);
    m.def("block_level_split", &block_level_split,
          "Split CSR into (16,1)-BSR + CSR hybrid dict by block density (GPU)", pybind11::arg("crow_ptr"),
          pybind11::arg("col_indices"), pybind11::arg("values"), pybind11::arg("nrows"), pybind11::arg("ncols"),
          pybind11::arg("a"), pybind11::arg("window_size") = 16);
    m.def("pack_rows", &pack_rows, "dst[index[i]] = src[i]; other rows zero (pack_node_tensor helper)");
    m.def("restore_rows", &restore_rows, "dst[i] = src[index[i]] (restore_node_tensor helper)");
    m.def("device_status", &device_status, "Sticky device-side validation status (code, detail)",
          pybind11::arg("reset") = false);
}
