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
    m.def("spmm_ascend_cube", &spmm_ascend_cube_impl,
          "CUDA mixed window/CSR SpMM; width divisible by 16, MAXD=1024 for FP16 and 512 for FP32");
    m.def("spmm_ascend_cube_aic_without_pipeline", &spmm_ascend_cube_aic_without_pipeline_impl,
          "Window-path ablation: single-stage block stream instead of the multi-stage ring");
    m.def("spmm_ascend_cube_aiv_mb", &spmm_ascend_cube_aiv_mb_impl,
          "CSR-path ablation: deeper gather batches (bitwise-identical CSR results)");
    m.def("spmm_csr_aiv_mb_batch", &spmm_csr_aiv_mb_batch_impl,
          "CSR ablation: deeper gather batches (bitwise-identical results)");
    m.def("pack_rows", &pack_rows, "dst[index[i]] = src[i]; other rows zero (pack_node_tensor helper)");
    m.def("restore_rows", &restore_rows, "dst[i] = src[index[i]] (restore_node_tensor helper)");
    m.def("device_status", &device_status, "Sticky device-side validation status (code, detail)",
          pybind11::arg("reset") = false);
}
