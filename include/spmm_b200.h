/*
 * spmm_b200.h - C ABI of the B200 SpMM engine (libspmm_b200.so).
 *
 * Plain pointers, sizes and status codes; no framework types.  Every SpMM
 * entry point mirrors one operator of the reference's `spmm_npu` module
 * (IDMG-Lab/Ascend-SpMM, extension/custom_op.cpp) and is what an FFI
 * binding of that operator calls.  Citations are path:line in the
 * reference project.
 *
 * Conventions
 *   - All array pointers are DEVICE pointers on the current CUDA device,
 *     contiguous, unless stated otherwise.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *     Launches are asynchronous on that stream, like the reference's
 *     EXEC_NPU_CMD on the current NPU stream (pytorch_npu_helper.hpp:516-581).
 *   - Index arrays are int32 (SPMM_I32) or int64 (SPMM_I64): the reference
 *     registers both index types (kernels/op_host/spmm_ascend_cube.cpp:77-126).
 *   - Value/dense/output dtype is SPMM_F16 or SPMM_F32; products accumulate
 *     in fp32 and the fp16 output is rounded to nearest once.
 *   - The `start` arrays of the reference ops (per-core first rows,
 *     tests/task_mapping/common.py:119-127) are accepted for signature
 *     compatibility and ignored: the engine plans its own nnz-balanced split.
 *   - Ops that need scratch take a caller-provided device workspace whose
 *     size the matching *_workspace_bytes() reports; they allocate nothing.
 *   - Output arrays are fully written by the launch (no pre-zeroing needed).
 *   - Invalid indices found on the device never fault: the entry is skipped
 *     and a sticky device status is raised (spmm_device_status()).
 *
 * Return value: SPMM_OK or an SPMM_ERR_* code; spmm_last_error() gives a
 * message (thread-local, valid until the next call on the same thread).
 */
#ifndef SPMM_B200_H_
#define SPMM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum spmm_status {
    SPMM_OK = 0,
    SPMM_ERR_ARG = 1,          /* invalid argument (shape, dtype, contract) */
    SPMM_ERR_CUDA = 2,         /* a CUDA runtime call failed */
    SPMM_ERR_DEVICE_CHECK = 3, /* device-side validation found invalid data */
    SPMM_ERR_UNSUPPORTED = 4,  /* valid request this build does not serve */
    SPMM_ERR_ALLOC = 5,        /* the caller's allocator returned NULL */
    SPMM_ERR_WORKSPACE = 6     /* workspace smaller than *_workspace_bytes() */
};

enum spmm_dtype { SPMM_F16 = 0, SPMM_F32 = 1, SPMM_F64 = 2 };
enum spmm_itype { SPMM_I32 = 0, SPMM_I64 = 1 };

/* Device-status codes raised by kernels (see spmm_device_status). */
enum spmm_device_code {
    SPMM_DEV_OK = 0,
    SPMM_DEV_BAD_COLUMN = 1,   /* a column index outside [0, K) was skipped */
    SPMM_DEV_BAD_ROWPTR = 2,   /* a row pointer was non-monotone or > nnz */
    SPMM_DEV_UNSORTED = 3,     /* a row's columns are not strictly ascending */
    SPMM_DEV_OCCUPANCY = 4,    /* a block column occupied > window_size times */
    SPMM_DEV_TIMEOUT = 5       /* a bounded device wait gave up */
};

const char *spmm_last_error(void);
int spmm_abi_version(void);

/* Sticky device status of the current device: first error code and a detail
 * value (the offending position).  Synchronises `stream`.  With reset != 0
 * the status is cleared after reading. */
int spmm_device_status(int *code, int64_t *detail, int reset, void *stream);

/* ---------------------------------------------------------------------- */
/* CSR SpMM: out[M, N] = A[M, K] * dense[K, N].                            */
/* Replaces spmm_csr_impl_npu (extension/custom_op.cpp:67-88; kernel       */
/* kernels/op_kernel/spmm_csr.cpp:226-569).  Width contract: fp16 N % 16,  */
/* N <= 1024; fp32 N % 8, N <= 512 (custom_op.cpp:39-57).                   */
/* ---------------------------------------------------------------------- */
size_t spmm_csr_workspace_bytes(int64_t M, int64_t N, int64_t nnz, int dtype);

int spmm_csr_launch(const void *rowptr, const void *col, const void *value,
                    const void *dense, const int32_t *start, int64_t n_start,
                    void *out, int64_t M, int64_t K, int64_t N, int64_t nnz,
                    int itype, int dtype, void *workspace, size_t workspace_bytes,
                    void *stream);

/* L2 residency plan of spmm_csr_launch (no counterpart in the reference:
 * the 910B's gathers have no L2 eviction priorities).  For rows of B of at
 * least 1 KB, a dense operand of at least 16x the L2 size and at least 2^26
 * nonzeros (SPMM_B200_L2PLAN=on: any size, =off: never), the launch first
 * samples 2^22 column indices on the device, marks the hottest B rows that
 * fit in half of L2, and - when they hold at least a quarter of the samples
 * - gathers them with an evict_last L2 policy and the other rows with
 * evict_first.  Results are bitwise the same either way; the plan lives in
 * the workspace.  This returns the byte offset of its header inside a
 * spmm_csr workspace (SIZE_MAX when the problem reserves no plan); after a
 * launch the header holds: */
struct spmm_l2_plan_header {
    uint32_t threshold;      /* a column bin is hot at this many samples (0: none) */
    uint32_t hot_bins;       /* hot bins (column id modulo 2^24) */
    uint32_t budget;         /* hot bins allowed: half of L2 in B rows */
    uint32_t reserved;
    uint64_t samples;        /* column indices sampled */
    uint64_t hot_samples;    /* of which in hot bins; enabled when 4x >= samples */
};
size_t spmm_csr_l2_plan_offset(int64_t M, int64_t N, int64_t nnz, int dtype);

/* Replaces spmm_csr_aiv_mb_batch_impl_npu (custom_op.cpp:154-187; kernel
 * kernels/op_kernel/spmm_csr_aiv_mb_batch.cpp).  Same math and the same
 * nnz split as spmm_csr_launch (bitwise-identical output); it issues its
 * gathers in deeper batches.  Same workspace. */
int spmm_csr_aiv_mb_batch_launch(const void *rowptr, const void *col, const void *value,
                                 const void *dense, const int32_t *start, int64_t n_start,
                                 void *out, int64_t M, int64_t K, int64_t N, int64_t nnz,
                                 int itype, int dtype, void *workspace,
                                 size_t workspace_bytes, void *stream);

/* Row-sharded CSR SpMM with the whole C replicated on every GPU of a job
 * (one process per GPU, each multiplying its own row shard): as
 * spmm_csr_launch, but every row of this call's C is stored once through
 * `out_multicast`, an NVLink multicast (NVLS) address of `out` - the
 * multicast object binds the same buffer of every GPU at the same offset -
 * so the switch writes each row into all copies while the kernel runs; `out`
 * itself receives the rows the same way.  The caller puts a cross-GPU
 * barrier after the call before any GPU reads the copies.  No counterpart in
 * the reference (a single-device operator): the multi-GPU form of
 * spmm_csr_impl_npu (extension/custom_op.cpp:67-88) fused with the row all-gather
 * that would follow it.  Same workspace as spmm_csr_launch; out_multicast
 * 16-byte aligned. */
int spmm_csr_launch_multicast(const void *rowptr, const void *col, const void *value,
                              const void *dense, void *out, void *out_multicast, int64_t M,
                              int64_t K, int64_t N, int64_t nnz, int itype, int dtype,
                              void *workspace, size_t workspace_bytes, void *stream);

/* CSR SpMM for callers that cannot allocate device memory when they call
 * (for example a service binding this ABI through cgo/JNI/FFI with a device
 * memory budget fixed at start-up, or a latency-critical loop where a
 * cudaMalloc would synchronise the device).  No counterpart in the
 * reference: it is spmm_csr_launch without the workspace argument.  Its
 * scratch (fp32 partial rows) lives in a 32 MiB static device array that
 * every GPU loading this library keeps until the process exits; it
 * allocates nothing, neither by CUDA nor by any library.  The first call on
 * a device looks the array up with cudaGetSymbolAddress, so make that first
 * call before any stream capture.  Problems whose partial rows do not fit
 * even with coarser work units return SPMM_ERR_UNSUPPORTED.  All calls share
 * the array: calls that overlap on the GPU (other streams or threads) race. */
int spmm_csr_launch_noalloc(const void *rowptr, const void *col, const void *value, const void *dense,
                            void *out, int64_t M, int64_t K, int64_t N, int64_t nnz, int itype, int dtype,
                            void *stream);

/* ---------------------------------------------------------------------- */
/* Mixed window/CSR SpMM.  Output rows = max(16 * n_windows, v_rows)       */
/* (custom_op.cpp:146).  Window slot s adds its (16 x 1)-block products to  */
/* rows [16s, 16s + 16); the CSR part adds to its own rows; both parts are */
/* summed in fp32 before a single rounding.                                */
/* Replaces spmm_ascend_cube_impl_npu (custom_op.cpp:115-152; kernel        */
/* kernels/op_kernel/spmm_ascend_cube.cpp:887-907).  N % 16 == 0.           */
/*   Crowptr  [n_windows + 1]  block offsets per window                     */
/*   Ccol_ids [n_blocks]       block column ids                             */
/*   Cvalue   [16 * n_blocks]  Cvalue[16 b + i] = A[row i of window, col b] */
/*   Vrowptr  [v_rows + 1], Vcol_ids [v_nnz], Vvalue [v_nnz]                */
/* The workspace holds the window kernel's item schedule (heavy windows    */
/* first, claimed dynamically; 8 bytes per window and 64-feature slice)    */
/* and the scratch of the CSR rows beyond the windows.                     */
/* ---------------------------------------------------------------------- */
size_t spmm_ascend_cube_workspace_bytes(int64_t n_windows, int64_t n_blocks, int64_t v_rows,
                                        int64_t v_nnz, int64_t N, int dtype);

int spmm_ascend_cube_launch(const void *Crowptr, const void *Ccol_ids, const void *Cvalue,
                            const void *Vrowptr, const void *Vcol_ids, const void *Vvalue,
                            const void *dense, const int32_t *Cstart, int64_t n_cstart,
                            const int32_t *Vstart, int64_t n_vstart, void *out,
                            int64_t n_windows, int64_t n_blocks, int64_t v_rows, int64_t v_nnz,
                            int64_t K, int64_t N, int itype, int dtype, void *workspace,
                            size_t workspace_bytes, void *stream);

/* Replaces spmm_ascend_cube_aic_without_pipeline_impl_npu (custom_op.cpp:
 * 189-245): the window path with a single-stage (unpipelined) block stream,
 * the analogue of the reference's SPTILE=16 ablation. Same arguments. */
int spmm_ascend_cube_aic_without_pipeline_launch(
    const void *Crowptr, const void *Ccol_ids, const void *Cvalue, const void *Vrowptr,
    const void *Vcol_ids, const void *Vvalue, const void *dense, const int32_t *Cstart,
    int64_t n_cstart, const int32_t *Vstart, int64_t n_vstart, void *out, int64_t n_windows,
    int64_t n_blocks, int64_t v_rows, int64_t v_nnz, int64_t K, int64_t N, int itype,
    int dtype, void *workspace, size_t workspace_bytes, void *stream);

/* Replaces spmm_ascend_cube_aiv_mb_impl_npu (custom_op.cpp:247-264): the CSR
 * part with deeper gather batching (bitwise-identical CSR results). */
int spmm_ascend_cube_aiv_mb_launch(
    const void *Crowptr, const void *Ccol_ids, const void *Cvalue, const void *Vrowptr,
    const void *Vcol_ids, const void *Vvalue, const void *dense, const int32_t *Cstart,
    int64_t n_cstart, const int32_t *Vstart, int64_t n_vstart, void *out, int64_t n_windows,
    int64_t n_blocks, int64_t v_rows, int64_t v_nnz, int64_t K, int64_t N, int itype,
    int dtype, void *workspace, size_t workspace_bytes, void *stream);

/* Replaces spmm_cube_impl_npu (custom_op.cpp:91-113; kernel
 * op_kernel/spmm_cube.cpp:51-147).  rowptr [n_windows + 1] holds the entry
 * offsets of each 16-row window; col[i] = (column << 4) | row; output
 * [16 * n_windows, N].  Inside a window, a run of entries with equal column
 * is one (16 x 1) block and the last entry of a row in a run wins.  fp16
 * and fp32 widths: N % 16 == 0 (custom_op.cpp:102).  The workspace holds the
 * normalised block stream (bounded by nnz blocks). */
size_t spmm_cube_workspace_bytes(int64_t n_windows, int64_t nnz, int64_t N, int itype, int dtype);
int spmm_cube_launch(const void *rowptr, const void *col, const void *value, const void *dense,
                     const int32_t *start, int64_t n_start, void *out, int64_t n_windows, int64_t K,
                     int64_t N, int64_t nnz, int itype, int dtype, void *workspace,
                     size_t workspace_bytes, void *stream);

/* Consumer of csr_to_ascend_cube's 16 x 16 tiles (custom_op.cpp:429-592;
 * the reference ships the producer only).  crow_window_ptr [n_windows + 1]
 * in tiles, unique_col_ids [16 * n_tiles], value [256 * n_tiles] with
 * value[256 t + 16 row + k]; output [16 * n_windows, N], rows in original
 * order.  Padding columns of a window's last tile (column 0, values 0) are
 * summed like any other entry.  N % 16 == 0 for fp16 and fp32; with int32
 * indices 16 * n_tiles must fit in int32. */
size_t spmm_ascend_cube_tiles_workspace_bytes(int64_t n_windows, int64_t n_tiles, int64_t N, int itype,
                                              int dtype);
int spmm_ascend_cube_tiles_launch(const void *crow_window_ptr, const void *unique_col_ids, const void *value,
                                  const void *dense, void *out, int64_t n_windows, int64_t n_tiles, int64_t K,
                                  int64_t N, int itype, int dtype, void *workspace, size_t workspace_bytes,
                                  void *stream);

/* ---------------------------------------------------------------------- */
/* Layout builders (GPU, bit-exact with the reference's CPU preprocessing). */
/* Inputs: CSR on the device (crow [nrows + 1], col [nnz], val [nnz] with  */
/* val element size vbytes = 2, 4 or 8).  Output sizes depend on the data, */
/* so these calls synchronise `stream`; every output and temporary array is */
/* obtained from the caller's allocator (outputs stay owned by the caller, */
/* temporaries are handed back through `release`).  Output index arrays    */
/* have the input index type; empty arrays have data == NULL, len == 0.    */
/* ---------------------------------------------------------------------- */
typedef struct spmm_allocator {
    void *ctx;
    void *(*alloc)(void *ctx, size_t bytes);  /* device memory, >= 16-byte aligned; NULL on failure */
    void (*release)(void *ctx, void *ptr);    /* temporaries; may be NULL */
} spmm_allocator;

typedef struct spmm_array {
    void *data;   /* device pointer */
    int64_t len;  /* elements */
} spmm_array;

typedef struct spmm_layout {
    spmm_array crow_window_ptr, unique_col_ids, value;
    spmm_array vrow_window_ptr, vcol_indices, vvalue;
} spmm_layout;

typedef struct spmm_preprocess_result {
    spmm_layout fwd;
    spmm_layout transpose;                       /* graph layout only */
    spmm_array renumbered_unique_col_ids;        /* graph layout only */
    spmm_array renumbered_vcol_indices;          /* graph layout only */
    spmm_array permutation;                      /* int64 [packed_rows] */
    spmm_array inv_permutation;                  /* int64 [nrows] */
    int64_t packed_rows, packed_layout_supported, marginal_window, marginal_aic_blocks,
        marginal_total_blocks, shared_windows;
    double estimated_aic_cost, estimated_aiv_cost, estimated_max_cost;
} spmm_preprocess_result;

/* Replaces csr_to_bcsr / ToBCSR (custom_op.cpp:594-746): per 16-row window,
 * ascending distinct columns; value[16 b + row].  Rows must be sorted. */
int spmm_csr_to_bcsr_run(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                         int64_t nnz, int64_t window_size, int itype, int vbytes,
                         const spmm_allocator *alloc, spmm_layout *out, void *stream);

/* Replaces csr_to_ascend_cube (custom_op.cpp:429-592): distinct columns in
 * 16-column tiles (last tile zero-padded); value[256 t + 16 row + k]. */
int spmm_csr_to_ascend_cube_run(const void *crow, const void *col, const void *val, int64_t nrows,
                                int64_t ncols, int64_t nnz, int64_t window_size, int itype, int vbytes,
                                const spmm_allocator *alloc, spmm_layout *out, void *stream);

/* Producer of spmm_cube's input (the reference ships the consumer only):
 * crow_window_ptr [nwin + 1] = crow[min(16 w, nrows)], unique_col_ids [nnz]
 * = (column << 4) | row with each window's entries in (column, row) order
 * (ToBCSR's merge order, custom_op.cpp:611-671; equal pairs keep CSR
 * order), value [nnz].  vrow/vcol/vvalue stay empty.  With int32 indices
 * ncols must be <= 2^27 so the encoding fits. */
int spmm_csr_to_spmm_cube_run(const void *crow, const void *col, const void *val, int64_t nrows,
                              int64_t ncols, int64_t nnz, int64_t window_size, int itype, int vbytes,
                              const spmm_allocator *alloc, spmm_layout *out, void *stream);

/* Replaces block_level_split / hybrid_split_impl (custom_op.cpp:1146-1348,
 * 1390-1412): the k least-dense blocks move to CSR, k = first argmin of
 * |(#blocks - k) / moved_nnz - a|. */
int spmm_block_level_split_run(const void *crow, const void *col, const void *val, int64_t nrows,
                               int64_t ncols, int64_t nnz, double a, int64_t window_size, int itype,
                               int vbytes, const spmm_allocator *alloc, spmm_layout *out, void *stream);

/* Replaces preprocess / taskmapping (custom_op.cpp:765-1137): calibrated
 * 295/505 GB/s window split, marginal-window block split, packed row order,
 * window and CSR packs; with graph_layout on a square matrix also the
 * P A P^T relabel and its fixed-layout transpose. */
int spmm_preprocess_run(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                        int64_t nnz, int64_t window_size, int graph_layout, int itype, int vbytes,
                        const spmm_allocator *alloc, spmm_preprocess_result *out, void *stream);

/* ---------------------------------------------------------------------- */
/* Graph-layout row permutation (P and P^T on node tensors).               */
/* ---------------------------------------------------------------------- */

/* Replaces pack_node_tensor (spmm_npu.py:22-47): dst[inv[i], :] = src[i, :]
 * for i < n; all other of the packed_rows rows of dst are zeroed.  Rows are
 * row_bytes bytes; inv is int64 on the device. */
int spmm_pack_rows_launch(const void *src, const int64_t *inv, int64_t n, int64_t row_bytes, void *dst,
                          int64_t packed_rows, void *stream);

/* Replaces restore_node_tensor (spmm_npu.py:50-61): dst[i, :] = src[inv[i], :]
 * for i < n; src has src_rows rows. */
int spmm_restore_rows_launch(const void *src, int64_t src_rows, const int64_t *inv, int64_t n,
                             int64_t row_bytes, void *dst, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SPMM_B200_H_ */
