// Internal host-side interface between the C ABI (capi.cu) and the kernel
// translation units.  Not installed; the public ABI is include/spmm_b200.h.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/spmm_b200.h"

namespace spmmb {

struct DevStatus;

// Records the thread-local error message of the C ABI and returns `code`.
int capi_error(int code, const char *fmt, ...);

// Argument contract shared by every CSR entry point (capi.cu): the width and
// dtype rules of the reference's check_dense_contract (custom_op.cpp:39-57),
// index type, sizes, null and 16-byte-aligned arrays.  Returns SPMM_OK (also
// for M == 0, when nothing else is checked) or an error code with the
// message set.  Workspace checks stay with each entry point.
int check_csr_args(const void *rowptr, const void *col, const void *value, const void *dense, const void *out,
                   int64_t M, int64_t K, int64_t N, int64_t nnz, int itype, int dtype, const char *op);

// Units of `unit` nonzeros covering nnz (at least one), without the overflow
// of (nnz + unit - 1) / unit near INT64_MAX.
inline int64_t units_for(int64_t nnz, int64_t unit)
{
    const int64_t n = nnz / unit + (nnz % unit != 0);
    return n > 0 ? n : 1;
}

// Per-device sticky status word (status.cu).
DevStatus *device_status_ptr(cudaError_t *err);
int device_sm_count();

// ---- CSR gather path (gather.cu) ------------------------------------------

// Work decomposition of one CSR gather launch: the nonzeros are cut into
// equal units of `unit` positions; rows crossing a unit boundary are summed
// from per-unit fp32 partials by a fix-up pass in unit order, so the result
// is deterministic and independent of the grid.
struct GatherPlan {
    int64_t unit = 0;        // nonzeros per unit
    int64_t unit_begin = 0;  // first unit index (absolute)
    int64_t unit_end = 0;    // one past the last unit
    int64_t N = 0;           // features
    int64_t nunits() const { return unit_end - unit_begin; }
    // fp32 head/tail partial rows, two per unit
    size_t partial_bytes() const { return (size_t)nunits() * 2 * (size_t)N * sizeof(float); }
    // then one int64 per unit boundary (nunits + 1 entries): the first row of
    // each unit for the tensor-core kernel, or the split row of each unit
    // that the ring kernel records for the fix-up
    size_t rows_offset() const { return (partial_bytes() + 255) & ~size_t(255); }
    size_t rows_end() const { return rows_offset() + (size_t)(nunits() + 1) * sizeof(int64_t); }
    // then, when l2 is set, the L2 residency plan of the B rows (l2plan.cu)
    bool l2 = false;
    size_t l2_offset() const { return (rows_end() + 255) & ~size_t(255); }
    size_t workspace_bytes() const { return l2 ? l2_offset() + l2_plan_bytes() : rows_end(); }
    static size_t l2_plan_bytes();
};

// with_l2: reserve the L2 residency plan where l2_plan_wanted() says so
// (spmm_csr and its variants); the mixed operator and the no-allocation
// entry point plan without it.
GatherPlan plan_gather(int64_t nnz, int64_t N, int dtype, bool with_l2 = false);

// ---- L2 residency plan for the B rows (l2plan.cu) ----------------------------
//
// For a dense operand far larger than L2 whose columns are skewed (power-law
// graphs: a few hub rows of B take most of the gathers), L2's replacement
// lets the long tail of once-used B rows evict the hub rows.  The plan
// samples the column indices on the device, marks the hottest columns that
// fit in half of L2 (a bitmap over column ids modulo kL2Bins) and, when the
// marked columns hold at least a quarter of the samples (l2_plan_enabled),
// the ring kernel copies their B rows with an evict_last L2 policy and every
// other B row with evict_first.  Only cache priorities change: results are
// bitwise the same with or without the plan.
constexpr int64_t kL2Bins = int64_t(1) << 24;
struct L2PlanHeader {
    unsigned threshold;      // a bin is hot when its sample count is at least this (0: none)
    unsigned hot_bins;       // bins at or above the threshold (the budget bounds them)
    unsigned budget;         // hot bins allowed: half of L2 in B rows
    unsigned pad;
    unsigned long long samples;      // column indices sampled
    unsigned long long hot_samples;  // of which in hot bins (exact)
    unsigned hist[1024];     // bins by sample count (capped at 1023)
};
static_assert(offsetof(L2PlanHeader, samples) == offsetof(spmm_l2_plan_header, samples) &&
                  offsetof(L2PlanHeader, hot_samples) == offsetof(spmm_l2_plan_header, hot_samples),
              "the public header mirrors the plan's first fields");
__host__ __device__ inline bool l2_plan_enabled(const L2PlanHeader &h)
{
    return h.threshold > 0 && h.samples > 0 && 4 * h.hot_samples >= h.samples;
}
// Whether a spmm_csr problem reserves the plan in its workspace: rows of at
// least 1 KB and at least 2^26 nonzeros; SPMM_B200_L2PLAN=on reserves it for
// every problem with 1 KB rows, =off never.
bool l2_plan_wanted(int64_t nnz, int64_t N, int dtype);

struct GatherArgs {
    const void *rowptr;
    const void *col;
    const void *val;
    const void *B;
    void *out;
    int64_t M;          // rows of the CSR (rowptr has M + 1 entries)
    int64_t K;          // rows of B (valid column range)
    int64_t N;          // features
    int64_t nnz;
    int64_t row_begin;  // rows below this are not written
    int64_t unit;
    int64_t unit_begin;
    int64_t unit_end;
    float *partial;     // (unit_end - unit_begin) * 2 * N floats
    int64_t *unit_rows; // (unit_end - unit_begin) + 1 entries of scratch
    DevStatus *status;
    // Optional, set by the ring kernel's launcher (pointing at unit_rows):
    // split_rows[u] = the row that starts in unit u and continues past its
    // end (its tail partial was written), else -1; the fix-up then needs no
    // search for it.
    int64_t *split_rows;
    // Optional NVLink multicast address of `out` (same layout): every row
    // of C is then stored once through it with multimem.st, and the switch
    // writes it into each GPU's copy bound to the multicast object; `out`
    // itself is not written directly.  nullptr: plain stores to `out`.
    void *out_mc;
    // Optional L2 residency plan (launch_l2_plan): hot-column bitmap and its
    // header; the ring kernel with rows of 1 KB or more uses them.
    const unsigned *l2_bits;
    const L2PlanHeader *l2_hdr;
};

// Runs the L2 plan into `region` (GatherPlan::l2_plan_bytes() bytes) on
// `stream` when the dense operand is at least 16x L2 (SPMM_B200_L2PLAN=on:
// always) and the column ids fit in 31 bits; sets a.l2_bits / a.l2_hdr,
// else leaves them null.
cudaError_t launch_l2_plan(GatherArgs &a, int itype, int dtype, void *region, cudaStream_t stream);

// Points a's scratch arrays into a workspace of plan.workspace_bytes().
inline void set_workspace(GatherArgs &a, const GatherPlan &plan, void *ws)
{
    a.partial = static_cast<float *>(ws);
    a.unit_rows = ws ? reinterpret_cast<int64_t *>(static_cast<char *>(ws) + plan.rows_offset()) : nullptr;
}

// batch_depth: 0 = default gather batch, 1 = deeper batches (same sums).
cudaError_t launch_gather(const GatherArgs &a, int itype, int dtype, int batch_depth,
                          cudaStream_t stream);

// Tensor-core variant for fp16 rows of a multiple of 64 features
// (gather_mma.cu); launch_gather picks it by default when eligible.  It may
// coarsen the units (a is updated: the partial and unit_rows scratch of the
// original plan is large enough); the caller then launches the fix-up of
// split rows with the updated a.
bool gather_mma_eligible(const GatherArgs &a, int dtype);
cudaError_t launch_gather_mma(GatherArgs &a, int itype, int batch_depth, cudaStream_t stream);

// ---- window path (window.cu) ----------------------------------------------

struct WindowArgs {
    const void *cptr;   // [nwin + 1] block offsets
    const void *ccol;   // [nblocks]
    const void *cval;   // [16 * nblocks]
    const void *vptr;   // [vrows + 1]
    const void *vcol;   // [vnnz]
    const void *vval;   // [vnnz]
    const void *B;
    void *out;
    int64_t nwin;
    int64_t nblocks;
    int64_t vrows;      // rows of the CSR part (only rows < 16 * nwin are fused here)
    int64_t vnnz;
    int64_t K;
    int64_t N;
    DevStatus *status;
    // Optional scratch of window_sched_bytes(nwin, N) bytes for the
    // warp-pipelined kernels' item schedule (heavy items first, claimed
    // dynamically); nullptr keeps the static item order.
    void *sched;
};

// Bytes of WindowArgs::sched for nwin windows of width N (a multiple of 256).
size_t window_sched_bytes(int64_t nwin, int64_t N);

// pipelined: 1 = multi-stage block stream (default), 0 = single stage.
cudaError_t launch_window(const WindowArgs &a, int itype, int dtype, int pipelined,
                          cudaStream_t stream);

// Warp-pipelined window kernels (window_warp.cu): fp16 N % 64 == 0 on
// tensor cores, fp32 N % 128 == 0 on CUDA cores; 16-byte aligned arrays;
// launch_window uses them when eligible.
bool window_warp_eligible(const WindowArgs &a, int dtype);
cudaError_t launch_window_warp(const WindowArgs &a, int itype, int dtype, cudaStream_t stream);

// Window kernel on tcgen05 tensor cores with TMEM accumulators
// (window_tc.cu): fp16, N % 128 == 0, 16-byte aligned values, B and out.
bool window_tc_eligible(const WindowArgs &a, int dtype);
cudaError_t launch_window_tc(const WindowArgs &a, int itype, cudaStream_t stream);

// ---- spmm_cube (cube.cu) -----------------------------------------------------

struct CubeArgs {
    const void *rowptr;  // [nwin + 1] entry offsets of each 16-row window
    const void *col;     // [nnz] (column << 4) | row
    const void *val;     // [nnz]
    const void *B;
    void *out;           // [16 * nwin, N]
    int64_t nwin;
    int64_t K;
    int64_t N;
    int64_t nnz;
    DevStatus *status;
};

size_t cube_workspace_bytes(int64_t nwin, int64_t nnz, int itype, int dtype);
cudaError_t launch_cube(const CubeArgs &a, int itype, int dtype, void *workspace, cudaStream_t stream);

// 16 x 16 tiles of csr_to_ascend_cube (cube.cu): tile t = blocks 16t..16t+15.
struct TileArgs {
    const void *tptr;    // [nwin + 1] tile offsets of each 16-row window
    const void *col;     // [16 * ntiles] tile columns (last tile of a window zero-padded)
    const void *val;     // [256 * ntiles] value[256 t + 16 row + k]
    const void *B;
    void *out;           // [16 * nwin, N]
    int64_t nwin;
    int64_t ntiles;
    int64_t K;
    int64_t N;
    DevStatus *status;
};

size_t tiles_workspace_bytes(int64_t nwin, int64_t ntiles, int itype, int dtype);
cudaError_t launch_tiles(const TileArgs &a, int itype, int dtype, void *workspace, cudaStream_t stream);

// ---- row permutation copies (rows.cu) ---------------------------------------

cudaError_t launch_pack_rows(const void *src, const int64_t *inv, int64_t n, int64_t row_bytes, void *dst,
                             int64_t packed_rows, DevStatus *st, cudaStream_t stream);
cudaError_t launch_restore_rows(const void *src, int64_t src_rows, const int64_t *inv, int64_t n,
                                int64_t row_bytes, void *dst, DevStatus *st, cudaStream_t stream);

// ---- layout builders (preprocess.cu) ----------------------------------------

int pre_csr_to_bcsr(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols, int64_t nnz,
                    int64_t window_size, int itype, int vbytes, const spmm_allocator *alloc, spmm_layout *out,
                    void *stream, bool cube);
int pre_csr_to_spmm_cube(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                         int64_t nnz, int64_t window_size, int itype, int vbytes, const spmm_allocator *alloc,
                         spmm_layout *out, void *stream);
int pre_block_level_split(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                          int64_t nnz, double a, int64_t window_size, int itype, int vbytes,
                          const spmm_allocator *alloc, spmm_layout *out, void *stream);
int pre_preprocess(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols, int64_t nnz,
                   int64_t window_size, int graph_layout, int itype, int vbytes, const spmm_allocator *alloc,
                   spmm_preprocess_result *out, void *stream);

}  // namespace spmmb
