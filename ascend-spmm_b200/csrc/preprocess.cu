// GPU layout builders, bit-exact with the reference's CPU code.
//
//   csr_to_bcsr         extension/custom_op.cpp:594-746   (ToBCSR)
//   csr_to_ascend_cube  extension/custom_op.cpp:429-592
//   block_level_split   extension/custom_op.cpp:1146-1348 (hybrid_split_impl)
//   preprocess          extension/custom_op.cpp:765-1137  (taskmapping), with
//                       extension/boundary_bucket_sort.h and
//                       extension/packed_column_reindex.h
//
// The reference walks windows one at a time on one CPU core (16-way merges,
// epoch arrays, std::stable_sort).  Here every layout derives from ONE sort:
// each nonzero p of row r gets the key (window = r / 16, column, r % 16) and
// the radix sort is stable in p.  Then
//   * a run of equal (window, column) is one (16 x 1) block; runs come out
//     in window-major, ascending-column order (the merge order of ToBCSR);
//   * the run length is the block's nonzero count (duplicates included, as
//     hybrid_split_impl counts them) and its first entry holds the smallest
//     p, i.e. the block's first-seen position in row-major order;
//   * within a run, equal (window, column, row) entries are ordered by p, so
//     the last one is the "last write wins" value of every reference loop.
// Orderings the reference gets from std::stable_sort / bucket sorts become
// radix sorts on keys that include the tie-break (window id, first-seen
// position), and its argmin/first-match loops become reductions that pick
// the smallest index among equal values.  Every cost is evaluated in IEEE
// double with explicit round-to-nearest division (__ddiv_rn), exactly the
// operations and operand order of the reference, so every decision matches.
//
// Generic primitives (radix sort, prefix sums) come from CUB; the domain
// steps are the kernels below.  Temporaries and outputs come from the
// caller's allocator (the torch layer hands out caching-allocator memory).
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

constexpr double kAicBw = 295.0;   // custom_op.cpp:778
constexpr double kAivBw = 505.0;   // custom_op.cpp:779
constexpr int kThreads = 256;

int bits_for(int64_t v)  // bits needed to hold values in [0, v]
{
    int b = 1;
    while (b < 63 && (int64_t(1) << b) <= v) ++b;
    return b;
}

unsigned grid_for(int64_t n, int per_thread = 1)
{
    const int64_t blocks = (n + (int64_t)kThreads * per_thread - 1) / ((int64_t)kThreads * per_thread);
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, 65535LL * 16));
}

#define GRID_STRIDE(i, n) \
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n); i += (int64_t)gridDim.x * blockDim.x)

// ---------------------------------------------------------------------------
// Host-side context: allocator, error state, synchronous reads.
// ---------------------------------------------------------------------------
struct Ctx {
    const spmm_allocator *A;
    cudaStream_t s;
    std::vector<void *> temps;
    int rc = SPMM_OK;
    std::string msg;
    DevStatus *dstat = nullptr;   // per-call device validation status

    Ctx(const spmm_allocator *a, cudaStream_t st) : A(a), s(st) {}
    ~Ctx()
    {
        if (A && A->release)
            for (void *p : temps) A->release(A->ctx, p);
    }
    bool ok() const { return rc == SPMM_OK; }
    void fail(int code, const char *fmt, ...)
    {
        if (rc != SPMM_OK) return;
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        rc = code;
        msg = buf;
    }
    bool cuda(cudaError_t e, const char *where)
    {
        if (e != cudaSuccess) fail(SPMM_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
        return e == cudaSuccess;
    }
    void *raw(size_t bytes, bool keep)
    {
        if (!ok()) return nullptr;
        void *p = A->alloc(A->ctx, std::max<size_t>(bytes, 16));
        if (!p) {
            fail(SPMM_ERR_ALLOC, "allocator returned NULL for %zu bytes", bytes);
            return nullptr;
        }
        if (!keep) temps.push_back(p);
        return p;
    }
    template <typename T> T *tmp(int64_t n) { return static_cast<T *>(raw(sizeof(T) * (size_t)std::max<int64_t>(n, 1), false)); }
    template <typename T> T *out(int64_t n) { return static_cast<T *>(raw(sizeof(T) * (size_t)std::max<int64_t>(n, 1), true)); }
    void zero(void *p, size_t bytes)
    {
        if (ok() && bytes) cuda(cudaMemsetAsync(p, 0, bytes, s), "memset");
    }
    template <typename T> T read(const T *dev)
    {
        T h{};
        if (!ok()) return h;
        if (cuda(cudaMemcpyAsync(&h, dev, sizeof(T), cudaMemcpyDeviceToHost, s), "read")) cuda(cudaStreamSynchronize(s), "sync");
        return h;
    }
    void launched(const char *what) { cuda(cudaGetLastError(), what); }
    // Fails the call if a kernel flagged invalid input.
    bool check_device(const char *op)
    {
        const DevStatus st = read(dstat);
        if (!ok()) return false;
        switch (st.code) {
        case SPMM_DEV_OK: return true;
        case SPMM_DEV_BAD_COLUMN: fail(SPMM_ERR_DEVICE_CHECK, "column index out of range"); break;
        case SPMM_DEV_BAD_ROWPTR:
            fail(SPMM_ERR_DEVICE_CHECK, "%s: invalid CSR row pointer (must start at 0, be non-decreasing and end at nnz)", op);
            break;
        case SPMM_DEV_UNSORTED:
            fail(SPMM_ERR_DEVICE_CHECK, "%s requires each row's col_indices to be sorted in ascending order (row of position %lld)",
                 op, (long long)st.detail);
            break;
        case SPMM_DEV_OCCUPANCY:
            fail(SPMM_ERR_DEVICE_CHECK, "block occupancy must be in [1, window_size]; coalesce duplicate CSR entries");
            break;
        default: fail(SPMM_ERR_DEVICE_CHECK, "%s: device check %d failed", op, st.code);
        }
        return false;
    }
};

template <typename K, typename V>
void sort_pairs(Ctx &c, const K *kin, K *kout, const V *vin, V *vout, int64_t n, int end_bit)
{
    if (!c.ok() || n <= 0) return;
    size_t bytes = 0;
    if (!c.cuda(cub::DeviceRadixSort::SortPairs(nullptr, bytes, kin, kout, vin, vout, n, 0, end_bit, c.s), "sort"))
        return;
    void *t = c.raw(bytes, false);
    if (!t) return;
    c.cuda(cub::DeviceRadixSort::SortPairs(t, bytes, kin, kout, vin, vout, n, 0, end_bit, c.s), "sort");
}

// out[0..n] = exclusive prefix sum of in[0..n) (out has n + 1 entries).
template <typename T>
void exclusive_scan_n1(Ctx &c, const T *in, T *out, int64_t n)
{
    if (!c.ok()) return;
    if (n == 0) {
        c.zero(out, sizeof(T));
        return;
    }
    size_t bytes = 0;
    if (!c.cuda(cub::DeviceScan::InclusiveSum(nullptr, bytes, in, out + 1, n, c.s), "scan")) return;
    void *t = c.raw(bytes, false);
    if (!t) return;
    c.zero(out, sizeof(T));
    c.cuda(cub::DeviceScan::InclusiveSum(t, bytes, in, out + 1, n, c.s), "scan");
}

// ---------------------------------------------------------------------------
// Kernels: sort keys and block runs
// ---------------------------------------------------------------------------

// One warp per row: key = (window, column, row % 16), value = position p.
template <typename I>
__global__ void __launch_bounds__(kThreads)
make_keys_kernel(const I *rowptr, const I *col, int64_t nrows, int64_t ncols, int64_t nnz, int cbits,
                 bool require_sorted, uint64_t *keys, int64_t *vals, DevStatus *st)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    if (warp == 0 && lane == 0 && (rowptr[0] != 0 || (int64_t)rowptr[nrows] != nnz))
        raise_status(st, SPMM_DEV_BAD_ROWPTR, 0);
    for (int64_t r = warp; r < nrows; r += nwarps) {
        int64_t beg = (int64_t)rowptr[r], end = (int64_t)rowptr[r + 1];
        if (beg < 0 || end < beg || end > nnz) {
            if (lane == 0) raise_status(st, SPMM_DEV_BAD_ROWPTR, r);
            continue;
        }
        const uint64_t hi = ((uint64_t)(r >> 4) << (cbits + 4)) | (uint64_t)(r & 15);
        for (int64_t p = beg + lane; p < end; p += 32) {
            const int64_t c = (int64_t)col[p];
            if (c < 0 || c >= ncols) {
                raise_status(st, SPMM_DEV_BAD_COLUMN, p);
                keys[p] = hi;
            } else {
                keys[p] = hi | ((uint64_t)c << 4);
            }
            vals[p] = p;
            if (require_sorted && p > beg && (int64_t)col[p - 1] > c) raise_status(st, SPMM_DEV_UNSORTED, r);
        }
    }
}

__global__ void block_flags_kernel(const uint64_t *sk, int64_t n, int64_t *flag)
{
    GRID_STRIDE(i, n) flag[i] = (i == 0 || (sk[i] >> 4) != (sk[i - 1] >> 4)) ? 1 : 0;
}

// bidx = inclusive count of block starts; fill the per-block arrays.
__global__ void block_fill_kernel(const uint64_t *sk, const int64_t *sp, const int64_t *bidx, int64_t n, int cbits,
                                  int64_t nblocks, int64_t *bstart, int64_t *bcol, int64_t *bwin, int64_t *bfirst)
{
    GRID_STRIDE(i, n)
    {
        if (i == 0 || (sk[i] >> 4) != (sk[i - 1] >> 4)) {
            const int64_t b = bidx[i] - 1;
            bstart[b] = i;
            bcol[b] = (int64_t)((sk[i] >> 4) & ((uint64_t(1) << cbits) - 1));
            bwin[b] = (int64_t)(sk[i] >> (cbits + 4));
            bfirst[b] = sp[i];
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) bstart[nblocks] = n;
}

// wptr[w] = first block of window w (blocks are sorted by window).
__global__ void window_ptr_kernel(const int64_t *bwin, int64_t nblocks, int64_t nwin, int64_t *wptr)
{
    GRID_STRIDE(w, nwin + 1)
    {
        int64_t lo = 0, hi = nblocks;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (bwin[mid] < w) lo = mid + 1;
            else hi = mid;
        }
        wptr[w] = lo;
    }
}

__device__ __forceinline__ bool last_of_group(const uint64_t *sk, int64_t i, int64_t n)
{
    return i == n - 1 || sk[i] != sk[i + 1];
}

template <typename W>
__device__ __forceinline__ void copy_val(void *dst, int64_t di, const void *src, int64_t si)
{
    static_cast<W *>(dst)[di] = static_cast<const W *>(src)[si];
}

template <typename W, typename I>
__global__ void cast_copy_kernel(const W *in, I *out, int64_t n)
{
    GRID_STRIDE(i, n) out[i] = (I)in[i];
}

// ---------------------------------------------------------------------------
// Block analysis shared by every builder
// ---------------------------------------------------------------------------
struct Blocks {
    int64_t n = 0;          // nonzeros
    int64_t nwin = 0;
    int64_t nblocks = 0;
    int cbits = 1;
    uint64_t *sk = nullptr; // sorted keys
    int64_t *sp = nullptr;  // sorted positions
    int64_t *bidx = nullptr;   // per sorted entry: block index + 1
    int64_t *bstart = nullptr; // [nblocks + 1]
    int64_t *bcol = nullptr, *bwin = nullptr, *bfirst = nullptr;
    int64_t *wptr = nullptr;   // [nwin + 1]
};

template <typename I>
bool analyse(Ctx &c, const I *rowptr, const I *col, int64_t nrows, int64_t ncols, int64_t nnz, bool require_sorted,
             const char *op, Blocks &B)
{
    B.n = nnz;
    B.nwin = (nrows + 15) / 16;
    B.cbits = bits_for(std::max<int64_t>(ncols - 1, 0));
    const int wbits = bits_for(std::max<int64_t>(B.nwin - 1, 0));
    if (B.cbits + wbits + 4 > 64) {
        c.fail(SPMM_ERR_UNSUPPORTED, "%s: matrix too large for 64-bit sort keys", op);
        return false;
    }
    if (nrows == 0) return c.ok();
    uint64_t *keys = c.tmp<uint64_t>(nnz);
    int64_t *vals = c.tmp<int64_t>(nnz);
    B.sk = c.tmp<uint64_t>(nnz);
    B.sp = c.tmp<int64_t>(nnz);
    if (!c.ok()) return false;
    make_keys_kernel<I><<<grid_for(nrows * 32), kThreads, 0, c.s>>>(rowptr, col, nrows, ncols, nnz, B.cbits,
                                                                       require_sorted, keys, vals, c.dstat);
    c.launched("make_keys");
    if (!c.check_device(op)) return false;
    sort_pairs(c, keys, B.sk, vals, B.sp, nnz, B.cbits + wbits + 4);
    int64_t *flag = c.tmp<int64_t>(nnz);
    B.bidx = c.tmp<int64_t>(nnz);
    if (!c.ok()) return false;
    if (nnz > 0) {
        block_flags_kernel<<<grid_for(nnz), kThreads, 0, c.s>>>(B.sk, nnz, flag);
        size_t bytes = 0;
        c.cuda(cub::DeviceScan::InclusiveSum(nullptr, bytes, flag, B.bidx, nnz, c.s), "scan");
        void *t = c.raw(bytes, false);
        if (t) c.cuda(cub::DeviceScan::InclusiveSum(t, bytes, flag, B.bidx, nnz, c.s), "scan");
        B.nblocks = c.read(B.bidx + nnz - 1);
    }
    B.bstart = c.tmp<int64_t>(B.nblocks + 1);
    B.bcol = c.tmp<int64_t>(B.nblocks);
    B.bwin = c.tmp<int64_t>(B.nblocks);
    B.bfirst = c.tmp<int64_t>(B.nblocks);
    B.wptr = c.tmp<int64_t>(B.nwin + 1);
    if (!c.ok()) return false;
    if (nnz > 0)
        block_fill_kernel<<<grid_for(nnz), kThreads, 0, c.s>>>(B.sk, B.sp, B.bidx, nnz, B.cbits, B.nblocks, B.bstart,
                                                               B.bcol, B.bwin, B.bfirst);
    else
        c.zero(B.bstart, sizeof(int64_t));
    window_ptr_kernel<<<grid_for(B.nwin + 1), kThreads, 0, c.s>>>(B.bwin, B.nblocks, B.nwin, B.wptr);
    c.launched("analyse");
    return c.ok();
}

// ---------------------------------------------------------------------------
// Deterministic first-argmin reductions
// ---------------------------------------------------------------------------
struct ArgMin {
    double v;
    int64_t i;
};

__device__ __forceinline__ ArgMin better(ArgMin a, ArgMin b)
{
    // smaller value wins; equal values -> smaller index (first occurrence)
    if (b.v < a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ ArgMin block_reduce(ArgMin m)
{
    __shared__ double sv[kThreads / 32];
    __shared__ int64_t si[kThreads / 32];
    for (int o = 16; o > 0; o >>= 1) {
        ArgMin t{__shfl_down_sync(0xffffffffu, m.v, o), __shfl_down_sync(0xffffffffu, m.i, o)};
        m = better(m, t);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { sv[wid] = m.v; si[wid] = m.i; }
    __syncthreads();
    if (wid == 0) {
        m = lane < (int)(blockDim.x / 32) ? ArgMin{sv[lane], si[lane]} : ArgMin{INFINITY, INT64_MAX};
        for (int o = 16; o > 0; o >>= 1) {
            ArgMin t{__shfl_down_sync(0xffffffffu, m.v, o), __shfl_down_sync(0xffffffffu, m.i, o)};
            m = better(m, t);
        }
    }
    return m;
}

__global__ void argmin_finish_kernel(const double *pv, const int64_t *pi, int nparts, ArgMin *out)
{
    ArgMin m{INFINITY, INT64_MAX};
    for (int j = threadIdx.x; j < nparts; j += blockDim.x) m = better(m, ArgMin{pv[j], pi[j]});
    m = block_reduce(m);
    if (threadIdx.x == 0) *out = m;
}

// block_level_split k search (custom_op.cpp:1209-1220): diff(k) =
// |ratio(k) - a|, ratio = (nblocks - k) / prefix[k] (+inf / 0 at prefix 0);
// the first k with the strictly smallest finite diff, else k = 0.
__global__ void bls_argmin_kernel(const int64_t *pref, int64_t nblocks, double a, double *pv, int64_t *pi)
{
    ArgMin m{INFINITY, INT64_MAX};
    GRID_STRIDE(k, nblocks + 1)
    {
        const int64_t rem = nblocks - k, nz = pref[k];
        const double ratio = nz == 0 ? (rem > 0 ? INFINITY : 0.0) : __ddiv_rn((double)rem, (double)nz);
        double diff = fabs(__dsub_rn(ratio, a));
        if (!(diff < INFINITY)) diff = INFINITY;   // NaN / inf never beat the initial +inf
        if (diff < INFINITY) m = better(m, ArgMin{diff, k});
    }
    m = block_reduce(m);
    if (threadIdx.x == 0) { pv[blockIdx.x] = m.v; pi[blockIdx.x] = m.i; }
}

template <typename Kern, typename... Args>
int64_t run_argmin(Ctx &c, Kern kern, int64_t n, Args... args)
{
    const unsigned g = std::min<unsigned>(grid_for(n), 1024);
    double *pv = c.tmp<double>(g);
    int64_t *pi = c.tmp<int64_t>(g);
    ArgMin *res = c.tmp<ArgMin>(1);
    if (!c.ok()) return 0;
    kern<<<g, kThreads, 0, c.s>>>(args..., pv, pi);
    argmin_finish_kernel<<<1, kThreads, 0, c.s>>>(pv, pi, (int)g, res);
    c.launched("argmin");
    const ArgMin r = c.read(res);
    return r.i == INT64_MAX ? 0 : r.i;
}

// ---------------------------------------------------------------------------
// csr_to_bcsr / csr_to_ascend_cube
// ---------------------------------------------------------------------------
template <typename W>
__global__ void bcsr_values_kernel(const uint64_t *sk, const int64_t *sp, const int64_t *bidx, int64_t n,
                                   const void *val, void *out)
{
    GRID_STRIDE(i, n)
    {
        if (!last_of_group(sk, i, n)) continue;
        copy_val<W>(out, 16 * (bidx[i] - 1) + (int64_t)(sk[i] & 15), val, sp[i]);
    }
}

__global__ void cube_tiles_kernel(const int64_t *wptr, int64_t nwin, int64_t *ntiles)
{
    GRID_STRIDE(w, nwin) ntiles[w] = (wptr[w + 1] - wptr[w] + 15) / 16;
}

template <typename I>
__global__ void cube_cols_kernel(const int64_t *bcol, const int64_t *bwin, const int64_t *wptr, const int64_t *tptr,
                                 int64_t nblocks, I *uniq)
{
    GRID_STRIDE(b, nblocks)
    {
        const int64_t w = bwin[b];
        uniq[16 * tptr[w] + (b - wptr[w])] = (I)bcol[b];
    }
}

template <typename W>
__global__ void cube_values_kernel(const uint64_t *sk, const int64_t *sp, const int64_t *bidx, const int64_t *bwin,
                                   const int64_t *wptr, const int64_t *tptr, int64_t n, const void *val, void *out)
{
    GRID_STRIDE(i, n)
    {
        if (!last_of_group(sk, i, n)) continue;
        const int64_t b = bidx[i] - 1, w = bwin[b], lb = b - wptr[w];
        const int64_t t = tptr[w] + lb / 16;
        copy_val<W>(out, 256 * t + 16 * (int64_t)(sk[i] & 15) + lb % 16, val, sp[i]);
    }
}

// ---------------------------------------------------------------------------
// block_level_split
// ---------------------------------------------------------------------------
__global__ void bls_key_kernel(const int64_t *bstart, const int64_t *bfirst, int64_t nblocks, uint64_t *key,
                               int64_t *ids, int64_t *cnt)
{
    GRID_STRIDE(b, nblocks)
    {
        const int64_t c = bstart[b + 1] - bstart[b];
        cnt[b] = c;
        key[b] = ((uint64_t)c << 32) | (uint64_t)bfirst[b];
        ids[b] = b;
    }
}

__global__ void gather_cnt_kernel(const int64_t *order, const int64_t *cnt, int64_t n, int64_t *out)
{
    GRID_STRIDE(i, n) out[i] = cnt[order[i]];
}

__global__ void bls_moved_kernel(const int64_t *order, int64_t nblocks, int64_t best_k, int64_t *kept)
{
    GRID_STRIDE(i, nblocks) kept[order[i]] = i < best_k ? 0 : 1;
}

template <typename I>
__global__ void bls_cols_kernel(const int64_t *kept, const int64_t *kscan, const int64_t *bcol, int64_t nblocks,
                                I *uniq)
{
    GRID_STRIDE(b, nblocks) if (kept[b]) uniq[kscan[b]] = (I)bcol[b];
}

template <typename I>
__global__ void window_ptr_from_scan_kernel(const int64_t *wptr, const int64_t *scan, int64_t nwin, I *out)
{
    GRID_STRIDE(w, nwin + 1) out[w] = (I)scan[wptr[w]];
}

template <typename W>
__global__ void bls_values_kernel(const uint64_t *sk, const int64_t *sp, const int64_t *bidx, const int64_t *kept,
                                  const int64_t *kscan, int64_t n, const void *val, void *out)
{
    GRID_STRIDE(i, n)
    {
        if (!last_of_group(sk, i, n)) continue;
        const int64_t b = bidx[i] - 1;
        if (kept[b]) copy_val<W>(out, 16 * kscan[b] + (int64_t)(sk[i] & 15), val, sp[i]);
    }
}

// moved-nonzero flag per original position
__global__ void moved_flag_kernel(const int64_t *sp, const int64_t *bidx, const int64_t *kept, int64_t n, int64_t *mf)
{
    GRID_STRIDE(i, n) mf[sp[i]] = 1 - kept[bidx[i] - 1];
}

template <typename I>
__global__ void vrow_ptr_kernel(const I *rowptr, int64_t nrows, int64_t nnz, const int64_t *pscan, int64_t m_pad, I *vptr)
{
    GRID_STRIDE(r, m_pad + 1) vptr[r] = (I)pscan[r < nrows ? (int64_t)rowptr[r] : nnz];
}

template <typename I, typename W>
__global__ void compact_kernel(const int64_t *flag, const int64_t *scan, const I *col, const void *val, int64_t n,
                               I *ocol, void *oval)
{
    GRID_STRIDE(p, n)
    {
        if (!flag[p]) continue;
        ocol[scan[p]] = col[p];
        copy_val<W>(oval, scan[p], val, p);
    }
}

// ---------------------------------------------------------------------------
// preprocess
// ---------------------------------------------------------------------------
template <typename I>
__global__ void window_stats_kernel(const I *rowptr, int64_t nrows, const int64_t *wptr, int64_t nwin,
                                    int64_t *wnnz, int64_t *wblk, uint64_t *key, int64_t *ids)
{
    GRID_STRIDE(w, nwin)
    {
        const int64_t r0 = 16 * w, r1 = min(r0 + 16, nrows);
        const int64_t nz = (int64_t)rowptr[r1] - (int64_t)rowptr[r0];
        const int64_t nb = wptr[w + 1] - wptr[w];
        const double density = nb ? __ddiv_rn((double)nz, (double)nb) : 0.0;   // custom_op.cpp:801-805
        wnnz[w] = nz;
        wblk[w] = nb;
        key[w] = ~(uint64_t)__double_as_longlong(density);   // descending density, stable in id
        ids[w] = w;
    }
}

__global__ void gather2_kernel(const int64_t *order, const int64_t *a, const int64_t *b, int64_t n, int64_t *oa,
                               int64_t *ob)
{
    GRID_STRIDE(i, n)
    {
        oa[i] = a[order[i]];
        ob[i] = b[order[i]];
    }
}

// First sorted position where the AIC side would be at least as slow
// (custom_op.cpp:813-826).
__global__ void boundary_kernel(const int64_t *sblk, const int64_t *snnz, const int64_t *pblk, const int64_t *pnnz,
                                int64_t nwin, int64_t nnz, double *pv, int64_t *pi)
{
    ArgMin m{INFINITY, INT64_MAX};
    GRID_STRIDE(pos, nwin)
    {
        const double aic_after = __ddiv_rn((double)(pblk[pos] + sblk[pos]), kAicBw);
        const double aiv_after = __ddiv_rn((double)(nnz - pnnz[pos] - snnz[pos]), kAivBw);
        if (aic_after >= aiv_after) m = better(m, ArgMin{0.0, pos});
    }
    m = block_reduce(m);
    if (threadIdx.x == 0) { pv[blockIdx.x] = m.v; pi[blockIdx.x] = m.i; }
}

// Marginal window: bucket order = occupancy descending, first-seen
// ascending (extension/boundary_bucket_sort.h:13-56).
__global__ void marginal_key_kernel(const int64_t *bstart, const int64_t *bfirst, int64_t b0, int64_t nb, int64_t p0,
                                    uint64_t *key, int64_t *ids, DevStatus *st)
{
    GRID_STRIDE(j, nb)
    {
        const int64_t b = b0 + j;
        const int64_t occ = bstart[b + 1] - bstart[b];
        if (occ < 1 || occ > 16) raise_status(st, SPMM_DEV_OCCUPANCY, b);
        const int64_t o = min(max(occ, (int64_t)1), (int64_t)16);
        key[j] = ((uint64_t)(16 - o) << 40) | (uint64_t)(bfirst[b] - p0);
        ids[j] = j;
    }
}

__global__ void marginal_occ_kernel(const int64_t *order, const int64_t *bstart, int64_t b0, int64_t nb, int64_t *occ)
{
    GRID_STRIDE(j, nb) occ[j] = bstart[b0 + order[j] + 1] - bstart[b0 + order[j]];
}

// q search (custom_op.cpp:866-880): the first q with the smallest
// max(aic_cost, aiv_cost).
__global__ void marginal_q_kernel(const int64_t *assigned, int64_t nb, int64_t prefix_blocks, int64_t suffix_nnz,
                                  int64_t win_nnz, double *pv, int64_t *pi)
{
    ArgMin m{INFINITY, INT64_MAX};
    GRID_STRIDE(q, nb + 1)
    {
        const double aic = __ddiv_rn((double)(prefix_blocks + q), kAicBw);
        const double aiv = __ddiv_rn((double)(suffix_nnz + win_nnz - assigned[q]), kAivBw);
        const double mc = (aic < aiv) ? aiv : aic;   // std::max
        m = better(m, ArgMin{mc, q});
    }
    m = block_reduce(m);
    if (threadIdx.x == 0) { pv[blockIdx.x] = m.v; pi[blockIdx.x] = m.i; }
}

__global__ void marginal_to_aic_kernel(const int64_t *order, int64_t nb, int64_t best_q, int64_t *to_aic)
{
    GRID_STRIDE(j, nb) to_aic[order[j]] = j < best_q ? 1 : 0;
}

__global__ void slot_of_window_kernel(const int64_t *sorted_w, int64_t nwin, int64_t naic, int64_t *slot,
                                      int64_t *rows_aiv, int64_t nrows)
{
    GRID_STRIDE(i, nwin)
    {
        const int64_t w = sorted_w[i];
        slot[w] = i < naic ? i : -1;
        if (i >= naic) rows_aiv[i - naic] = min((int64_t)16, nrows - 16 * w);
    }
}

__global__ void permutation_kernel(const int64_t *sorted_w, int64_t nwin, int64_t naic, const int64_t *aiv_base,
                                   int64_t nrows, int64_t *perm, int64_t *inv)
{
    GRID_STRIDE(t, nwin * 16)
    {
        const int64_t i = t >> 4, j = t & 15;
        const int64_t w = sorted_w[i], r = 16 * w + j;
        if (r >= nrows) continue;
        const int64_t o = i < naic ? 16 * i + j : 16 * naic + aiv_base[i - naic] + j;
        perm[o] = r;
        inv[r] = o;
    }
}

// Block kept in the AIC pack: its window is an AIC slot and, for a shared
// marginal window, the block was assigned to the matrix side.
__device__ __forceinline__ bool aic_block(int64_t b, const int64_t *bwin, const int64_t *slot, int64_t mwin,
                                          int64_t mb0, const int64_t *to_aic, bool shared)
{
    const int64_t w = bwin[b];
    if (slot[w] < 0) return false;
    if (shared && w == mwin) return to_aic[b - mb0] != 0;
    return true;
}

__global__ void aic_flag_kernel(const int64_t *bwin, const int64_t *slot, int64_t nblocks, int64_t mwin, int64_t mb0,
                                const int64_t *to_aic, bool shared, int64_t *inc)
{
    GRID_STRIDE(b, nblocks) inc[b] = aic_block(b, bwin, slot, mwin, mb0, to_aic, shared) ? 1 : 0;
}

__global__ void aic_slot_count_kernel(const int64_t *sorted_w, const int64_t *wptr, const int64_t *iscan, int64_t naic,
                                      int64_t *cnt)
{
    GRID_STRIDE(s, naic)
    {
        const int64_t w = sorted_w[s];
        cnt[s] = iscan[wptr[w + 1]] - iscan[wptr[w]];
    }
}

template <typename I>
__global__ void aic_cols_kernel(const int64_t *inc, const int64_t *iscan, const int64_t *bwin, const int64_t *bcol,
                                const int64_t *wptr, const int64_t *slot, const int64_t *cptr, int64_t nblocks, I *uniq)
{
    GRID_STRIDE(b, nblocks)
    {
        if (!inc[b]) continue;
        const int64_t w = bwin[b];
        uniq[cptr[slot[w]] + iscan[b] - iscan[wptr[w]]] = (I)bcol[b];
    }
}

template <typename W>
__global__ void aic_values_kernel(const uint64_t *sk, const int64_t *sp, const int64_t *bidx, const int64_t *inc,
                                  const int64_t *iscan, const int64_t *bwin, const int64_t *wptr, const int64_t *slot,
                                  const int64_t *cptr, int64_t n, const void *val, void *out)
{
    GRID_STRIDE(i, n)
    {
        if (!last_of_group(sk, i, n)) continue;
        const int64_t b = bidx[i] - 1;
        if (!inc[b]) continue;
        const int64_t w = bwin[b];
        const int64_t pos = cptr[slot[w]] + iscan[b] - iscan[wptr[w]];
        copy_val<W>(out, 16 * pos + (int64_t)(sk[i] & 15), val, sp[i]);
    }
}

// Marginal-window nonzeros assigned to the matrix side (excluded from the
// CSR residual), indexed by position relative to the window's first nonzero.
__global__ void marginal_p_flag_kernel(const int64_t *sp, const int64_t *bidx, const int64_t *to_aic, int64_t i0,
                                       int64_t i1, int64_t mb0, int64_t p0, int64_t *pflag)
{
    GRID_STRIDE(t, i1 - i0)
    {
        const int64_t i = i0 + t;
        pflag[sp[i] - p0] = to_aic[bidx[i] - 1 - mb0];
    }
}

// CSR part over packed rows (custom_op.cpp:981-1001); one warp per row.
template <typename I>
__global__ void aiv_count_kernel(const I *rowptr, const int64_t *perm, int64_t out_rows, int64_t naic, bool shared,
                                 int64_t mwin, const int64_t *pflag, int64_t p0, int64_t *cnt)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t o = warp; o < out_rows; o += nwarps) {
        const int64_t r = perm[o];
        int64_t c = 0;
        if (r >= 0) {
            const bool owned = o >= 16 * naic;
            const bool residual = shared && (r >> 4) == mwin;
            if (owned || residual) {
                const int64_t beg = (int64_t)rowptr[r], end = (int64_t)rowptr[r + 1];
                if (!residual) {
                    c = end - beg;
                } else {
                    for (int64_t p = beg + lane; p < end; p += 32) c += pflag[p - p0] ? 0 : 1;
                    for (int off = 16; off > 0; off >>= 1) c += __shfl_down_sync(0xffffffffu, c, off);
                }
            }
        }
        if (lane == 0) cnt[o] = c;
    }
}

template <typename I, typename W>
__global__ void aiv_fill_kernel(const I *rowptr, const I *col, const void *val, const int64_t *perm, int64_t out_rows,
                                int64_t naic, bool shared, int64_t mwin, const int64_t *pflag, int64_t p0,
                                const int64_t *vscan, I *vcol, void *vval)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t o = warp; o < out_rows; o += nwarps) {
        const int64_t r = perm[o];
        if (r < 0) continue;
        const bool owned = o >= 16 * naic;
        const bool residual = shared && (r >> 4) == mwin;
        if (!owned && !residual) continue;
        const int64_t beg = (int64_t)rowptr[r], end = (int64_t)rowptr[r + 1];
        int64_t dst = vscan[o];
        for (int64_t p0b = beg; p0b < end; p0b += 32) {
            const int64_t p = p0b + lane;
            const bool take = p < end && (!residual || !pflag[p - p0]);
            const unsigned m = __ballot_sync(0xffffffffu, take);
            if (take) {
                const int64_t d = dst + __popc(m & ((1u << lane) - 1));
                vcol[d] = col[p];
                copy_val<W>(vval, d, val, p);
            }
            dst += __popc(m);
        }
    }
}

template <typename I>
__global__ void renumber_kernel(const I *in, const int64_t *inv, int64_t n, I *out)
{
    GRID_STRIDE(i, n) out[i] = (I)inv[(int64_t)in[i]];
}

// Transpose into packed ids (packed_column_reindex.h:43-101): nonzero p of
// row r, column c goes to packed row inv[c] with packed column inv[r];
// a stable sort by inv[c] keeps original-row order inside each new row.
template <typename I>
__global__ void transpose_key_kernel(const I *col, const int64_t *inv, int64_t n, uint64_t *key, int64_t *ids)
{
    GRID_STRIDE(p, n)
    {
        key[p] = (uint64_t)inv[(int64_t)col[p]];
        ids[p] = p;
    }
}

template <typename I>
__global__ void transpose_ptr_kernel(const uint64_t *sk, int64_t n, int64_t rows, I *tptr)
{
    GRID_STRIDE(t, rows + 1)
    {
        int64_t lo = 0, hi = n;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if ((int64_t)sk[mid] < t) lo = mid + 1;
            else hi = mid;
        }
        tptr[t] = (I)lo;
    }
}

template <typename I, typename W>
__global__ void transpose_fill_kernel(const int64_t *sp, const I *rowptr, int64_t nrows, const int64_t *inv,
                                      const void *val, int64_t n, I *tcol, void *tval)
{
    GRID_STRIDE(d, n)
    {
        const int64_t p = sp[d];
        int64_t lo = 0, hi = nrows;   // row r with rowptr[r] <= p < rowptr[r + 1]
        while (hi - lo > 1) {
            const int64_t mid = (lo + hi) >> 1;
            if ((int64_t)rowptr[mid] <= p) lo = mid;
            else hi = mid;
        }
        tcol[d] = (I)inv[lo];
        copy_val<W>(tval, d, val, p);
    }
}

// ---------------------------------------------------------------------------
// Builders
// ---------------------------------------------------------------------------
template <typename F>
void dispatch_w(int vbytes, F f)
{
    if (vbytes == 2) f((uint16_t)0);
    else if (vbytes == 4) f((uint32_t)0);
    else f((uint64_t)0);
}

void set_array(spmm_array &a, void *p, int64_t n)
{
    a.data = n > 0 ? p : nullptr;
    a.len = n;
}

template <typename I>
void build_bcsr(Ctx &c, const I *rowptr, const I *col, const void *val, int64_t nrows, int64_t ncols, int64_t nnz,
                int vbytes, bool cube, spmm_layout *out)
{
    const char *op = cube ? "csr_to_ascend_cube" : "csr_to_bcsr";
    Blocks B;
    if (!analyse<I>(c, rowptr, col, nrows, ncols, nnz, true, op, B)) return;
    const int64_t nwin = B.nwin;
    I *cptr = c.out<I>(nwin + 1);
    if (!c.ok()) return;
    if (!cube) {
        I *uniq = c.out<I>(B.nblocks);
        void *value = c.raw((size_t)16 * B.nblocks * vbytes, true);
        if (!c.ok()) return;
        if (nwin > 0) cast_copy_kernel<int64_t, I><<<grid_for(nwin + 1), kThreads, 0, c.s>>>(B.wptr, cptr, nwin + 1);
        else c.zero(cptr, sizeof(I));
        cast_copy_kernel<int64_t, I><<<grid_for(B.nblocks), kThreads, 0, c.s>>>(B.bcol, uniq, B.nblocks);
        c.zero(value, (size_t)16 * B.nblocks * vbytes);
        dispatch_w(vbytes, [&](auto w) {
            using W = decltype(w);
            if (nnz > 0) bcsr_values_kernel<W><<<grid_for(nnz), kThreads, 0, c.s>>>(B.sk, B.sp, B.bidx, nnz, val, value);
        });
        c.launched(op);
        set_array(out->crow_window_ptr, cptr, nwin + 1);
        set_array(out->unique_col_ids, uniq, B.nblocks);
        set_array(out->value, value, 16 * B.nblocks);
        return;
    }
    int64_t *ntiles = c.tmp<int64_t>(nwin);
    int64_t *tptr = c.tmp<int64_t>(nwin + 1);
    if (!c.ok()) return;
    if (nwin > 0) cube_tiles_kernel<<<grid_for(nwin), kThreads, 0, c.s>>>(B.wptr, nwin, ntiles);
    exclusive_scan_n1(c, ntiles, tptr, nwin);
    const int64_t T = c.read(tptr + nwin);
    I *uniq = c.out<I>(16 * T);
    void *value = c.raw((size_t)256 * T * vbytes, true);
    if (!c.ok()) return;
    cast_copy_kernel<int64_t, I><<<grid_for(nwin + 1), kThreads, 0, c.s>>>(tptr, cptr, nwin + 1);
    c.zero(uniq, sizeof(I) * 16 * T);
    c.zero(value, (size_t)256 * T * vbytes);
    if (B.nblocks > 0)
        cube_cols_kernel<I><<<grid_for(B.nblocks), kThreads, 0, c.s>>>(B.bcol, B.bwin, B.wptr, tptr, B.nblocks, uniq);
    dispatch_w(vbytes, [&](auto w) {
        using W = decltype(w);
        if (nnz > 0)
            cube_values_kernel<W><<<grid_for(nnz), kThreads, 0, c.s>>>(B.sk, B.sp, B.bidx, B.bwin, B.wptr, tptr, nnz, val,
                                                                       value);
    });
    c.launched(op);
    set_array(out->crow_window_ptr, cptr, nwin + 1);
    set_array(out->unique_col_ids, uniq, 16 * T);
    set_array(out->value, value, 256 * T);
}

// ---- producer of the spmm_cube window encoding ------------------------------

template <typename I, typename W>
__global__ void cube_encode_kernel(const uint64_t *sk, const int64_t *sp, int64_t n, int cbits, const void *val,
                                   I *col_out, void *val_out)
{
    const uint64_t cmask = (uint64_t(1) << cbits) - 1;
    GRID_STRIDE(i, n)
    {
        const uint64_t k = sk[i];
        col_out[i] = (I)((((k >> 4) & cmask) << 4) | (k & 15));
        copy_val<W>(val_out, i, val, sp[i]);
    }
}

template <typename I>
__global__ void cube_window_ptr_kernel(const I *rowptr, int64_t nrows, int64_t nwin, I *out)
{
    GRID_STRIDE(w, nwin + 1) out[w] = rowptr[std::min<int64_t>(16 * w, nrows)];
}

// Sorting by (window, column, row) with a stable radix sort puts each
// window's entries in ToBCSR's merge order (custom_op.cpp:611-671); the
// window's entries keep their CSR offsets, so the window pointer is the CSR
// row pointer sampled every 16 rows.
template <typename I>
void build_spmm_cube(Ctx &c, const I *rowptr, const I *col, const void *val, int64_t nrows, int64_t ncols,
                     int64_t nnz, int vbytes, spmm_layout *out)
{
    const char *op = "csr_to_spmm_cube";
    if (sizeof(I) == 4 && ncols > (int64_t(1) << 27)) {
        c.fail(SPMM_ERR_ARG, "%s: int32 (column << 4 | row) needs ncols <= 2^27, got %lld", op, (long long)ncols);
        return;
    }
    const int64_t nwin = (nrows + 15) / 16;
    const int cbits = bits_for(std::max<int64_t>(ncols - 1, 0));
    const int wbits = bits_for(std::max<int64_t>(nwin - 1, 0));
    if (cbits + wbits + 4 > 64) {
        c.fail(SPMM_ERR_UNSUPPORTED, "%s: matrix too large for 64-bit sort keys", op);
        return;
    }
    I *wptr = c.out<I>(nwin + 1);
    I *ecol = c.out<I>(nnz);
    void *eval = c.raw((size_t)std::max<int64_t>(nnz, 1) * vbytes, true);
    if (!c.ok()) return;
    if (nrows == 0) {
        c.zero(wptr, sizeof(I));
    } else {
        uint64_t *keys = c.tmp<uint64_t>(nnz), *sk = c.tmp<uint64_t>(nnz);
        int64_t *vals = c.tmp<int64_t>(nnz), *sp = c.tmp<int64_t>(nnz);
        if (!c.ok()) return;
        make_keys_kernel<I><<<grid_for(nrows * 32), kThreads, 0, c.s>>>(rowptr, col, nrows, ncols, nnz, cbits, false,
                                                                           keys, vals, c.dstat);
        c.launched("make_keys");
        if (!c.check_device(op)) return;
        sort_pairs(c, keys, sk, vals, sp, nnz, cbits + wbits + 4);
        cube_window_ptr_kernel<I><<<grid_for(nwin + 1), kThreads, 0, c.s>>>(rowptr, nrows, nwin, wptr);
        dispatch_w(vbytes, [&](auto w) {
            using W = decltype(w);
            if (nnz > 0) cube_encode_kernel<I, W><<<grid_for(nnz), kThreads, 0, c.s>>>(sk, sp, nnz, cbits, val, ecol, eval);
        });
        c.launched(op);
    }
    set_array(out->crow_window_ptr, wptr, nwin + 1);
    set_array(out->unique_col_ids, ecol, nnz);
    set_array(out->value, eval, nnz);
}

template <typename I>
void build_bls(Ctx &c, const I *rowptr, const I *col, const void *val, int64_t nrows, int64_t ncols, int64_t nnz,
               int vbytes, double a, spmm_layout *out)
{
    const char *op = "block_level_split";
    Blocks B;
    if (!analyse<I>(c, rowptr, col, nrows, ncols, nnz, false, op, B)) return;
    const int64_t nwin = B.nwin, nb = B.nblocks, m_pad = nwin * 16;
    // stable ascending order by count, first-seen tie-break
    uint64_t *key = c.tmp<uint64_t>(nb), *skey = c.tmp<uint64_t>(nb);
    int64_t *ids = c.tmp<int64_t>(nb), *order = c.tmp<int64_t>(nb), *cnt = c.tmp<int64_t>(nb);
    int64_t *ocnt = c.tmp<int64_t>(nb), *pref = c.tmp<int64_t>(nb + 1);
    int64_t *kept = c.tmp<int64_t>(nb), *kscan = c.tmp<int64_t>(nb + 1);
    int64_t *mflag = c.tmp<int64_t>(nnz), *pscan = c.tmp<int64_t>(nnz + 1);
    if (!c.ok()) return;
    if (nb > 0) {
        bls_key_kernel<<<grid_for(nb), kThreads, 0, c.s>>>(B.bstart, B.bfirst, nb, key, ids, cnt);
        sort_pairs(c, key, skey, ids, order, nb, 64);
        gather_cnt_kernel<<<grid_for(nb), kThreads, 0, c.s>>>(order, cnt, nb, ocnt);
    }
    exclusive_scan_n1(c, ocnt, pref, nb);
    const int64_t best_k = run_argmin(c, bls_argmin_kernel, nb + 1, (const int64_t *)pref, nb, a);
    if (!c.ok()) return;
    if (nb > 0) bls_moved_kernel<<<grid_for(nb), kThreads, 0, c.s>>>(order, nb, best_k, kept);
    exclusive_scan_n1(c, kept, kscan, nb);
    const int64_t n_kept = c.read(kscan + nb);
    if (nnz > 0) moved_flag_kernel<<<grid_for(nnz), kThreads, 0, c.s>>>(B.sp, B.bidx, kept, nnz, mflag);
    exclusive_scan_n1(c, mflag, pscan, nnz);
    const int64_t n_v = c.read(pscan + nnz);
    I *cptr = c.out<I>(nwin + 1), *uniq = c.out<I>(n_kept), *vptr = c.out<I>(m_pad + 1), *vcol = c.out<I>(n_v);
    void *value = c.raw((size_t)16 * n_kept * vbytes, true);
    void *vval = c.raw((size_t)n_v * vbytes, true);
    if (!c.ok()) return;
    window_ptr_from_scan_kernel<I><<<grid_for(nwin + 1), kThreads, 0, c.s>>>(B.wptr, kscan, nwin, cptr);
    if (nb > 0) bls_cols_kernel<I><<<grid_for(nb), kThreads, 0, c.s>>>(kept, kscan, B.bcol, nb, uniq);
    c.zero(value, (size_t)16 * n_kept * vbytes);
    vrow_ptr_kernel<I><<<grid_for(m_pad + 1), kThreads, 0, c.s>>>(rowptr, nrows, nnz, pscan, m_pad, vptr);
    dispatch_w(vbytes, [&](auto w) {
        using W = decltype(w);
        if (nnz > 0) {
            bls_values_kernel<W><<<grid_for(nnz), kThreads, 0, c.s>>>(B.sk, B.sp, B.bidx, kept, kscan, nnz, val, value);
            compact_kernel<I, W><<<grid_for(nnz), kThreads, 0, c.s>>>(mflag, pscan, col, val, nnz, vcol, vval);
        }
    });
    c.launched(op);
    set_array(out->crow_window_ptr, cptr, nwin + 1);
    set_array(out->unique_col_ids, uniq, n_kept);
    set_array(out->value, value, 16 * n_kept);
    set_array(out->vrow_window_ptr, vptr, m_pad + 1);
    set_array(out->vcol_indices, vcol, n_v);
    set_array(out->vvalue, vval, n_v);
}

template <typename I>
void build_preprocess(Ctx &c, const I *rowptr, const I *col, const void *val, int64_t nrows, int64_t ncols,
                      int64_t nnz, int vbytes, bool graph_layout, spmm_preprocess_result *R)
{
    const char *op = "preprocess";
    Blocks B;
    if (!analyse<I>(c, rowptr, col, nrows, ncols, nnz, false, op, B)) return;
    const int64_t nwin = B.nwin, nb = B.nblocks;

    // window statistics and density order (custom_op.cpp:784-811)
    int64_t *wnnz = c.tmp<int64_t>(nwin), *wblk = c.tmp<int64_t>(nwin), *wids = c.tmp<int64_t>(nwin);
    int64_t *sorted_w = c.tmp<int64_t>(nwin);
    uint64_t *wkey = c.tmp<uint64_t>(nwin), *wkey_s = c.tmp<uint64_t>(nwin);
    int64_t *sblk = c.tmp<int64_t>(nwin), *snnz = c.tmp<int64_t>(nwin);
    int64_t *pblk = c.tmp<int64_t>(nwin + 1), *pnnz = c.tmp<int64_t>(nwin + 1);
    if (!c.ok()) return;
    if (nwin > 0) {
        window_stats_kernel<I><<<grid_for(nwin), kThreads, 0, c.s>>>(rowptr, nrows, B.wptr, nwin, wnnz, wblk, wkey, wids);
        sort_pairs(c, wkey, wkey_s, wids, sorted_w, nwin, 64);
        gather2_kernel<<<grid_for(nwin), kThreads, 0, c.s>>>(sorted_w, wblk, wnnz, nwin, sblk, snnz);
    }
    exclusive_scan_n1(c, sblk, pblk, nwin);
    exclusive_scan_n1(c, snnz, pnnz, nwin);
    int64_t bpos = -1;
    if (nwin > 0) {
        const int64_t r = run_argmin(c, boundary_kernel, nwin, (const int64_t *)sblk, (const int64_t *)snnz,
                                     (const int64_t *)pblk, (const int64_t *)pnnz, nwin, nnz);
        // run_argmin maps "none" to 0; re-check the predicate on the host
        if (c.ok()) {
            const int64_t pb = c.read(pblk + r), pn = c.read(pnnz + r), sbk = c.read(sblk + r), snz = c.read(snnz + r);
            const double aic_after = (double)(pb + sbk) / kAicBw;
            const double aiv_after = (double)(nnz - pn - snz) / kAivBw;
            bpos = aic_after >= aiv_after ? r : -1;
        }
    }
    if (!c.ok()) return;

    // marginal window split (custom_op.cpp:828-885)
    int64_t mwin = -1, mblocks = 0, best_q = 0, mb0 = 0, p0 = 0, win_nnz = 0;
    double e_aic = 0.0, e_aiv = 0.0, e_max = 0.0;
    int64_t *to_aic = c.tmp<int64_t>(1);
    if (bpos >= 0) {
        mwin = c.read(sorted_w + bpos);
        const int64_t prefix_blocks = c.read(pblk + bpos);
        const int64_t remaining = nnz - c.read(pnnz + bpos);
        win_nnz = c.read(snnz + bpos);
        mblocks = c.read(sblk + bpos);
        mb0 = c.read(B.wptr + mwin);
        p0 = (int64_t)c.read(rowptr + 16 * mwin);
        uint64_t *mkey = c.tmp<uint64_t>(mblocks), *mkey_s = c.tmp<uint64_t>(mblocks);
        int64_t *mids = c.tmp<int64_t>(mblocks), *morder = c.tmp<int64_t>(mblocks);
        int64_t *mocc = c.tmp<int64_t>(mblocks), *assigned = c.tmp<int64_t>(mblocks + 1);
        to_aic = c.tmp<int64_t>(mblocks);
        if (!c.ok()) return;
        if (mblocks > 0) {
            marginal_key_kernel<<<grid_for(mblocks), kThreads, 0, c.s>>>(B.bstart, B.bfirst, mb0, mblocks, p0, mkey, mids,
                                                                         c.dstat);
            if (!c.check_device(op)) return;
            sort_pairs(c, mkey, mkey_s, mids, morder, mblocks, 64);
            marginal_occ_kernel<<<grid_for(mblocks), kThreads, 0, c.s>>>(morder, B.bstart, mb0, mblocks, mocc);
        }
        exclusive_scan_n1(c, mocc, assigned, mblocks);
        const int64_t suffix_nnz = remaining - win_nnz;
        best_q = run_argmin(c, marginal_q_kernel, mblocks + 1, (const int64_t *)assigned, mblocks, prefix_blocks,
                            suffix_nnz, win_nnz);
        if (mblocks > 0) marginal_to_aic_kernel<<<grid_for(mblocks), kThreads, 0, c.s>>>(morder, mblocks, best_q, to_aic);
        const int64_t asg = c.read(assigned + best_q);
        e_aic = (double)(prefix_blocks + best_q) / kAicBw;
        e_aiv = (double)(suffix_nnz + win_nnz - asg) / kAivBw;
        e_max = std::max(e_aic, e_aiv);
    }
    if (!c.ok()) return;
    const bool shared = best_q > 0 && best_q < mblocks;
    const int64_t naic = bpos < 0 ? 0 : bpos + (best_q > 0 ? 1 : 0);

    // row permutation (custom_op.cpp:905-940)
    int64_t *slot = c.tmp<int64_t>(nwin), *rows_aiv = c.tmp<int64_t>(nwin - naic), *aiv_base = c.tmp<int64_t>(nwin - naic + 1);
    if (!c.ok()) return;
    if (nwin > 0) slot_of_window_kernel<<<grid_for(nwin), kThreads, 0, c.s>>>(sorted_w, nwin, naic, slot, rows_aiv, nrows);
    exclusive_scan_n1(c, rows_aiv, aiv_base, nwin - naic);
    const int64_t aiv_rows = c.read(aiv_base + (nwin - naic));
    const int64_t aic_real_rows = nrows - aiv_rows;
    const int64_t real_extent = 16 * naic + (nrows - aic_real_rows);
    const int64_t packed_ok = (graph_layout && nrows == ncols) ? 1 : 0;
    const int64_t out_rows = packed_ok ? nwin * 16 : real_extent;
    int64_t *perm = c.out<int64_t>(out_rows), *inv = c.out<int64_t>(nrows);
    if (!c.ok()) return;
    c.cuda(cudaMemsetAsync(perm, 0xff, sizeof(int64_t) * out_rows, c.s), "memset");
    c.cuda(cudaMemsetAsync(inv, 0xff, sizeof(int64_t) * nrows, c.s), "memset");
    if (nwin > 0) permutation_kernel<<<grid_for(nwin * 16), kThreads, 0, c.s>>>(sorted_w, nwin, naic, aiv_base, nrows, perm, inv);

    // AIC pack (custom_op.cpp:942-979)
    int64_t *inc = c.tmp<int64_t>(nb), *iscan = c.tmp<int64_t>(nb + 1);
    int64_t *scount = c.tmp<int64_t>(naic), *cscan = c.tmp<int64_t>(naic + 1);
    if (!c.ok()) return;
    if (nb > 0) aic_flag_kernel<<<grid_for(nb), kThreads, 0, c.s>>>(B.bwin, slot, nb, mwin, mb0, to_aic, shared, inc);
    exclusive_scan_n1(c, inc, iscan, nb);
    if (naic > 0) aic_slot_count_kernel<<<grid_for(naic), kThreads, 0, c.s>>>(sorted_w, B.wptr, iscan, naic, scount);
    exclusive_scan_n1(c, scount, cscan, naic);
    const int64_t n_aic_blocks = c.read(cscan + naic);
    I *cptr = c.out<I>(naic + 1), *uniq = c.out<I>(n_aic_blocks);
    void *value = c.raw((size_t)16 * n_aic_blocks * vbytes, true);
    if (!c.ok()) return;
    cast_copy_kernel<int64_t, I><<<grid_for(naic + 1), kThreads, 0, c.s>>>(cscan, cptr, naic + 1);
    c.zero(value, (size_t)16 * n_aic_blocks * vbytes);
    if (nb > 0)
        aic_cols_kernel<I><<<grid_for(nb), kThreads, 0, c.s>>>(inc, iscan, B.bwin, B.bcol, B.wptr, slot, cscan, nb, uniq);

    // marginal nonzeros kept on the matrix side
    int64_t *pflag = c.tmp<int64_t>(1);
    if (shared) {
        const int64_t i0 = c.read(B.bstart + mb0), i1 = c.read(B.bstart + mb0 + mblocks);
        pflag = c.tmp<int64_t>(win_nnz);
        if (!c.ok()) return;
        marginal_p_flag_kernel<<<grid_for(i1 - i0), kThreads, 0, c.s>>>(B.sp, B.bidx, to_aic, i0, i1, mb0, p0, pflag);
    }

    // CSR part over packed rows (custom_op.cpp:981-1001)
    int64_t *vcount = c.tmp<int64_t>(out_rows), *vscan = c.tmp<int64_t>(out_rows + 1);
    if (!c.ok()) return;
    if (out_rows > 0)
        aiv_count_kernel<I><<<grid_for(out_rows * 32), kThreads, 0, c.s>>>(rowptr, perm, out_rows, naic, shared, mwin, pflag,
                                                                           p0, vcount);
    exclusive_scan_n1(c, vcount, vscan, out_rows);
    const int64_t n_v = c.read(vscan + out_rows);
    I *vptr = c.out<I>(out_rows + 1), *vcol = c.out<I>(n_v);
    void *vval = c.raw((size_t)n_v * vbytes, true);
    if (!c.ok()) return;
    cast_copy_kernel<int64_t, I><<<grid_for(out_rows + 1), kThreads, 0, c.s>>>(vscan, vptr, out_rows + 1);
    dispatch_w(vbytes, [&](auto w) {
        using W = decltype(w);
        if (nnz > 0)
            aic_values_kernel<W><<<grid_for(nnz), kThreads, 0, c.s>>>(B.sk, B.sp, B.bidx, inc, iscan, B.bwin, B.wptr, slot,
                                                                       cscan, nnz, val, value);
        if (out_rows > 0)
            aiv_fill_kernel<I, W><<<grid_for(out_rows * 32), kThreads, 0, c.s>>>(rowptr, col, val, perm, out_rows, naic,
                                                                                 shared, mwin, pflag, p0, vscan, vcol,
                                                                                 vval);
    });
    c.launched(op);

    spmm_layout &F = R->fwd;
    set_array(F.crow_window_ptr, cptr, naic + 1);
    set_array(F.unique_col_ids, uniq, n_aic_blocks);
    set_array(F.value, value, 16 * n_aic_blocks);
    set_array(F.vrow_window_ptr, vptr, out_rows + 1);
    set_array(F.vcol_indices, vcol, n_v);
    set_array(F.vvalue, vval, n_v);
    set_array(R->permutation, perm, out_rows);
    set_array(R->inv_permutation, inv, nrows);
    R->packed_rows = out_rows;
    R->packed_layout_supported = packed_ok;
    R->marginal_window = mwin;
    R->marginal_aic_blocks = best_q;
    R->marginal_total_blocks = mblocks;
    R->shared_windows = shared ? 1 : 0;
    R->estimated_aic_cost = e_aic;
    R->estimated_aiv_cost = e_aiv;
    R->estimated_max_cost = e_max;

    if (!packed_ok) return;
    // graph layout: P A P^T relabel + fixed-layout transpose (custom_op.cpp:1006-1035)
    I *ru = c.out<I>(n_aic_blocks), *rv = c.out<I>(n_v);
    uint64_t *tkey = c.tmp<uint64_t>(nnz), *tkey_s = c.tmp<uint64_t>(nnz);
    int64_t *tids = c.tmp<int64_t>(nnz), *tsp = c.tmp<int64_t>(nnz);
    I *tptr = c.tmp<I>(out_rows + 1), *tcol = c.tmp<I>(nnz);
    void *tval = c.raw((size_t)nnz * vbytes, false);
    if (!c.ok()) return;
    if (n_aic_blocks > 0) renumber_kernel<I><<<grid_for(n_aic_blocks), kThreads, 0, c.s>>>(uniq, inv, n_aic_blocks, ru);
    if (n_v > 0) renumber_kernel<I><<<grid_for(n_v), kThreads, 0, c.s>>>(vcol, inv, n_v, rv);
    set_array(R->renumbered_unique_col_ids, ru, n_aic_blocks);
    set_array(R->renumbered_vcol_indices, rv, n_v);
    if (nnz > 0) {
        transpose_key_kernel<I><<<grid_for(nnz), kThreads, 0, c.s>>>(col, inv, nnz, tkey, tids);
        sort_pairs(c, tkey, tkey_s, tids, tsp, nnz, bits_for(out_rows));
    }
    transpose_ptr_kernel<I><<<grid_for(out_rows + 1), kThreads, 0, c.s>>>(tkey_s, nnz, out_rows, tptr);
    dispatch_w(vbytes, [&](auto w) {
        using W = decltype(w);
        if (nnz > 0)
            transpose_fill_kernel<I, W><<<grid_for(nnz), kThreads, 0, c.s>>>(tsp, rowptr, nrows, inv, val, nnz, tcol, tval);
    });
    c.launched("transpose");
    build_bls<I>(c, tptr, tcol, tval, out_rows, out_rows, nnz, vbytes, 295.0 / 505.0, &R->transpose);
}

template <typename F>
int run_entry(const spmm_allocator *alloc, void *stream, int itype, int vbytes, int64_t nrows, int64_t ncols,
              int64_t nnz, int64_t window_size, bool window16_only, const char *op, F body)
{
    if (!alloc || !alloc->alloc) return capi_error(SPMM_ERR_ARG, "%s: allocator required", op);
    if (itype != SPMM_I32 && itype != SPMM_I64) return capi_error(SPMM_ERR_ARG, "%s: index arrays must be int32 or int64", op);
    if (vbytes != 2 && vbytes != 4 && vbytes != 8)
        return capi_error(SPMM_ERR_ARG, "%s: values must be float16, float32 or float64", op);
    if (nrows < 0 || ncols < 0 || nnz < 0) return capi_error(SPMM_ERR_ARG, "%s: negative size", op);
    if (window_size != 16)
        return capi_error(SPMM_ERR_ARG, window16_only ? "Ascend-SpMM requires a 16-row window"
                                                      : "%s: this engine builds 16-row windows only", op);
    if (nnz >= (int64_t(1) << 32)) return capi_error(SPMM_ERR_UNSUPPORTED, "%s: nnz must be below 2^32", op);
    Ctx c(alloc, static_cast<cudaStream_t>(stream));
    c.dstat = c.tmp<DevStatus>(1);
    c.zero(c.dstat, sizeof(DevStatus));
    if (c.ok()) body(c);
    if (c.ok()) c.cuda(cudaStreamSynchronize(c.s), op);
    if (!c.ok()) return capi_error(c.rc, "%s", c.msg.c_str());
    return SPMM_OK;
}

}  // namespace

// ---- entry points (called from capi.cu) -------------------------------------

int pre_csr_to_bcsr(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols, int64_t nnz,
                    int64_t window_size, int itype, int vbytes, const spmm_allocator *alloc, spmm_layout *out,
                    void *stream, bool cube)
{
    *out = spmm_layout{};
    return run_entry(alloc, stream, itype, vbytes, nrows, ncols, nnz, window_size, false,
                     cube ? "csr_to_ascend_cube" : "csr_to_bcsr", [&](Ctx &c) {
                         if (itype == SPMM_I32)
                             build_bcsr<int>(c, (const int *)crow, (const int *)col, val, nrows, ncols, nnz, vbytes, cube, out);
                         else
                             build_bcsr<int64_t>(c, (const int64_t *)crow, (const int64_t *)col, val, nrows, ncols, nnz,
                                                 vbytes, cube, out);
                     });
}

int pre_csr_to_spmm_cube(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                         int64_t nnz, int64_t window_size, int itype, int vbytes, const spmm_allocator *alloc,
                         spmm_layout *out, void *stream)
{
    *out = spmm_layout{};
    return run_entry(alloc, stream, itype, vbytes, nrows, ncols, nnz, window_size, false, "csr_to_spmm_cube",
                     [&](Ctx &c) {
                         if (itype == SPMM_I32)
                             build_spmm_cube<int>(c, (const int *)crow, (const int *)col, val, nrows, ncols, nnz, vbytes,
                                                  out);
                         else
                             build_spmm_cube<int64_t>(c, (const int64_t *)crow, (const int64_t *)col, val, nrows, ncols,
                                                      nnz, vbytes, out);
                     });
}

int pre_block_level_split(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols,
                          int64_t nnz, double a, int64_t window_size, int itype, int vbytes,
                          const spmm_allocator *alloc, spmm_layout *out, void *stream)
{
    *out = spmm_layout{};
    return run_entry(alloc, stream, itype, vbytes, nrows, ncols, nnz, window_size, false, "block_level_split",
                     [&](Ctx &c) {
                         if (itype == SPMM_I32)
                             build_bls<int>(c, (const int *)crow, (const int *)col, val, nrows, ncols, nnz, vbytes, a, out);
                         else
                             build_bls<int64_t>(c, (const int64_t *)crow, (const int64_t *)col, val, nrows, ncols, nnz,
                                                vbytes, a, out);
                     });
}

int pre_preprocess(const void *crow, const void *col, const void *val, int64_t nrows, int64_t ncols, int64_t nnz,
                   int64_t window_size, int graph_layout, int itype, int vbytes, const spmm_allocator *alloc,
                   spmm_preprocess_result *out, void *stream)
{
    *out = spmm_preprocess_result{};
    out->marginal_window = -1;
    return run_entry(alloc, stream, itype, vbytes, nrows, ncols, nnz, window_size, true, "preprocess", [&](Ctx &c) {
        if (itype == SPMM_I32)
            build_preprocess<int>(c, (const int *)crow, (const int *)col, val, nrows, ncols, nnz, vbytes, graph_layout != 0,
                                  out);
        else
            build_preprocess<int64_t>(c, (const int64_t *)crow, (const int64_t *)col, val, nrows, ncols, nnz, vbytes,
                                      graph_layout != 0, out);
    });
}

}  // namespace spmmb
