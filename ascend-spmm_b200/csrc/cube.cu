// spmm_cube: SpMM over 16-row windows whose entries are encoded as
// (column << 4) | row-in-window (reference consumer:
// kernels/op_kernel/spmm_cube.cpp:51-147; host op custom_op.cpp:91-113).
//
// Semantics (reference kernel, one AI core walking a window's entries in
// order): an entry whose column differs from the previous entry's opens a
// new (16 x 1) block (spmm_cube.cpp:88-107; every window starts a new one,
// :61-82); the entry's value lands at row (col & 15) of the block and
// overwrites an earlier entry of the same row in the same block (:125-126);
// output rows [16w, 16w + 16) are the sum of block[r] * B[column, :].
//
// B200 design: the encoding is normalised on the device into the same
// (16 x 1)-block stream the window kernel of the mixed operator consumes
// (window.cu), then that kernel runs unchanged - every output row is summed
// in fp32 by one CTA and rounded once (the reference rounds each batch of
// 16 blocks to fp16 and adds them atomically, spmm_cube.cpp:227-236).
//   1. cube_count_kernel   CTA per window: number of blocks (runs);
//                          per-tile totals by integer atomics (order free)
//   2. cube_scan_tiles_kernel one CTA: exclusive scan of the tile totals
//   3. cube_fill_kernel    CTA per window: block offset (tile offset + sum
//                          of the earlier counts of its tile), block columns
//                          and the 16 values of every block (zeroed first;
//                          inside a chunk an entry is dropped when a later
//                          entry of its run has the same row, and chunks are
//                          written in order, so the last entry wins)
//   4. launch_window       the block-stream MMA / FFMA kernel
// The workspace bound uses #blocks <= nnz, so nothing is read back to the
// host and the call stays asynchronous.
#include <algorithm>

#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

constexpr int kCubeThreads = 128;   // entries per chunk
constexpr int kTileWindows = 256;   // windows per scan tile

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct CubeWorkspace {
    unsigned long long *tile;  // [ntiles + 1] tile totals, then exclusive offsets
    long long *count;          // [nwin] blocks per window
    void *cptr;                // I [nwin + 1]
    void *ccol;                // I [max(nnz, 1)]
    void *cval;                // T [16 * max(nnz, 1)]
    size_t bytes;
};

CubeWorkspace carve(void *base, int64_t nwin, int64_t nnz, int isz, int vsz)
{
    const int64_t ntiles = (nwin + kTileWindows - 1) / kTileWindows;
    const int64_t nb = std::max<int64_t>(nnz, 1);
    CubeWorkspace w{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = base ? static_cast<char *>(base) + off : nullptr;
        off += align256(bytes);
        return static_cast<void *>(p);
    };
    w.tile = static_cast<unsigned long long *>(take(8 * (size_t)(ntiles + 1)));
    w.count = static_cast<long long *>(take(8 * (size_t)std::max<int64_t>(nwin, 1)));
    w.cptr = take((size_t)isz * (size_t)(nwin + 1));
    w.ccol = take((size_t)isz * (size_t)nb);
    w.cval = take((size_t)vsz * 16 * (size_t)nb);
    w.bytes = off;
    return w;
}

// Entry range of window w, or an empty one (status raised) if invalid.
template <typename I>
__device__ __forceinline__ bool window_range(const I *rowptr, int64_t w, int64_t nnz, int64_t &e0, int64_t &e1,
                                             DevStatus *st)
{
    e0 = (int64_t)rowptr[w];
    e1 = (int64_t)rowptr[w + 1];
    if (e0 < 0 || e1 < e0 || e1 > nnz) {
        if (threadIdx.x == 0) raise_status(st, SPMM_DEV_BAD_ROWPTR, w);
        e0 = e1 = 0;
        return false;
    }
    return true;
}

// Column of an encoded entry (arithmetic shift: negative stays negative and
// is rejected by the window kernel's column check).
template <typename I> __device__ __forceinline__ int64_t cube_col(I x) { return (int64_t)x >> 4; }

template <typename I>
__global__ void __launch_bounds__(kCubeThreads)
cube_count_kernel(const I *rowptr, const I *col, int64_t nwin, int64_t nnz, long long *count,
                  unsigned long long *tile, DevStatus *st)
{
    for (int64_t w = blockIdx.x; w < nwin; w += gridDim.x) {
        int64_t e0, e1;
        window_range(rowptr, w, nnz, e0, e1, st);
        long long n = 0;
        for (int64_t b = e0; b < e1; b += kCubeThreads) {
            const int64_t i = b + threadIdx.x;
            bool start = false;
            if (i < e1) start = i == e0 || cube_col(col[i]) != cube_col(col[i - 1]);
            n += __syncthreads_count(start);
        }
        if (threadIdx.x == 0) {
            count[w] = n;
            if (n) atomicAdd(tile + w / kTileWindows, (unsigned long long)n);
        }
    }
}

// tile[0..ntiles) -> exclusive offsets, tile[ntiles] = total (one CTA).
__global__ void __launch_bounds__(1024) cube_scan_tiles_kernel(unsigned long long *tile, int64_t ntiles)
{
    using Scan = cub::BlockScan<unsigned long long, 1024>;
    __shared__ typename Scan::TempStorage tmp;
    unsigned long long carry = 0;
    for (int64_t b = 0; b < ntiles; b += 1024) {
        const int64_t i = b + threadIdx.x;
        const unsigned long long x = i < ntiles ? tile[i] : 0ull;
        unsigned long long y, agg;
        Scan(tmp).ExclusiveSum(x, y, agg);
        if (i < ntiles) tile[i] = carry + y;
        carry += agg;
        __syncthreads();
    }
    if (threadIdx.x == 0) tile[ntiles] = carry;
}

template <typename T, typename I>
__global__ void __launch_bounds__(kCubeThreads)
cube_fill_kernel(const I *rowptr, const I *col, const T *val, int64_t nwin, int64_t nnz, const long long *count,
                 const unsigned long long *tile, I *cptr, I *ccol, T *cval, DevStatus *st)
{
    using Reduce = cub::BlockReduce<long long, kCubeThreads>;
    using Scan = cub::BlockScan<int, kCubeThreads>;
    __shared__ union {
        typename Reduce::TempStorage red;
        typename Scan::TempStorage scan;
    } tmp;
    __shared__ I s_col[kCubeThreads];
    __shared__ long long s_base;

    for (int64_t w = blockIdx.x; w < nwin; w += gridDim.x) {
        // Block offset of window w: its tile's offset plus the counts of the
        // earlier windows of the tile.
        const int64_t t0 = (w / kTileWindows) * kTileWindows;
        long long part = 0;
        for (int64_t j = t0 + threadIdx.x; j < w; j += kCubeThreads) part += count[j];
        const long long before = Reduce(tmp.red).Sum(part);
        if (threadIdx.x == 0) s_base = (long long)tile[w / kTileWindows] + before;
        __syncthreads();
        const long long base = s_base;
        const long long nblk = count[w];
        if (threadIdx.x == 0) {
            cptr[w] = (I)base;
            if (w == nwin - 1) cptr[nwin] = (I)(base + nblk);
        }
        // Zero the window's block values (16 per block, 16-byte stores).
        {
            constexpr int kVecPerBlock = 16 * (int)sizeof(T) / 16;
            uint4 *z = reinterpret_cast<uint4 *>(cval + 16 * base);
            for (long long k = threadIdx.x; k < nblk * kVecPerBlock; k += kCubeThreads) z[k] = make_uint4(0, 0, 0, 0);
        }
        int64_t e0, e1;
        window_range(rowptr, w, nnz, e0, e1, st);
        long long run = -1;   // block (within the window) of the previous entry
        __syncthreads();      // zeroing before the scatter
        for (int64_t b = e0; b < e1; b += kCubeThreads) {
            const int64_t i = b + threadIdx.x;
            const int len = (int)std::min<int64_t>(kCubeThreads, e1 - b);
            const bool valid = threadIdx.x < len;
            I x = 0;
            if (valid) x = col[i];
            s_col[threadIdx.x] = x;
            __syncthreads();
            const int64_t c = cube_col(x);
            bool start = false;
            if (valid) {
                const I prev = threadIdx.x > 0 ? s_col[threadIdx.x - 1] : (i > e0 ? col[i - 1] : x);
                start = i == e0 || c != cube_col(prev);
            }
            int rank, starts;
            Scan(tmp.scan).InclusiveSum(start ? 1 : 0, rank, starts);
            if (valid) {
                const long long blk = base + run + rank;
                if (start) ccol[blk] = (I)c;
                const int r = (int)(x & 15);
                bool later = false;   // a later entry of this run in this chunk has the same row
                for (int j = threadIdx.x + 1; j < len; ++j) {
                    const I y = s_col[j];
                    if (cube_col(y) != c) break;
                    if ((int)(y & 15) == r) { later = true; break; }
                }
                if (!later) cval[16 * blk + r] = val[i];
            }
            run += starts;
            __syncthreads();   // chunk order: later chunks overwrite earlier ones
        }
    }
}

unsigned cube_grid(int64_t nwin)
{
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(nwin, (int64_t)device_sm_count() * 16));
}

template <typename T, typename I>
cudaError_t run_cube(const CubeArgs &a, const CubeWorkspace &ws, cudaStream_t s)
{
    const int64_t ntiles = (a.nwin + kTileWindows - 1) / kTileWindows;
    cudaError_t e = cudaMemsetAsync(ws.tile, 0, 8 * (size_t)(ntiles + 1), s);
    if (e != cudaSuccess) return e;
    const I *rowptr = static_cast<const I *>(a.rowptr);
    const I *col = static_cast<const I *>(a.col);
    cube_count_kernel<I><<<cube_grid(a.nwin), kCubeThreads, 0, s>>>(rowptr, col, a.nwin, a.nnz, ws.count, ws.tile,
                                                                     a.status);
    cube_scan_tiles_kernel<<<1, 1024, 0, s>>>(ws.tile, ntiles);
    cube_fill_kernel<T, I><<<cube_grid(a.nwin), kCubeThreads, 0, s>>>(
        rowptr, col, static_cast<const T *>(a.val), a.nwin, a.nnz, ws.count, ws.tile, static_cast<I *>(ws.cptr),
        static_cast<I *>(ws.ccol), static_cast<T *>(ws.cval), a.status);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    WindowArgs w{};
    w.cptr = ws.cptr; w.ccol = ws.ccol; w.cval = ws.cval;
    w.vptr = nullptr; w.vcol = nullptr; w.vval = nullptr;
    w.B = a.B; w.out = a.out;
    w.nwin = a.nwin; w.nblocks = std::max<int64_t>(a.nnz, 1); w.vrows = 0; w.vnnz = 0;
    w.K = a.K; w.N = a.N; w.status = a.status;
    return launch_window(w, sizeof(I) == 4 ? SPMM_I32 : SPMM_I64, sizeof(T) == 2 ? SPMM_F16 : SPMM_F32, 1, s);
}

// ---- 16 x 16 tiles of csr_to_ascend_cube -------------------------------------
// The producer (custom_op.cpp:429-592) stores per window its distinct columns
// in tiles of 16 (unique_col_ids[16 t + k], the last tile zero-padded) and
// value[256 t + 16 r + k] = A[row r of the window, column k of tile t].  Tile
// t is exactly blocks 16 t .. 16 t + 15 of the (16 x 1)-block stream with
// each 16 x 16 value tile transposed, so the consumer transposes the tiles,
// scales the window pointer by 16 and runs the window kernel with the
// producer's column array as is.  Padding blocks (column 0, values 0) are
// summed like any other block.

struct TileWorkspace {
    void *cptr;   // I [nwin + 1]
    void *cval;   // T [256 * max(ntiles, 1)]
    size_t bytes;
};

TileWorkspace carve_tiles(void *base, int64_t nwin, int64_t ntiles, int isz, int vsz)
{
    TileWorkspace w{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = base ? static_cast<char *>(base) + off : nullptr;
        off += align256(bytes);
        return static_cast<void *>(p);
    };
    w.cptr = take((size_t)isz * (size_t)(nwin + 1));
    w.cval = take((size_t)vsz * 256 * (size_t)std::max<int64_t>(ntiles, 1));
    w.bytes = off;
    return w;
}

// One 256-thread CTA per tile (grid-stride): coalesced load of the tile,
// transposed through shared memory, coalesced store.  CTA 0 also writes the
// block pointer; a window pointer outside [0, ntiles] becomes -1, which the
// window kernel reports as a malformed pointer.
template <typename T, typename I>
__global__ void __launch_bounds__(256)
tiles_to_blocks_kernel(const I *tptr, const T *tval, int64_t nwin, int64_t ntiles, I *cptr, T *cval)
{
    __shared__ T s[16][17];
    if (blockIdx.x == 0) {
        for (int64_t w = threadIdx.x; w <= nwin; w += blockDim.x) {
            const int64_t p = (int64_t)tptr[w];
            cptr[w] = (p < 0 || p > ntiles) ? (I)-1 : (I)(16 * p);
        }
    }
    const int r = threadIdx.x >> 4, k = threadIdx.x & 15;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        s[r][k] = tval[256 * t + threadIdx.x];                  // value[256 t + 16 r + k]
        __syncthreads();
        cval[256 * t + threadIdx.x] = s[k][r];                  // block 16 t + r, row k
        __syncthreads();
    }
}

template <typename T, typename I>
cudaError_t run_tiles(const TileArgs &a, const TileWorkspace &ws, cudaStream_t s)
{
    const unsigned grid = (unsigned)std::max<int64_t>(
        1, std::min<int64_t>(a.ntiles, (int64_t)device_sm_count() * 8));
    tiles_to_blocks_kernel<T, I><<<grid, 256, 0, s>>>(static_cast<const I *>(a.tptr), static_cast<const T *>(a.val),
                                                      a.nwin, a.ntiles, static_cast<I *>(ws.cptr),
                                                      static_cast<T *>(ws.cval));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    WindowArgs w{};
    w.cptr = ws.cptr; w.ccol = a.col; w.cval = ws.cval;
    w.vptr = nullptr; w.vcol = nullptr; w.vval = nullptr;
    w.B = a.B; w.out = a.out;
    w.nwin = a.nwin; w.nblocks = 16 * a.ntiles; w.vrows = 0; w.vnnz = 0;
    w.K = a.K; w.N = a.N; w.status = a.status;
    return launch_window(w, sizeof(I) == 4 ? SPMM_I32 : SPMM_I64, sizeof(T) == 2 ? SPMM_F16 : SPMM_F32, 1, s);
}

}  // namespace

size_t tiles_workspace_bytes(int64_t nwin, int64_t ntiles, int itype, int dtype)
{
    return carve_tiles(nullptr, nwin, ntiles, itype == SPMM_I32 ? 4 : 8, dtype == SPMM_F16 ? 2 : 4).bytes;
}

cudaError_t launch_tiles(const TileArgs &a, int itype, int dtype, void *workspace, cudaStream_t stream)
{
    if (a.nwin <= 0) return cudaSuccess;
    const TileWorkspace ws = carve_tiles(workspace, a.nwin, a.ntiles, itype == SPMM_I32 ? 4 : 8,
                                         dtype == SPMM_F16 ? 2 : 4);
    if (dtype == SPMM_F16)
        return itype == SPMM_I32 ? run_tiles<__half, int>(a, ws, stream) : run_tiles<__half, int64_t>(a, ws, stream);
    return itype == SPMM_I32 ? run_tiles<float, int>(a, ws, stream) : run_tiles<float, int64_t>(a, ws, stream);
}

size_t cube_workspace_bytes(int64_t nwin, int64_t nnz, int itype, int dtype)
{
    return carve(nullptr, nwin, nnz, itype == SPMM_I32 ? 4 : 8, dtype == SPMM_F16 ? 2 : 4).bytes;
}

cudaError_t launch_cube(const CubeArgs &a, int itype, int dtype, void *workspace, cudaStream_t stream)
{
    if (a.nwin <= 0) return cudaSuccess;
    const CubeWorkspace ws = carve(workspace, a.nwin, a.nnz, itype == SPMM_I32 ? 4 : 8, dtype == SPMM_F16 ? 2 : 4);
    if (dtype == SPMM_F16)
        return itype == SPMM_I32 ? run_cube<__half, int>(a, ws, stream) : run_cube<__half, int64_t>(a, ws, stream);
    return itype == SPMM_I32 ? run_cube<float, int>(a, ws, stream) : run_cube<float, int64_t>(a, ws, stream);
}

}  // namespace spmmb
