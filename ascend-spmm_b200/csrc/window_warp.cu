// Window path, warp-pipelined kernels: tensor cores for fp16 (N % 64 == 0),
// CUDA cores for fp32 (N % 128 == 0).
//
// Same semantics as window.cu (reference: op_kernel/spmm_ascend_cube.cpp:
// 52-165, 265-288, and the vector-core rows added on top, :782-875): window
// slot s owns output rows [16s, 16s + 16) = sum over its (16 x 1) blocks of
// Cvalue[16b + i] * B[Ccol[b], :] plus the CSR entries of those rows, summed
// in fp32 and rounded once.
//
// Design: a warp owns (window, feature slice of FW = 64, 128 or 256 features) and
// runs on its own, no block-wide barrier.  The window's stream - its blocks,
// then the CSR entries of its rows - is consumed in chunks of 16 entries:
//  * gathers: the 16 B-row slices of a chunk go by 16-byte cp.async into the
//    warp's STAGES-deep shared-memory ring together with the chunk's 16 x 16
//    value tile (blocks) or its 16 values (CSR entries); the column indices
//    of chunk x travel one pipeline depth earlier, in the copy group of chunk
//    x - STAGES + 1, so no global load is ever waited on inside the loop;
//  * math: D[feature, row] += sum_k Bg[k, feature] * V[k, row] with
//    mma.sync m16n8k16, features as M (ldmatrix.trans of the staged rows),
//    window rows as N in two halves of 8; for blocks the value tile is read
//    with one ldmatrix.x4.trans, for CSR entries a value is placed at its
//    row by comparing its position with the row ranges held in lanes;
//  * epilogue: the 16 x FW fp32 tile is rounded to fp16 and written through
//    a stmatrix.trans transpose as 16-byte row segments.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ void cp16(unsigned dst, const void *src, int bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void wait_groups() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
__device__ __forceinline__ void ldsm4t(unsigned addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void stsm4t(unsigned addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3)
{
    asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(r0),
                 "r"(r1), "r"(r2), "r"(r3)
                 : "memory");
}
__device__ __forceinline__ void mma(float *d, const uint32_t *a, uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2(float lo, float hi)
{
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ unsigned lds16u(unsigned addr)
{
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ int64_t lds_idx(unsigned addr, int isz)
{
    if (isz == 4) {
        int v;
        asm volatile("ld.shared.s32 %0, [%1];\n" : "=r"(v) : "r"(addr));
        return v;
    }
    long long v;
    asm volatile("ld.shared.s64 %0, [%1];\n" : "=l"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds128(unsigned addr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ int64_t ld_pinned(const int64_t *p)
{
    long long v;
    asm volatile("ld.global.nc.s64 %0, [%1];\n" : "=l"(v) : "l"(p));
    return v;
}

// ---------------------------------------------------------------------------
// Item schedule (WindowArgs::sched).  Windows differ in length by two orders
// of magnitude and are not sorted (config 2: 4 to 277 chunks per item), so a
// static item order leaves the warp with the heaviest items running long
// after the others (SMs active 58 % of the kernel on config 2).  The schedule
// lists the items of at least kHeavyChunks chunks first and the rest after
// them; warps claim positions in that list with an atomic counter, the
// heavy items going out first (longest-first list scheduling).  Which warp
// computes an item does not change how it is computed, so results are the
// same bit for bit under any schedule.
// Layout: three 64-bit counters (heavy and light windows placed, claim
// counter) in a kSchedHeader-byte header, then the item order (int64 per
// item; item = window * slices + slice).
// ---------------------------------------------------------------------------
constexpr int kSchedHeader = 256;
constexpr int kHeavyChunks = 16;

// One block per contiguous range of windows.  A window's slices share its
// cost, so heaviness is decided per window: pass 1 counts the block's heavy
// and light windows, one atomic per list reserves the block's positions,
// pass 2 writes the items (window-major, slices consecutive).
template <typename I>
__global__ void __launch_bounds__(256)
window_order_kernel(const WindowArgs a, int nslices)
{
    __shared__ unsigned long long s_count[2], s_base[2];
    unsigned long long *cursor = static_cast<unsigned long long *>(a.sched);
    int64_t *order = reinterpret_cast<int64_t *>(static_cast<char *>(a.sched) + kSchedHeader);
    const I *cptr = static_cast<const I *>(a.cptr);
    const I *vptr = static_cast<const I *>(a.vptr);
    const int64_t nitems = a.nwin * nslices;
    const int64_t per = (a.nwin + gridDim.x - 1) / gridDim.x;
    const int64_t w0 = min(a.nwin, (int64_t)blockIdx.x * per), w1 = min(a.nwin, w0 + per);
    const int lane = threadIdx.x & 31;
    const unsigned below = (1u << lane) - 1u;
    // malformed bounds count as empty here; the window kernel reports them
    auto heavy_window = [&](int64_t s) {
        const int64_t cb = ld_idx(cptr + s), ce = ld_idx(cptr + s + 1);
        const int64_t nb = (cb >= 0 && ce >= cb && ce <= a.nblocks) ? ce - cb : 0;
        int64_t nv = 0;
        if (a.vrows > 0 && 16 * s < a.vrows) {
            const int64_t vb = ld_idx(vptr + 16 * s), ve = ld_idx(vptr + min(16 * s + 16, a.vrows));
            nv = (vb >= 0 && ve >= vb && ve <= a.vnnz) ? ve - vb : 0;
        }
        return (nb + 15) / 16 + (nv + 15) / 16 >= kHeavyChunks;
    };
    if (threadIdx.x < 2) s_count[threadIdx.x] = 0;
    __syncthreads();
    for (int64_t base = w0 + (threadIdx.x & ~31); base < w1; base += blockDim.x) {
        const int64_t s = base + lane;
        const bool valid = s < w1;
        const unsigned hm = __ballot_sync(kFull, valid && heavy_window(s));
        const unsigned vm = __ballot_sync(kFull, valid);
        if (lane == 0) {
            atomicAdd(&s_count[0], (unsigned long long)__popc(hm));
            atomicAdd(&s_count[1], (unsigned long long)__popc(vm & ~hm));
        }
    }
    __syncthreads();
    if (threadIdx.x < 2) {
        s_base[threadIdx.x] = s_count[threadIdx.x] ? atomicAdd(cursor + threadIdx.x, s_count[threadIdx.x]) : 0;
        s_count[threadIdx.x] = 0;
    }
    __syncthreads();
    for (int64_t base = w0 + (threadIdx.x & ~31); base < w1; base += blockDim.x) {
        const int64_t s = base + lane;
        const bool valid = s < w1;
        const bool heavy = valid && heavy_window(s);
        const unsigned hm = __ballot_sync(kFull, heavy);
        const unsigned lm = __ballot_sync(kFull, valid && !heavy);
        unsigned long long ho = 0, lo = 0;
        if (lane == 0) {
            if (hm) ho = atomicAdd(&s_count[0], (unsigned long long)__popc(hm));
            if (lm) lo = atomicAdd(&s_count[1], (unsigned long long)__popc(lm));
        }
        ho = __shfl_sync(kFull, ho, 0);
        lo = __shfl_sync(kFull, lo, 0);
        if (valid) {
            const int64_t rank = heavy ? (int64_t)(s_base[0] + ho + __popc(hm & below))
                                       : (int64_t)(s_base[1] + lo + __popc(lm & below));
            for (int k = 0; k < nslices; ++k) {
                const int64_t item = s * nslices + k;
                if (heavy) order[rank * nslices + k] = item;
                else order[nitems - 1 - (rank * nslices + k)] = item;
            }
        }
    }
}

// Zeroes the counters and writes the item order (stream-ordered, so a
// captured graph replays it too).
template <typename I>
cudaError_t build_schedule(const WindowArgs &a, int nslices, cudaStream_t stream)
{
    cudaError_t e = cudaMemsetAsync(a.sched, 0, 3 * sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return e;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((a.nwin + 255) / 256, 8 * (int64_t)device_sm_count()));
    window_order_kernel<I><<<(unsigned)grid, 256, 0, stream>>>(a, nslices);
    return cudaGetLastError();
}

template <int FW, int STAGES, int WARPS> struct WinShape {
    static constexpr int kPitch = FW * 2 + 16;     // staged B row (16-byte pad: conflict-free ldmatrix)
    static constexpr int kVPitch = 48;             // value-tile row: 16 values + pad (conflict-free ldmatrix)
    static constexpr int kRows = 0;
    static constexpr int kTile = kRows + 16 * kPitch;   // 16 x 16 value tile, or the values of 16 CSR entries
    static constexpr int kCols = kTile + 16 * kVPitch;  // column indices of a later chunk (aligned copy)
    static constexpr int kStage = kCols + 160;
    // The 16-row epilogue tile reuses the ring (it is written only after the
    // last copy of the window has landed).
    static_assert(16 * kPitch <= STAGES * kStage, "epilogue tile fits in the ring");
    static constexpr int kWarp = (STAGES * kStage + 127) / 128 * 128;
    static constexpr int kBlock = WARPS * kWarp;
};

template <typename I, int FW, int STAGES, int WARPS, int MINB>
__global__ void __launch_bounds__(WARPS * 32, MINB)
window_warp_kernel(const WindowArgs a, int nslices)
{
    using L = WinShape<FW, STAGES, WARPS>;
    constexpr int PITCH = L::kPitch;
    constexpr int NMT = FW / 16;
    constexpr int PIECES = FW / 8;
    constexpr int ISZ = sizeof(I);
    extern __shared__ __align__(128) unsigned char win_smem[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const unsigned base = (unsigned)__cvta_generic_to_shared(win_smem) + (unsigned)(wid * L::kWarp);
    const unsigned epi = base;   // epilogue tile over the drained ring

    const I *cptr = static_cast<const I *>(a.cptr);
    const I *ccol = static_cast<const I *>(a.ccol);
    const char *cval = static_cast<const char *>(a.cval);
    const I *vptr = static_cast<const I *>(a.vptr);
    const I *vcol = static_cast<const I *>(a.vcol);
    const char *vval = static_cast<const char *>(a.vval);
    const char *B = static_cast<const char *>(a.B);
    char *out = static_cast<char *>(a.out);
    const int64_t rowbytes = a.N * 2;
    const int rowb = (int)rowbytes;   // N <= 1024 (the operators' width contract)

    const int64_t nitems = a.nwin * nslices;
    // items: claimed from the schedule when there is one (the next claim is
    // in flight while an item runs), else a static grid stride
    unsigned long long *claim = a.sched ? static_cast<unsigned long long *>(a.sched) + 2 : nullptr;
    const int64_t *order =
        a.sched ? reinterpret_cast<const int64_t *>(static_cast<const char *>(a.sched) + kSchedHeader) : nullptr;
    int64_t it = (int64_t)blockIdx.x * WARPS + wid;
    if (claim) {
        unsigned long long p = 0;
        if (lane == 0) p = atomicAdd(claim, 1ull);
        p = __shfl_sync(kFull, p, 0);
        it = p < (unsigned long long)nitems ? ld_pinned(order + p) : nitems;
    }
    while (it < nitems) {
        unsigned long long np = 0;   // lane 0: the next claimed position
        if (claim && lane == 0) np = atomicAdd(claim, 1ull);
        const int64_t s = it / nslices;
        const int f0 = (int)(it % nslices) * FW;
        const char *Bf = B + f0 * 2 + (lane % PIECES) * 16;   // this lane's piece of B row 0's slice

        // ---- the window's stream: blocks [cb, cb + nb), CSR entries [vb, vb + nv)
        int64_t cb = ld_idx(cptr + s), ce = ld_idx(cptr + s + 1);
        if (cb < 0 || ce < cb || ce > a.nblocks) {
            if (lane == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, s);
            cb = ce = 0;
        }
        // lane r < 17 holds vptr[16 s + r] (rows past vrows are empty)
        int64_t vr = 0;
        if (a.vrows > 0 && 16 * s < a.vrows) vr = ld_idx(vptr + min(16 * s + min(lane, 16), a.vrows));
        int64_t vb = __shfl_sync(kFull, vr, 0), ve = __shfl_sync(kFull, vr, 16);
        {
            const int64_t nxt = __shfl_down_sync(kFull, vr, 1);
            const bool bad = (lane == 0 && (vb < 0 || ve > a.vnnz)) || (lane < 16 && nxt < vr);
            if (__any_sync(kFull, bad)) {
                if (lane == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, 16 * s);
                vb = ve = 0;
                vr = 0;
            }
        }
        const int nb = (int)(ce - cb), nv = (int)(ve - vb);
        const int nbc = (nb + 15) >> 4, nvc = (nv + 15) >> 4;
        const int nch = nbc + nvc;
        // row ranges of window rows g and 8 + g, relative to vb (CSR entries)
        const int rb0 = (int)(__shfl_sync(kFull, vr, g) - vb), re0 = (int)(__shfl_sync(kFull, vr, g + 1) - vb);
        const int rb1 = (int)(__shfl_sync(kFull, vr, g + 8) - vb), re1 = (int)(__shfl_sync(kFull, vr, g + 9) - vb);
        const int misb = (int)((cb * ISZ) & 15), misv = (int)((vb * ISZ) & 15);   // column-array misalignment
        const int misval = (int)((vb * 2) & 15);                                  // value-array misalignment

        // Column indices of chunk x into the col slot of stage st: the
        // aligned 16-byte pieces covering its 16 (or fewer) indices.
        auto stage_cols = [&](int x, unsigned st) {
            if (x >= nch) return;
            const bool blk = x < nbc;
            const char *arr = blk ? reinterpret_cast<const char *>(ccol) : reinterpret_cast<const char *>(vcol);
            const int64_t first = blk ? cb + 16 * x : vb + 16 * (x - nbc);
            const int64_t count = blk ? min(16, nb - 16 * x) : min(16, nv - 16 * (x - nbc));
            const int64_t b0 = first * ISZ, b1 = (first + count) * ISZ;
            const int64_t p0 = b0 & ~int64_t(15);
            const int npieces = (int)((b1 - p0 + 15) >> 4);
            if (lane < npieces) {
                const int64_t pb = p0 + 16 * lane;
                const int bytes = (int)max((int64_t)0, min((int64_t)16, b1 - pb));
                cp16(st + L::kCols + 16 * lane, arr + (bytes > 0 ? pb : 0), bytes);
            }
        };
        // Gathers (and values) of chunk x into stage st; its columns sit in
        // that stage's col slot already.
        auto stage_rows = [&](int x, unsigned st) {
            if (x >= nch) return;
            const bool blk = x < nbc;
            const int k = lane & 15;
            const int cnt = blk ? min(16, nb - 16 * x) : min(16, nv - 16 * (x - nbc));
            const int mis = blk ? misb : misv;
            int64_t c = -1;
            if (k < cnt) {
                c = lds_idx(st + L::kCols + mis + k * ISZ, ISZ);
                if (c < 0 || c >= a.K) {
                    if (lane < 16) raise_status(a.status, SPMM_DEV_BAD_COLUMN, s);
                    c = -1;
                }
            }
            const int cc = (int)c;
            constexpr int RPI = 32 / PIECES;   // rows per instruction
            const int v = lane % PIECES;
#pragma unroll
            for (int i = 0; i < 16 / RPI; ++i) {
                const int kk = lane / PIECES + RPI * i;
                const int ck = __shfl_sync(kFull, cc, kk);
                const char *src = Bf + (int64_t)(ck >= 0 ? ck : 0) * rowb;   // 32 x 32 -> 64-bit multiply-add
                cp16(st + (unsigned)(kk * PITCH + v * 16), src, ck >= 0 ? 16 : 0);
            }
            if (blk) {
                // 16 blocks x 16 values, contiguous: lane -> half a block column
                const int kk = lane >> 1, h = lane & 1;
                const bool ok = kk < cnt;
                const char *src = cval + ((cb + 16 * x + (ok ? kk : 0)) * 16 + 8 * h) * 2;
                cp16(st + L::kTile + (unsigned)(kk * L::kVPitch + 16 * h), src, ok ? 16 : 0);
            } else if (lane < 3) {
                // the chunk's values: aligned pieces covering 16 fp16 entries
                const int64_t b0 = (vb + 16 * (x - nbc)) * 2, b1 = b0 + 2 * cnt;
                const int64_t pb = (b0 & ~int64_t(15)) + 16 * lane;
                const int bytes = (int)max((int64_t)0, min((int64_t)16, b1 - pb));
                cp16(st + L::kTile + 16 * lane, vval + (bytes > 0 ? pb : 0), bytes);
            }
        };
        auto stage_of = [&](int x) -> unsigned { return base + (unsigned)((x % STAGES) * L::kStage); };

        float acc0[NMT][4], acc1[NMT][4];
#pragma unroll
        for (int m = 0; m < NMT; ++m)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc0[m][e] = acc1[m][e] = 0.f;

        // prologue: columns of chunks 0 .. STAGES-2, then their gathers (each
        // group also carries the columns of the chunk STAGES-1 further on)
#pragma unroll
        for (int x = 0; x < STAGES - 1; ++x) stage_cols(x, stage_of(x));
        commit();
        wait_groups<0>();
        __syncwarp();
#pragma unroll
        for (int x = 0; x < STAGES - 1; ++x) {
            stage_rows(x, stage_of(x));
            stage_cols(x + STAGES - 1, stage_of(x + STAGES - 1));
            commit();
        }
        // the next item (its order entry loads while this one runs)
        int64_t nit = it + (int64_t)gridDim.x * WARPS;
        if (claim) {
            np = __shfl_sync(kFull, np, 0);
            nit = np < (unsigned long long)nitems ? ld_pinned(order + np) : nitems;
        }

        for (int c = 0; c < nch; ++c) {
            wait_groups<STAGES - 2>();
            __syncwarp();
            // group c + STAGES - 1: gathers of that chunk (columns arrived with
            // group c) and the columns of chunk c + 2 STAGES - 2
            {
                const int x = c + STAGES - 1;
                stage_rows(x, stage_of(x));
                stage_cols(x + STAGES - 1, stage_of(x + STAGES - 1));
                commit();
            }
            const unsigned st = stage_of(c);
            uint32_t bb[4];   // B operand: {b0, b1} for rows 0-7, then rows 8-15
            if (c < nbc) {
                const int tile = lane >> 3;
                ldsm4t(st + L::kTile + (unsigned)(((tile & 1) * 8 + (lane & 7)) * L::kVPitch + (tile >> 1) * 16),
                       bb[0], bb[1], bb[2], bb[3]);
            } else {
                const int q = 16 * (c - nbc) + 2 * t;   // positions q, q+1, q+8, q+9 (relative to vb)
                const unsigned vs = st + L::kTile + (unsigned)misval;
                const unsigned v0 = lds16u(vs + 2 * (2 * t)), v1 = lds16u(vs + 2 * (2 * t + 1));
                const unsigned v2 = lds16u(vs + 2 * (2 * t + 8)), v3 = lds16u(vs + 2 * (2 * t + 9));
                const unsigned w0 = (unsigned)(re0 - rb0), w1 = (unsigned)(re1 - rb1);
                bb[0] = (((unsigned)(q - rb0) < w0) ? v0 : 0u) | ((((unsigned)(q + 1 - rb0) < w0) ? v1 : 0u) << 16);
                bb[1] = (((unsigned)(q + 8 - rb0) < w0) ? v2 : 0u) | ((((unsigned)(q + 9 - rb0) < w0) ? v3 : 0u) << 16);
                bb[2] = (((unsigned)(q - rb1) < w1) ? v0 : 0u) | ((((unsigned)(q + 1 - rb1) < w1) ? v1 : 0u) << 16);
                bb[3] = (((unsigned)(q + 8 - rb1) < w1) ? v2 : 0u) | ((((unsigned)(q + 9 - rb1) < w1) ? v3 : 0u) << 16);
            }
#pragma unroll
            for (int m = 0; m < NMT; ++m) {
                const int tile = lane >> 3;
                uint32_t af[4];
                ldsm4t(st + (unsigned)(((tile >> 1) * 8 + (lane & 7)) * PITCH + (16 * m + 8 * (tile & 1)) * 2), af[0],
                       af[1], af[2], af[3]);
                mma(acc0[m], af, bb[0], bb[1]);
                mma(acc1[m], af, bb[2], bb[3]);
            }
        }
        wait_groups<0>();
        __syncwarp();

        // ---- epilogue: rows 16 s .. 16 s + 15, fp16, through the transpose tile
#pragma unroll
        for (int m = 0; m < NMT; m += 2) {
            const int tile = lane >> 3;
            const unsigned fo = (unsigned)((16 * (m + (tile >> 1)) + 8 * (tile & 1)) * 2);
            stsm4t(epi + (unsigned)((lane & 7) * PITCH) + fo, h2(acc0[m][0], acc0[m][1]), h2(acc0[m][2], acc0[m][3]),
                   h2(acc0[m + 1][0], acc0[m + 1][1]), h2(acc0[m + 1][2], acc0[m + 1][3]));
            stsm4t(epi + (unsigned)((8 + (lane & 7)) * PITCH) + fo, h2(acc1[m][0], acc1[m][1]),
                   h2(acc1[m][2], acc1[m][3]), h2(acc1[m + 1][0], acc1[m + 1][1]), h2(acc1[m + 1][2], acc1[m + 1][3]));
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < PIECES / 2; ++i) {
            const int idx = lane + 32 * i;
            const int n = idx / PIECES, v = idx % PIECES;
            uint4 *o = reinterpret_cast<uint4 *>(out + (16 * s + n) * rowbytes + f0 * 2) + v;
            __stcs(o, lds128(epi + (unsigned)(n * PITCH + v * 16)));
        }
        __syncwarp();
        it = nit;
    }
}

template <typename I, int FW, int STAGES, int WARPS>
cudaError_t launch_ww(const WindowArgs &a, cudaStream_t stream)
{
    using L = WinShape<FW, STAGES, WARPS>;
    constexpr int MINB = std::max(1, (220 * 1024) / L::kBlock);
    auto kern = window_warp_kernel<I, FW, STAGES, WARPS, MINB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBlock);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, WARPS * 32, L::kBlock);
    if (e != cudaSuccess) return e;
    const int nslices = (int)(a.N / FW);
    const int64_t items = a.nwin * nslices;
    if (a.sched && (e = build_schedule<I>(a, nslices, stream)) != cudaSuccess) return e;
    int64_t blocks = (int64_t)std::max(per_sm, 1) * device_sm_count();
    blocks = std::max<int64_t>(1, std::min(blocks, (items + WARPS - 1) / WARPS));
    kern<<<(unsigned)blocks, WARPS * 32, L::kBlock, stream>>>(a, nslices);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// fp32: same stream and pipeline, CUDA-core math.  Lane l owns features
// f0 + 4 l .. f0 + 4 l + 3 of all 16 window rows (64 fp32 accumulators) and
// multiplies with packed fma.rn.f32x2 (an IEEE fp32 fma per lane half; TF32
// tensor cores would miss the 1e-4 tolerance).  A block updates all 16 rows
// from its value column; a CSR entry updates only its row, chosen by a
// warp-uniform switch.  Sums run over the window's blocks in order, then its
// CSR entries in order.
// ---------------------------------------------------------------------------
template <int STAGES, int WARPS> struct WinShapeF32 {
    static constexpr int kPitch = 512;             // 128 fp32 features per staged row
    static constexpr int kTile = 16 * kPitch;      // 16 x 16 fp32 value tile (k-major), or 16 CSR values
    static constexpr int kCols = kTile + 16 * 64 + 16;
    static constexpr int kStage = kCols + 160;
    static constexpr int kWarp = (STAGES * kStage + 127) / 128 * 128;
    static constexpr int kBlock = WARPS * kWarp;
};

__device__ __forceinline__ void fma2(float &x, float &y, float v, float bx, float by)
{
    asm("{\n\t.reg .b64 a, vv, bb;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 vv, {%2, %2};\n\tmov.b64 bb, {%3, %4};\n\t"
        "fma.rn.f32x2 a, vv, bb, a;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "+f"(x), "+f"(y)
        : "f"(v), "f"(bx), "f"(by));
}
__device__ __forceinline__ float4 lds_f4(unsigned addr)
{
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];\n" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float lds_f(unsigned addr)
{
    float v;
    asm volatile("ld.shared.f32 %0, [%1];\n" : "=f"(v) : "r"(addr));
    return v;
}

template <typename I, int STAGES, int WARPS, int MINB>
__global__ void __launch_bounds__(WARPS * 32, MINB)
window_warp_f32_kernel(const WindowArgs a, int nslices)
{
    using L = WinShapeF32<STAGES, WARPS>;
    constexpr int FW = 128;
    constexpr int ISZ = sizeof(I);
    extern __shared__ __align__(128) unsigned char win_smem[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const unsigned base = (unsigned)__cvta_generic_to_shared(win_smem) + (unsigned)(wid * L::kWarp);

    const I *cptr = static_cast<const I *>(a.cptr);
    const I *ccol = static_cast<const I *>(a.ccol);
    const char *cval = static_cast<const char *>(a.cval);
    const I *vptr = static_cast<const I *>(a.vptr);
    const I *vcol = static_cast<const I *>(a.vcol);
    const char *vval = static_cast<const char *>(a.vval);
    const char *B = static_cast<const char *>(a.B);
    char *out = static_cast<char *>(a.out);
    const int64_t rowbytes = a.N * 4;

    const int64_t nitems = a.nwin * nslices;
    // position q of the schedule's item order (heavy items on the first
    // blocks), or item q itself without a schedule
    const int64_t *order =
        a.sched ? reinterpret_cast<const int64_t *>(static_cast<const char *>(a.sched) + kSchedHeader) : nullptr;
    for (int64_t q = (int64_t)blockIdx.x * WARPS + wid; q < nitems; q += (int64_t)gridDim.x * WARPS) {
        const int64_t it = order ? ld_idx(order + q) : q;
        const int64_t s = it / nslices;
        const int f0 = (int)(it % nslices) * FW;

        int64_t cb = ld_idx(cptr + s), ce = ld_idx(cptr + s + 1);
        if (cb < 0 || ce < cb || ce > a.nblocks) {
            if (lane == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, s);
            cb = ce = 0;
        }
        int64_t vr = 0;
        if (a.vrows > 0 && 16 * s < a.vrows) vr = ld_idx(vptr + min(16 * s + min(lane, 16), a.vrows));
        int64_t vb = __shfl_sync(kFull, vr, 0), ve = __shfl_sync(kFull, vr, 16);
        {
            const int64_t nxt = __shfl_down_sync(kFull, vr, 1);
            const bool bad = (lane == 0 && (vb < 0 || ve > a.vnnz)) || (lane < 16 && nxt < vr);
            if (__any_sync(kFull, bad)) {
                if (lane == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, 16 * s);
                vb = ve = 0;
                vr = 0;
            }
        }
        const int nb = (int)(ce - cb), nv = (int)(ve - vb);
        const int nbc = (nb + 15) >> 4, nvc = (nv + 15) >> 4;
        const int nch = nbc + nvc;
        // lane r < 16: end of window row r (relative to vb)
        const int rend = (int)(__shfl_down_sync(kFull, vr, 1) - vb);
        const int misb = (int)((cb * ISZ) & 15), misv = (int)((vb * ISZ) & 15);
        const int misval = (int)((vb * 4) & 15);

        auto stage_cols = [&](int x, unsigned st) {
            if (x >= nch) return;
            const bool blk = x < nbc;
            const char *arr = blk ? reinterpret_cast<const char *>(ccol) : reinterpret_cast<const char *>(vcol);
            const int64_t first = blk ? cb + 16 * x : vb + 16 * (x - nbc);
            const int64_t count = blk ? min(16, nb - 16 * x) : min(16, nv - 16 * (x - nbc));
            const int64_t b0 = first * ISZ, b1 = (first + count) * ISZ;
            const int64_t p0 = b0 & ~int64_t(15);
            const int npieces = (int)((b1 - p0 + 15) >> 4);
            if (lane < npieces) {
                const int64_t pb = p0 + 16 * lane;
                const int bytes = (int)max((int64_t)0, min((int64_t)16, b1 - pb));
                cp16(st + L::kCols + 16 * lane, arr + (bytes > 0 ? pb : 0), bytes);
            }
        };
        auto stage_rows = [&](int x, unsigned st) {
            if (x >= nch) return;
            const bool blk = x < nbc;
            const int cnt = blk ? min(16, nb - 16 * x) : min(16, nv - 16 * (x - nbc));
            const int mis = blk ? misb : misv;
            // column of row k held by lane k
            int64_t c = -1;
            if (lane < cnt) {
                c = lds_idx(st + L::kCols + mis + lane * ISZ, ISZ);
                if (c < 0 || c >= a.K) {
                    raise_status(a.status, SPMM_DEV_BAD_COLUMN, s);
                    c = -1;
                }
            }
            const int cc = (int)c;
            // 16 rows x 512 bytes: one row per instruction, lane -> 16-byte piece
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int ck = __shfl_sync(kFull, cc, k);
                const char *src = B + (int64_t)(ck >= 0 ? ck : 0) * rowbytes + f0 * 4 + lane * 16;
                cp16(st + (unsigned)(k * L::kPitch + lane * 16), src, ck >= 0 ? 16 : 0);
            }
            if (blk) {
                // 16 blocks x 16 fp32 values, contiguous: 64 pieces
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int piece = lane + 32 * h, kk = piece >> 2;
                    const bool ok = kk < cnt;
                    const char *src = cval + ((cb + 16 * x + (ok ? kk : 0)) * 16 + 4 * (piece & 3)) * 4;
                    cp16(st + L::kTile + (unsigned)(piece * 16), src, ok ? 16 : 0);
                }
            } else if (lane < 5) {
                const int64_t b0 = (vb + 16 * (x - nbc)) * 4, b1 = b0 + 4 * cnt;
                const int64_t pb = (b0 & ~int64_t(15)) + 16 * lane;
                const int bytes = (int)max((int64_t)0, min((int64_t)16, b1 - pb));
                cp16(st + L::kTile + 16 * lane, vval + (bytes > 0 ? pb : 0), bytes);
            }
        };
        auto stage_of = [&](int x) -> unsigned { return base + (unsigned)((x % STAGES) * L::kStage); };

        float acc[16][4];
#pragma unroll
        for (int r = 0; r < 16; ++r) acc[r][0] = acc[r][1] = acc[r][2] = acc[r][3] = 0.f;

#pragma unroll
        for (int x = 0; x < STAGES - 1; ++x) stage_cols(x, stage_of(x));
        commit();
        wait_groups<0>();
        __syncwarp();
#pragma unroll
        for (int x = 0; x < STAGES - 1; ++x) {
            stage_rows(x, stage_of(x));
            stage_cols(x + STAGES - 1, stage_of(x + STAGES - 1));
            commit();
        }

        for (int c = 0; c < nch; ++c) {
            wait_groups<STAGES - 2>();
            __syncwarp();
            {
                const int x = c + STAGES - 1;
                stage_rows(x, stage_of(x));
                stage_cols(x + STAGES - 1, stage_of(x + STAGES - 1));
                commit();
            }
            const unsigned st = stage_of(c);
            if (c < nbc) {
                const int cnt = min(16, nb - 16 * c);
                for (int k = 0; k < cnt; ++k) {
                    const float4 b = lds_f4(st + (unsigned)(k * L::kPitch + lane * 16));
                    const unsigned vt = st + L::kTile + (unsigned)(k * 64);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 v = lds_f4(vt + 16 * q);
                        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            fma2(acc[4 * q + i][0], acc[4 * q + i][1], vv[i], b.x, b.y);
                            fma2(acc[4 * q + i][2], acc[4 * q + i][3], vv[i], b.z, b.w);
                        }
                    }
                }
            } else {
                const int p0 = 16 * (c - nbc);
                const int cnt = min(16, nv - p0);
                for (int k = 0; k < cnt; ++k) {
                    const float4 b = lds_f4(st + (unsigned)(k * L::kPitch + lane * 16));
                    const float v = lds_f(st + L::kTile + (unsigned)(misval + 4 * k));
                    // row of position p0 + k: number of window rows ending at or before it
                    const int row = __popc(__ballot_sync(kFull, lane < 16 && rend <= p0 + k));
                    switch (row) {
#define SPMM_ROW_CASE(R)                                  \
    case R:                                               \
        fma2(acc[R][0], acc[R][1], v, b.x, b.y);          \
        fma2(acc[R][2], acc[R][3], v, b.z, b.w);          \
        break;
                        SPMM_ROW_CASE(0) SPMM_ROW_CASE(1) SPMM_ROW_CASE(2) SPMM_ROW_CASE(3)
                        SPMM_ROW_CASE(4) SPMM_ROW_CASE(5) SPMM_ROW_CASE(6) SPMM_ROW_CASE(7)
                        SPMM_ROW_CASE(8) SPMM_ROW_CASE(9) SPMM_ROW_CASE(10) SPMM_ROW_CASE(11)
                        SPMM_ROW_CASE(12) SPMM_ROW_CASE(13) SPMM_ROW_CASE(14) SPMM_ROW_CASE(15)
#undef SPMM_ROW_CASE
                    default: break;
                    }
                }
            }
        }
        wait_groups<0>();
        __syncwarp();
        // rows 16 s .. 16 s + 15: lane l stores its 16 bytes of each row
#pragma unroll
        for (int r = 0; r < 16; ++r)
            __stcs(reinterpret_cast<float4 *>(out + (16 * s + r) * rowbytes + f0 * 4) + lane,
                   make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]));
    }
}

template <typename I, int STAGES, int WARPS>
cudaError_t launch_ww_f32(const WindowArgs &a, cudaStream_t stream)
{
    using L = WinShapeF32<STAGES, WARPS>;
    constexpr int MINB = std::max(1, (220 * 1024) / L::kBlock);
    auto kern = window_warp_f32_kernel<I, STAGES, WARPS, MINB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBlock);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, WARPS * 32, L::kBlock);
    if (e != cudaSuccess) return e;
    const int nslices = (int)(a.N / 128);
    const int64_t items = a.nwin * nslices;
    if (a.sched && (e = build_schedule<I>(a, nslices, stream)) != cudaSuccess) return e;
    // one item per warp, no persistent loop: the block scheduler hands out
    // blocks in order as others finish, heavy items first with a schedule
    // (without one, measured 4.5 % faster on config 4 than a persistent loop)
    (void)per_sm;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((items + WARPS - 1) / WARPS, INT_MAX));
    kern<<<(unsigned)blocks, WARPS * 32, L::kBlock, stream>>>(a, nslices);
    return cudaGetLastError();
}

}  // namespace

size_t window_sched_bytes(int64_t nwin, int64_t N)
{
    // one order entry per (window, feature slice); slices are >= 64 features
    const int64_t slices = std::max<int64_t>(1, N / 64);
    const int64_t bytes = kSchedHeader + 8 * std::max<int64_t>(0, nwin) * slices;
    return (size_t)((bytes + 255) / 256 * 256);
}

bool window_warp_eligible(const WindowArgs &a, int dtype)
{
    // index and value arrays are copied in 16-byte pieces from 16-byte
    // aligned bases; other layouts take the block-synchronous kernel
    auto al = [](const void *p) { return ((uintptr_t)p & 15u) == 0; };
    const bool width = dtype == SPMM_F16 ? a.N % 64 == 0 : (dtype == SPMM_F32 && a.N % 128 == 0);
    return width && a.K > 0 && a.K <= INT_MAX && al(a.ccol) && al(a.cval) && al(a.vcol) && al(a.vval) && al(a.B) &&
           al(a.out);
}

// Launch shape for measurement, read at every launch: SPMM_B200_WW =
// <FW>s<stages>w<warps per CTA>.  The default is the widest slice the width
// allows with 3 stages and 4 warps per CTA: 256 features (2 CTAs, 8 warps
// per SM, 244 registers), else 128 (3 CTAs) or 64 (5 CTAs).  On config 2
// (N = 256) the 256-feature slice halves the items and doubles the bytes of
// every chunk: window kernel 462 -> 407 us against 128s3w4 on one box; on
// config 3 (N = 128) 128s3w4 measured fastest.
static int ww_variant()
{
    const char *e = getenv("SPMM_B200_WW");
    if (!e) return 0;
    static const char *const names[] = {"",        "128s4w2", "128s5w2", "128s6w2", "128s5w1",
                                        "64s6w2",  "64s5w4",  "128s4w4", "64s3w4",  "256s3w4",
                                        "256s3w2", "256s4w2", "128s3w4"};
    for (int i = 1; i < (int)(sizeof(names) / sizeof(names[0])); ++i)
        if (strcmp(e, names[i]) == 0) return i;
    return 0;
}

template <typename I>
cudaError_t launch_ww_f16(const WindowArgs &a, cudaStream_t stream)
{
    const bool w128 = a.N % 128 == 0, w256 = a.N % 256 == 0;
    switch (ww_variant()) {
    case 1: if (w128) return launch_ww<I, 128, 4, 2>(a, stream); break;
    case 2: if (w128) return launch_ww<I, 128, 5, 2>(a, stream); break;
    case 3: if (w128) return launch_ww<I, 128, 6, 2>(a, stream); break;
    case 4: if (w128) return launch_ww<I, 128, 5, 1>(a, stream); break;
    case 5: return launch_ww<I, 64, 6, 2>(a, stream);
    case 6: return launch_ww<I, 64, 5, 4>(a, stream);
    case 7: if (w128) return launch_ww<I, 128, 4, 4>(a, stream); break;
    case 8: return launch_ww<I, 64, 3, 4>(a, stream);
    case 9: if (w256) return launch_ww<I, 256, 3, 4>(a, stream); break;
    case 10: if (w256) return launch_ww<I, 256, 3, 2>(a, stream); break;
    case 11: if (w256) return launch_ww<I, 256, 4, 2>(a, stream); break;
    case 12: if (w128) return launch_ww<I, 128, 3, 4>(a, stream); break;
    default: break;
    }
    if (w256) return launch_ww<I, 256, 3, 4>(a, stream);
    return w128 ? launch_ww<I, 128, 3, 4>(a, stream) : launch_ww<I, 64, 3, 4>(a, stream);
}

cudaError_t launch_window_warp(const WindowArgs &a, int itype, int dtype, cudaStream_t stream)
{
    if (a.nwin <= 0) return cudaSuccess;
    // fp32: 2 stages of 16 x 128 features per warp (12 warps per SM; 3 stages
    // fit only 8 and measured 3 % slower on config 4, 4 stages 14 % slower)
    if (dtype == SPMM_F32)
        return itype == SPMM_I32 ? launch_ww_f32<int, 2, 2>(a, stream) : launch_ww_f32<int64_t, 2, 2>(a, stream);
    return itype == SPMM_I32 ? launch_ww_f16<int>(a, stream) : launch_ww_f16<int64_t>(a, stream);
}

}  // namespace spmmb
