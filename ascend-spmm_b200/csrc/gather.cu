// CSR gather SpMM on CUDA cores (the sparse-row path).
//
// Semantics follow the reference's vector-core kernel
// (kernels/op_kernel/spmm_csr.cpp:383-423): out[r, :] = sum_p val[p] * B[col[p], :]
// with fp32 accumulation.  The B200 design is new:
//
//  * Work unit = a fixed range of `unit` nonzeros (not a row).  Units are
//    dealt round-robin to resident warps, so a 4096-nonzero row costs the
//    same per unit as 256 short rows and power-law skew cannot leave one
//    warp with the tail.  The reference instead splits nnz statically over
//    40 vector cores (op_host/spmm_csr.cpp:22-27).
//  * A warp processes a unit as 32/G row lanes-groups of G lanes; a group
//    owns one row at a time and each lane owns VPL 16-byte vectors of the
//    row's N features, so every gathered B row is read with coalesced
//    128-bit loads and U gathers per lane are kept in flight.
//  * Each output element is a sequential fp32 fma chain over the row's
//    nonzeros in CSR order.  A row crossing a unit boundary is accumulated
//    per unit into an fp32 partial (head slot for the unit where it ends or
//    continues, tail slot for the unit where it starts); csr_fixup_kernel sums
//    the partials in unit order.  The split depends only on nnz, never on the
//    grid, the feature width or the batching variant, so every variant is
//    bitwise identical (the reference's AIV-variant tests demand this,
//    tests/aic_aiv_ablation/bitwise_correctness.py:238-239) and no float
//    atomics are used (the reference atomically adds fp16 partials at core
//    boundaries, op_kernel/spmm_csr.cpp:472).
//  * fp16 output is rounded to nearest once (the reference casts with
//    round-toward-minus-infinity, spmm_csr.cpp:417).
//  * Invalid column indices or row pointers are skipped and reported through
//    the sticky device status instead of faulting.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

constexpr int kGatherThreads = 256;

// MINB: minimum resident blocks per SM requested from the register allocator
// (3 x 256 threads = 24 warps/SM for the default batch of narrow rows).
template <typename T, typename I, int G, int VPL, int U, int MINB>
__global__ void __launch_bounds__(kGatherThreads, MINB)
csr_gather_kernel(const GatherArgs a)
{
    constexpr int S = 32 / G;                   // row groups per warp
    constexpr int EPV = Vec<T>::kElems;         // elements per 16-byte vector
    const int lane = threadIdx.x & 31;
    const int sub = lane / G;
    const int gl = lane % G;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;

    const I *rowptr = static_cast<const I *>(a.rowptr);
    const I *col = static_cast<const I *>(a.col);
    const T *val = static_cast<const T *>(a.val);
    const uint4 *B = static_cast<const uint4 *>(a.B);
    const int NV = (int)(a.N / EPV);            // 16-byte vectors per row

    for (int64_t u = a.unit_begin + warp; u < a.unit_end; u += nwarps) {
        const int64_t lo = u * a.unit;
        const int64_t hi = min(lo + a.unit, a.nnz);
        const bool last = (u == a.unit_end - 1);
        const int64_t i0 = warp_lower_bound(rowptr, a.row_begin, a.M + 1, lo);
        int64_t r0 = i0;
        if (i0 > a.row_begin && (i0 > a.M || ld_idx(rowptr + i0) > lo)) r0 = i0 - 1;

        for (int64_t r = r0 + sub; r < a.M; r += S) {
            int64_t beg = ld_idx(rowptr + r);
            int64_t end = ld_idx(rowptr + r + 1);
            if (!(beg < hi || last)) break;
            if (beg < 0 || end < beg || end > a.nnz) {
                if (gl == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, r);
                beg = end = max((int64_t)0, min(beg, a.nnz));
            }
            const int64_t sb = max(beg, lo);
            const int n = (int)(min(end, hi) - sb);   // nonzeros of this row inside the unit
            const I *cp = col + sb;
            const T *vp = val + sb;

            float acc[VPL][EPV];
#pragma unroll
            for (int q = 0; q < VPL; ++q)
#pragma unroll
                for (int e = 0; e < EPV; ++e) acc[q][e] = 0.f;

            for (int p = 0; p < n; p += U) {
                // Entries past the row or with an invalid column contribute
                // fma(0, 0, acc); no per-entry predicate stays live.
                uint4 b[U][VPL];
                float v[U];
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    int c = -1;
                    v[j] = 0.f;
                    if (p + j < n) {
                        const int64_t cc = (int64_t)ld_stream(cp + p + j);
                        if (cc >= 0 && cc < a.K) {
                            c = (int)cc;
                            v[j] = to_f32(ld_stream(vp + p + j));
                        } else if (gl == 0) {
                            raise_status(a.status, SPMM_DEV_BAD_COLUMN, sb + p + j);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < VPL; ++q) {
                        const int vi = gl + q * G;
                        b[j][q] = (c >= 0 && vi < NV) ? __ldg(B + (int64_t)c * NV + vi)
                                                      : make_uint4(0, 0, 0, 0);
                    }
                }
#pragma unroll
                for (int j = 0; j < U; ++j)
#pragma unroll
                    for (int q = 0; q < VPL; ++q) {
                        float f[EPV];
                        unpack16<T>(b[j][q], f);
#pragma unroll
                        for (int e = 0; e < EPV; ++e) acc[q][e] = fmaf(v[j], f[e], acc[q][e]);
                    }
            }

            const bool head = beg < lo;
            const bool tail = end > hi;
            if (!head && !tail) {
                uint4 *orow = static_cast<uint4 *>(a.out) + r * NV;
#pragma unroll
                for (int q = 0; q < VPL; ++q) {
                    const int vi = gl + q * G;
                    if (vi < NV) store_c16(a.out, a.out_mc, orow + vi, pack16<T>(acc[q]));
                }
            } else {
                float *prow = a.partial + ((u - a.unit_begin) * 2 + (head ? 0 : 1)) * a.N;
#pragma unroll
                for (int q = 0; q < VPL; ++q) {
                    const int vi = gl + q * G;
                    if (vi >= NV) continue;
                    float4 *dst = reinterpret_cast<float4 *>(prow + (int64_t)vi * EPV);
#pragma unroll
                    for (int e = 0; e < EPV; e += 4)
                        dst[e / 4] = make_float4(acc[q][e], acc[q][e + 1], acc[q][e + 2], acc[q][e + 3]);
                }
            }
        }
    }
    release_c(a.out_mc);   // multicast rows ordered before the caller's barrier
}

// ---------------------------------------------------------------------------
// Stream kernel (rows of >= 16 vectors: N >= 128 fp16, N >= 64 fp32).
//
// A group of G lanes (a warp, or a half-warp for G = 16) consumes its unit as
// one flat nonzero stream instead of row by row: the next 32 column/value
// entries are prefetched into lanes while the current 32 are gathered, a
// batch of U gathers per lane is always in flight whatever the row lengths,
// and row boundaries are handled inline (flush, then advance through the
// row-pointer cache held in lanes).  The per-row fma order is the same as in
// csr_gather_kernel, so both produce identical bits.
// ---------------------------------------------------------------------------
template <typename I, int G>
__device__ __forceinline__ int64_t group_lower_bound(const I *a, int64_t L, int64_t H, int64_t key, unsigned gmask,
                                                     int gl, int shift)
{
    while (H - L > G) {
        const int64_t step = (H - L + G - 1) / G;
        const int64_t pos = L + (int64_t)gl * step;
        const bool ge = pos < H && ld_idx(a + pos) >= key;
        const unsigned m = (__ballot_sync(gmask, ge) & gmask) >> shift;
        if (m == 0) {
            const int64_t kmax = min((int64_t)(G - 1), (H - 1 - L) / step);
            L = L + kmax * step + 1;
        } else {
            const int f = __ffs(m) - 1;
            const int64_t pf = L + (int64_t)f * step;
            L = (f == 0) ? L : L + (int64_t)(f - 1) * step + 1;
            H = pf;
        }
    }
    const int64_t pos = L + gl;
    const bool ge = pos < H && ld_idx(a + pos) >= key;
    const unsigned m = (__ballot_sync(gmask, ge) & gmask) >> shift;
    return m ? L + (__ffs(m) - 1) : H;
}

// FULL: every lane owns VPL valid vectors (N * sizeof(T) / 16 == G * VPL).
template <typename T, typename I, int G, int VPL, int U, int MINB, bool FULL>
__global__ void __launch_bounds__(kGatherThreads, MINB)
csr_stream_kernel(const GatherArgs a)
{
    static_assert(G == 16 || G == 32, "stream groups are half-warps or warps");
    using F = FmaVec<T>;
    using Scalar = typename F::Scalar;
    constexpr int S = 32 / G;
    constexpr int EPV = Vec<T>::kElems;
    constexpr int CH = 32;          // nonzeros per prefetched chunk
    constexpr int PER = CH / G;     // chunk entries held per lane
    static_assert(CH % U == 0 && U <= 32, "batches tile the chunk");
    const int lane = threadIdx.x & 31;
    const int sub = lane / G, gl = lane % G, shift = sub * G;
    const unsigned gmask = (G == 32) ? 0xffffffffu : (((1u << G) - 1u) << shift);
    const int64_t stream = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * S + sub;
    const int64_t nstreams = (((int64_t)gridDim.x * blockDim.x) >> 5) * S;

    const I *rowptr = static_cast<const I *>(a.rowptr);
    const I *col = static_cast<const I *>(a.col);
    const T *val = static_cast<const T *>(a.val);
    const uint4 *B = static_cast<const uint4 *>(a.B);
    uint4 *out = static_cast<uint4 *>(a.out);
    const int NV = (int)(a.N / EPV);
    const uint4 *Bl = B + gl;

    for (int64_t u = a.unit_begin + stream; u < a.unit_end; u += nstreams) {
        const int64_t lo = u * a.unit;
        const int64_t hi = min(lo + a.unit, a.nnz);
        const bool last = (u == a.unit_end - 1);
        const int64_t i0 = group_lower_bound<I, G>(rowptr, a.row_begin, a.M + 1, lo, gmask, gl, shift);
        int64_t r = i0;
        if (i0 > a.row_begin && (i0 > a.M || ld_idx(rowptr + i0) > lo)) r = i0 - 1;

        // Row-pointer cache: lanes hold rowptr[rc + gl] and rowptr[rc + G + gl];
        // rp(x) follows the current row (x never decreases) and slides the
        // window forward.
        int64_t rc = r;
        int64_t rpa = ld_idx(rowptr + min(rc + gl, a.M));
        int64_t rpb = ld_idx(rowptr + min(rc + G + gl, a.M));
        auto rp = [&](int64_t x) -> int64_t {
            if (x < rc || x >= rc + 2 * G) {
                rc = x;
                rpa = ld_idx(rowptr + min(rc + gl, a.M));
                rpb = ld_idx(rowptr + min(rc + G + gl, a.M));
            } else if (x >= rc + G) {
                rc += G;
                rpa = rpb;
                rpb = ld_idx(rowptr + min(rc + G + gl, a.M));
            }
            return __shfl_sync(gmask, rpa, (int)(x - rc), G);
        };

        float acc[VPL][EPV];
#pragma unroll
        for (int q = 0; q < VPL; ++q)
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[q][e] = 0.f;

        // Current row: r with [beg, end); rows before it are finished.
        // Empty rows owned by this unit are written as zeros on the way.
        int64_t beg = 0, end = 0;
        bool have_row = false;
        auto zero_row = [&](int64_t row) {
#pragma unroll
            for (int q = 0; q < VPL; ++q) {
                const int vi = gl + q * G;
                if (vi < NV) store_c16(a.out, a.out_mc, out + row * NV + vi, make_uint4(0, 0, 0, 0));
            }
        };
        for (; r < a.M; ++r) {
            beg = rp(r);
            end = rp(r + 1);
            if (beg < 0 || end < beg || end > a.nnz) {
                if (gl == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, r);
                break;
            }
            if (beg >= hi && !last) break;
            if (end > beg) { have_row = true; break; }
            zero_row(r);
        }
        if (!have_row) continue;
        const int64_t s0 = max(lo, beg);
        bool head_pending = beg < lo;   // the first segment is a head partial

        // Invalid columns become column 0 with value 0 (this kernel runs only
        // with K > 0), so the gather needs no predicate beyond the batch end.
        auto load_chunk = [&](int64_t pos, int *cc, Scalar *vv) {
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int64_t e = pos + gl + k * G;
                cc[k] = 0;
                vv[k] = F::zero();
                if (e < hi) {
                    const int64_t c = (int64_t)ld_stream(col + e);
                    if (c >= 0 && c < a.K) {
                        cc[k] = (int)c;
                        vv[k] = F::load(val + e);
                    } else {
                        raise_status(a.status, SPMM_DEV_BAD_COLUMN, e);
                    }
                }
            }
        };
        // fp32 partial row of this unit: slot 0 = head (row began before lo),
        // slot 1 = tail (row continues past hi).
        auto store_partial = [&](int slot) {
            float *prow = a.partial + ((u - a.unit_begin) * 2 + slot) * a.N;
#pragma unroll
            for (int q = 0; q < VPL; ++q) {
                const int vi = gl + q * G;
                if (vi >= NV) continue;
                float4 *dst = reinterpret_cast<float4 *>(prow + (int64_t)vi * EPV);
#pragma unroll
                for (int e = 0; e < EPV; e += 4)
                    dst[e / 4] = make_float4(acc[q][e], acc[q][e + 1], acc[q][e + 2], acc[q][e + 3]);
            }
        };

        int ccur[PER];
        Scalar vcur[PER];
        load_chunk(s0, ccur, vcur);
        bool done = false;
        for (int64_t pb = s0; pb < hi && !done; pb += CH) {
            int cnext[PER];
            Scalar vnext[PER];
            load_chunk(pb + CH, cnext, vnext);
#pragma unroll 1
            for (int b = 0; b < CH && !done; b += U) {
                const int64_t pbase = pb + b;
                if (pbase >= hi) break;
                const int nvalid = (int)min((int64_t)U, hi - pbase);
                uint4 bv[U][VPL];
                Scalar vj[U];
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    const int e = b + j;
                    int cw = ccur[0];
                    Scalar vw = vcur[0];
#pragma unroll
                    for (int k = 1; k < PER; ++k)
                        if (e / G == k) { cw = ccur[k]; vw = vcur[k]; }
                    const int c = __shfl_sync(gmask, cw, e % G, G);
                    vj[j] = __shfl_sync(gmask, vw, e % G, G);
                    if (j < nvalid) {
                        const uint4 *brow = Bl + (int64_t)c * NV;
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
                            if (FULL || gl + q * G < NV) bv[j][q] = __ldg(brow + q * G);
                    }
                }
                // Row bookkeeping for the batch, done once while the gathers
                // are in flight: bit j of `ends` is set when a row segment
                // ends at position pbase + j, and lane j then holds that row;
                // `tails` marks a segment cut by the unit's end.
                unsigned ends = 0, tails = 0;
                int64_t myrow = 0;
                const int64_t bend = pbase + nvalid;
                for (;;) {
                    if (end <= bend) {                      // row r ends in this batch
                        const int jb = (int)(end - pbase - 1);
                        ends |= 1u << jb;
                        if (gl == jb) myrow = r;
                        int64_t prev = end;
                        bool next = false;
                        for (++r; r < a.M; ++r) {
                            beg = prev;
                            end = rp(r + 1);
                            if (end < beg || end > a.nnz) {
                                if (gl == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, r);
                                break;
                            }
                            if (beg >= hi && !last) break;
                            if (end > beg) { next = true; break; }
                            zero_row(r);
                        }
                        if (!next) { done = true; break; }
                        continue;
                    }
                    if (bend == hi) {                       // row r continues past the unit
                        ends |= 1u << (nvalid - 1);
                        tails |= 1u << (nvalid - 1);
                        if (gl == nvalid - 1) myrow = r;
                        done = true;
                    }
                    break;
                }
                if (ends == 0) {
                    // no row ends here: the batch is full and in one row
#pragma unroll
                    for (int j = 0; j < U; ++j)
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
                            if (FULL || gl + q * G < NV) F::run(acc[q], vj[j], bv[j][q]);
                    continue;
                }
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    if (j < nvalid) {
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
                            if (FULL || gl + q * G < NV) F::run(acc[q], vj[j], bv[j][q]);
                    }
                    if ((ends >> j) & 1u) {
                        if (head_pending || ((tails >> j) & 1u)) {
                            store_partial(head_pending ? 0 : 1);
                            head_pending = false;
                        } else {
                            const int64_t row = __shfl_sync(gmask, myrow, j, G);
#pragma unroll
                            for (int q = 0; q < VPL; ++q) {
                                const int vi = gl + q * G;
                                if (vi < NV) store_c16(a.out, a.out_mc, out + row * NV + vi, pack16<T>(acc[q]));
                            }
                        }
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
#pragma unroll
                            for (int e = 0; e < EPV; ++e) acc[q][e] = 0.f;
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                ccur[k] = cnext[k];
                vcur[k] = vnext[k];
            }
        }
    }
    release_c(a.out_mc);   // multicast rows ordered before the caller's barrier
}

// ---------------------------------------------------------------------------
// Ring kernel: the stream kernel with its gathers landing in shared memory.
//
// Each lane copies the 16-byte pieces of the B rows it will itself consume
// (cp.async.cg, L2 only) into a per-warp ring of 2 x U positions and reads
// them back with one 16-byte shared load per position: no cross-lane
// synchronisation is needed (cp.async.wait_group covers the thread's own
// copies), in-flight data holds no registers, so more warps fit per SM and
// two batches stay in flight.  Column indices and values are staged per
// 64-nonzero chunk in the warp's shared memory (two chunks resident, the
// next one in registers), so a batch reads its U columns and U values with
// a few broadcast vector loads instead of per-position register selects and
// shuffles; a batch with no row end inside skips the per-position row tests.
// Row ends are found warp-parallel: a rolling window holds the unit-local
// end positions of the next 32-64 rows (one lane per row, prefetched 32 rows
// ahead), one ballot per batch yields the batch's row-end mask and each
// ending row's index goes to a per-warp shared table; a batch that the
// current row spans skips this step.  The per-row fma order is that of
// csr_stream_kernel, so results are bitwise identical.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16_cg_s(unsigned saddr, const void *gmem)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gmem) : "memory");
}
// The same copy with an L2 eviction policy (createpolicy) for the line.
__device__ __forceinline__ void cp_async16_cg_hint(unsigned saddr, const void *gmem, uint64_t pol)
{
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(gmem), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_normal()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;\n" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint4 lds16(unsigned saddr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(saddr));
    return v;
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

// Shared memory of one warp in the ring kernel: the ring (2 batches of U
// positions x VPL 16-byte pieces per lane), then two staged chunks of 64
// column indices and 64 values.
template <typename T, int VPL, int U> struct RingShape {
    static constexpr int kChunk = 64;
    static constexpr int kRingBytes = 2 * U * VPL * 32 * 16;
    static constexpr int kColOff = kRingBytes;
    static constexpr int kValOff = kColOff + 2 * kChunk * 4;
    static constexpr int kRowOff = kValOff + 2 * kChunk * (int)sizeof(typename FmaVec<T>::Scalar);
    // a multiple of 128 bytes, so each 512-byte ring position starts on a
    // 128-byte boundary (4 shared-memory wavefronts per warp access, not 5)
    static constexpr int kWarpBytes = (kRowOff + 2 * U * 8 + 127) / 128 * 128;
};

// fp16 products of one nonzero (half SEL of the packed value word) with the
// 8 elements of a 16-byte B piece, accumulated in fp32.
__device__ __forceinline__ void fma8_f16_lo(float *acc, unsigned vw, const uint4 &b)
{
    asm("{\n\t.reg .f16 s, t, l0, u0, l1, u1, l2, u2, l3, u3;\n\t"
        "mov.b32 {s, t}, %8;\n\t"
        "mov.b32 {l0, u0}, %9;\n\tmov.b32 {l1, u1}, %10;\n\tmov.b32 {l2, u2}, %11;\n\tmov.b32 {l3, u3}, %12;\n\t"
        "fma.rn.f32.f16 %0, s, l0, %0;\n\tfma.rn.f32.f16 %1, s, u0, %1;\n\t"
        "fma.rn.f32.f16 %2, s, l1, %2;\n\tfma.rn.f32.f16 %3, s, u1, %3;\n\t"
        "fma.rn.f32.f16 %4, s, l2, %4;\n\tfma.rn.f32.f16 %5, s, u2, %5;\n\t"
        "fma.rn.f32.f16 %6, s, l3, %6;\n\tfma.rn.f32.f16 %7, s, u3, %7;\n\t}"
        : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc[4]), "+f"(acc[5]), "+f"(acc[6]),
          "+f"(acc[7])
        : "r"(vw), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w));
}
__device__ __forceinline__ void fma8_f16_hi(float *acc, unsigned vw, const uint4 &b)
{
    asm("{\n\t.reg .f16 s, t, l0, u0, l1, u1, l2, u2, l3, u3;\n\t"
        "mov.b32 {t, s}, %8;\n\t"
        "mov.b32 {l0, u0}, %9;\n\tmov.b32 {l1, u1}, %10;\n\tmov.b32 {l2, u2}, %11;\n\tmov.b32 {l3, u3}, %12;\n\t"
        "fma.rn.f32.f16 %0, s, l0, %0;\n\tfma.rn.f32.f16 %1, s, u0, %1;\n\t"
        "fma.rn.f32.f16 %2, s, l1, %2;\n\tfma.rn.f32.f16 %3, s, u1, %3;\n\t"
        "fma.rn.f32.f16 %4, s, l2, %4;\n\tfma.rn.f32.f16 %5, s, u2, %5;\n\t"
        "fma.rn.f32.f16 %6, s, l3, %6;\n\tfma.rn.f32.f16 %7, s, u3, %7;\n\t}"
        : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc[4]), "+f"(acc[5]), "+f"(acc[6]),
          "+f"(acc[7])
        : "r"(vw), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w));
}

// Product of nonzero j of a batch (its value packed in the words vw) with one
// 16-byte B piece; j is a compile-time constant after unrolling.
template <typename T> struct BatchFma;
template <> struct BatchFma<__half> {
    template <int NW>
    static __device__ __forceinline__ void run(float *acc, const unsigned (&vw)[NW], int j, const uint4 &b)
    {
        if (j & 1) fma8_f16_hi(acc, vw[j >> 1], b);
        else fma8_f16_lo(acc, vw[j >> 1], b);
    }
};
template <> struct BatchFma<float> {
    template <int NW>
    static __device__ __forceinline__ void run(float *acc, const unsigned (&vw)[NW], int j, const uint4 &b)
    {
        FmaVec<float>::run(acc, __uint_as_float(vw[j]), b);
    }
};

// NW consecutive 32-bit words from shared memory with the widest loads the
// alignment allows (callers keep 4 * NW-byte alignment); every lane reads the
// same address, so each load is a broadcast.
template <int NW>
__device__ __forceinline__ void lds_words(const void *p, unsigned (&w)[NW])
{
    if constexpr (NW % 4 == 0) {
#pragma unroll
        for (int i = 0; i < NW / 4; ++i) {
            const uint4 x = reinterpret_cast<const uint4 *>(p)[i];
            w[4 * i] = x.x; w[4 * i + 1] = x.y; w[4 * i + 2] = x.z; w[4 * i + 3] = x.w;
        }
    } else if constexpr (NW == 2) {
        const uint2 x = *reinterpret_cast<const uint2 *>(p);
        w[0] = x.x; w[1] = x.y;
    } else {
        static_assert(NW == 1, "1, 2 or a multiple of 4 words");
        w[0] = *reinterpret_cast<const unsigned *>(p);
    }
}

// L2H: copies of B rows carry the L2 residency plan's eviction priorities
// (evict_last for hot columns, evict_first for the rest; the normal priority
// for all when the plan is not enabled).  The plan's hot bit travels in bit
// 31 of the staged column index (column ids fit in 31 bits under a plan).
template <typename T, typename I, int G, int VPL, int U, int MINB, bool FULL, bool L2H = false>
__global__ void __launch_bounds__(kGatherThreads, MINB)
csr_ring_kernel(const GatherArgs a)
{
    static_assert(G == 32, "the ring serves whole-warp rows");
    using F = FmaVec<T>;
    using Scalar = typename F::Scalar;
    using Shape = RingShape<T, VPL, U>;
    constexpr int EPV = Vec<T>::kElems;
    constexpr int CH = Shape::kChunk;   // nonzeros per staged column/value chunk
    constexpr int PER = CH / 32;
    constexpr int VB = (int)sizeof(Scalar);
    static_assert(CH % U == 0 && 2 * U <= CH && (U * VB) % 4 == 0 && U <= 32, "batches tile the chunk");
    extern __shared__ __align__(16) uint4 ring_smem[];
    const int lane = threadIdx.x & 31;
    const int gl = lane;
    constexpr unsigned gmask = 0xffffffffu;
    char *wbase = reinterpret_cast<char *>(ring_smem) + (size_t)(threadIdx.x >> 5) * Shape::kWarpBytes;
    // this lane's column of the ring, as a 32-bit shared address
    const unsigned ring_s = (unsigned)__cvta_generic_to_shared(wbase) + (unsigned)lane * 16;
    int *s_col = reinterpret_cast<int *>(wbase + Shape::kColOff);            // [2][CH], chunk n in slot n & 1
    Scalar *s_val = reinterpret_cast<Scalar *>(wbase + Shape::kValOff);      // [2][CH]
    int64_t *s_row = reinterpret_cast<int64_t *>(wbase + Shape::kRowOff);    // [2][U] row ending at each position
    const int64_t stream = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nstreams = ((int64_t)gridDim.x * blockDim.x) >> 5;

    const I *rowptr = static_cast<const I *>(a.rowptr);
    const I *col = static_cast<const I *>(a.col);
    const T *val = static_cast<const T *>(a.val);
    const uint4 *Bl = static_cast<const uint4 *>(a.B) + gl;
    uint4 *out = static_cast<uint4 *>(a.out);
    const int NV = (int)(a.N / EPV);
    uint64_t pol_hot = 0, pol_cold = 0;
    if constexpr (L2H) {
        if (l2_plan_enabled(*a.l2_hdr)) {
            pol_hot = l2_policy_last();
            pol_cold = l2_policy_first();
        } else {
            pol_hot = pol_cold = l2_policy_normal();
        }
    }

    for (int64_t u = a.unit_begin + stream; u < a.unit_end; u += nstreams) {
        const int64_t lo = u * a.unit;
        const int64_t hi = min(lo + a.unit, a.nnz);
        const bool last = (u == a.unit_end - 1);
        const int64_t i0 = group_lower_bound<I, G>(rowptr, a.row_begin, a.M + 1, lo, gmask, gl, 0);
        int64_t r = i0;
        if (i0 > a.row_begin && (i0 > a.M || ld_idx(rowptr + i0) > lo)) r = i0 - 1;

        auto zero_row = [&](int64_t row) {
#pragma unroll
            for (int q = 0; q < VPL; ++q) {
                const int vi = gl + q * G;
                if (FULL || vi < NV) store_c16(a.out, a.out_mc, out + row * NV + vi, make_uint4(0, 0, 0, 0));
            }
        };
        // first row with a nonzero in the unit; the empty rows before it that
        // start inside the unit are written as zeros
        int64_t beg = 0, end = 0;
        bool have_row = false;
        {
            int64_t rc = r;
            int64_t rpa = ld_idx(rowptr + min(rc + gl, a.M));
            int64_t rpb = ld_idx(rowptr + min(rc + G + gl, a.M));
            auto rp = [&](int64_t x) -> int64_t {
                if (x < rc || x >= rc + 2 * G) {
                    rc = x;
                    rpa = ld_idx(rowptr + min(rc + gl, a.M));
                    rpb = ld_idx(rowptr + min(rc + G + gl, a.M));
                } else if (x >= rc + G) {
                    rc += G;
                    rpa = rpb;
                    rpb = ld_idx(rowptr + min(rc + G + gl, a.M));
                }
                return __shfl_sync(gmask, rpa, (int)(x - rc), G);
            };
            for (; r < a.M; ++r) {
                beg = rp(r);
                end = rp(r + 1);
                if (beg < 0 || end < beg || end > a.nnz) {
                    if (gl == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, r);
                    break;
                }
                if (beg >= hi && !last) break;
                if (end > beg) { have_row = true; break; }
                zero_row(r);
            }
        }
        if (a.split_rows && gl == 0) a.split_rows[u - a.unit_begin] = -1;
        if (!have_row) continue;
        const int64_t s0 = max(lo, beg);
        bool head_pending = beg < lo;   // the first segment is a head partial
        const int H = (int)(hi - s0);   // positions of the unit, local to s0
        const int nbatch = (H + U - 1) / U;

        // Row ends as unit-local positions: lane l of a window based at row w
        // holds rowptr[w + l + 1] - s0 (H + 1 past the unit, INT_MAX past M).
        // A = rows [w0, w0 + 32), B = the next 32, C = the 32 after (raw,
        // loaded 32 rows before it is needed).  rcur = first unfinished row.
        bool bad = false;
        auto load_raw = [&](int64_t w) -> int64_t { return ld_idx(rowptr + min(w + gl + 1, a.M)); };
        auto conv = [&](int64_t raw, int64_t w, int before) -> int {
            const int64_t row = w + gl;
            int le;
            bool wrong = false;
            if (row >= a.M) {
                le = INT_MAX;
            } else {
                wrong = raw > a.nnz || raw < s0;
                le = raw > hi ? H + 1 : (int)(raw - s0);
            }
            const int pl = __shfl_up_sync(gmask, le, 1);
            wrong = wrong || le < (gl ? pl : before);
            if (__any_sync(gmask, wrong)) {
                if (gl == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, w);
                bad = true;
            }
            return wrong ? INT_MAX : le;
        };
        int64_t w0 = r, rcur = r;
        int winA, winB;
        int64_t rawC;
        {
            const int64_t ra = load_raw(w0), rb = load_raw(w0 + 32);
            rawC = load_raw(w0 + 64);
            winA = conv(ra, w0, -1);
            winB = conv(rb, w0 + 32, __shfl_sync(gmask, winA, 31));
        }
        int carry = -1;   // local end of row rcur - 1
        int cur_le = __shfl_sync(gmask, winA, 0);   // local end of row rcur

        float acc[VPL][EPV];
#pragma unroll
        for (int q = 0; q < VPL; ++q)
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[q][e] = 0.f;

        // Invalid columns become column 0 with value 0 (this kernel runs only
        // with K > 0), so the gather needs no predicate beyond the batch end.
        auto load_chunk = [&](int64_t pos, int *cc, Scalar *vv) {
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int64_t e = pos + gl + k * G;
                cc[k] = 0;
                vv[k] = F::zero();
                if (e < hi) {
                    const int64_t c = (int64_t)ld_stream(col + e);
                    if (c >= 0 && c < a.K) {
                        cc[k] = (int)c;
                        vv[k] = F::load(val + e);
                    } else {
                        raise_status(a.status, SPMM_DEV_BAD_COLUMN, e);
                    }
                }
            }
        };
        auto stage = [&](int slot, const int *cc, const Scalar *vv) {
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                int c = cc[k];
                if constexpr (L2H) {   // the plan's hot bit of this column rides in bit 31
                    const unsigned bin = (unsigned)c & (unsigned)(kL2Bins - 1);
                    c |= (int)(((__ldg(a.l2_bits + (bin >> 5)) >> (bin & 31u)) & 1u) << 31);
                }
                s_col[slot * CH + gl + k * G] = c;
                s_val[slot * CH + gl + k * G] = vv[k];
            }
        };
        // chunks 0 and 1 staged in shared memory, chunk 2 in registers
        int colR[PER];
        Scalar valR[PER];
        __syncwarp();   // the previous unit's reads of the staging slots are done
        {
            int c0[PER];
            Scalar v0[PER];
            load_chunk(s0, c0, v0);
            load_chunk(s0 + CH, colR, valR);
            stage(0, c0, v0);
            stage(1, colR, valR);
            load_chunk(s0 + 2 * CH, colR, valR);
        }
        __syncwarp();

        auto issue = [&](int k) {
            if (k < nbatch) {
                const int o0 = k * U;
                const int nv = min(U, H - o0);
                unsigned cw[U];
                lds_words<U>(s_col + ((o0 / CH) & 1) * CH + (o0 % CH), cw);
                const unsigned slot0 = ring_s + (unsigned)((k & 1) * U * VPL * G * 16);
                // one B row: this lane's VPL pieces of it (under L2H with the
                // plan's policy; bit 31 of the staged index is the hot bit)
                auto copy_row = [&](int j) {
                    if constexpr (L2H) {
                        const uint4 *src = Bl + (int64_t)(int)(cw[j] & 0x7fffffffu) * NV;
                        const uint64_t pol = (cw[j] >> 31) ? pol_hot : pol_cold;
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
                            if (FULL || gl + q * G < NV)
                                cp_async16_cg_hint(slot0 + (j * VPL + q) * G * 16, src + q * G, pol);
                    } else {
                        const uint4 *src = Bl + (int64_t)(int)cw[j] * NV;
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
                            if (FULL || gl + q * G < NV) cp_async16_cg_s(slot0 + (j * VPL + q) * G * 16, src + q * G);
                    }
                };
                if (nv == U) {
#pragma unroll
                    for (int j = 0; j < U; ++j) copy_row(j);
                } else {
#pragma unroll
                    for (int j = 0; j < U; ++j)
                        if (j < nv) copy_row(j);
                }
            }
            cp_async_commit_group();
        };
        issue(0);
        issue(1);

        for (int k = 0; k < nbatch && !bad; ++k) {
            const int o0 = k * U;
            const int nvalid = min(U, H - o0);
            const int lim = o0 + nvalid;
            const int buf = k & 1;
            // Rows ending in this batch, warp-parallel over the window: their
            // end positions form the mask `ends`, s_row[buf][j] names the row
            // ending at position o0 + j; empty rows among them are zeroed.
            // Empty rows starting at hi belong to the next unit (unless last).
            unsigned ends = 0, tails = 0;
            const bool any_end = cur_le <= lim;
            if (any_end) __syncwarp();   // earlier reads of s_row[buf] are done
            for (; cur_le <= lim;) {   // some row ends in this batch
                const int d = (int)(rcur - w0);
                const int src = (d + gl) & 31;
                const int va = __shfl_sync(gmask, winA, src);
                const int vb = __shfl_sync(gmask, winB, src);
                const int le = (d + gl < 32) ? va : vb;
                const int up = __shfl_up_sync(gmask, le, 1);
                const bool empty = le == (gl ? up : carry);
                const bool in = le <= lim && (last || !empty || le < H);
                const int nin = __popc(__ballot_sync(gmask, in));
                const int pos = le - 1 - o0;   // in [0, nvalid) for every row ending here
                const bool endhere = in && !empty && (unsigned)pos < (unsigned)U;
                ends |= __reduce_or_sync(gmask, endhere ? 1u << pos : 0u);
                if (endhere) s_row[buf * U + pos] = rcur + gl;
                unsigned em = __ballot_sync(gmask, in && empty);
                while (em) {
                    const int b = __ffs(em) - 1;
                    em &= em - 1;
                    zero_row(rcur + b);
                }
                if (nin) carry = __shfl_sync(gmask, le, nin - 1);
                cur_le = __shfl_sync(gmask, le, nin & 31);   // row rcur + nin (re-read below when nin == 32)
                rcur += nin;
                if (rcur - w0 >= 32) {
                    winA = winB;
                    winB = conv(rawC, w0 + 64, __shfl_sync(gmask, winB, 31));
                    w0 += 32;
                    rawC = load_raw(w0 + 64);
                }
                if (nin < 32 || bad) break;
                cur_le = __shfl_sync(gmask, (int)(rcur - w0) < 32 ? winA : winB, (int)(rcur - w0) & 31);
            }
            if (lim == H && !((ends >> (nvalid - 1)) & 1u)) {   // a row continues past the unit
                ends |= 1u << (nvalid - 1);
                tails |= 1u << (nvalid - 1);
            }
            unsigned vw[U * VB / 4];
            lds_words<U * VB / 4>(s_val + ((o0 / CH) & 1) * CH + (o0 % CH), vw);
            if (any_end) __syncwarp();   // s_row entries of this batch are visible
            cp_async_wait_1();   // this lane's copies of batch k have landed
            const unsigned slot0 = ring_s + (unsigned)((k & 1) * U * VPL * G * 16);
            if (ends == 0) {
                // the batch is full and inside one row
#pragma unroll
                for (int j = 0; j < U; ++j)
#pragma unroll
                    for (int q = 0; q < VPL; ++q)
                        if (FULL || gl + q * G < NV)
                            BatchFma<T>::run(acc[q], vw, j, lds16(slot0 + (j * VPL + q) * G * 16));
            } else {
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    if (j < nvalid) {
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
                            if (FULL || gl + q * G < NV)
                                BatchFma<T>::run(acc[q], vw, j, lds16(slot0 + (j * VPL + q) * G * 16));
                    }
                    if ((ends >> j) & 1u) {
                        if (head_pending || ((tails >> j) & 1u)) {
                            float *prow = a.partial + ((u - a.unit_begin) * 2 + (head_pending ? 0 : 1)) * a.N;
                            if (!head_pending && a.split_rows && gl == 0) a.split_rows[u - a.unit_begin] = rcur;
#pragma unroll
                            for (int q = 0; q < VPL; ++q) {
                                const int vi = gl + q * G;
                                if (!FULL && vi >= NV) continue;
                                float4 *dst = reinterpret_cast<float4 *>(prow + (int64_t)vi * EPV);
#pragma unroll
                                for (int e = 0; e < EPV; e += 4)
                                    dst[e / 4] = make_float4(acc[q][e], acc[q][e + 1], acc[q][e + 2], acc[q][e + 3]);
                            }
                            head_pending = false;
                        } else {
                            const int64_t row = s_row[buf * U + j];
#pragma unroll
                            for (int q = 0; q < VPL; ++q) {
                                const int vi = gl + q * G;
                                if (FULL || vi < NV) store_c16(a.out, a.out_mc, out + row * NV + vi, pack16<T>(acc[q]));
                            }
                        }
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
#pragma unroll
                            for (int e = 0; e < EPV; ++e) acc[q][e] = 0.f;
                    }
                }
            }
            // chunk n = o0 / CH is finished after its last batch: its slot
            // takes chunk n + 2 (held in registers), and chunk n + 3 is loaded
            if (((k + 1) * U) % CH == 0) {
                const int n = o0 / CH;
                __syncwarp();
                stage(n & 1, colR, valR);
                __syncwarp();
                load_chunk(s0 + (int64_t)(n + 3) * CH, colR, valR);
            }
            issue(k + 2);
        }
        asm volatile("cp.async.wait_all;\n" ::: "memory");
    }
    release_c(a.out_mc);   // multicast rows ordered before the caller's barrier
}


// Sums the per-unit partials of every row that crosses a unit boundary, in
// unit order: tail(u0) + head(u0 + 1) + ... + head(u1).  One warp per unit;
// a unit owns the fix-up of the split row that starts inside it.
template <typename T, typename I>
__global__ void __launch_bounds__(kGatherThreads)
csr_fixup_kernel(const GatherArgs a)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const I *rowptr = static_cast<const I *>(a.rowptr);

    for (int64_t u = a.unit_begin + warp; u < a.unit_end - 1; u += nwarps) {
        const int64_t lo = u * a.unit;
        const int64_t hi = lo + a.unit;
        int64_t r;
        if (a.split_rows) {
            r = a.split_rows[u - a.unit_begin];   // written by the ring kernel
            if (r < 0) continue;
        } else {
            r = warp_lower_bound(rowptr, a.row_begin, a.M + 1, hi) - 1;
        }
        if (r < a.row_begin || r >= a.M) continue;
        const int64_t beg = ld_idx(rowptr + r);
        const int64_t end = ld_idx(rowptr + r + 1);
        if (!(end > hi && beg >= lo && beg <= end && end <= a.nnz)) continue;
        const int64_t u1 = min((end - 1) / a.unit, a.unit_end - 1);
        for (int64_t f = (int64_t)lane * 4; f < a.N; f += 128) {
            const float *base = a.partial + f;
            float4 s = *reinterpret_cast<const float4 *>(base + ((u - a.unit_begin) * 2 + 1) * a.N);
            for (int64_t w = u + 1; w <= u1; ++w) {
                const float4 h = *reinterpret_cast<const float4 *>(base + ((w - a.unit_begin) * 2) * a.N);
                s.x += h.x; s.y += h.y; s.z += h.z; s.w += h.w;
            }
            T *o = static_cast<T *>(a.out) + r * a.N + f;
            if constexpr (sizeof(T) == 2) {
                const __half2 lo = __floats2half2_rn(s.x, s.y), hi = __floats2half2_rn(s.z, s.w);
                store_c8(a.out, a.out_mc, o,
                         make_uint2(*reinterpret_cast<const unsigned *>(&lo), *reinterpret_cast<const unsigned *>(&hi)));
            } else {
                store_c16(a.out, a.out_mc, o,
                          make_uint4(__float_as_uint(s.x), __float_as_uint(s.y), __float_as_uint(s.z), __float_as_uint(s.w)));
            }
        }
    }
    release_c(a.out_mc);   // multicast rows ordered before the caller's barrier
}

template <typename T, typename I>
cudaError_t launch_fixup(const GatherArgs &a, cudaStream_t stream)
{
    const int64_t units = a.unit_end - a.unit_begin;
    if (units <= 1) return cudaSuccess;
    const int64_t fb = std::min<int64_t>((units + 7) / 8, 8LL * device_sm_count());
    csr_fixup_kernel<T, I><<<(unsigned)std::max<int64_t>(fb, 1), kGatherThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

template <typename T, typename I, typename Kern>
cudaError_t launch_kernel(Kern kern, const GatherArgs &a, int64_t units_per_warp, cudaStream_t stream)
{
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGatherThreads, 0);
    if (e != cudaSuccess) return e;
    const int64_t units = a.unit_end - a.unit_begin;
    const int64_t warps_needed = (units + units_per_warp - 1) / units_per_warp;
    int64_t blocks = (int64_t)std::max(per_sm, 1) * device_sm_count();
    blocks = std::min(blocks, (warps_needed + 7) / 8);
    blocks = std::max<int64_t>(blocks, 1);
    kern<<<(unsigned)blocks, kGatherThreads, 0, stream>>>(a);
    e = cudaGetLastError();
    return e != cudaSuccess ? e : launch_fixup<T, I>(a, stream);
}

// Kernel choice.  Default: the tensor-core kernel where eligible (fp16,
// N % 64 == 0), else the ring kernel for whole-warp rows, the stream kernel
// for half-warp rows and the row kernel for narrower rows.  The environment
// variable SPMM_B200_GATHER = ring | stream | row selects one of the CUDA-core
// kernels (all three produce bitwise-identical sums) for A/B measurement.
int gather_kernel_choice()
{
    static const int choice = [] {
        const char *v = getenv("SPMM_B200_GATHER");
        if (v && strcmp(v, "row") == 0) return 2;
        if (v && strcmp(v, "stream") == 0) return 1;
        if (v && strcmp(v, "ring") == 0) return 0;
        return -1;
    }();
    return choice;
}

template <typename T, typename I, typename Kern>
cudaError_t launch_ring(Kern kern, const GatherArgs &a, int units_per_warp, size_t smem, cudaStream_t stream)
{
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGatherThreads, smem);
    if (e != cudaSuccess) return e;
    const int64_t units = a.unit_end - a.unit_begin;
    const int64_t warps_needed = (units + units_per_warp - 1) / units_per_warp;
    int64_t blocks = (int64_t)std::max(per_sm, 1) * device_sm_count();
    blocks = std::max<int64_t>(1, std::min(blocks, (warps_needed + 7) / 8));
    GatherArgs b = a;
    b.split_rows = a.unit_rows;   // the ring kernel records the split row of each unit
    kern<<<(unsigned)blocks, kGatherThreads, smem, stream>>>(b);
    e = cudaGetLastError();
    return e != cudaSuccess ? e : launch_fixup<T, I>(b, stream);
}

template <typename T, typename I, int G, int VPL, int U, int MINB>
cudaError_t launch_cfg(const GatherArgs &a, cudaStream_t stream)
{
    if constexpr (G >= 16) {
        const int choice = gather_kernel_choice();
        const bool full = a.N / Vec<T>::kElems == G * VPL;
        if constexpr (G == 32) {
        if (choice <= 0 && a.K > 0) {
            // ring (measured faster when a whole warp serves one row; half-warp
            // groups stay on the stream kernel): 2 * U positions x VPL
            // vectors per lane, 8 warps per block
            const size_t smem = (size_t)(kGatherThreads / 32) * RingShape<T, VPL, U>::kWarpBytes;
            constexpr int RMINB = (VPL == 1) ? 3 : 2;
            if constexpr (VPL >= 2) {   // rows of 1 KB or more: the L2 plan applies
                if (full && a.l2_bits)
                    return launch_ring<T, I>(csr_ring_kernel<T, I, G, VPL, U, RMINB, true, true>, a, 32 / G, smem,
                                             stream);
            }
            if (full)
                return launch_ring<T, I>(csr_ring_kernel<T, I, G, VPL, U, RMINB, true>, a, 32 / G, smem, stream);
            return launch_ring<T, I>(csr_ring_kernel<T, I, G, VPL, U, RMINB, false>, a, 32 / G, smem, stream);
        }
        }
        if (choice <= 1 && a.K > 0) {
            if (full)
                return launch_kernel<T, I>(csr_stream_kernel<T, I, G, VPL, U, MINB, true>, a, 32 / G, stream);
            return launch_kernel<T, I>(csr_stream_kernel<T, I, G, VPL, U, MINB, false>, a, 32 / G, stream);
        }
    }
    return launch_kernel<T, I>(csr_gather_kernel<T, I, G, VPL, U, (G >= 16 && MINB < 3 && VPL == 1) ? MINB + 1 : MINB>,
                               a, 1, stream);
}

// U x VPL = 8 sixteen-byte gathers in flight per lane (128 B) at 24 warps/SM
// by default; the deep-batch variant keeps 16 in flight at 16 warps/SM.
// Both consume the nonzeros of a row in the same order, so their sums are
// bitwise identical.
template <typename T, typename I>
cudaError_t launch_typed(const GatherArgs &a, int batch_depth, cudaStream_t s)
{
    if constexpr (sizeof(T) == 2) {
        if (gather_kernel_choice() < 0 && gather_mma_eligible(a, SPMM_F16)) {
            GatherArgs m = a;   // the tensor-core kernel may use coarser units
            const cudaError_t e = launch_gather_mma(m, sizeof(I) == 4 ? SPMM_I32 : SPMM_I64, batch_depth, s);
            return e != cudaSuccess ? e : launch_fixup<T, I>(m, s);
        }
    }
    const int64_t NV = a.N / Vec<T>::kElems;
    const bool deep = batch_depth != 0;
#define SPMM_GATHER_CFG(G, VPL, U)                                                         \
    return deep ? launch_cfg<T, I, G, VPL, 2 * (U), ((G) >= 16 || (VPL) > 1 ? 1 : 2)>(a, s)  \
                : launch_cfg<T, I, G, VPL, U, ((G) >= 16 || (VPL) > 1 ? 2 : 3)>(a, s)
    if (NV <= 2) SPMM_GATHER_CFG(2, 1, 8);
    if (NV <= 4) SPMM_GATHER_CFG(4, 1, 8);
    if (NV <= 8) SPMM_GATHER_CFG(8, 1, 8);
    if (NV <= 16) SPMM_GATHER_CFG(16, 1, 8);
    if (NV <= 32) SPMM_GATHER_CFG(32, 1, 8);
    if (NV <= 64) SPMM_GATHER_CFG(32, 2, 4);
    SPMM_GATHER_CFG(32, 4, 2);
#undef SPMM_GATHER_CFG
}

}  // namespace

GatherPlan plan_gather(int64_t nnz, int64_t N, int dtype, bool with_l2)
{
    GatherPlan p;
    p.l2 = with_l2 && l2_plan_wanted(nnz, N, dtype);
    p.N = N;
    // Unit size depends on nnz only (never on N, the device or the variant):
    // about 32K units, 256..8192 nonzeros each, a power of two; below 2^20
    // nonzeros the floor is 64, so small matrices still spread over all SMs
    // (config 1, 164K nonzeros: 34.9 -> 21.7 us; a floor under 256 measured
    // slower on power-law matrices of 1.6M nonzeros).
    const int64_t target = units_for(nnz, 32768);
    int64_t unit = nnz < (int64_t(1) << 20) ? 64 : 256;
    while (unit < target && unit < 8192) unit <<= 1;
    p.unit = unit;
    p.unit_begin = 0;
    p.unit_end = units_for(nnz, unit);
    return p;
}

cudaError_t launch_gather(const GatherArgs &a, int itype, int dtype, int batch_depth,
                          cudaStream_t stream)
{
    if (a.M <= a.row_begin) return cudaSuccess;
    if (dtype == SPMM_F16) {
        return itype == SPMM_I32 ? launch_typed<__half, int>(a, batch_depth, stream)
                                 : launch_typed<__half, int64_t>(a, batch_depth, stream);
    }
    return itype == SPMM_I32 ? launch_typed<float, int>(a, batch_depth, stream)
                             : launch_typed<float, int64_t>(a, batch_depth, stream);
}

}  // namespace spmmb
