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
                    if (vi < NV) __stcs(orow + vi, pack16<T>(acc[q]));
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
                if (vi < NV) __stcs(out + row * NV + vi, make_uint4(0, 0, 0, 0));
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
                                if (vi < NV) __stcs(out + row * NV + vi, pack16<T>(acc[q]));
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
}

// ---------------------------------------------------------------------------
// Ring kernel: the stream kernel with its gathers landing in shared memory.
//
// Each lane copies the 16-byte pieces of the B rows it will itself consume
// (cp.async.cg, L2 only) into a per-group ring of 2 x U positions and reads
// them back with one 16-byte shared load per position: no cross-lane
// synchronisation is needed (cp.async.wait_group covers the thread's own
// copies), in-flight data holds no registers, so more groups fit per SM and
// two batches stay in flight.  Row bookkeeping and the per-row fma order are
// those of csr_stream_kernel, so results are bitwise identical.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16_cg_s(unsigned saddr, const void *gmem)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gmem) : "memory");
}
__device__ __forceinline__ uint4 lds16(unsigned saddr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(saddr));
    return v;
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

template <typename T, typename I, int G, int VPL, int U, int MINB, bool FULL>
__global__ void __launch_bounds__(kGatherThreads, MINB)
csr_ring_kernel(const GatherArgs a)
{
    static_assert(G == 16 || G == 32, "ring groups are half-warps or warps");
    using F = FmaVec<T>;
    using Scalar = typename F::Scalar;
    constexpr int S = 32 / G;
    constexpr int EPV = Vec<T>::kElems;
    constexpr int CH = 64;          // nonzeros per prefetched column/value chunk
    constexpr int PER = CH / G;
    constexpr int RING = 2 * U;     // positions in the ring (two batches)
    static_assert(CH % U == 0 && U <= G, "batches tile the chunk");
    extern __shared__ __align__(16) uint4 ring_smem[];
    const int lane = threadIdx.x & 31;
    const int sub = lane / G, gl = lane % G, shift = sub * G;
    const unsigned gmask = (G == 32) ? 0xffffffffu : (((1u << G) - 1u) << shift);
    const int group_in_block = (threadIdx.x >> 5) * S + sub;
    // this lane's column of the ring, as a 32-bit shared address
    const unsigned ring_s = (unsigned)__cvta_generic_to_shared(ring_smem + (size_t)group_in_block * RING * VPL * G + gl);
    const int64_t stream = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * S + sub;
    const int64_t nstreams = (((int64_t)gridDim.x * blockDim.x) >> 5) * S;

    const I *rowptr = static_cast<const I *>(a.rowptr);
    const I *col = static_cast<const I *>(a.col);
    const T *val = static_cast<const T *>(a.val);
    const uint4 *Bl = static_cast<const uint4 *>(a.B) + gl;
    uint4 *out = static_cast<uint4 *>(a.out);
    const int NV = (int)(a.N / EPV);

    for (int64_t u = a.unit_begin + stream; u < a.unit_end; u += nstreams) {
        const int64_t lo = u * a.unit;
        const int64_t hi = min(lo + a.unit, a.nnz);
        const bool last = (u == a.unit_end - 1);
        const int64_t i0 = group_lower_bound<I, G>(rowptr, a.row_begin, a.M + 1, lo, gmask, gl, shift);
        int64_t r = i0;
        if (i0 > a.row_begin && (i0 > a.M || ld_idx(rowptr + i0) > lo)) r = i0 - 1;

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
        auto zero_row = [&](int64_t row) {
#pragma unroll
            for (int q = 0; q < VPL; ++q) {
                const int vi = gl + q * G;
                if (FULL || vi < NV) __stcs(out + row * NV + vi, make_uint4(0, 0, 0, 0));
            }
        };

        int64_t beg = 0, end = 0;
        bool have_row = false;
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
        bool head_pending = beg < lo;
        const int nbatch = (int)((hi - s0 + U - 1) / U);

        float acc[VPL][EPV];
#pragma unroll
        for (int q = 0; q < VPL; ++q)
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[q][e] = 0.f;

        // column/value chunks: A holds chunk ka, B chunk ka + 1
        int colA[PER], colB[PER];
        Scalar valA[PER], valB[PER];
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
        int ka = 0;
        load_chunk(s0, colA, valA);
        load_chunk(s0 + CH, colB, valB);
        // Entry o (offset from s0) lives in chunk o / CH (A = chunk ka,
        // B = chunk ka + 1), register slot (o % CH) / G, lane o % G.  A batch
        // never straddles a slot (U divides G), so the register is chosen once
        // per batch and each entry costs one shuffle.
        auto pick_col = [&](int o0) -> int {
            const bool inA = (o0 / CH) == ka;
            const int slot = (o0 % CH) / G;
            int cw = inA ? colA[0] : colB[0];
#pragma unroll
            for (int k = 1; k < PER; ++k)
                if (slot == k) cw = inA ? colA[k] : colB[k];
            return cw;
        };
        auto pick_val = [&](int o0) -> Scalar {
            const bool inA = (o0 / CH) == ka;
            const int slot = (o0 % CH) / G;
            Scalar vw = inA ? valA[0] : valB[0];
#pragma unroll
            for (int k = 1; k < PER; ++k)
                if (slot == k) vw = inA ? valA[k] : valB[k];
            return vw;
        };
        auto issue = [&](int k) {
            if (k < nbatch) {
                const int o0 = k * U;
                const int nv = (int)min((int64_t)U, hi - (s0 + o0));
                const int cw = pick_col(o0);
                const unsigned slot0 = ring_s + (unsigned)((k & 1) * U * VPL * G * 16);
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    const int c = __shfl_sync(gmask, cw, (o0 + j) % G, G);
                    if (j < nv) {
                        const uint4 *src = Bl + (int64_t)c * NV;
#pragma unroll
                        for (int q = 0; q < VPL; ++q)
                            if (FULL || gl + q * G < NV) cp_async16_cg_s(slot0 + (j * VPL + q) * G * 16, src + q * G);
                    }
                }
            }
            cp_async_commit_group();
        };
        issue(0);
        issue(1);

        bool done = false;
        for (int k = 0; k < nbatch && !done; ++k) {
            const int64_t pbase = s0 + (int64_t)k * U;
            const int nvalid = (int)min((int64_t)U, hi - pbase);
            const int64_t bend = pbase + nvalid;
            // row bookkeeping of this batch (as in csr_stream_kernel)
            unsigned ends = 0, tails = 0;
            int64_t myrow = 0;
            for (;;) {
                if (end <= bend) {
                    const int jb = (int)(end - pbase - 1);
                    ends |= 1u << jb;
                    if (gl == jb) myrow = r;
                    const int64_t prev = end;
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
                if (bend == hi) {
                    ends |= 1u << (nvalid - 1);
                    tails |= 1u << (nvalid - 1);
                    if (gl == nvalid - 1) myrow = r;
                    done = true;
                }
                break;
            }
            cp_async_wait_1();   // this lane's copies of batch k have landed
            const unsigned slot0 = ring_s + (unsigned)((k & 1) * U * VPL * G * 16);
            const Scalar vw = pick_val(k * U);
#pragma unroll
            for (int j = 0; j < U; ++j) {
                if (j < nvalid) {
                    const Scalar v = __shfl_sync(gmask, vw, (k * U + j) % G, G);
#pragma unroll
                    for (int q = 0; q < VPL; ++q)
                        if (FULL || gl + q * G < NV) F::run(acc[q], v, lds16(slot0 + (j * VPL + q) * G * 16));
                }
                if ((ends >> j) & 1u) {
                    if (head_pending || ((tails >> j) & 1u)) {
                        float *prow = a.partial + ((u - a.unit_begin) * 2 + (head_pending ? 0 : 1)) * a.N;
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
                        const int64_t row = __shfl_sync(gmask, myrow, j, G);
#pragma unroll
                        for (int q = 0; q < VPL; ++q) {
                            const int vi = gl + q * G;
                            if (FULL || vi < NV) __stcs(out + row * NV + vi, pack16<T>(acc[q]));
                        }
                    }
#pragma unroll
                    for (int q = 0; q < VPL; ++q)
#pragma unroll
                        for (int e = 0; e < EPV; ++e) acc[q][e] = 0.f;
                }
            }
            // consumption moves to the next chunk: B becomes A and the chunk
            // after it is loaded, 6 batches before the issue stage needs it
            if (((k + 1) * U) % CH == 0) {
#pragma unroll
                for (int i = 0; i < PER; ++i) {
                    colA[i] = colB[i];
                    valA[i] = valB[i];
                }
                ++ka;
                load_chunk(s0 + (int64_t)(ka + 1) * CH, colB, valB);
            }
            issue(k + 2);
        }
        asm volatile("cp.async.wait_all;\n" ::: "memory");
    }
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
        const int64_t i = warp_lower_bound(rowptr, a.row_begin, a.M + 1, hi);
        const int64_t r = i - 1;
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
                __half2 *o2 = reinterpret_cast<__half2 *>(o);
                o2[0] = __floats2half2_rn(s.x, s.y);
                o2[1] = __floats2half2_rn(s.z, s.w);
            } else {
                *reinterpret_cast<float4 *>(o) = s;
            }
        }
    }
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
    kern<<<(unsigned)blocks, kGatherThreads, smem, stream>>>(a);
    e = cudaGetLastError();
    return e != cudaSuccess ? e : launch_fixup<T, I>(a, stream);
}

template <typename T, typename I, int G, int VPL, int U, int MINB>
cudaError_t launch_cfg(const GatherArgs &a, cudaStream_t stream)
{
    if constexpr (G >= 16) {
        const int choice = gather_kernel_choice();
        const bool full = a.N / Vec<T>::kElems == G * VPL;
        if (choice <= 0 && a.K > 0 && G == 32) {
            // ring (measured faster when a whole warp serves one row; half-warp
            // groups stay on the stream kernel): 2 * U positions x VPL
            // vectors per lane, 8 warps per block
            const size_t smem = (size_t)kGatherThreads * 2 * U * VPL * 16;
            constexpr int RMINB = (VPL == 1) ? 3 : 2;
            if (full)
                return launch_ring<T, I>(csr_ring_kernel<T, I, G, VPL, U, RMINB, true>, a, 32 / G, smem, stream);
            return launch_ring<T, I>(csr_ring_kernel<T, I, G, VPL, U, RMINB, false>, a, 32 / G, smem, stream);
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

GatherPlan plan_gather(int64_t nnz, int64_t N, int dtype)
{
    (void)dtype;
    GatherPlan p;
    p.N = N;
    // Unit size depends on nnz only (never on N, the device or the variant):
    // about 32K units, 256..8192 nonzeros each, a power of two.
    int64_t target = (nnz + 32767) / 32768;
    int64_t unit = 256;
    while (unit < target && unit < 8192) unit <<= 1;
    p.unit = unit;
    p.unit_begin = 0;
    p.unit_end = std::max<int64_t>(1, (nnz + unit - 1) / unit);
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
