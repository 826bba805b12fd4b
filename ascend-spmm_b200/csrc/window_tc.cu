// Window path on the fifth-generation tensor cores: tcgen05.mma with the
// accumulators in tensor memory (TMEM), fp16 in, fp32 accumulate, for
// feature widths that are a multiple of 128.
//
// Same semantics as window_warp.cu / window.cu (reference:
// op_kernel/spmm_ascend_cube.cpp:52-165, 265-288, and the vector-core rows
// added on top, :782-875): window slot s owns output rows [16 s, 16 s + 16) =
// sum over its (16 x 1) blocks of Cvalue[16 b + i] * B[Ccol[b], :] plus the
// CSR entries of those rows, summed in fp32 and rounded to fp16 once.
//
// Design.  A CTA is one warpgroup (128 threads); an item is (window, slice of
// 128 features).  The window's stream - its blocks, then the CSR entries of
// its rows - is cut into chunks of 16 entries and every chunk becomes one
//     D[feature, row] += sum_k G[k, feature] * V[k, row]
// with M = 128 features, N = 16 window rows and K = 16 entries
// (tcgen05.mma.cta_group::1.kind::f16, D in 16 TMEM columns):
//  * G (the 16 gathered B-row slices) is the A operand, MN-major (features
//    contiguous) in the canonical 128-byte-swizzled layout: two 64-feature
//    atoms of 8 entries x 128 bytes per 8-entry group.  All 128 threads fill
//    it with 16-byte cp.async copies (zero-filled past the stream) that
//    complete on the stage's mbarrier (cp.async.mbarrier.arrive.noinc);
//  * V (values) is the B operand, MN-major (rows contiguous), no swizzle:
//    core matrices of 8 entries x 8 rows.  A block's 16 values are copied
//    the same way; a CSR entry's value is written at its row by a thread
//    (st.shared, then fence.proxy.async before the arrive);
//  * thread 0 issues the MMAs a few chunks behind the copies and commits
//    each to the stage's "empty" mbarrier, which frees the stage for the
//    copies STAGES chunks later; the last chunk of an item also commits to
//    the item's accumulator mbarrier;
//  * the epilogue runs one item behind: each thread reads its feature's 16
//    rows from TMEM (tcgen05.ld 32x32b, lane = feature), rounds to fp16 and
//    stores them.  Two accumulators alternate between items.
// Several CTAs share an SM (36 KB of shared memory and 32 TMEM columns
// each), so one CTA's index loads overlap another's gathers.
//
// Numerics: every product of fp16 inputs is exact in fp32; the tensor core
// adds each chunk's 16 products into the fp32 accumulator, chunk after chunk
// in stream order; one rounding to fp16 at the end.  As in any dense-tile
// product, a non-finite B element reaches the other rows of its window
// (0 * inf); finite inputs contribute exactly what the reference sums.
//
// Every mbarrier wait is bounded; on expiry the kernel records
// SPMM_DEV_TIMEOUT, stops issuing work, waits (bounded) for what it issued
// and frees its TMEM before returning.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

constexpr int kTcThreads = 128;   // one warpgroup: TMEM lane t = feature t of the slice
constexpr int kTcFW = 128;        // features per item
constexpr int kTcAcc = 2;         // accumulators (16 TMEM columns each)
constexpr int kTcCols = 32;       // TMEM columns allocated per CTA (power of two >= 32)
constexpr int kTcSeg = 8;         // chunks whose entries are staged per index segment (128 entries)
constexpr long long kTcSpin = 1ll << 26;   // polls per bounded wait
constexpr long long kTcCycles = 1ll << 32; // ... or about 2 s of SM cycles

template <int STAGES> struct TcShape {
    static constexpr int kA = 4096;                       // gathered rows of one chunk: 16 x 128 fp16
    static constexpr int kV = 512;                        // value tile: 16 entries x 16 rows fp16
    static constexpr int kAOff = 0;                       // STAGES A tiles, 1024-byte aligned
    static constexpr int kVOff = kAOff + STAGES * kA;     // STAGES value tiles
    static constexpr int kColOff = kVOff + STAGES * kV;   // segment: 128 columns (int32)
    static constexpr int kValOff = kColOff + 128 * 4;     // segment: 128 CSR values (fp16 bits)
    static constexpr int kRowOff = kValOff + 128 * 2;     // segment: 128 CSR rows in the window (int8)
    static constexpr int kMetaOff = kRowOff + 128;        // per item: 4 stream sizes, then 17 row pointers
    static constexpr int kBarOff = kMetaOff + 8 * (8 + 17);
    static constexpr int kFull = kBarOff;                 // STAGES mbarriers
    static constexpr int kEmpty = kFull + 8 * STAGES;     // STAGES mbarriers
    static constexpr int kAccF = kEmpty + 8 * STAGES;     // kTcAcc mbarriers
    static constexpr int kDone = kAccF + 8 * kTcAcc;      // final drain
    static constexpr int kStageMeta = kDone + 8;          // per stage: accumulator | first << 8 | last << 9
    static constexpr int kTmemSlot = kStageMeta + 4 * STAGES;
    static constexpr int kFlag = kTmemSlot + 4;
    static constexpr int kBytes = kFlag + 16 + 1024;      // + slack to align the base to 1024
};

// ---- PTX helpers -------------------------------------------------------------
__device__ __forceinline__ void tc_cp16(unsigned dst, const void *src, int bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_init(unsigned bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}\n" ::"r"(bar) : "memory");
}
// An arrival triggered when every cp.async this thread issued so far has landed.
__device__ __forceinline__ void mbar_arrive_cpasync(unsigned bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");
}
// POLL = 0: try_wait (the thread may be suspended until the phase
// completes); POLL = 1: test_wait (never suspends; a spin).
template <int POLL>
__device__ __forceinline__ bool mbar_test(unsigned bar, unsigned parity)
{
    unsigned ok;
    if constexpr (POLL == 0)
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}\n"
                     : "=r"(ok)
                     : "r"(bar), "r"(parity)
                     : "memory");
    else
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}\n"
                     : "=r"(ok)
                     : "r"(bar), "r"(parity)
                     : "memory");
    return ok != 0;
}
// Bounded wait for the phase of the given parity; false on expiry.
template <int POLL>
__device__ __forceinline__ bool mbar_wait(unsigned bar, unsigned parity)
{
    if (mbar_test<POLL>(bar, parity)) return true;
    const long long t0 = clock64();
    for (long long i = 0; i < kTcSpin; ++i) {
        if (mbar_test<POLL>(bar, parity)) return true;
        if (clock64() - t0 > kTcCycles) break;
    }
    return false;
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]; accumulate = 0 overwrites D.
__device__ __forceinline__ void tc_mma(unsigned tmem_d, uint64_t adesc, uint64_t bdesc, unsigned idesc, unsigned acc)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
                 : "memory");
}
// mbarrier arrival once every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(unsigned bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_ld16(unsigned taddr, float *v)
{
    unsigned r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                 "[%16];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (sm100 format): start address, leading
// and stride byte offsets (16-byte units), version 1, layout type.
__device__ __forceinline__ uint64_t smem_desc(unsigned addr, unsigned lbo, unsigned sbo, unsigned layout)
{
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3fffu);
    d |= (uint64_t)((lbo >> 4) & 0x3fffu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3fffu) << 32;
    d |= (uint64_t)1 << 46;                   // descriptor version for sm100
    d |= (uint64_t)(layout & 7u) << 61;       // 0 = no swizzle, 2 = 128-byte swizzle
    return d;
}

// Instruction descriptor: fp32 accumulator, fp16 A and B, both MN-major,
// N = 16, M = 128.
constexpr unsigned kTcIdesc = (1u << 4) | (1u << 15) | (1u << 16) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

// Byte offset of 16-byte piece j (features 8 j .. 8 j + 7) of entry k in the
// A tile: [feature atom][entry group][8 entries x 128 bytes], swizzled.
__device__ __forceinline__ unsigned a_offset(int k, int j)
{
    const int atom = j >> 3, jj = j & 7, kg = k >> 3, kr = k & 7;
    return (unsigned)(atom * 2048 + kg * 1024 + kr * 128 + ((jj ^ kr) << 4));
}
// Byte offset of the 8 values of entry k for window rows 8 g .. 8 g + 7 in
// the V tile: [row group][entry group][8 entries x 16 bytes].
__device__ __forceinline__ unsigned v_offset(int k, int g) { return (unsigned)(g * 256 + (k >> 3) * 128 + (k & 7) * 16); }

template <typename I, int STAGES, int MINB, int POLL>
__global__ void __launch_bounds__(kTcThreads, MINB)
window_tc_kernel(const WindowArgs a, int nslices)
{
    using L = TcShape<STAGES>;
    extern __shared__ unsigned char tc_smem_raw[];
    const unsigned raw = (unsigned)__cvta_generic_to_shared(tc_smem_raw);
    const unsigned sbase = (raw + 1023u) & ~1023u;   // the A tiles need 1024-byte alignment
    unsigned char *gbase = tc_smem_raw + (sbase - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    int *s_col = reinterpret_cast<int *>(gbase + L::kColOff);
    unsigned short *s_val = reinterpret_cast<unsigned short *>(gbase + L::kValOff);
    signed char *s_row = reinterpret_cast<signed char *>(gbase + L::kRowOff);
    unsigned *s_stage_meta = reinterpret_cast<unsigned *>(gbase + L::kStageMeta);
    volatile unsigned *s_tmem = reinterpret_cast<volatile unsigned *>(gbase + L::kTmemSlot);
    volatile int *s_abort = reinterpret_cast<volatile int *>(gbase + L::kFlag);
    const unsigned bar_full = sbase + L::kFull, bar_empty = sbase + L::kEmpty, bar_acc = sbase + L::kAccF;
    const unsigned bar_done = sbase + L::kDone;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 2 * kTcThreads);   // a copy arrival and a plain arrival per thread
            mbar_init(bar_empty + 8 * s, 1);               // tcgen05.commit
        }
        for (int x = 0; x < kTcAcc; ++x) mbar_init(bar_acc + 8 * x, 1);
        mbar_init(bar_done, 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(sbase + L::kTmemSlot),
                     "r"(kTcCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const unsigned tmem = *s_tmem;

    const I *cptr = static_cast<const I *>(a.cptr);
    const I *ccol = static_cast<const I *>(a.ccol);
    const char *cval = static_cast<const char *>(a.cval);
    const I *vptr = static_cast<const I *>(a.vptr);
    const I *vcol = static_cast<const I *>(a.vcol);
    const unsigned short *vval = static_cast<const unsigned short *>(a.vval);
    const char *B = static_cast<const char *>(a.B);
    __half *out = static_cast<__half *>(a.out);
    const int64_t rowbytes = a.N * 2;

    uint32_t gchunk = 0;    // chunks produced by this CTA
    uint32_t gmma = 0;      // chunks multiplied (thread 0)
    uint32_t gitem = 0;     // items produced
    bool fail = false;      // this thread gave up a wait (then it only follows the loop structure)
    bool abort = false;     // some thread gave up (uniform: read at CTA barriers)
    int64_t prev_item = -1; // item whose epilogue is pending
    uint32_t prev_last = 0; // one past its last chunk
    auto give_up = [&](long long detail) {
        if (!fail) raise_status(a.status, SPMM_DEV_TIMEOUT, detail);
        fail = true;
        *s_abort = 1;
    };

    // Warp 0, converged: MMAs for chunks [gmma, upto), issued by lane 0.
    auto mma_until = [&](uint32_t upto) {
        while (gmma < upto) {
            const int st = (int)(gmma % STAGES);
            const bool ok = !fail && mbar_wait<POLL>(bar_full + 8 * st, (gmma / STAGES) & 1u);
            if (!ok) give_up(gmma);
            if (!__all_sync(0xffffffffu, ok)) {
                fail = true;
                break;
            }
            tc_fence_after();
            if (lane == 0) {
                const unsigned meta = s_stage_meta[st];
                const unsigned acc = meta & 0xffu, first = (meta >> 8) & 1u, last = (meta >> 9) & 1u;
                const uint64_t ad = smem_desc(sbase + L::kAOff + st * L::kA, 2048, 1024, 2);
                const uint64_t bd = smem_desc(sbase + L::kVOff + st * L::kV, 128, 256, 0);
                tc_mma(tmem + acc * 16, ad, bd, kTcIdesc, first ? 0u : 1u);
                tc_commit(bar_empty + 8 * st);
                if (last) tc_commit(bar_acc + 8 * acc);
            }
            __syncwarp();
            ++gmma;
        }
    };
    // All threads: the pending item's rows from TMEM to C.
    auto epilogue = [&](int64_t item, uint32_t seq) {
        const unsigned acc = seq % kTcAcc;
        const bool ok = !fail && mbar_wait<POLL>(bar_acc + 8 * acc, (seq / kTcAcc) & 1u);
        if (!ok) give_up(item);
        __syncwarp();
        if (!__all_sync(0xffffffffu, ok)) return;   // tcgen05.ld is warp-collective
        tc_fence_after();
        float v[16];
        tc_ld16(tmem + ((unsigned)(warp * 32) << 16) + acc * 16, v);
        tc_fence_before();
        const int64_t s = item / nslices;
        const int f = (int)(item % nslices) * kTcFW + tid;
        __half *o = out + 16 * s * a.N + f;
#pragma unroll
        for (int r = 0; r < 16; ++r) __stcs(o + r * a.N, __float2half_rn(v[r]));
    };

    long long *s_meta = reinterpret_cast<long long *>(gbase + L::kMetaOff);
    const volatile long long *vrs = s_meta + 8;                                // vptr[16 s + r], r = 0..16
    const int64_t nitems = a.nwin * nslices;
    for (int64_t it = blockIdx.x; it < nitems && !abort; it += gridDim.x) {
        const int64_t s = it / nslices;
        const int f0 = (int)(it % nslices) * kTcFW;
        // ---- the window's stream: blocks [cb, cb + nb), CSR entries [vb, vb + nv);
        // every thread reads the four bounds itself (broadcast loads), the 17
        // row pointers go to shared memory for the CSR rows of the entries
        __syncthreads();   // every read of the previous item's row pointers is done
        if (tid < 17) {
            int64_t vr = 0;
            if (a.vrows > 0 && 16 * s < a.vrows) vr = ld_idx(vptr + min(16 * s + tid, a.vrows));
            s_meta[8 + tid] = vr;
        }
        int64_t cb = ld_idx(cptr + s), ce = ld_idx(cptr + s + 1);
        if (cb < 0 || ce < cb || ce > a.nblocks) {
            if (tid == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, s);
            cb = ce = 0;
        }
        int64_t vb = 0, ve = 0;
        if (a.vrows > 0 && 16 * s < a.vrows) {
            vb = ld_idx(vptr + 16 * s);
            ve = ld_idx(vptr + min(16 * s + 16, a.vrows));
        }
        __syncthreads();
        {
            bool bad = vb < 0 || ve < vb || ve > a.vnnz;
            for (int r = 0; r < 16; ++r) bad = bad || vrs[r + 1] < vrs[r];
            if (bad) {
                if (tid == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, 16 * s);
                vb = ve = 0;
            }
        }
        const int nb = (int)(ce - cb), nv = (int)(ve - vb);
        const int nbc = (nb + 15) >> 4, nvc = (nv + 15) >> 4;
        const int nch = max(1, nbc + nvc);
        const uint32_t acc = gitem % kTcAcc;

        for (int x0 = 0; x0 < nch; x0 += kTcSeg) {
            // ---- stage the segment's entries: thread t = entry t % 16 of chunk x0 + t / 16
            if (x0 > 0) __syncthreads();   // the previous segment's entries have been read
            {
                const int x = x0 + tid / 16, k = tid % 16;
                int c = -1, row = -1;
                unsigned short val = 0;
                bool valid = false;
                int64_t cc = 0;
                if (x < nbc) {
                    const int e = 16 * x + k;
                    valid = e < nb;
                    if (valid) cc = (int64_t)ld_stream(ccol + cb + e);
                } else if (x < nbc + nvc) {
                    const int e = 16 * (x - nbc) + k;
                    valid = e < nv;
                    if (valid) {
                        const int64_t p = vb + e;
                        cc = (int64_t)ld_stream(vcol + p);
                        val = __ldcs(vval + p);
                        row = 0;
                        for (int r = 1; r < 16; ++r) row += vrs[r] <= p;
                    }
                }
                if (valid) {
                    if (cc >= 0 && cc < a.K) {
                        c = (int)cc;
                    } else {
                        raise_status(a.status, SPMM_DEV_BAD_COLUMN, s);
                        row = -1;
                    }
                }
                s_col[tid] = c;
                s_val[tid] = val;
                s_row[tid] = (signed char)row;
            }
            if (__syncthreads_or(*s_abort)) abort = true;
            if (abort) break;

            const int xend = min(nch, x0 + kTcSeg);
            for (int x = x0; x < xend; ++x) {
                const int st = (int)(gchunk % STAGES);
                if (!fail && !mbar_wait<POLL>(bar_empty + 8 * st, ((gchunk / STAGES) & 1u) ^ 1u)) give_up(gchunk);
                const unsigned As = sbase + L::kAOff + st * L::kA;
                const unsigned Vs = sbase + L::kVOff + st * L::kV;
                const int lx = x - x0;
                if (!fail) {
                    // gathered rows: pieces tid and tid + 128 (entry p / 16, piece p % 16)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int p = tid + 128 * h, k = p >> 4, j = p & 15;
                        const int c = s_col[16 * lx + k];
                        const char *src = B + (int64_t)(c >= 0 ? c : 0) * rowbytes + (f0 + 8 * j) * 2;
                        tc_cp16(As + a_offset(k, j), src, c >= 0 ? 16 : 0);
                    }
                    // values: thread t < 32 = entry t / 2, row group t % 2
                    if (tid < 32) {
                        const int k = tid >> 1, g = tid & 1;
                        if (x < nbc) {
                            const bool ok = 16 * x + k < nb;
                            const char *src = cval + ((cb + 16 * x + (ok ? k : 0)) * 16 + 8 * g) * 2;
                            tc_cp16(Vs + v_offset(k, g), src, ok ? 16 : 0);
                        } else {
                            const int row = s_row[16 * lx + k];
                            const unsigned val = s_val[16 * lx + k];
                            // the value at its row, zeros elsewhere (16-bit lane q of 8)
                            const int q = row - 8 * g;
                            const bool here = row >= 0 && (unsigned)q < 8u;
                            const unsigned word = here ? ((q & 1) ? (val << 16) : val) : 0u;
                            const int wi = here ? (q >> 1) : -1;
                            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(Vs + v_offset(k, g)),
                                         "r"(wi == 0 ? word : 0u), "r"(wi == 1 ? word : 0u), "r"(wi == 2 ? word : 0u),
                                         "r"(wi == 3 ? word : 0u)
                                         : "memory");
                        }
                    }
                    if (tid == 0) s_stage_meta[st] = acc | (x == 0 ? 1u << 8 : 0u) | (x == nch - 1 ? 1u << 9 : 0u);
                    // the value tile of a CSR chunk was written by st.shared: order it
                    // before the tensor core's (async-proxy) reads
                    if (tid < 32 && x >= nbc) fence_async_smem();
                    mbar_arrive_cpasync(bar_full + 8 * st);
                    mbar_arrive(bar_full + 8 * st);
                }
                ++gchunk;
                if (warp == 0 && gchunk > (uint32_t)(STAGES - 2)) mma_until(gchunk - (STAGES - 2));
            }
        }
        if (abort) break;
        // ---- the previous item is complete once its MMAs are: write it out
        if (prev_item >= 0) {
            if (warp == 0) mma_until(prev_last);
            epilogue(prev_item, gitem - 1);
            tc_fence_before();
            __syncthreads();   // every thread has read the accumulator before it is overwritten
            tc_fence_after();
        }
        prev_item = it;
        prev_last = gchunk;
        ++gitem;
        if (__syncthreads_or(*s_abort)) abort = true;
    }
    // ---- drain: the last item's MMAs and epilogue
    if (!abort && prev_item >= 0) {
        if (warp == 0) mma_until(prev_last);
        epilogue(prev_item, gitem - 1);
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    if (warp == 0 && gmma > 0) {
        // every MMA issued has completed before TMEM is released (bounded)
        if (lane == 0) tc_commit(bar_done);
        __syncwarp();
        mbar_wait<POLL>(bar_done, 0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    __syncwarp();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTcCols) : "memory");
}

template <typename I, int STAGES, int POLL>
cudaError_t launch_tc(const WindowArgs &a, cudaStream_t stream)
{
    using L = TcShape<STAGES>;
    constexpr int MINB = 4;
    auto kern = window_tc_kernel<I, STAGES, MINB, POLL>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    // all of the unified L1/shared array as shared memory, so several CTAs fit
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTcThreads, L::kBytes);
    if (e != cudaSuccess) return e;
    // SPMM_B200_TC_CTAS=n asks for n resident CTAs per SM (measurement)
    if (const char *v = getenv("SPMM_B200_TC_CTAS")) per_sm = atoi(v);
    per_sm = std::min(std::max(per_sm, 1), 512 / kTcCols);   // TMEM columns of one SM
    const int nslices = (int)(a.N / kTcFW);
    const int64_t items = a.nwin * nslices;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((int64_t)per_sm * device_sm_count(), items));
    kern<<<(unsigned)blocks, kTcThreads, L::kBytes, stream>>>(a, nslices);
    return cudaGetLastError();
}

}  // namespace

bool window_tc_eligible(const WindowArgs &a, int dtype)
{
    auto al = [](const void *p) { return ((uintptr_t)p & 15u) == 0; };
    return dtype == SPMM_F16 && a.N % kTcFW == 0 && a.K > 0 && a.K <= INT_MAX && al(a.cval) && al(a.B) &&
           al(a.out);
}

cudaError_t launch_window_tc(const WindowArgs &a, int itype, cudaStream_t stream)
{
    if (a.nwin <= 0) return cudaSuccess;
    // SPMM_B200_TC_POLL=spin selects the test_wait polling variant (measurement)
    static const bool spin = [] {
        const char *v = getenv("SPMM_B200_TC_POLL");
        return v && strcmp(v, "spin") == 0;
    }();
    if (spin) return itype == SPMM_I32 ? launch_tc<int, 8, 1>(a, stream) : launch_tc<int64_t, 8, 1>(a, stream);
    return itype == SPMM_I32 ? launch_tc<int, 8, 0>(a, stream) : launch_tc<int64_t, 8, 0>(a, stream);
}

}  // namespace spmmb
