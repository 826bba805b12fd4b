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
// Design (one CTA per SM, warp-specialised; an item is (window, slice of 128
// features)).  The window's stream - its blocks, then the CSR entries of its
// rows - is cut into chunks of 16 entries and every chunk becomes one
//     D[feature, row] += sum_k G[k, feature] * V[k, row]
// with M = 128 features, N = 16 window rows and K = 16 entries
// (tcgen05.mma.cta_group::1.kind::f16, D in 16 TMEM columns):
//  * 8 producer warps, each with its own item sequence and a ring of 5
//    stages: G (the 16 gathered B-row slices, the A operand) goes MN-major
//    (features contiguous) into the canonical 128-byte-swizzled layout - two
//    64-feature atoms of 8 entries x 128 bytes per 8-entry group - by 16-byte
//    cp.async copies (zero-filled past the stream) that complete on the
//    stage's mbarrier (cp.async.mbarrier.arrive.noinc); V (values, the B
//    operand) goes MN-major (rows contiguous) without swizzle, in core
//    matrices of 8 entries x 8 rows: a block's 16 values by cp.async, a CSR
//    entry's value written at its row by st.shared + fence.proxy.async.  The
//    next 32 entries' columns are loaded while a chunk's copies are issued;
//  * one MMA warp serves whichever producer has a chunk ready: lane 0 issues
//    the MMA into that producer's accumulator (two per producer, alternating
//    between its items) and commits it to the stage's "empty" mbarrier; an
//    item's last chunk also commits to the accumulator's mbarrier and
//    appends (accumulator, item) to a completion queue;
//  * 4 epilogue warps drain the queue in order: each thread reads its
//    feature's 16 rows from TMEM (tcgen05.ld 32x32b: warp w reads lanes
//    32 w .. 32 w + 31), rounds to fp16 and stores them, then releases the
//    accumulator to its producer's next-but-one item.
// No CTA-wide barrier runs between the set-up and the teardown.
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

constexpr int kTcFW = 128;        // features per item (TMEM lane t = feature t of the slice)
constexpr int kTcProducers = 12;  // producer warps, each with its own item sequence, stage ring and accumulators
constexpr int kTcStages = 4;      // stages per producer
constexpr int kTcLag = 3;         // a chunk's MMA is issued this many chunks after its copies
constexpr int kTcEpi = 4;         // epilogue warps (TMEM lane quarters 0-3); warp 0 owns TMEM
constexpr int kTcProd0 = kTcEpi;  // first producer warp
constexpr int kTcThreads = 32 * (kTcEpi + kTcProducers);
constexpr int kTcCols = 512;      // TMEM columns: 2 accumulators of 16 columns per producer (384 used)
constexpr long long kTcSpin = 1ll << 26;   // polls per bounded wait
constexpr long long kTcCycles = 1ll << 32; // ... or about 2 s of SM cycles

struct TcShape {
    static constexpr int kStagesAll = kTcProducers * kTcStages;
    static constexpr int kA = 4096;                        // gathered rows of one chunk: 16 x 128 fp16
    static constexpr int kV = 512;                         // value tile: 16 entries x 16 rows fp16
    static constexpr int kAOff = 0;                        // A tiles, 1024-byte aligned
    static constexpr int kVOff = kAOff + kStagesAll * kA;  // value tiles
    static constexpr int kBarOff = kVOff + kStagesAll * kV;
    static constexpr int kFull = kBarOff;                  // kStagesAll mbarriers
    static constexpr int kEmpty = kFull + 8 * kStagesAll;  // kStagesAll mbarriers
    static constexpr int kAccF = kEmpty + 8 * kStagesAll;  // 2 per producer: accumulator written
    static constexpr int kAccE = kAccF + 16 * kTcProducers; // 2 per producer: accumulator read out
    static constexpr int kQFull = kAccE + 16 * kTcProducers;      // 2 per producer: completion-queue slots
    static constexpr int kDone = kQFull + 16 * kTcProducers;       // final drain of the MMAs
    static constexpr int kQueue = kDone + 8;                        // 2 P entries: accumulator, parity, item
    static constexpr int kQTail = kQueue + 16 * 2 * kTcProducers;   // completion-queue tail counter
    static constexpr int kStageMeta = kQTail + 16;                  // (unused)
    static constexpr int kTmemSlot = kStageMeta + 4 * kStagesAll;
    static constexpr int kFlag = kTmemSlot + 4;
    static constexpr int kBytes = kFlag + 16 + 1024;       // + slack to align the base to 1024
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
// POLL = 0: try_wait with a suspend-time hint (the thread sleeps until the
// phase completes or about 20 us pass, so waiting warps leave the issue
// slots to the working ones); POLL = 1: test_wait (never suspends; a spin).
template <int POLL>
__device__ __forceinline__ bool mbar_test(unsigned bar, unsigned parity)
{
    unsigned ok;
    if constexpr (POLL == 0)   // suspended (up to ~20 us, woken when the phase completes)
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}\n"
                     : "=r"(ok)
                     : "r"(bar), "r"(parity), "r"(20000)
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

template <typename I, int POLL>
__global__ void __launch_bounds__(kTcThreads, 1)
window_tc_kernel(const WindowArgs a, int nslices)
{
    using L = TcShape;
    constexpr unsigned kAll = 0xffffffffu;
    constexpr int kQ = 2 * kTcProducers;   // at most two items per producer await their epilogue
    extern __shared__ unsigned char tc_smem_raw[];
    const unsigned raw = (unsigned)__cvta_generic_to_shared(tc_smem_raw);
    const unsigned sbase = (raw + 1023u) & ~1023u;   // the A tiles need 1024-byte alignment
    unsigned char *gbase = tc_smem_raw + (sbase - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    volatile unsigned *s_tmem = reinterpret_cast<volatile unsigned *>(gbase + L::kTmemSlot);
    volatile int *s_abort = reinterpret_cast<volatile int *>(gbase + L::kFlag);
    volatile long long *s_queue = reinterpret_cast<volatile long long *>(gbase + L::kQueue);
    int *s_qtail = reinterpret_cast<int *>(gbase + L::kQTail);
    const unsigned bar_full = sbase + L::kFull, bar_empty = sbase + L::kEmpty;
    const unsigned bar_accf = sbase + L::kAccF, bar_acce = sbase + L::kAccE;
    const unsigned bar_qfull = sbase + L::kQFull, bar_done = sbase + L::kDone;

    if (tid == 0) {
        for (int x = 0; x < L::kStagesAll; ++x) {
            mbar_init(bar_full + 8 * x, 64);   // a copy arrival and a plain arrival per producer lane
            mbar_init(bar_empty + 8 * x, 1);   // tcgen05.commit of the chunk's MMA
        }
        for (int x = 0; x < 2 * kTcProducers; ++x) {
            mbar_init(bar_accf + 8 * x, 1);                // tcgen05.commit of an item's last chunk
            mbar_init(bar_acce + 8 * x, 32 * kTcEpi);      // every epilogue thread has read it
            mbar_init(bar_qfull + 8 * x, 1);               // a producer has written the queue slot
        }
        mbar_init(bar_done, kTcProducers);                 // one tcgen05.commit per producer at the end
        *s_abort = 0;
        *s_qtail = 0;
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

    const int64_t nitems = a.nwin * nslices;
    bool fail = false;
    auto give_up = [&](long long detail) {
        if (!fail) raise_status(a.status, SPMM_DEV_TIMEOUT, detail);
        fail = true;
        *s_abort = 1;
    };

    if (warp >= kTcProd0) {
        // ========== producer warp: gathers, value tiles and its own MMAs ==========
        const int p = warp - kTcProd0;
        const I *cptr = static_cast<const I *>(a.cptr);
        const I *ccol = static_cast<const I *>(a.ccol);
        const char *cval = static_cast<const char *>(a.cval);
        const I *vptr = static_cast<const I *>(a.vptr);
        const I *vcol = static_cast<const I *>(a.vcol);
        const unsigned short *vval = static_cast<const unsigned short *>(a.vval);
        const char *B = static_cast<const char *>(a.B);
        const int64_t rowbytes = a.N * 2;
        uint32_t chunkc = 0;   // chunks whose copies were issued
        uint32_t mmac = 0;     // chunks multiplied
        // Per stage, the pending MMA's description (lane 0 only):
        // accumulator | first << 8 | last << 9 | accumulator-use parity << 10, and the item.
        unsigned pend_meta[kTcStages];
        int64_t pend_item[kTcStages];
        // MMA of chunk mmac: its copies have landed (the stage's mbarrier), one
        // lane issues it into the producer's accumulator and commits it to the
        // stage's "empty" mbarrier; an item's last chunk is committed to the
        // accumulator's mbarrier and queued for the epilogue.
        auto issue_mma = [&]() {
            const int sl = (int)(mmac % kTcStages);
            const int st = p * kTcStages + sl;
            const bool ok = mbar_wait<POLL>(bar_full + 8 * st, (mmac / kTcStages) & 1u);
            if (!__all_sync(kAll, ok)) { give_up(mmac); return; }
            unsigned meta = 0;
            int64_t item = 0;
#pragma unroll
            for (int i = 0; i < kTcStages; ++i)
                if (i == sl) { meta = pend_meta[i]; item = pend_item[i]; }
            const unsigned acc = meta & 0xffu, par = (meta >> 10) & 1u;
            if (meta & (1u << 8)) {   // first chunk of an item: its accumulator's previous item was read out
                const uint32_t use = (uint32_t)(((item - ((int64_t)blockIdx.x * kTcProducers + p)) /
                                                 ((int64_t)gridDim.x * kTcProducers)) >> 1);
                if (use >= 1) {
                    const bool ok2 = mbar_wait<POLL>(bar_acce + 8 * acc, (use - 1) & 1u);
                    if (!__all_sync(kAll, ok2)) { give_up(item); return; }
                    tc_fence_after();
                }
            }
            if (lane == 0) {
                const uint64_t ad = smem_desc(sbase + L::kAOff + st * L::kA, 2048, 1024, 2);
                const uint64_t bd = smem_desc(sbase + L::kVOff + st * L::kV, 128, 256, 0);
                tc_mma(tmem + acc * 16, ad, bd, kTcIdesc, (meta & (1u << 8)) ? 0u : 1u);
                tc_commit(bar_empty + 8 * st);
                if (meta & (1u << 9)) {
                    tc_commit(bar_accf + 8 * acc);
                    const int slot = atomicAdd(s_qtail, 1) % kQ;
                    s_queue[2 * slot] = (long long)(acc | (par << 8));
                    s_queue[2 * slot + 1] = (long long)item;
                    mbar_arrive(bar_qfull + 8 * slot);
                }
            }
            __syncwarp();
            ++mmac;
        };
        uint32_t r = 0;   // items started by this producer
        for (int64_t it = (int64_t)blockIdx.x * kTcProducers + p; it < nitems && !fail;
             it += (int64_t)gridDim.x * kTcProducers, ++r) {
            if (*s_abort) break;
            const int64_t s = it / nslices;
            const int f0 = (int)(it % nslices) * kTcFW;
            const unsigned acc = (unsigned)(p * 2 + (r & 1)), par = (r >> 1) & 1u;
            // ---- the window's stream: blocks [cb, cb + nb), CSR entries [vb, vb + nv)
            int64_t cb = ld_idx(cptr + s), ce = ld_idx(cptr + s + 1);
            if (cb < 0 || ce < cb || ce > a.nblocks) {
                if (lane == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, s);
                cb = ce = 0;
            }
            int64_t vr = 0;   // lane r < 17: row pointer of window row r
            if (a.vrows > 0 && 16 * s < a.vrows) vr = ld_idx(vptr + min(16 * s + min(lane, 16), a.vrows));
            int64_t vb = __shfl_sync(kAll, vr, 0), ve = __shfl_sync(kAll, vr, 16);
            {
                const int64_t nxt = __shfl_down_sync(kAll, vr, 1);
                const bool bad = (lane == 0 && (vb < 0 || ve > a.vnnz)) || (lane < 16 && nxt < vr);
                if (__any_sync(kAll, bad)) {
                    if (lane == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, 16 * s);
                    vb = ve = 0;
                    vr = 0;
                }
            }
            const int nb = (int)(ce - cb), nv = (int)(ve - vb);
            const int nbc = (nb + 15) >> 4, nvc = (nv + 15) >> 4;
            const int nch = max(1, nbc + nvc);
            // Lane l holds entry l of superchunk q (chunks 2 q, 2 q + 1): its
            // column (-1 if none), and for CSR entries its value and row.
            auto load_entry = [&](int q, int &c, unsigned &val) {
                const int x = 2 * q + (lane >> 4), k = lane & 15;
                c = -1;
                val = 0u;
                int64_t cc = -1;
                bool valid = false;
                if (x < nbc) {
                    const int e = 16 * x + k;
                    valid = e < nb;
                    if (valid) cc = (int64_t)ld_stream(ccol + cb + e);
                } else if (x < nbc + nvc) {
                    const int e = 16 * (x - nbc) + k;
                    valid = e < nv;
                    if (valid) {
                        cc = (int64_t)ld_stream(vcol + vb + e);
                        val = __ldcs(vval + vb + e);
                    }
                }
                if (valid) {
                    if (cc >= 0 && cc < a.K) c = (int)cc;
                    else raise_status(a.status, SPMM_DEV_BAD_COLUMN, s);
                }
            };
            auto row_of = [&](int q, int c) -> int {   // window row of this lane's CSR entry
                const int x = 2 * q + (lane >> 4);
                const int64_t pos = vb + 16 * (x - nbc) + (lane & 15);
                int row = 0;
#pragma unroll
                for (int rr = 1; rr < 16; ++rr) row += __shfl_sync(kAll, vr, rr) <= pos;
                return (x >= nbc && c >= 0) ? row : -1;
            };
            int cq, rq, cn = -1;
            unsigned vq, vn = 0u;
            load_entry(0, cq, vq);
            rq = row_of(0, cq);
            const int nsc = (nch + 1) >> 1;
            for (int q = 0; q < nsc && !fail; ++q) {
                if (q + 1 < nsc) load_entry(q + 1, cn, vn);   // in flight while this superchunk is issued
                for (int h = 0; h < 2 && !fail; ++h) {
                    const int x = 2 * q + h;
                    if (x >= nch) break;
                    const int sl = (int)(chunkc % kTcStages);
                    const int st = p * kTcStages + sl;
                    const bool ok = mbar_wait<POLL>(bar_empty + 8 * st, ((chunkc / kTcStages) & 1u) ^ 1u);
                    if (!__all_sync(kAll, ok)) { give_up(chunkc); break; }
                    const unsigned As = sbase + L::kAOff + st * L::kA;
                    const unsigned Vs = sbase + L::kVOff + st * L::kV;
                    // gathered rows: lane l copies pieces l + 32 i (entry 2 i + l / 16, piece l % 16)
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int k = 2 * i + (lane >> 4), j = lane & 15;
                        const int c = __shfl_sync(kAll, cq, 16 * h + k);
                        const char *src = B + (int64_t)(c >= 0 ? c : 0) * rowbytes + (f0 + 8 * j) * 2;
                        tc_cp16(As + a_offset(k, j), src, c >= 0 ? 16 : 0);
                    }
                    // values: lane l = entry l / 2, row group l % 2
                    {
                        const int k = lane >> 1, g = lane & 1;
                        if (x < nbc) {
                            const bool okv = 16 * x + k < nb;
                            const char *src = cval + ((cb + 16 * x + (okv ? k : 0)) * 16 + 8 * g) * 2;
                            tc_cp16(Vs + v_offset(k, g), src, okv ? 16 : 0);
                        } else {
                            const int row = __shfl_sync(kAll, rq, 16 * h + k);
                            const unsigned val = __shfl_sync(kAll, vq, 16 * h + k);
                            const int qq = row - 8 * g;
                            const bool here = row >= 0 && (unsigned)qq < 8u;
                            const unsigned word = here ? ((qq & 1) ? (val << 16) : val) : 0u;
                            const int wi = here ? (qq >> 1) : -1;
                            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(Vs + v_offset(k, g)),
                                         "r"(wi == 0 ? word : 0u), "r"(wi == 1 ? word : 0u), "r"(wi == 2 ? word : 0u),
                                         "r"(wi == 3 ? word : 0u)
                                         : "memory");
                            fence_async_smem();   // the st.shared precede the tensor core's reads
                        }
                    }
#pragma unroll
                    for (int i = 0; i < kTcStages; ++i)
                        if (i == sl) {
                            pend_meta[i] = acc | (x == 0 ? 1u << 8 : 0u) | (x == nch - 1 ? 1u << 9 : 0u) | (par << 10);
                            pend_item[i] = it;
                        }
                    mbar_arrive_cpasync(bar_full + 8 * st);
                    mbar_arrive(bar_full + 8 * st);
                    ++chunkc;
                    if (chunkc - mmac > (uint32_t)kTcLag) issue_mma();
                }
                if (q + 1 < nsc) {
                    cq = cn;
                    vq = vn;
                    rq = row_of(q + 1, cn);
                }
            }
        }
        while (mmac < chunkc && !fail) issue_mma();
        asm volatile("cp.async.wait_all;\n" ::: "memory");
        // every MMA this warp issued has completed before TMEM is released (bounded)
        if (lane == 0) tc_commit(bar_done);
        __syncwarp();
    } else {
        // ================= epilogue warps: TMEM -> fp16 rows of C, in queue order =================
        __half *out = static_cast<__half *>(a.out);
        int64_t total = 0;
        for (int q = 0; q < kTcProducers; ++q) {
            const int64_t first = (int64_t)blockIdx.x * kTcProducers + q, stride = (int64_t)gridDim.x * kTcProducers;
            total += first < nitems ? (nitems - first + stride - 1) / stride : 0;
        }
        for (int64_t n = 0; n < total && !fail; ++n) {
            const int slot = (int)(n % kQ);
            bool ok = mbar_wait<POLL>(bar_qfull + 8 * slot, (uint32_t)((n / kQ) & 1));
            if (!__all_sync(kAll, ok)) { give_up(n); break; }
            const unsigned word = (unsigned)s_queue[2 * slot];
            const int64_t it = (int64_t)s_queue[2 * slot + 1];
            const unsigned acc = word & 0xffu, parity = (word >> 8) & 1u;
            ok = mbar_wait<POLL>(bar_accf + 8 * acc, parity);
            if (!__all_sync(kAll, ok)) { give_up(it); break; }
            tc_fence_after();
            float v[16];
            tc_ld16(tmem + ((unsigned)(warp * 32) << 16) + acc * 16, v);
            tc_fence_before();
            mbar_arrive(bar_acce + 8 * acc);
            const int64_t s = it / nslices;
            const int f = (int)(it % nslices) * kTcFW + warp * 32 + lane;
            __half *o = out + 16 * s * a.N + f;
#pragma unroll
            for (int rr = 0; rr < 16; ++rr) __stcs(o + rr * a.N, __float2half_rn(v[rr]));
        }
        if (warp == 0) mbar_wait<POLL>(bar_done, 0);   // every producer's MMAs have completed
    }
    // ---- teardown: every copy landed, every MMA complete (or abandoned), TMEM freed
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTcCols) : "memory");
    }
}

template <typename I, int POLL>
cudaError_t launch_tc(const WindowArgs &a, cudaStream_t stream)
{
    using L = TcShape;
    auto kern = window_tc_kernel<I, POLL>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    const int nslices = (int)(a.N / kTcFW);
    const int64_t items = a.nwin * nslices;
    // one CTA per SM (its TMEM holds every producer's accumulators)
    const int64_t blocks = std::max<int64_t>(
        1, std::min<int64_t>(device_sm_count(), (items + kTcProducers - 1) / kTcProducers));
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
    if (spin) return itype == SPMM_I32 ? launch_tc<int, 1>(a, stream) : launch_tc<int64_t, 1>(a, stream);
    return itype == SPMM_I32 ? launch_tc<int, 0>(a, stream) : launch_tc<int64_t, 0>(a, stream);
}

}  // namespace spmmb
