// Tensor-core CSR gather (fp16, feature width a multiple of 64).
//
// Same work split as the CUDA-core gather kernels (gather.cu): the nonzeros
// are cut into units of `unit` positions (here twice the CUDA-core unit),
// rows crossing a unit boundary go to fp32 head/tail partials summed by
// csr_fixup_kernel in unit order, empty rows are zeroed by the unit their
// (empty) position range falls in.  What changes is how a unit is
// multiplied:
//
//  * A warp owns (unit, feature slice of FW = 64, 128 or 256 features).  It
//    walks the unit's positions in chunks of 16.  The 16 gathered B rows of a
//    chunk (FW features each) are fetched into a per-warp shared-memory ring
//    by 16-byte cp.async.cg copies (L2 only; rows past the unit end or with
//    an invalid column are zero-filled), STAGES - 1 chunks ahead.  The
//    chunk is then one k16 step of
//        D[feature, row] += sum_k Bg[k, feature] * V[k, row]
//    with mma.sync m16n8k16 (fp16 x fp16 -> fp32): the A operand is the
//    staged rows read with ldmatrix.trans (features as M), the B operand is
//    the chunk's values placed at their row inside an 8-row window (rows as
//    N).  Per nonzero and 16 features this costs one ldmatrix and one mma;
//    the gather costs one instruction per row.
//  * An 8-row window accumulates in registers until the walk leaves it; the
//    window is then flushed: rows completed inside the unit are rounded to
//    fp16 once and written through a small shared-memory transpose
//    (stmatrix.trans) as coalesced 16-byte vectors, the unit's head and tail
//    rows are written as fp32 partials.
//  * Row bookkeeping never searches per nonzero: lane g holds the position
//    range of window row g, a chunk entry belongs to row g iff it falls in
//    that range, and the row ends after the window are prefetched into
//    lanes while the window is multiplied.
//  * No wait in the kernel depends on another warp or CTA: cp.async groups
//    complete on their own.
//
// Numerics: per output element the sum runs over the row's nonzeros in
// 16-position chunks; each chunk's products are exact in fp32 and added by
// the tensor core, chunk after chunk, in fp32; the result is rounded to fp16
// once.  The chunk grid depends only on nnz, so the result is deterministic
// and the pipeline-depth ablation (spmm_csr_aiv_mb_batch) is bitwise
// identical.  It is not bitwise identical to the CUDA-core kernels
// (different summation order); both are within the reference's fp16
// tolerance.  As in any dense-tile product, a non-finite B element also
// reaches the other rows of its 8-row window (0 * inf), unlike the
// CUDA-core kernels.
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

__device__ __forceinline__ void ldsm_x4_trans(unsigned addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void stsm_x4_trans(unsigned addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3)
{
    asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(r0),
                 "r"(r1), "r"(r2), "r"(r3)
                 : "memory");
}
__device__ __forceinline__ void mma16816(float *d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi)
{
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ uint4 lds128(unsigned addr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
template <int FW, int STAGES, int WARPS> struct MmaShape {
    static constexpr int kWarps = WARPS;                      // warps per CTA
    static constexpr int kPitch = FW * 2 + 16;                // bytes per staged row (pad: conflict-free ldmatrix)
    static constexpr int kStage = 16 * kPitch;                // one chunk: 16 gathered rows
    static constexpr int kEpi = 8 * kPitch;                   // 8-row output transpose tile
    // ring + epilogue tile, rounded so that every warp's ring starts
    // 128-byte aligned
    static constexpr int kWarp = (STAGES * kStage + kEpi + 127) / 128 * 128;
    static constexpr int kBlock = kWarps * kWarp;
    static constexpr int kSuper = STAGES / 2 + 3;             // superchunks of columns held in registers
};

__device__ __forceinline__ void cp_async16_zfill(unsigned dst, const void *src, bool valid)
{
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Gathers by 16-byte cp.async.cg (zero-filling invalid rows), completing per
// commit group.
template <typename I, int FW, int STAGES, int WARPS, int MINB>
__global__ void __launch_bounds__(WARPS * 32, MINB)
csr_mma_kernel(const GatherArgs a, int nslices)
{
    using L = MmaShape<FW, STAGES, WARPS>;
    constexpr int PITCH = L::kPitch;
    constexpr int NMT = FW / 16;        // m16 feature tiles per slice
    constexpr int PIECES = FW / 8;      // 16-byte pieces per staged row
    extern __shared__ __align__(128) unsigned char mma_smem[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const unsigned ring = (unsigned)__cvta_generic_to_shared(mma_smem) + (unsigned)(wid * L::kWarp);
    const unsigned epi = ring + STAGES * L::kStage;

    const I *rowptr = static_cast<const I *>(a.rowptr);
    const I *col = static_cast<const I *>(a.col);
    const unsigned short *val = static_cast<const unsigned short *>(a.val);
    const char *B = static_cast<const char *>(a.B);
    char *out = static_cast<char *>(a.out);
    const int64_t rowbytes = a.N * 2;
    uint32_t gbase = 0;   // chunks this warp has issued and consumed, over all its items

    const int64_t nitems = (a.unit_end - a.unit_begin) * nslices;
    for (int64_t it = (int64_t)blockIdx.x * WARPS + wid; it < nitems; it += (int64_t)gridDim.x * WARPS) {
        const int64_t u = a.unit_begin + it / nslices;
        const int f0 = (int)(it % nslices) * FW;
        const int64_t lo = u * a.unit;
        const int64_t hi = min(lo + a.unit, a.nnz);
        const bool last = u == a.unit_end - 1;

        // ---- rows whose (possibly empty) range starts in [lo, hi): zero the
        // empty ones (unit_rows[k] = first row at or after row_begin whose
        // range starts at or after position (unit_begin + k) * unit)
        const int64_t ra = a.unit_rows[u - a.unit_begin];
        const int64_t rb = last ? a.M : min(a.M, a.unit_rows[u - a.unit_begin + 1]);
        for (int64_t r = ra + lane; r < rb; r += 32) {
            const int64_t b0 = ld_idx(rowptr + r), b1 = ld_idx(rowptr + r + 1);
            if (b1 < b0 || b0 < 0 || b1 > a.nnz) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, r);
            if (b1 == b0) {
                uint4 *o = reinterpret_cast<uint4 *>(out + r * rowbytes + f0 * 2);
#pragma unroll
                for (int v = 0; v < PIECES; ++v) store_c16(a.out, a.out_mc, o + v, make_uint4(0, 0, 0, 0));
            }
        }

        const int64_t s0 = max(lo, ld_idx(rowptr + a.row_begin));
        if (s0 >= hi) continue;
        const int span = (int)(hi - s0);   // positions of the walk, relative to s0
        const int nchunks = (span + 15) >> 4;

        // ---- window state: lane g describes row wbase + g
        int64_t r0 = ra;
        if (ra > a.row_begin && (ra > a.M || ld_idx(rowptr + ra) > lo)) r0 = ra - 1;
        int64_t wbase = r0 & ~int64_t(7);
        int eb = 0, ee = 0;          // row's positions inside the walk, relative to s0
        bool hd = false, tl = false; // row started before the unit / continues after it
        int64_t wend = 0;            // rowptr[wbase + 8]: first position after the window
        int64_t rpn = 0;             // rowptr[wbase + 9 + lane]: row ends after the window
        auto set_row = [&](int64_t b, int64_t e, int64_t r) {
            if (r < a.row_begin || r >= a.M) {
                b = e = s0;
            } else if (e < b || b < 0 || e > a.nnz) {
                if (t == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, r);
                b = e = s0;
            }
            eb = (int)(min(max(b, s0), hi) - s0);
            ee = (int)(min(max(e, s0), hi) - s0);
            hd = b < lo;
            tl = e > hi;
        };
        auto load_window = [&](int64_t wb) {
            const int64_t r = wb + g;
            set_row(ld_idx(rowptr + min(r, a.M)), ld_idx(rowptr + min(r + 1, a.M)), r);
            wend = ld_idx(rowptr + min(wb + 8, a.M));
            rpn = ld_idx(rowptr + min(wb + 9 + lane, a.M));
        };
        load_window(wbase);

        float acc[NMT][4];
#pragma unroll
        for (int m = 0; m < NMT; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;

        // Flush the accumulated window: direct rows as fp16 through the
        // epilogue tile, head / tail rows as fp32 partials.
        auto flush = [&]() {
            const bool touched = eb < ee;
            const bool head = touched && hd;
            const bool tail = touched && !hd && tl;
            const unsigned dmask = __ballot_sync(kFull, t == 0 && touched && !head && !tail);
            const unsigned pmask = __ballot_sync(kFull, t == 0 && (head || tail));
            const unsigned hmask = __ballot_sync(kFull, t == 0 && head);
            if (dmask) {
#pragma unroll
                for (int m = 0; m < NMT; m += 2) {
                    const int tile = lane >> 3;
                    const unsigned addr =
                        epi + (unsigned)((lane & 7) * PITCH + (16 * (m + (tile >> 1)) + 8 * (tile & 1)) * 2);
                    stsm_x4_trans(addr, pack_h2(acc[m][0], acc[m][1]), pack_h2(acc[m][2], acc[m][3]),
                                  pack_h2(acc[m + 1][0], acc[m + 1][1]), pack_h2(acc[m + 1][2], acc[m + 1][3]));
                }
                __syncwarp();
#pragma unroll
                for (int i = 0; i < PIECES / 4; ++i) {
                    const int idx = lane + 32 * i;
                    const int n = idx / PIECES, v = idx % PIECES;
                    if ((dmask >> (4 * n)) & 1u) {
                        uint4 *o = reinterpret_cast<uint4 *>(out + (wbase + n) * rowbytes + f0 * 2) + v;
                        store_c16(a.out, a.out_mc, o, lds128(epi + (unsigned)(n * PITCH + v * 16)));
                    }
                }
                __syncwarp();
            }
            if (pmask) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int n = 2 * t + h;
                    if ((pmask >> (4 * n)) & 1u) {
                        const int slot = ((hmask >> (4 * n)) & 1u) ? 0 : 1;
                        float *prow = a.partial + ((u - a.unit_begin) * 2 + slot) * a.N + f0;
#pragma unroll
                        for (int m = 0; m < NMT; ++m) {
                            prow[16 * m + g] = acc[m][h];
                            prow[16 * m + g + 8] = acc[m][2 + h];
                        }
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < NMT; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
        };

        // Move to the window holding position pos (> every position of the
        // current window); the row ends prefetched in rpn cover 32 rows.
        // Returns false (status raised) if the row pointer does not move the
        // walk forward, i.e. it is not a valid CSR row pointer.
        auto advance = [&](int64_t pos) -> bool {
            const unsigned m = __ballot_sync(kFull, rpn > pos);
            int64_t row;
            if (m) row = wbase + 8 + (__ffs(m) - 1);
            else row = warp_lower_bound(rowptr, min(wbase + 41, a.M + 1), a.M + 1, pos + 1) - 1;
            const int64_t wb = row & ~int64_t(7);
            if (row >= a.M || wb <= wbase) {
                if (lane == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, row);
                return false;
            }
            const int64_t j0 = wb - (wbase + 9);   // lane of rowptr[wb + 1] in rpn
            if (j0 >= -1 && j0 + 8 <= 31) {
                const int lb = (int)j0 + g;
                const int64_t xb = __shfl_sync(kFull, rpn, max(lb, 0));
                const int64_t xe = __shfl_sync(kFull, rpn, lb + 1);
                const int64_t w8 = __shfl_sync(kFull, rpn, (int)j0 + 8);
                set_row(lb < 0 ? wend : xb, xe, wb + g);
                wend = w8;
                wbase = wb;
                rpn = ld_idx(rowptr + min(wb + 9 + lane, a.M));
            } else {
                wbase = wb;
                load_window(wb);
            }
            return true;
        };

        // ---- superchunk j = positions [s0 + 32 j, +32): lane l holds its
        // column (-1 past the walk or if invalid) and value bits.  NSC
        // superchunks j .. j + NSC - 1 are held while chunks of superchunk j
        // are multiplied; the next is requested on entering a new superchunk,
        // so a column arrives several chunks before its gather is issued.
        constexpr int NSC = L::kSuper;
        auto load_sc = [&](int j, int &cc, unsigned &vv) {
            const int q = 32 * j + lane;
            cc = -1;
            vv = 0u;
            if (q < span) {
                const int64_t c = (int64_t)ld_stream(col + s0 + q);
                vv = (unsigned)__ldcs(val + s0 + q);
                if (c >= 0 && c < a.K) cc = (int)c;
                else raise_status(a.status, SPMM_DEV_BAD_COLUMN, s0 + q);
            }
        };
        int colq[NSC];
        unsigned valq[NSC];
#pragma unroll
        for (int i = 0; i < NSC; ++i) load_sc(i, colq[i], valq[i]);
        static_assert((STAGES - 1 + 1) / 2 + 1 <= NSC, "column prefetch covers the issue distance");
        auto col_of = [&](int x, int c) -> int {
            const int d = (x >> 1) - (c >> 1);
            int r = colq[0];
#pragma unroll
            for (int i = 1; i < NSC; ++i)
                if (d == i) r = colq[i];
            return r;
        };
        const char *Bs = B + f0 * 2;
        // Gathers of chunk c: lane l copies 16-byte pieces l % PIECES of rows
        // l / PIECES + 32 i / PIECES; one commit group per chunk (empty past
        // the walk, so the group count stays uniform).
        auto issue = [&](int c, int cc) {
            if (c < nchunks) {
                const uint32_t gc = gbase + (uint32_t)c;
                const unsigned st = ring + (gc % STAGES) * L::kStage;
                const int half = 16 * (c & 1);
                constexpr int RPI = 32 / PIECES;   // rows per instruction
                const int v = lane % PIECES;
#pragma unroll
                for (int i = 0; i < 16 / RPI; ++i) {
                    const int k = lane / PIECES + RPI * i;
                    const int ck = __shfl_sync(kFull, cc, half + k);
                    const char *src = Bs + (int64_t)(ck >= 0 ? ck : 0) * rowbytes + v * 16;
                    cp_async16_zfill(st + (unsigned)(k * PITCH + v * 16), src, ck >= 0);
                }
            }
            cp_commit();
        };

#pragma unroll
        for (int c = 0; c < STAGES - 1; ++c) issue(c, col_of(c, 0));

        bool ok = true;
        int c = 0;
        for (; c < nchunks && ok; ++c) {
            const uint32_t gc = gbase + (uint32_t)c;
            cp_wait<STAGES - 2>();   // this lane's copies of chunk c have landed
            __syncwarp();            // ... and every other lane's
            issue(c + STAGES - 1, col_of(c + STAGES - 1, c));
            const unsigned vc = valq[0];
            const int vh = 16 * (c & 1);
            if (c & 1) {   // leaving superchunk c >> 1
#pragma unroll
                for (int i = 0; i + 1 < NSC; ++i) {
                    colq[i] = colq[i + 1];
                    valq[i] = valq[i + 1];
                }
                load_sc((c >> 1) + NSC, colq[NSC - 1], valq[NSC - 1]);
            }

            const unsigned st = ring + (gc % STAGES) * L::kStage;
            const unsigned v0 = __shfl_sync(kFull, vc, vh + 2 * t);
            const unsigned v1 = __shfl_sync(kFull, vc, vh + 2 * t + 1);
            const unsigned v2 = __shfl_sync(kFull, vc, vh + 2 * t + 8);
            const unsigned v3 = __shfl_sync(kFull, vc, vh + 2 * t + 9);
            const int q = 16 * c + 2 * t;   // this lane's B-operand positions q, q+1, q+8, q+9
            const int64_t cend = s0 + min(16 * c + 16, span);
            for (;;) {
                const unsigned w = (unsigned)(ee - eb);
                const unsigned h0 = ((unsigned)(q - eb) < w) ? v0 : 0u;
                const unsigned h1 = ((unsigned)(q + 1 - eb) < w) ? v1 : 0u;
                const unsigned h2 = ((unsigned)(q + 8 - eb) < w) ? v2 : 0u;
                const unsigned h3 = ((unsigned)(q + 9 - eb) < w) ? v3 : 0u;
                const uint32_t b0 = h0 | (h1 << 16), b1 = h2 | (h3 << 16);
#pragma unroll
                for (int m = 0; m < NMT; ++m) {
                    const int tile = lane >> 3;
                    const unsigned addr =
                        st + (unsigned)(((tile >> 1) * 8 + (lane & 7)) * PITCH + (16 * m + 8 * (tile & 1)) * 2);
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_trans(addr, a0, a1, a2, a3);
                    mma16816(acc[m], a0, a1, a2, a3, b0, b1);
                }
                if (cend <= wend) break;
                flush();
                if (!(ok = advance(max(wend, s0 + 16 * c)))) break;
            }
        }
        if (ok) flush();
        // Chunks issued but not consumed (only after a bad row pointer) land
        // before the warp moves on.
        const int issued = min(nchunks, c + STAGES - 1);
        cp_wait<0>();
        gbase += (uint32_t)issued;
        __syncwarp();
        if (!ok) break;
    }
    release_c(a.out_mc);   // multicast rows ordered before the caller's barrier
}

// unit_rows[k] = first row r in [row_begin, M] with rowptr[r] >= (unit_begin
// + k) * unit (M + 1 if none), for k = 0 .. nunits; one warp per entry.
template <typename I>
__global__ void __launch_bounds__(256) unit_rows_kernel(const GatherArgs a)
{
    const I *rowptr = static_cast<const I *>(a.rowptr);
    const int64_t n = a.unit_end - a.unit_begin + 1;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t k = warp; k < n; k += nwarps) {
        const int64_t r = warp_lower_bound(rowptr, a.row_begin, a.M + 1, (a.unit_begin + k) * a.unit);
        if ((threadIdx.x & 31) == 0) a.unit_rows[k] = r;
    }
}

template <typename I, int FW, int STAGES, int WARPS>
cudaError_t launch_fw(const GatherArgs &a, cudaStream_t stream)
{
    using L = MmaShape<FW, STAGES, WARPS>;
    constexpr int MINB = std::max(1, (220 * 1024) / L::kBlock);
    auto kern = csr_mma_kernel<I, FW, STAGES, WARPS, MINB>;
    constexpr int smem = L::kBlock;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, L::kWarps * 32, smem);
    if (e != cudaSuccess) return e;
    const int nslices = (int)(a.N / FW);
    const int64_t items = (a.unit_end - a.unit_begin) * nslices;
    int64_t blocks = (int64_t)std::max(per_sm, 1) * device_sm_count();
    blocks = std::max<int64_t>(1, std::min(blocks, (items + L::kWarps - 1) / L::kWarps));
    kern<<<(unsigned)blocks, L::kWarps * 32, smem, stream>>>(a, nslices);
    return cudaGetLastError();
}

// Variant for measurement: SPMM_B200_MMA = c<width>s<stages>, e.g. "c128s6"
// (128-feature slices, 6 stages, one warp per CTA).
int mma_variant()
{
    static const int v = [] {
        const char *e = getenv("SPMM_B200_MMA");
        if (!e) return 0;
        static const char *names[] = {"", "c128s6", "c128s8", "c64s8", "c256s4", "c256s6", "c128s3"};
        for (int i = 1; i < (int)(sizeof(names) / sizeof(names[0])); ++i)
            if (strcmp(e, names[i]) == 0) return i;
        return 0;
    }();
    return v;
}

template <typename I>
cudaError_t launch_width(const GatherArgs &a, bool deep, cudaStream_t stream)
{
    switch (mma_variant()) {
    case 1: if (a.N % 128 == 0) return launch_fw<I, 128, 6, 1>(a, stream); break;
    case 2: if (a.N % 128 == 0) return launch_fw<I, 128, 8, 1>(a, stream); break;
    case 3: return launch_fw<I, 64, 8, 1>(a, stream);
    case 4: if (a.N % 256 == 0) return launch_fw<I, 256, 4, 1>(a, stream); break;
    case 5: if (a.N % 256 == 0) return launch_fw<I, 256, 6, 1>(a, stream); break;
    case 6: if (a.N % 128 == 0) return launch_fw<I, 128, 3, 4>(a, stream); break;
    default: break;
    }
    if (a.N % 128 == 0) return deep ? launch_fw<I, 128, 4, 4>(a, stream) : launch_fw<I, 128, 3, 4>(a, stream);
    return deep ? launch_fw<I, 64, 4, 4>(a, stream) : launch_fw<I, 64, 3, 4>(a, stream);
}

}  // namespace

bool gather_mma_eligible(const GatherArgs &a, int dtype)
{
    // Column indices travel as 32-bit integers inside the kernel.  Chosen
    // for one 64- or 128-feature slice per row (measured faster than the
    // CUDA-core ring kernel there); wider rows keep the ring kernel unless
    // SPMM_B200_MMA names a variant.
    const bool shape = dtype == SPMM_F16 && a.K > 0 && a.K <= INT_MAX && a.N % 64 == 0 && a.unit_rows != nullptr;
    return shape && (a.N <= 128 || mma_variant() != 0);
}

cudaError_t launch_gather_mma(GatherArgs &a, int itype, int batch_depth, cudaStream_t stream)
{
    // Units twice as coarse as the CUDA-core kernels' (fewer per-unit row
    // lookups and partial rows; the scratch of the original plan covers
    // them).  Like the original split, this depends on nnz only.
    if (a.unit_begin == 0) {
        a.unit *= 2;
        a.unit_end = units_for(a.nnz, a.unit);
    }
    {
        const int64_t n = a.unit_end - a.unit_begin + 1;
        const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, 16LL * device_sm_count()));
        if (itype == SPMM_I32) unit_rows_kernel<int><<<(unsigned)blocks, 256, 0, stream>>>(a);
        else unit_rows_kernel<int64_t><<<(unsigned)blocks, 256, 0, stream>>>(a);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const bool deep = batch_depth != 0;
    return itype == SPMM_I32 ? launch_width<int>(a, deep, stream) : launch_width<int64_t>(a, deep, stream);
}

}  // namespace spmmb
