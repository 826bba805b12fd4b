// Window path: 16-row windows stored as (16 x 1)-block BCSR.
//
// Semantics follow the reference's matrix-core part
// (kernels/op_kernel/spmm_ascend_cube.cpp:52-165, 265-288): window slot s
// computes rows [16s, 16s + 16) as  sum_b Cvalue[16b + i] * B[Ccol[b], :].
// In the mixed operator the reference's vector cores atomically add the CSR
// rows of the same output range on top (spmm_ascend_cube.cpp:785); here the
// CSR entries of a window's rows are appended to the window's block stream
// as one-nonzero blocks, so each output row is produced by one CTA, summed
// in fp32 and rounded once - no atomics, deterministic.
//
// Block stream of window s:  [Crowptr[s], Crowptr[s+1]) blocks, then the CSR
// entries of rows [16s, min(16s + 16, vrows)).  It is consumed in chunks of
// 16 entries (one MMA K step).  For every chunk the CTA gathers the 16 B rows
// (16-byte cp.async, L2-only) and the 16 x 16 value tile into a shared-memory
// ring of STAGES buffers, so the gathers of the next chunks are in flight
// while the current one is multiplied.
//  * fp16: mma.sync m16n8k16 (fp16 x fp16 -> fp32).  A 16-row window is
//    below the M >= 64 of tcgen05 UMMA, and the path is bound by the B-row
//    gather, not by tensor throughput (16 MACs per gathered element).
//  * fp32: shared-memory FFMA (TF32 would miss the 1e-4 tolerance).
// STAGES = 1 is the unpipelined variant (the reference's SPTILE = 16
// ablation, op_kernel/spmm_ascend_cube_aic_without_pipeline.cpp:6).
#include <algorithm>
#include <cstring>
#include <cstdlib>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

constexpr int kChunk = 16;

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Per-window stream bounds, validated against the array extents.
struct WinStream {
    int64_t cb, nb;   // first block, block count
    int64_t vb, nv;   // first CSR entry, entry count
};

template <typename I>
__device__ __forceinline__ WinStream window_stream(const WindowArgs &a, int64_t s, int64_t *s_vptr)
{
    const I *cptr = static_cast<const I *>(a.cptr);
    const I *vptr = static_cast<const I *>(a.vptr);
    WinStream w;
    int64_t cb = ld_idx(cptr + s), ce = ld_idx(cptr + s + 1);
    if (cb < 0 || ce < cb || ce > a.nblocks) {
        if (threadIdx.x == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, s);
        cb = ce = 0;
    }
    w.cb = cb;
    w.nb = ce - cb;
    // CSR rows of this window that the window path fuses.
    const int64_t r0 = 16 * s;
    if (threadIdx.x <= 16) {
        const int64_t r = min(r0 + (int64_t)threadIdx.x, a.vrows);
        s_vptr[threadIdx.x] = (a.vrows > 0 && r0 < a.vrows) ? ld_idx(vptr + r) : 0;
    }
    __syncthreads();
    int64_t vb = s_vptr[0], ve = s_vptr[16];
    bool bad = vb < 0 || ve < vb || ve > a.vnnz;
    for (int i = 0; i < 16 && !bad; ++i) bad = s_vptr[i + 1] < s_vptr[i];
    if (bad) {
        if (threadIdx.x == 0) raise_status(a.status, SPMM_DEV_BAD_ROWPTR, r0);
        vb = ve = 0;
    }
    w.vb = vb;
    w.nv = ve - vb;
    __syncthreads();
    if (bad && threadIdx.x <= 16) s_vptr[threadIdx.x] = 0;
    __syncthreads();
    return w;
}

// Column of stream entry kk (-1 past the end or if invalid).
template <typename I>
__device__ __forceinline__ int64_t stream_col(const WindowArgs &a, const WinStream &w, int64_t kk)
{
    int64_t c = -1;
    if (kk < w.nb) c = ld_idx(static_cast<const I *>(a.ccol) + w.cb + kk);
    else if (kk < w.nb + w.nv) c = ld_idx(static_cast<const I *>(a.vcol) + w.vb + (kk - w.nb));
    else return -1;
    if (c < 0 || c >= a.K) {
        raise_status(a.status, SPMM_DEV_BAD_COLUMN, kk);
        return -1;
    }
    return c;
}

// Row (0..15) of CSR entry e of the window.
__device__ __forceinline__ int entry_row(const int64_t *s_vptr, int64_t e)
{
    int i = 0;
#pragma unroll
    for (int j = 1; j < 16; ++j) i += (s_vptr[j] <= e) ? 1 : 0;
    return i;
}

// Stage chunk c of window w: 16 gathered B rows (row pitch `bpitch` elements)
// and the 16 x 16 value tile A_s[k][row] (row pitch `apitch` elements).
template <typename T, typename I>
__device__ __forceinline__ void load_chunk(const WindowArgs &a, const WinStream &w, const int64_t *s_vptr,
                                           int64_t c, T *As, int apitch, T *Bs, int bpitch)
{
    constexpr int EPV = Vec<T>::kElems;
    const int nthreads = blockDim.x;
    const int NV = (int)(a.N / EPV);
    const uint4 *B = static_cast<const uint4 *>(a.B);
    for (int idx = threadIdx.x; idx < kChunk * NV; idx += nthreads) {
        const int k = idx / NV, v = idx % NV;
        const int64_t col = stream_col<I>(a, w, c * kChunk + k);
        T *dst = Bs + k * bpitch + v * EPV;
        if (col >= 0) cp_async16(dst, B + col * NV + v);
        else *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
    }
    constexpr int APV = 16 / EPV;  // 16-byte vectors per 16-value block column
    for (int idx = threadIdx.x; idx < kChunk * APV; idx += nthreads) {
        const int k = idx / APV, h = idx % APV;
        const int64_t kk = c * kChunk + k;
        T *dst = As + k * apitch + h * EPV;
        if (kk < w.nb) {
            cp_async16(dst, static_cast<const T *>(a.cval) + 16 * (w.cb + kk) + h * EPV);
        } else {
            float f[EPV];
#pragma unroll
            for (int e = 0; e < EPV; ++e) f[e] = 0.f;
            if (kk < w.nb + w.nv) {
                const int64_t e = w.vb + (kk - w.nb);
                const int row = entry_row(s_vptr, e);
                if (row >= h * EPV && row < (h + 1) * EPV)
                    f[row - h * EPV] = to_f32(static_cast<const T *>(a.vval)[e]);
            }
            *reinterpret_cast<uint4 *>(dst) = pack16<T>(f);
        }
    }
}

// ---------------------------------------------------------------------------
// fp16: tensor-core MMA.  Warp w owns n8 tiles [w * tpw, (w + 1) * tpw).
// ---------------------------------------------------------------------------
constexpr int kApitchH = 24;   // 48-byte rows: conflict-free ldmatrix.trans

template <typename I, int STAGES>
__global__ void __launch_bounds__(512)
window_mma_f16_kernel(const WindowArgs a, int tpw)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int bpitch = (int)a.N + 8;                       // +16 bytes: no bank conflicts
    int64_t *s_vptr = reinterpret_cast<int64_t *>(smem);   // 17 entries
    __half *As = reinterpret_cast<__half *>(smem + 256);
    __half *Bs = As + STAGES * kChunk * kApitchH;
    const int stageB = kChunk * bpitch;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int NT = (int)(a.N / 8);
    const int tile0 = warp * tpw;
    const int ntile = max(0, min(tpw, NT - tile0));

    for (int64_t s = blockIdx.x; s < a.nwin; s += gridDim.x) {
        const WinStream w = window_stream<I>(a, s, s_vptr);
        const int64_t L = w.nb + w.nv;
        const int64_t nchunks = (L + kChunk - 1) / kChunk;

        float acc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;

        auto compute = [&](int st) {
            const __half *A = As + st * kChunk * kApitchH;
            const __half *Bt = Bs + st * stageB;
            uint32_t af[4];
            {
                const int m = lane >> 3, i = lane & 7;
                const __half *p = A + ((m >> 1) * 8 + i) * kApitchH + (m & 1) * 8;
                const unsigned addr = (unsigned)__cvta_generic_to_shared(p);
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                             : "=r"(af[0]), "=r"(af[1]), "=r"(af[2]), "=r"(af[3]) : "r"(addr));
            }
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                if (j >= ntile) break;
                const int m = lane >> 3, i = lane & 7;
                const int tj = min(j + (m >> 1), ntile - 1);
                const __half *p = Bt + ((m & 1) * 8 + i) * bpitch + (tile0 + tj) * 8;
                const unsigned addr = (unsigned)__cvta_generic_to_shared(p);
                uint32_t bf[4];
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                             : "=r"(bf[0]), "=r"(bf[1]), "=r"(bf[2]), "=r"(bf[3]) : "r"(addr));
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (j + h < ntile) {
                        float *d = acc[j + h];
                        asm volatile(
                            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
                            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                            : "r"(af[0]), "r"(af[1]), "r"(af[2]), "r"(af[3]),
                              "r"(bf[2 * h]), "r"(bf[2 * h + 1]));
                    }
                }
            }
        };

        if constexpr (STAGES == 1) {
            for (int64_t c = 0; c < nchunks; ++c) {
                load_chunk<__half, I>(a, w, s_vptr, c, As, kApitchH, Bs, bpitch);
                cp_async_commit();
                cp_async_wait<0>();
                __syncthreads();
                compute(0);
                __syncthreads();
            }
        } else {
#pragma unroll
            for (int c = 0; c < STAGES - 1; ++c) {
                if (c < nchunks)
                    load_chunk<__half, I>(a, w, s_vptr, c, As + c * kChunk * kApitchH, kApitchH,
                                          Bs + c * stageB, bpitch);
                cp_async_commit();
            }
            for (int64_t c = 0; c < nchunks; ++c) {
                cp_async_wait<STAGES - 2>();
                __syncthreads();
                const int64_t cn = c + STAGES - 1;
                if (cn < nchunks) {
                    const int sn = (int)(cn % STAGES);
                    load_chunk<__half, I>(a, w, s_vptr, cn, As + sn * kChunk * kApitchH, kApitchH,
                                          Bs + sn * stageB, bpitch);
                }
                cp_async_commit();
                compute((int)(c % STAGES));
            }
            cp_async_wait<0>();
            __syncthreads();
        }

        // Epilogue: fp32 accumulators -> fp16, rows 16s + g and 16s + g + 8.
        __half *out = static_cast<__half *>(a.out);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j >= ntile) break;
            const int64_t col0 = (int64_t)(tile0 + j) * 8 + 2 * t;
            *reinterpret_cast<__half2 *>(out + (16 * s + g) * a.N + col0) = __floats2half2_rn(acc[j][0], acc[j][1]);
            *reinterpret_cast<__half2 *>(out + (16 * s + g + 8) * a.N + col0) = __floats2half2_rn(acc[j][2], acc[j][3]);
        }
    }
}

// ---------------------------------------------------------------------------
// fp32: shared-memory FFMA.  Thread t owns columns [4t, 4t + 4) of all 16 rows.
// ---------------------------------------------------------------------------
template <typename I, int STAGES>
__global__ void __launch_bounds__(128)
window_ffma_f32_kernel(const WindowArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    int64_t *s_vptr = reinterpret_cast<int64_t *>(smem);
    float *As = reinterpret_cast<float *>(smem + 256);
    float *Bs = As + STAGES * kChunk * 16;
    const int bpitch = (int)a.N;
    const int stageB = kChunk * bpitch;
    const int tcol = threadIdx.x * 4;
    const bool active = tcol < a.N;

    for (int64_t s = blockIdx.x; s < a.nwin; s += gridDim.x) {
        const WinStream w = window_stream<I>(a, s, s_vptr);
        const int64_t L = w.nb + w.nv;
        const int64_t nchunks = (L + kChunk - 1) / kChunk;
        float acc[16][4];
#pragma unroll
        for (int i = 0; i < 16; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;

        auto compute = [&](int st) {
            if (!active) return;
            const float *A = As + st * kChunk * 16;
            const float *Bt = Bs + st * stageB;
#pragma unroll 4
            for (int k = 0; k < kChunk; ++k) {
                const float4 b = *reinterpret_cast<const float4 *>(Bt + k * bpitch + tcol);
                float av[16];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 x = *reinterpret_cast<const float4 *>(A + k * 16 + 4 * q);
                    av[4 * q] = x.x; av[4 * q + 1] = x.y; av[4 * q + 2] = x.z; av[4 * q + 3] = x.w;
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    acc[i][0] = fmaf(av[i], b.x, acc[i][0]);
                    acc[i][1] = fmaf(av[i], b.y, acc[i][1]);
                    acc[i][2] = fmaf(av[i], b.z, acc[i][2]);
                    acc[i][3] = fmaf(av[i], b.w, acc[i][3]);
                }
            }
        };

        if constexpr (STAGES == 1) {
            for (int64_t c = 0; c < nchunks; ++c) {
                load_chunk<float, I>(a, w, s_vptr, c, As, 16, Bs, bpitch);
                cp_async_commit();
                cp_async_wait<0>();
                __syncthreads();
                compute(0);
                __syncthreads();
            }
        } else {
#pragma unroll
            for (int c = 0; c < STAGES - 1; ++c) {
                if (c < nchunks)
                    load_chunk<float, I>(a, w, s_vptr, c, As + c * kChunk * 16, 16, Bs + c * stageB, bpitch);
                cp_async_commit();
            }
            for (int64_t c = 0; c < nchunks; ++c) {
                cp_async_wait<STAGES - 2>();
                __syncthreads();
                const int64_t cn = c + STAGES - 1;
                if (cn < nchunks) {
                    const int sn = (int)(cn % STAGES);
                    load_chunk<float, I>(a, w, s_vptr, cn, As + sn * kChunk * 16, 16, Bs + sn * stageB, bpitch);
                }
                cp_async_commit();
                compute((int)(c % STAGES));
            }
            cp_async_wait<0>();
            __syncthreads();
        }

        if (active) {
            float *out = static_cast<float *>(a.out);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                __stcs(reinterpret_cast<float4 *>(out + (16 * s + i) * a.N + tcol),
                       make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]));
        }
    }
}

template <typename I, int STAGES>
cudaError_t launch_f16(const WindowArgs &a, cudaStream_t stream)
{
    const int NT = (int)(a.N / 8);
    const int nw = (NT + 7) / 8;
    const int tpw = (NT + nw - 1) / nw;
    const size_t smem = 256 + (size_t)STAGES * kChunk * (kApitchH + (a.N + 8)) * sizeof(__half);
    auto kern = window_mma_f16_kernel<I, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, nw * 32, smem);
    if (e != cudaSuccess) return e;
    const int64_t grid = std::min<int64_t>(a.nwin, (int64_t)std::max(per_sm, 1) * device_sm_count() * 4);
    kern<<<(unsigned)grid, nw * 32, smem, stream>>>(a, tpw);
    return cudaGetLastError();
}

template <typename I, int STAGES>
cudaError_t launch_f32(const WindowArgs &a, cudaStream_t stream)
{
    const int threads = (int)std::max<int64_t>(32, ((a.N / 4 + 31) / 32) * 32);
    const size_t smem = 256 + (size_t)STAGES * kChunk * (16 + a.N) * sizeof(float);
    auto kern = window_ffma_f32_kernel<I, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
    if (e != cudaSuccess) return e;
    const int64_t grid = std::min<int64_t>(a.nwin, (int64_t)std::max(per_sm, 1) * device_sm_count() * 4);
    kern<<<(unsigned)grid, threads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

// Window kernel choice, read at every launch: SPMM_B200_WINDOW = block
// (block-synchronous window.cu kernels), warp (window_warp.cu) or tc
// (tcgen05, window_tc.cu); the default is the warp-pipelined kernel where
// eligible.
int window_kernel_choice()
{
    const char *v = getenv("SPMM_B200_WINDOW");
    if (v && strcmp(v, "block") == 0) return 1;
    if (v && strcmp(v, "tc") == 0) return 2;
    if (getenv("SPMM_B200_WINDOW_BLOCK")) return 1;
    return 0;
}

cudaError_t launch_window(const WindowArgs &a, int itype, int dtype, int pipelined, cudaStream_t stream)
{
    if (a.nwin <= 0) return cudaSuccess;
    if (pipelined && window_kernel_choice() == 2 && window_tc_eligible(a, dtype))
        return launch_window_tc(a, itype, stream);
    if (pipelined && window_kernel_choice() != 1 && window_warp_eligible(a, dtype))
        return launch_window_warp(a, itype, dtype, stream);
    if (dtype == SPMM_F16) {
        if (itype == SPMM_I32) return pipelined ? launch_f16<int, 3>(a, stream) : launch_f16<int, 1>(a, stream);
        return pipelined ? launch_f16<int64_t, 3>(a, stream) : launch_f16<int64_t, 1>(a, stream);
    }
    if (itype == SPMM_I32) return pipelined ? launch_f32<int, 3>(a, stream) : launch_f32<int, 1>(a, stream);
    return pipelined ? launch_f32<int64_t, 3>(a, stream) : launch_f32<int64_t, 1>(a, stream);
}

}  // namespace spmmb
