// Shared device helpers for the B200 SpMM engine (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace spmmb {

// Sticky device status: the first kernel that meets invalid data records a
// code and the offending position; nothing faults or traps.  One instance
// per device lives in status.cu; kernels receive its address.
struct DevStatus {
    int code;
    int pad;
    long long detail;
};

__device__ __forceinline__ void raise_status(DevStatus *st, int code, long long detail)
{
    if (atomicCAS(&st->code, 0, code) == 0) atomicExch((unsigned long long *)&st->detail,
                                                       (unsigned long long)detail);
}

// ---- stores of C --------------------------------------------------------

// 16 bytes of C at p (an address inside `out`): a streaming store, or with a
// multicast address `mc` for `out`, one multimem.st to the same offset
// through it (NVLS: the switch writes every GPU's copy).  The bits are
// stored as they are; the .f32 type only names the operand size.
__device__ __forceinline__ void store_c16(void *out, void *mc, void *p, const uint4 &v)
{
    if (mc) {
        char *q = static_cast<char *>(mc) + (static_cast<char *>(p) - static_cast<char *>(out));
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(q),
                     "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
                     "f"(__uint_as_float(v.w))
                     : "memory");
    } else {
        __stcs(static_cast<uint4 *>(p), v);
    }
}

// 8 bytes of C at p, as store_c16.
__device__ __forceinline__ void store_c8(void *out, void *mc, void *p, const uint2 &v)
{
    if (mc) {
        char *q = static_cast<char *>(mc) + (static_cast<char *>(p) - static_cast<char *>(out));
        asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};\n" ::"l"(q), "f"(__uint_as_float(v.x)),
                     "f"(__uint_as_float(v.y))
                     : "memory");
    } else {
        *static_cast<uint2 *>(p) = v;
    }
}

// After the last multicast store of a thread: orders its stores before any
// later signal at system scope (the caller's cross-GPU barrier).
__device__ __forceinline__ void release_c(const void *mc)
{
    if (mc) __threadfence_system();
}

// ---- element conversions ------------------------------------------------

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }

// Elements per 16-byte vector.
template <typename T> struct Vec { static constexpr int kElems = 16 / sizeof(T); };

// Unpack a 16-byte vector into fp32 lanes.
template <typename T> __device__ __forceinline__ void unpack16(const uint4 &v, float *f);
template <> __device__ __forceinline__ void unpack16<__half>(const uint4 &v, float *f)
{
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}
template <> __device__ __forceinline__ void unpack16<float>(const uint4 &v, float *f)
{
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}

// Same conversion, written as volatile asm so the compiler keeps it at its
// use site: in loops that revisit the same vectors under different
// predicates, hoisting the conversion of every vector would multiply the
// live registers.
template <typename T> __device__ __forceinline__ void unpack16_at_use(const uint4 &v, float *f);
template <> __device__ __forceinline__ void unpack16_at_use<__half>(const uint4 &v, float *f)
{
    const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
        asm volatile("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
                     "cvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
                     : "=f"(f[2 * i]), "=f"(f[2 * i + 1])
                     : "r"(w[i]));
}
template <> __device__ __forceinline__ void unpack16_at_use<float>(const uint4 &v, float *f) { unpack16<float>(v, f); }

// acc[e] += v * b[e] over one 16-byte vector of B, fp32 accumulation.
// fp16: fma.rn.f32.f16 takes the fp16 operands directly; both are exact in
// fp32 and so is their product, so each step rounds once, bit-identical to
// fmaf((float)v, (float)b[e], acc[e]) without separate conversions.
// fp32: two packed fma.rn.f32x2 (each lane an IEEE fp32 fma).
template <typename T> struct FmaVec;
template <> struct FmaVec<__half> {
    using Scalar = unsigned short;   // fp16 bits of the nonzero's value
    static __device__ __forceinline__ void run(float *acc, Scalar v, const uint4 &b)
    {
        const unsigned w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            asm("{\n\t.reg .f16 s, l, u;\n\tmov.b16 s, %2;\n\tmov.b32 {l, u}, %3;\n\t"
                "fma.rn.f32.f16 %0, s, l, %0;\n\tfma.rn.f32.f16 %1, s, u, %1;\n\t}"
                : "+f"(acc[2 * i]), "+f"(acc[2 * i + 1])
                : "h"(v), "r"(w[i]));
    }
    static __device__ __forceinline__ Scalar load(const __half *p)
    {
        return __ldcs(reinterpret_cast<const unsigned short *>(p));
    }
    static __device__ __forceinline__ Scalar zero() { return 0; }
};
template <> struct FmaVec<float> {
    using Scalar = float;
    static __device__ __forceinline__ void run(float *acc, Scalar v, const uint4 &b)
    {
        asm("{\n\t.reg .b64 a, x, vv;\n\tmov.b64 vv, {%4, %4};\n\t"
            "mov.b64 a, {%0, %1};\n\tmov.b64 x, {%5, %6};\n\tfma.rn.f32x2 a, vv, x, a;\n\tmov.b64 {%0, %1}, a;\n\t"
            "mov.b64 a, {%2, %3};\n\tmov.b64 x, {%7, %8};\n\tfma.rn.f32x2 a, vv, x, a;\n\tmov.b64 {%2, %3}, a;\n\t}"
            : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3])
            : "f"(v), "f"(__uint_as_float(b.x)), "f"(__uint_as_float(b.y)), "f"(__uint_as_float(b.z)),
              "f"(__uint_as_float(b.w)));
    }
    static __device__ __forceinline__ Scalar load(const float *p) { return __ldcs(p); }
    static __device__ __forceinline__ Scalar zero() { return 0.f; }
};

// Pack fp32 lanes into a 16-byte vector (round to nearest even for fp16).
template <typename T> __device__ __forceinline__ uint4 pack16(const float *f);
template <> __device__ __forceinline__ uint4 pack16<__half>(const float *f)
{
    uint4 v;
    __half2 *h = reinterpret_cast<__half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return v;
}
template <> __device__ __forceinline__ uint4 pack16<float>(const float *f)
{
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
}

// ---- loads -----------------------------------------------------------------

// Streaming (evict-first) loads for data touched once (A's index/value arrays)
// so that L2 keeps the reused rows of the dense operand.
__device__ __forceinline__ int ld_stream(const int *p) { return __ldcs(p); }
__device__ __forceinline__ long long ld_stream(const long long *p) { return __ldcs(p); }
__device__ __forceinline__ int64_t ld_stream(const int64_t *p)
{
    return (int64_t)__ldcs(reinterpret_cast<const long long *>(p));
}
__device__ __forceinline__ float ld_stream(const float *p) { return __ldcs(p); }
__device__ __forceinline__ __half ld_stream(const __half *p)
{
    const unsigned short u = __ldcs(reinterpret_cast<const unsigned short *>(p));
    return __ushort_as_half(u);
}

__device__ __forceinline__ int64_t ld_idx(const int *p) { return (int64_t)__ldg(p); }
__device__ __forceinline__ int64_t ld_idx(const int64_t *p)
{
    return (int64_t)__ldg(reinterpret_cast<const long long *>(p));
}

// ---- warp-cooperative search -------------------------------------------------

// First i in [L, H) with a[i] >= key (a non-decreasing), or H if none.
// All 32 lanes must call it with the same arguments.  Each round samples 32
// evenly spaced positions, so a range of n entries takes ~log32(n) rounds of
// parallel loads instead of log2(n) dependent ones.
template <typename I>
__device__ __forceinline__ int64_t warp_lower_bound(const I *a, int64_t L, int64_t H, int64_t key)
{
    const int lane = threadIdx.x & 31;
    while (H - L > 32) {
        const int64_t step = (H - L + 31) / 32;
        const int64_t pos = L + (int64_t)lane * step;
        const bool ge = pos < H && ld_idx(a + pos) >= key;
        const unsigned m = __ballot_sync(0xffffffffu, ge);
        if (m == 0) {
            const int64_t kmax = min((int64_t)31, (H - 1 - L) / step);
            L = L + kmax * step + 1;
        } else {
            const int f = __ffs(m) - 1;
            const int64_t pf = L + (int64_t)f * step;
            L = (f == 0) ? L : L + (int64_t)(f - 1) * step + 1;
            H = pf;
        }
    }
    const int64_t pos = L + lane;
    const bool ge = pos < H && ld_idx(a + pos) >= key;
    const unsigned m = __ballot_sync(0xffffffffu, ge);
    return m ? L + (__ffs(m) - 1) : H;
}

}  // namespace spmmb
