// L2 residency plan for the B rows of one CSR SpMM (see engine.h).
//
// Why: on a power-law matrix whose dense operand is far larger than L2
// (config 5: B = 34 GB, 126 MB of L2) every nonzero gathers one B row; the
// hub columns take most of the gathers, but L2's replacement also admits
// the long tail of rows that are used once or twice, which evicts hub rows
// between their uses (47 % of the B-row reads hit in L2 without a plan).
// The ring kernel can give each 16-byte copy an L2 eviction priority; this
// file decides which columns are worth keeping.
//
// How, on the caller's stream, all on the device (no host synchronisation):
//  1. zero the counters and the header (one memset);
//  2. l2_sample_kernel: S = min(nnz, 2^22) column indices at evenly spaced
//     positions, counted per bin (column id modulo kL2Bins = 2^24: exact
//     for matrices of up to 16.8M columns), the hub columns in a per-block
//     shared-memory table first;
//  3. l2_hist_kernel: histogram of the bins' counts (capped at 1023);
//  4. l2_select_kernel: the smallest threshold t >= 2 whose bins (count >= t)
//     fit in the budget - half of L2 in B rows of this width;
//  5. l2_bits_kernel: bitmap of the hot bins, and the exact number of
//     samples they hold.
// The ring kernel reads the header: with at least a quarter of the samples
// in hot bins (l2_plan_enabled) it copies hot rows with evict_last and the
// rest with evict_first; otherwise every copy keeps the normal priority.
// A column sampled once is never hot (t >= 2); on a uniform matrix the bins
// that fit the budget hold far less than a quarter of the samples (for
// about two samples per column, Poisson counts put ~14 % of them in the
// bins above the threshold), so the plan stays off.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

constexpr int64_t kL2Samples = int64_t(1) << 22;
constexpr size_t kHdrBytes = (sizeof(L2PlanHeader) + 255) / 256 * 256;
constexpr size_t kCountBytes = (size_t)kL2Bins * sizeof(unsigned);
constexpr size_t kBitBytes = (size_t)kL2Bins / 8;
constexpr int kHistBins = 1024;

// SPMM_B200_L2PLAN = off | on | auto (default), read at every call.
int l2_mode()
{
    const char *v = getenv("SPMM_B200_L2PLAN");
    if (v && strcmp(v, "off") == 0) return 0;
    if (v && strcmp(v, "on") == 0) return 2;
    return 1;
}

// Hub columns take a large share of the samples (config 5: the hottest
// column about 6 %), and increments of one global counter serialise, so each
// block first counts in a small shared-memory table: a bin claims a free
// slot (first come), samples of a bin that holds its slot are counted there,
// everything else goes straight to the global counters; the table is added
// to them at the end.
constexpr int kSlots = 4096;

template <typename I>
__global__ void __launch_bounds__(256) l2_sample_kernel(const I *col, int64_t nnz, int64_t K, int64_t S,
                                                        unsigned *count, L2PlanHeader *hdr)
{
    __shared__ int s_key[kSlots];
    __shared__ unsigned s_cnt[kSlots];
    for (int i = threadIdx.x; i < kSlots; i += blockDim.x) {
        s_key[i] = -1;
        s_cnt[i] = 0;
    }
    __syncthreads();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    constexpr int kIlp = 4;   // independent column loads in flight per thread
    // position of sample i = floor(i * nnz / S), as i * q + floor(i * r / S)
    // with nnz = q * S + r, so no product exceeds 2^22 * nnz / S or 2^44
    const int64_t q = nnz / S, r = nnz % S;
    unsigned long long taken = 0;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < S; i0 += kIlp * stride) {
        int64_t c[kIlp];
#pragma unroll
        for (int u = 0; u < kIlp; ++u) {
            const int64_t i = i0 + u * stride;
            c[u] = i < S ? (int64_t)ld_stream(col + (i * q + i * r / S)) : int64_t(-1);
        }
#pragma unroll
        for (int u = 0; u < kIlp; ++u) {
            if (c[u] < 0 || c[u] >= K) continue;
            const int bin = (int)(c[u] & (kL2Bins - 1));
            const int slot = (int)(((unsigned)bin * 2654435761u) >> 20);   // 12 bits
            int k = s_key[slot];
            if (k < 0) {
                const int old = atomicCAS(&s_key[slot], -1, bin);
                k = old < 0 ? bin : old;
            }
            if (k == bin) atomicAdd(&s_cnt[slot], 1u);
            else atomicAdd(count + bin, 1u);
            ++taken;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kSlots; i += blockDim.x)
        if (s_key[i] >= 0 && s_cnt[i]) atomicAdd(count + s_key[i], s_cnt[i]);
    // warp sum of the samples taken (invalid columns are skipped)
    for (int o = 16; o; o >>= 1) taken += __shfl_down_sync(0xffffffffu, taken, o);
    if ((threadIdx.x & 31) == 0 && taken) atomicAdd(&hdr->samples, taken);
}

__global__ void __launch_bounds__(256) l2_hist_kernel(const unsigned *count, L2PlanHeader *hdr)
{
    __shared__ unsigned h[kHistBins];
    for (int i = threadIdx.x; i < kHistBins; i += blockDim.x) h[i] = 0;
    __syncthreads();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < kL2Bins; b += stride) {
        const unsigned v = count[b];
        if (v) atomicAdd(&h[min(v, (unsigned)kHistBins - 1)], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kHistBins; i += blockDim.x)
        if (h[i]) atomicAdd(&hdr->hist[i], h[i]);
}

// The histogram goes to shared memory; one thread then walks it down from
// the top while the bins at or above the count still fit in the budget.
__global__ void __launch_bounds__(kHistBins) l2_select_kernel(L2PlanHeader *hdr, unsigned budget)
{
    __shared__ unsigned h[kHistBins];
    for (int i = threadIdx.x; i < kHistBins; i += blockDim.x) h[i] = hdr->hist[i];
    __syncthreads();
    if (threadIdx.x != 0) return;
    unsigned long long bins = 0;
    unsigned t = 0;
    for (int v = kHistBins - 1; v >= 2; --v) {
        const unsigned long long more = bins + h[v];
        if (more > budget) break;
        bins = more;
        if (h[v]) t = (unsigned)v;
    }
    hdr->threshold = t;
    hdr->hot_bins = (unsigned)bins;
    hdr->budget = budget;
}

// One bit per bin; lane 0 of each warp writes the word of its 32 bins (the
// grid stride is a multiple of 32 and kL2Bins of the stride's warps, so a
// warp is always wholly inside or outside the range).
__global__ void __launch_bounds__(256) l2_bits_kernel(const unsigned *count, L2PlanHeader *hdr, unsigned *bits)
{
    const unsigned t = hdr->threshold;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    unsigned long long hot = 0;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < kL2Bins; b += stride) {
        const unsigned v = count[b];
        const bool h = t > 0 && v >= t;
        const unsigned w = __ballot_sync(0xffffffffu, h);
        if ((threadIdx.x & 31) == 0) bits[b >> 5] = w;
        if (h) hot += v;
    }
    for (int o = 16; o; o >>= 1) hot += __shfl_down_sync(0xffffffffu, hot, o);
    if ((threadIdx.x & 31) == 0 && hot) atomicAdd(&hdr->hot_samples, hot);
}

size_t device_l2_bytes()
{
    static std::mutex mu;
    static int cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return size_t(126) << 20;
    std::lock_guard<std::mutex> lock(mu);
    if (!cached[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrL2CacheSize, dev) != cudaSuccess || v <= 0) v = 126 << 20;
        cached[dev] = v;
    }
    return (size_t)cached[dev];
}

}  // namespace

size_t GatherPlan::l2_plan_bytes() { return kHdrBytes + kCountBytes + kBitBytes; }

bool l2_plan_wanted(int64_t nnz, int64_t N, int dtype)
{
    const int64_t rowbytes = N * (dtype == SPMM_F16 ? 2 : 4);
    const int mode = l2_mode();
    if (mode == 0 || rowbytes < 1024 || nnz <= 0) return false;
    return mode == 2 || nnz >= (int64_t(1) << 26);
}

cudaError_t launch_l2_plan(GatherArgs &a, int itype, int dtype, void *region, cudaStream_t stream)
{
    a.l2_bits = nullptr;
    a.l2_hdr = nullptr;
    const int mode = l2_mode();
    const int64_t rowbytes = a.N * (dtype == SPMM_F16 ? 2 : 4);
    if (!region || mode == 0 || a.nnz <= 0 || a.K <= 0 || a.K > INT32_MAX || rowbytes < 1024) return cudaSuccess;
    const size_t l2 = device_l2_bytes();
    if (mode == 1 && (double)a.K * (double)rowbytes < 16.0 * (double)l2) return cudaSuccess;
    auto *hdr = static_cast<L2PlanHeader *>(region);
    auto *count = reinterpret_cast<unsigned *>(static_cast<char *>(region) + kHdrBytes);
    auto *bits = reinterpret_cast<unsigned *>(static_cast<char *>(region) + kHdrBytes + kCountBytes);
    cudaError_t e = cudaMemsetAsync(region, 0, kHdrBytes + kCountBytes, stream);
    if (e != cudaSuccess) return e;
    const int64_t S = std::min<int64_t>(a.nnz, kL2Samples);
    const unsigned blocks =
        (unsigned)std::max<int64_t>(1, std::min<int64_t>((S + 255) / 256, 4LL * device_sm_count()));
    if (itype == SPMM_I32)
        l2_sample_kernel<int><<<blocks, 256, 0, stream>>>(static_cast<const int *>(a.col), a.nnz, a.K, S, count, hdr);
    else
        l2_sample_kernel<int64_t>
            <<<blocks, 256, 0, stream>>>(static_cast<const int64_t *>(a.col), a.nnz, a.K, S, count, hdr);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const unsigned sweep = (unsigned)(4 * device_sm_count());
    l2_hist_kernel<<<sweep, 256, 0, stream>>>(count, hdr);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t budget = std::max<size_t>(1, (l2 / 2) / (size_t)rowbytes);
    l2_select_kernel<<<1, kHistBins, 0, stream>>>(hdr, (unsigned)std::min<size_t>(budget, 0xffffffffu));
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    l2_bits_kernel<<<sweep, 256, 0, stream>>>(count, hdr, bits);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    a.l2_bits = bits;
    a.l2_hdr = hdr;
    return cudaSuccess;
}

}  // namespace spmmb
