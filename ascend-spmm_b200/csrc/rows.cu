// Row permutation copies for the graph-layout helpers.
//
// pack:    dst[inv[i], :] = src[i, :] for i < n, every other dst row zero
//          (reference spmm_npu.py:22-47, index_copy_ into zero rows)
// restore: dst[i, :] = src[inv[i], :] for i < n
//          (reference spmm_npu.py:50-61, index_select)
// One warp per row; 16-byte vectors when the row pitch and the base
// pointers allow it, 4-byte or 1-byte words otherwise.  Out-of-range
// indices are skipped and raise the sticky device status.
#include <algorithm>

#include "../../include/spmm_b200.h"
#include "common.cuh"
#include "engine.h"

namespace spmmb {

namespace {

template <typename W, bool kScatter>
__global__ void __launch_bounds__(256)
permute_rows_kernel(const W *src, W *dst, const int64_t *inv, int64_t n, int64_t src_rows, int64_t dst_rows,
                    int64_t words, DevStatus *status)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t i = warp; i < n; i += nwarps) {
        const int64_t j = __ldg(reinterpret_cast<const long long *>(inv) + i);
        const int64_t limit = kScatter ? dst_rows : src_rows;
        if (j < 0 || j >= limit) {
            if (lane == 0) raise_status(status, SPMM_DEV_BAD_ROWPTR, i);
            continue;
        }
        const W *s = src + (kScatter ? i : j) * words;
        W *d = dst + (kScatter ? j : i) * words;
        for (int64_t w = lane; w < words; w += 32) d[w] = s[w];
    }
}

template <bool kScatter>
cudaError_t launch_perm(const void *src, void *dst, const int64_t *inv, int64_t n, int64_t src_rows,
                        int64_t dst_rows, int64_t row_bytes, DevStatus *st, cudaStream_t stream)
{
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, 16LL * device_sm_count()));
    const uintptr_t align = (uintptr_t)src | (uintptr_t)dst | (uintptr_t)row_bytes;
    if (align % 16 == 0)
        permute_rows_kernel<uint4, kScatter><<<(unsigned)blocks, 256, 0, stream>>>(
            (const uint4 *)src, (uint4 *)dst, inv, n, src_rows, dst_rows, row_bytes / 16, st);
    else if (align % 4 == 0)
        permute_rows_kernel<uint32_t, kScatter><<<(unsigned)blocks, 256, 0, stream>>>(
            (const uint32_t *)src, (uint32_t *)dst, inv, n, src_rows, dst_rows, row_bytes / 4, st);
    else
        permute_rows_kernel<unsigned char, kScatter><<<(unsigned)blocks, 256, 0, stream>>>(
            (const unsigned char *)src, (unsigned char *)dst, inv, n, src_rows, dst_rows, row_bytes, st);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_pack_rows(const void *src, const int64_t *inv, int64_t n, int64_t row_bytes, void *dst,
                             int64_t packed_rows, DevStatus *st, cudaStream_t stream)
{
    cudaError_t e = cudaMemsetAsync(dst, 0, (size_t)packed_rows * (size_t)row_bytes, stream);
    if (e != cudaSuccess || n == 0 || row_bytes == 0) return e;
    return launch_perm<true>(src, dst, inv, n, n, packed_rows, row_bytes, st, stream);
}

cudaError_t launch_restore_rows(const void *src, int64_t src_rows, const int64_t *inv, int64_t n,
                                int64_t row_bytes, void *dst, DevStatus *st, cudaStream_t stream)
{
    if (n == 0 || row_bytes == 0) return cudaSuccess;
    return launch_perm<false>(src, dst, inv, n, src_rows, n, row_bytes, st, stream);
}

}  // namespace spmmb
