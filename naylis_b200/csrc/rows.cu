// Rows of a token-ordered activation copied into routing-plan row order:
// dst[r, :] = src[perm[r], :], r < N (perm from mom_bucket).
//
// The tensor-core read kernels stream a tile of 128 plan rows per (item, head).
// Scattered rows cost the loader ~2 us per tile however they are fetched (TMA
// gather4 or cp.async), while one 2-D TMA box over 128 contiguous plan rows issues
// in ~0.1 us; so Q (forward) and dO (backward) are copied once into plan order by
// this bandwidth-bound kernel (one read and one write of the tensor).
#include "common.cuh"
#include "launch.h"

namespace mom {

// One warp per row, 16-B vectors; row_bytes is a multiple of 16.
__global__ void __launch_bounds__(256)
permute_rows_kernel(const uint4 *__restrict__ src, const int *__restrict__ perm, int64_t N, int vec_per_row,
                    uint4 *__restrict__ dst) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < N; r += nwarps) {
        const int64_t t = perm[r];
        const uint4 *s = src + t * vec_per_row;
        uint4 *d = dst + r * vec_per_row;
        for (int i = lane; i < vec_per_row; i += 32) d[i] = s[i];
    }
}

cudaError_t launch_permute_rows(const void *src, int64_t N, int64_t row_bytes, const int *perm, void *dst,
                                cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    if (row_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
        return cudaErrorInvalidValue;
    const int64_t want = (N + 7) / 8;
    const int grid = static_cast<int>(std::min<int64_t>(want, 148 * 16));
    permute_rows_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4 *>(src), perm, N,
                                              static_cast<int>(row_bytes / 16), static_cast<uint4 *>(dst));
    count_launch();
    return cudaGetLastError();
}

}  // namespace mom
