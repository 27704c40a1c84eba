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
                    int rows_per_src, uint4 *__restrict__ dst) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < N; r += nwarps) {
        const int64_t t = perm[r] / rows_per_src;
        const uint4 *s = src + t * vec_per_row;
        uint4 *d = dst + r * vec_per_row;
        for (int i = lane; i < vec_per_row; i += 32) d[i] = s[i];
    }
}

cudaError_t launch_permute_rows(const void *src, int64_t N, int64_t row_bytes, const int *perm, void *dst,
                                cudaStream_t st, int rows_per_src) {
    if (N == 0) return cudaSuccess;
    if (row_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
        return cudaErrorInvalidValue;
    const int64_t want = (N + 7) / 8;
    const int grid = static_cast<int>(std::min<int64_t>(want, 148 * 16));
    permute_rows_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4 *>(src), perm, N,
                                              static_cast<int>(row_bytes / 16), rows_per_src,
                                              static_cast<uint4 *>(dst));
    count_launch();
    return cudaGetLastError();
}

// delta[h][r] = sum_d dO[perm[r], h, d] * O[perm[r], h, d] (fp32 accumulation of the
// bf16 products: the softmax-backward's row term, as the reference forms it from
// the bf16 output), with dO's row copied to do_rows[r] when do_rows is given.
// With row_w (a block-split plan): the row's dO is bf16(row_w[perm[r]][h] *
// dout[perm[r] / rows_per_out]) (zero where the weight is 0), the same values the
// split path's weighted copy forms, and delta is taken over those.
// Warp per plan row; lane l reads 16-B vectors l, l+32, ...; the vph = hd / 8
// lanes that share a head combine their partial sums by shuffles.
__global__ void __launch_bounds__(256)
row_delta_kernel(const uint4 *__restrict__ dout, const uint4 *__restrict__ out, const int *__restrict__ perm,
                 int64_t N, int H, int hd, int rows_per_out, uint4 *__restrict__ do_rows, float *__restrict__ delta,
                 const float *__restrict__ row_w) {
    const int lane = threadIdx.x & 31;
    const int vpr = H * hd / 8, vph = hd / 8;            // 16-B vectors per row / per head
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < N; r += nwarps) {
        const int64_t t = perm[r];
        const int64_t tq = t / rows_per_out;
        const uint4 *dr = dout + (row_w ? tq : t) * vpr;
        const uint4 *orow = out + tq * vpr;
        for (int v0 = 0; v0 < vpr; v0 += 32) {
            const int v = v0 + lane;
            float acc = 0.0f;
            if (v < vpr) {
                uint4 a = dr[v];
                const uint4 b = orow[v];
                if (row_w) {
                    const float w = row_w[t * H + v / vph];
                    if (w == 0.0f) {
                        a = make_uint4(0u, 0u, 0u, 0u);
                    } else {
                        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
                        uint32_t sw[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            sw[q] = pack_bf16x2(w * __uint_as_float(aw[q] << 16),
                                                w * __uint_as_float(aw[q] & 0xFFFF0000u));
                        a = make_uint4(sw[0], sw[1], sw[2], sw[3]);
                    }
                }
                if (do_rows) do_rows[r * vpr + v] = a;
                const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    acc = fmaf(__uint_as_float(aw[q] << 16), __uint_as_float(bw[q] << 16), acc);
                    acc = fmaf(__uint_as_float(aw[q] & 0xFFFF0000u), __uint_as_float(bw[q] & 0xFFFF0000u), acc);
                }
            }
            for (int o = 1; o < vph; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (v < vpr && (v % vph) == 0) delta[static_cast<int64_t>(v / vph) * N + r] = acc;
        }
    }
}

cudaError_t launch_row_delta(const void *dout, const void *out, int64_t N, int H, int hd, const int *perm,
                             void *do_rows, float *delta, cudaStream_t st, int rows_per_out, const float *row_w) {
    if (N == 0) return cudaSuccess;
    if ((hd % 8) || (32 % (hd / 8)) || (reinterpret_cast<uintptr_t>(dout) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(do_rows) & 15))
        return cudaErrorInvalidValue;
    const int64_t want = (N + 7) / 8;
    const int grid = static_cast<int>(std::min<int64_t>(want, 148 * 16));
    row_delta_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4 *>(dout), static_cast<const uint4 *>(out), perm,
                                           N, H, hd, rows_per_out, static_cast<uint4 *>(do_rows), delta, row_w);
    count_launch();
    return cudaGetLastError();
}

}  // namespace mom
