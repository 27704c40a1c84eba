// Block-split read: top-k routing whose block sets are too many for the set
// bucketing (top-4 of 32 blocks has 35,960 sets) is read as N*top rows, one per
// (token, k) pair, each reading its one block with top = 1. The same read kernels
// run on that plan (PlanView::rows_per_q = top: every row's q is its token's);
// these kernels do what is left:
//
//   prep     the rows' log-gates; a block chosen twice by one token is one read
//            with the sum of its log-gates (mom_kernels/reference.py:14-29 sums
//            them in its one-hot einsum), so the first occurrence gets the sum
//            and later ones are dead rows (weight 0 in the combine).
//   combine  per token and head, lse = logsumexp_k lse_k over the live rows and
//            out = sum_k a_k out_k with a_k = exp(lse_k - lse): the softmax over
//            the union of the blocks, as the single-pass read forms it.
//   gate_do  g_k = a_k dO, the backward's per-row dO. With it, and delta taken
//            from the combined output (rows_per_q again), every dS = P (dP - delta)
//            of the split rows equals the full softmax's, so dK, dV and the
//            per-row gate gradient come out exact, with no extra term. (The
//            tensor-core path forms g_k inside its row copy of dO instead, rows.cu;
//            this kernel serves the warp-level kernels, which read dO per token.)
//   dq_sum   dQ = sum_k dQ_k, and the dead rows' gate gradient = their first
//            occurrence's (d bias / d log_gate = 1 for both).
//
// All are HBM-bound row passes: a warp per token (or row), 16-B vectors.
#include "common.cuh"
#include "launch.h"

namespace mom {
namespace {

__device__ __forceinline__ int64_t load_idx(const void *idx, int idx64, int64_t i) {
    return idx64 ? static_cast<const int64_t *>(idx)[i] : static_cast<const int32_t *>(idx)[i];
}

// bit k set: slot k repeats a block chosen at an earlier slot of the same token;
// first[k] = the earliest slot with slot k's block. Unrolled over TOPM >= top so
// that the arrays stay in registers.
template <int TOPM>
__device__ __forceinline__ uint32_t dead_mask(const void *idx, int idx64, int64_t t, int top, int (&first)[TOPM]) {
    int64_t b[TOPM];
#pragma unroll
    for (int k = 0; k < TOPM; ++k) b[k] = k < top ? load_idx(idx, idx64, t * top + k) : 0;
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < TOPM; ++k) {
        int f = k;
#pragma unroll
        for (int j = k - 1; j >= 0; --j)
            if (b[j] == b[k]) f = j;
        first[k] = f;
        if (k < top && f != k) m |= 1u << k;
    }
    return m;
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__global__ void __launch_bounds__(256)
split_prep_kernel(const void *__restrict__ idx, int idx64, const float *__restrict__ lg, int64_t N, int top,
                  float *__restrict__ lg_rows) {
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < N;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int first[kMaxTop];
        const uint32_t dead = dead_mask<kMaxTop>(idx, idx64, t, top, first);
        for (int k = 0; k < top; ++k) {
            float s = lg[t * top + k];
            if (!((dead >> k) & 1))
                for (int j = k + 1; j < top; ++j)
                    if (first[j] == k) s += lg[t * top + j];
            lg_rows[t * top + k] = s;
        }
    }
}

// w[perm[r]][h] = lse_rows[h][r]: the rows' log-sum-exp in (token, k) order.
__global__ void __launch_bounds__(256)
split_lse_scatter_kernel(const float *__restrict__ lse_rows, const int *__restrict__ perm, int64_t M, int H,
                         float *__restrict__ w) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < M * H;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t h = i / M, r = i - h * M;
        w[static_cast<int64_t>(perm[r]) * H + h] = lse_rows[i];
    }
}

// Warp per token. w holds the rows' lse on entry and the weights a_k on exit
// (each (token, head) entry read and rewritten by the same lane). TOPM >= top is
// the unroll bound; each lane combines two 16-B vectors per step with all rows'
// loads in flight first.
template <int TOPM>
__global__ void __launch_bounds__(256)
split_combine_kernel(const uint4 *__restrict__ out_rows, const void *__restrict__ idx, int idx64, int64_t N,
                     int top, int H, int hd, float *__restrict__ w, uint4 *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int vph = hd / 8, vpr = H * vph;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < N; t += nwarps) {
        int first[TOPM];
        const uint32_t dead = dead_mask<TOPM>(idx, idx64, t, top, first);
        float *wt = w + t * top * H;
        for (int h = lane; h < H; h += 32) {
            float lv[TOPM];
            float m = -INFINITY;
#pragma unroll
            for (int k = 0; k < TOPM; ++k) {
                const bool live = k < top && !((dead >> k) & 1);
                lv[k] = k < top ? wt[k * H + h] : -INFINITY;
                if (live) m = fmaxf(m, lv[k]);
            }
            float e[TOPM], sum = 0.0f;
#pragma unroll
            for (int k = 0; k < TOPM; ++k) {
                const bool live = k < top && !((dead >> k) & 1);
                e[k] = (live && m != -INFINITY) ? expf(lv[k] - m) : 0.0f;
                sum += e[k];
            }
            const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
#pragma unroll
            for (int k = 0; k < TOPM; ++k)
                if (k < top) wt[k * H + h] = e[k] * inv;
        }
        __syncwarp();
        for (int v0 = lane; v0 < vpr; v0 += 64) {
            float a[2][TOPM];
            uint4 x[2][TOPM];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int v = v0 + 32 * u;
                const int h = (v < vpr ? v : v0) / vph;
#pragma unroll
                for (int k = 0; k < TOPM; ++k) {
                    a[u][k] = (k < top && v < vpr) ? wt[k * H + h] : 0.0f;
                    x[u][k] = a[u][k] != 0.0f ? out_rows[(t * top + k) * vpr + v] : make_uint4(0u, 0u, 0u, 0u);
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int v = v0 + 32 * u;
                if (v >= vpr) break;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int k = 0; k < TOPM; ++k) {
                    const uint32_t xw[4] = {x[u][k].x, x[u][k].y, x[u][k].z, x[u][k].w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        acc[2 * q] = fmaf(a[u][k], bf_lo(xw[q]), acc[2 * q]);
                        acc[2 * q + 1] = fmaf(a[u][k], bf_hi(xw[q]), acc[2 * q + 1]);
                    }
                }
                out[t * vpr + v] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                              pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
            }
        }
        __syncwarp();
    }
}

// Warp per (token, k) row: g[row] = a_k * dO[token] (bf16).
__global__ void __launch_bounds__(256)
split_gate_do_kernel(const uint4 *__restrict__ dout, const float *__restrict__ w, int64_t M, int top, int H, int hd,
                     uint4 *__restrict__ g) {
    const int lane = threadIdx.x & 31;
    const int vph = hd / 8, vpr = H * vph;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < M; r += nwarps) {
        const int64_t t = r / top;
        for (int v = lane; v < vpr; v += 32) {
            const float a = w[r * H + v / vph];
            uint4 y = make_uint4(0u, 0u, 0u, 0u);
            if (a != 0.0f) {
                const uint4 x = dout[t * vpr + v];
                y = make_uint4(pack_bf16x2(a * bf_lo(x.x), a * bf_hi(x.x)), pack_bf16x2(a * bf_lo(x.y), a * bf_hi(x.y)),
                               pack_bf16x2(a * bf_lo(x.z), a * bf_hi(x.z)), pack_bf16x2(a * bf_lo(x.w), a * bf_hi(x.w)));
            }
            g[r * vpr + v] = y;
        }
    }
}

// Warp per token: dq[t] = sum_k dq_rows[t*top + k] (fp32 sum, bf16 out); the
// dead slots' gate gradient copied from their first occurrence.
template <int TOPM>
__global__ void __launch_bounds__(256)
split_dq_sum_kernel(const uint4 *__restrict__ dq_rows, const void *__restrict__ idx, int idx64, int64_t N, int top,
                    int vpr, uint4 *__restrict__ dq, float *__restrict__ dlog_gates) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < N; t += nwarps) {
        for (int v = lane; v < vpr; v += 32) {
            uint4 x[TOPM];
#pragma unroll
            for (int k = 0; k < TOPM; ++k)
                x[k] = k < top ? dq_rows[(t * top + k) * vpr + v] : make_uint4(0u, 0u, 0u, 0u);
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < TOPM; ++k) {
                const uint32_t xw[4] = {x[k].x, x[k].y, x[k].z, x[k].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    acc[2 * q] += bf_lo(xw[q]);
                    acc[2 * q + 1] += bf_hi(xw[q]);
                }
            }
            dq[t * vpr + v] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                         pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
        }
        if (lane == 0) {
            int first[TOPM];
            const uint32_t dead = dead_mask<TOPM>(idx, idx64, t, top, first);
#pragma unroll
            for (int k = 0; k < TOPM; ++k)
                if ((dead >> k) & 1) dlog_gates[t * top + k] = dlog_gates[t * top + first[k]];
        }
    }
}

// iperm[perm[r]] = r: each (token, k) row's position in plan order.
__global__ void __launch_bounds__(256)
split_iperm_kernel(const int *__restrict__ perm, int64_t M, int *__restrict__ iperm) {
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < M;
         r += static_cast<int64_t>(gridDim.x) * blockDim.x)
        iperm[perm[r]] = static_cast<int>(r);
}

// Warp per token: q[t] read once, copied to the plan rows of its top (token, k) rows.
__global__ void __launch_bounds__(256)
split_permute_q_kernel(const uint4 *__restrict__ q, const int *__restrict__ iperm, int64_t N, int top, int vpr,
                       uint4 *__restrict__ q_rows) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < N; t += nwarps) {
        int64_t dst[kMaxTop];
#pragma unroll
        for (int k = 0; k < kMaxTop; ++k) dst[k] = k < top ? static_cast<int64_t>(iperm[t * top + k]) * vpr : 0;
        for (int v = lane; v < vpr; v += 32) {
            const uint4 x = q[t * vpr + v];
#pragma unroll
            for (int k = 0; k < kMaxTop; ++k)
                if (k < top) q_rows[dst[k] + v] = x;
        }
    }
}

// Warp per token, the block-split backward's row copy on the tensor-core path:
// for each of the token's rows p = t*top + k, do_rows[iperm[p]] = bf16(w_k dO[t])
// (zero where w_k = 0) and delta[h][iperm[p]] = <that row, O[t]> per head (fp32
// sums of the bf16 products, as rows.cu's row_delta_kernel forms them). dO[t] and
// O[t] are read once per token instead of once per row.
template <int TOPM>
__global__ void __launch_bounds__(256)
split_row_delta_kernel(const uint4 *__restrict__ dout, const uint4 *__restrict__ out,
                       const float *__restrict__ w, const int *__restrict__ iperm, int64_t N, int top, int H,
                       int hd, uint4 *__restrict__ do_rows, float *__restrict__ delta) {
    const int lane = threadIdx.x & 31;
    const int vph = hd / 8, vpr = H * vph;
    const int64_t M = N * top;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < N; t += nwarps) {
        int row[TOPM];
#pragma unroll
        for (int k = 0; k < TOPM; ++k) row[k] = k < top ? iperm[t * top + k] : 0;
        // two 16-B vectors per lane and step (v0 and v0 + 32), both loaded first
        for (int v0 = 0; v0 < vpr; v0 += 64) {
            uint4 a[2], b[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int v = v0 + 32 * u + lane;
                a[u] = make_uint4(0u, 0u, 0u, 0u);
                b[u] = a[u];
                if (v < vpr) {
                    a[u] = dout[t * vpr + v];
                    b[u] = out[t * vpr + v];
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                if (v0 + 32 * u >= vpr) break;   // warp-uniform
                const int v = v0 + 32 * u + lane;
                const bool in = v < vpr;
                const int h = in ? v / vph : 0;
                const uint32_t aw[4] = {a[u].x, a[u].y, a[u].z, a[u].w}, bw[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
#pragma unroll
                for (int k = 0; k < TOPM; ++k) {
                    if (k >= top) break;
                    const float wk = in ? w[(t * top + k) * H + h] : 0.0f;
                    uint32_t g[4] = {0u, 0u, 0u, 0u};
                    float acc = 0.0f;
                    if (wk != 0.0f) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            g[q] = pack_bf16x2(wk * bf_lo(aw[q]), wk * bf_hi(aw[q]));
                            acc = fmaf(bf_lo(g[q]), bf_lo(bw[q]), acc);
                            acc = fmaf(bf_hi(g[q]), bf_hi(bw[q]), acc);
                        }
                    }
                    if (in) do_rows[static_cast<int64_t>(row[k]) * vpr + v] = make_uint4(g[0], g[1], g[2], g[3]);
                    for (int o = 1; o < vph; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                    if (in && (v % vph) == 0) delta[static_cast<int64_t>(h) * M + row[k]] = acc;
                }
            }
        }
    }
}

int grid_for(int64_t work, int per_block) {
    const int64_t want = (work + per_block - 1) / per_block;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 148 * 16)));
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

cudaError_t launch_split_prep(const void *top_idx, int idx64, const float *log_gates, int64_t N, int top,
                              float *lg_rows, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    if (top < 1 || top > kMaxTop) return cudaErrorInvalidValue;
    split_prep_kernel<<<grid_for(N, 256), 256, 0, st>>>(top_idx, idx64, log_gates, N, top, lg_rows);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_split_combine(const void *out_rows, const float *lse_rows, const int *perm, const void *top_idx,
                                 int idx64, int64_t N, int top, int H, int hd, float *weights, void *out,
                                 cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    if (top < 1 || top > kMaxTop || hd % 8 || !aligned16(out_rows) || !aligned16(out)) return cudaErrorInvalidValue;
    const int64_t M = N * top;
    split_lse_scatter_kernel<<<grid_for(M * H, 256), 256, 0, st>>>(lse_rows, perm, M, H, weights);
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    auto kern = top <= 4 ? split_combine_kernel<4> : split_combine_kernel<kMaxTop>;
    kern<<<grid_for(N, 8), 256, 0, st>>>(static_cast<const uint4 *>(out_rows), top_idx, idx64, N, top, H, hd, weights,
                                         static_cast<uint4 *>(out));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_split_iperm(const int *perm, int64_t M, int *iperm, cudaStream_t st) {
    if (M == 0) return cudaSuccess;
    split_iperm_kernel<<<grid_for(M, 256), 256, 0, st>>>(perm, M, iperm);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_split_permute_q(const void *q, const int *iperm, int64_t N, int top, int64_t row_bytes,
                                   void *q_rows, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    if (top < 1 || top > kMaxTop || row_bytes % 16 || !aligned16(q) || !aligned16(q_rows))
        return cudaErrorInvalidValue;
    split_permute_q_kernel<<<grid_for(N, 8), 256, 0, st>>>(static_cast<const uint4 *>(q), iperm, N, top,
                                                           static_cast<int>(row_bytes / 16),
                                                           static_cast<uint4 *>(q_rows));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_split_row_delta(const void *dout, const void *out, const float *weights, const int *iperm,
                                   int64_t N, int top, int H, int hd, void *do_rows, float *delta, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    if (top < 1 || top > kMaxTop || hd % 8 || (32 % (hd / 8)) || !aligned16(dout) || !aligned16(out) ||
        !aligned16(do_rows))
        return cudaErrorInvalidValue;
    auto kern = top <= 4 ? split_row_delta_kernel<4> : split_row_delta_kernel<kMaxTop>;
    kern<<<grid_for(N, 8), 256, 0, st>>>(static_cast<const uint4 *>(dout), static_cast<const uint4 *>(out), weights,
                                         iperm, N, top, H, hd, static_cast<uint4 *>(do_rows), delta);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_split_gate_do(const void *dout, const float *weights, int64_t N, int top, int H, int hd, void *g,
                                 cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    if (hd % 8 || !aligned16(dout) || !aligned16(g)) return cudaErrorInvalidValue;
    const int64_t M = N * top;
    split_gate_do_kernel<<<grid_for(M, 8), 256, 0, st>>>(static_cast<const uint4 *>(dout), weights, M, top, H, hd,
                                                         static_cast<uint4 *>(g));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_split_dq_sum(const void *dq_rows, const void *top_idx, int idx64, int64_t N, int top, int H,
                                int hd, void *dq, float *dlog_gates, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    if (top < 1 || top > kMaxTop || hd % 8 || !aligned16(dq_rows) || !aligned16(dq)) return cudaErrorInvalidValue;
    auto kern = top <= 4 ? split_dq_sum_kernel<4> : split_dq_sum_kernel<kMaxTop>;
    kern<<<grid_for(N, 8), 256, 0, st>>>(static_cast<const uint4 *>(dq_rows), top_idx, idx64, N, top, H * hd / 8,
                                         static_cast<uint4 *>(dq), dlog_gates);
    count_launch();
    return cudaGetLastError();
}

}  // namespace mom
