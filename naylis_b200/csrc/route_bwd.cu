// Router backward: the autograd of model.py:186-220 (prefix mean -> bf16/fp32
// router_down -> tanh -> router_up -> softmax / top-k / gate softmax).
//
//   token     per token: gate-softmax and probs-softmax adjoints -> dlogits;
//             da = dlogits . Wu; dz = da * (1 - act^2)
//   revscan   u[b,t,:] = sum_{s>=t} dz[b,s,:] / (s+1): the adjoint of the prefix
//             mean, done in rank-r space (r = 32) instead of d-space (d = 1024)
//   dxdw      dx = u . Wd (N x r).(r x d) and dWd = u^T . x (r x N).(N x d) in one
//             pass over the tokens (x read once, dx written once)
//   dwup      dWu = dlogits^T . act         (nb x N) . (N x r), per-CTA partial sums
//
// Only tolerance-level parity applies to the backward, so the reverse scan is a
// parallel chunked scan and the two rank-r GEMMs run on the tensor cores with
// u split into a bf16 high part and a bf16 residual (about 16 mantissa bits),
// when the router computes in bf16; fp32 routers use fp32 FMA throughout.
#include "common.cuh"
#include "launch.h"

namespace mom {

namespace {
constexpr int kMaxNbB = 64;
constexpr int kMaxRankB = 128;
}  // namespace

// ---------------------------------------------------------------- per token
// Warp per token: dlogits and dz.
template <int CDT>
__global__ void __launch_bounds__(256)
route_bwd_token_kernel(int64_t ntok, int r, int nb, int top, const float *__restrict__ probs,
                       const void *__restrict__ top_idx, int idx64, const float *__restrict__ gates,
                       const typename Elem<CDT>::T *__restrict__ act,
                       const typename Elem<CDT>::T *__restrict__ w_up,
                       const float *__restrict__ dlog_gates, const float *__restrict__ dgates,
                       const float *__restrict__ dprobs, float *__restrict__ dlogits, float *__restrict__ dz) {
    const int lane = threadIdx.x & 31;
    {
        const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
        if (t >= ntok) return;
        float g = 0.0f, dg = 0.0f;
        int idx = -1;
        if (lane < top) {
            g = gates[t * top + lane];
            if (dlog_gates) dg += (g >= 1e-9f) ? dlog_gates[t * top + lane] / fmaxf(g, 1e-9f) : 0.0f;
            if (dgates) dg += dgates[t * top + lane];
            idx = idx64 ? static_cast<int>(reinterpret_cast<const int64_t *>(top_idx)[t * top + lane])
                        : reinterpret_cast<const int32_t *>(top_idx)[t * top + lane];
        }
        const float sgdg = warp_sum(g * dg);
        const float dtv = g * (dg - sgdg);
        float sp = 0.0f;
        if (dprobs) {
            float part = 0.0f;
            for (int e = lane; e < nb; e += 32) part += probs[t * nb + e] * dprobs[t * nb + e];
            sp = warp_sum(part);
        }
        // Every shuffle below runs on all 32 lanes: the loops have warp-uniform
        // trip counts and only the loads/stores are predicated.
        float dl0 = 0.0f, dl1 = 0.0f;   // dlogits for e = lane and e = lane + 32
#pragma unroll
        for (int half = 0; half < kMaxNbB / 32; ++half) {
            const int e = half * 32 + lane;
            float v = 0.0f;
            for (int k = 0; k < top; ++k) {
                const int ik = __shfl_sync(0xffffffffu, idx, k);
                const float dk = __shfl_sync(0xffffffffu, dtv, k);
                if (ik == e) v += dk;
            }
            if (e < nb) {
                if (dprobs) {
                    const float p = probs[t * nb + e];
                    v += p * (dprobs[t * nb + e] - sp);
                }
                dlogits[t * nb + e] = v;
            } else {
                v = 0.0f;
            }
            if (half == 0) dl0 = v; else dl1 = v;
        }
        for (int j0 = 0; j0 < r; j0 += 32) {
            const int j = j0 + lane;
            const float a = j < r ? Elem<CDT>::load(act, t * r + j) : 0.0f;
            float da = 0.0f;
            for (int e = 0; e < nb; ++e) {
                const float dle = __shfl_sync(0xffffffffu, e < 32 ? dl0 : dl1, e & 31);
                if (j < r) da = fmaf(dle, Elem<CDT>::load(w_up, static_cast<int64_t>(e) * r + j), da);
            }
            if (j < r) dz[t * r + j] = da * (1.0f - a * a);
        }
    }
}

// dWu[e, j] += sum_t dlogits[t, e] * act[t, j]: warp = a run of tokens with its
// partial sums in registers (lane j, all e), 4 tokens' loads in flight at a
// time; the CTA's 8 warps meet in shared memory, one reduction per CTA.
template <int CDT, int NB>
__global__ void __launch_bounds__(256)
route_bwd_dwup_kernel(const float *__restrict__ dlogits, const typename Elem<CDT>::T *__restrict__ act,
                      int64_t ntok, int r, int nb, int64_t per_warp, float *__restrict__ dw_up) {
    __shared__ float s_acc[8][NB][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + warp;
    const int64_t t0 = gw * per_warp, t1 = min(ntok, t0 + per_warp);
    for (int j0 = 0; j0 < r; j0 += 32) {
        const int j = j0 + lane;
        float acc[NB];
#pragma unroll
        for (int e = 0; e < NB; ++e) acc[e] = 0.0f;
        for (int64_t t = t0; t < t1; t += 4) {
            float a[4], dl[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const bool ok = t + u < t1;
                a[u] = (ok && j < r) ? Elem<CDT>::load(act, (t + u) * r + j) : 0.0f;
                dl[u] = (ok && lane < nb) ? dlogits[(t + u) * nb + lane] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int e = 0; e < NB; ++e) acc[e] = fmaf(__shfl_sync(0xffffffffu, dl[u], e), a[u], acc[e]);
        }
#pragma unroll
        for (int e = 0; e < NB; ++e) s_acc[warp][e][lane] = acc[e];
        __syncthreads();
        for (int i = threadIdx.x; i < NB * 32; i += 256) {
            const int e = i / 32, jj = i % 32;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) v += s_acc[w][e][jj];
            if (e < nb && j0 + jj < r) atomicAdd(dw_up + e * r + j0 + jj, v);
        }
        __syncthreads();
    }
}

// General (nb > 16) dWu: thread per output element over a token range.
template <int CDT>
__global__ void __launch_bounds__(256)
route_bwd_dwup_any_kernel(const float *__restrict__ dlogits, const typename Elem<CDT>::T *__restrict__ act,
                          int64_t ntok, int r, int nb, int64_t per_cta, float *__restrict__ dw_up) {
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * per_cta, t1 = min(ntok, t0 + per_cta);
    for (int o = blockIdx.x * 256 + threadIdx.x; o < nb * r; o += gridDim.x * 256) {
        const int e = o / r, j = o % r;
        float acc = 0.0f;
        for (int64_t t = t0; t < t1; ++t) acc = fmaf(dlogits[t * nb + e], Elem<CDT>::load(act, t * r + j), acc);
        atomicAdd(dw_up + o, acc);
    }
}

// ---------------------------------------------------------------- reverse scan
// CTA = 8 columns x 128 chunks of the sequence (1024 threads) of one batch row.
// Phase 1: chunk sums; phase 2: suffix scan of the chunk sums per column;
// phase 3: each thread walks its chunk backwards from its carry.
constexpr int kRsCols = 8, kRsChunks = 128;
__global__ void __launch_bounds__(1024)
route_bwd_revscan_kernel(const float *__restrict__ dz, float *__restrict__ u, int S, int r) {
    __shared__ float s_tot[kRsCols][kRsChunks + 1];
    const int c = threadIdx.x % kRsCols, k = threadIdx.x / kRsCols;
    const int b = blockIdx.y;
    const int j = blockIdx.x * kRsCols + c;
    const int len = (S + kRsChunks - 1) / kRsChunks;
    const int t0 = k * len, t1 = min(S, t0 + len);
    const float *src = dz + static_cast<int64_t>(b) * S * r + j;
    float *dst = u + static_cast<int64_t>(b) * S * r + j;
    float acc = 0.0f;
    if (j < r) {
#pragma unroll 8
        for (int t = t0; t < t1; ++t) acc += src[static_cast<int64_t>(t) * r] / static_cast<float>(t + 1);
    }
    s_tot[c][k] = acc;
    __syncthreads();
    {   // exclusive suffix scan over the 128 chunks of a column: warp w < 8 takes
        // column w, lane l chunks 4l .. 4l+3
        static_assert(kRsChunks == 128 && kRsCols <= 32, "suffix-scan layout");
        const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
        if (w < kRsCols) {
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = s_tot[w][4 * l + q];
            const float tot = v[0] + v[1] + v[2] + v[3];
            float incl = tot;   // sum over lanes >= l
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float n = __shfl_down_sync(0xffffffffu, incl, o);
                if (l + o < 32) incl += n;
            }
            float run = incl - tot;   // the chunks after this lane's
#pragma unroll
            for (int q = 3; q >= 0; --q) {
                s_tot[w][4 * l + q] = run;   // exclusive: sum of the chunks after 4l+q
                run += v[q];
            }
        }
    }
    __syncthreads();
    if (j >= r) return;
    float run = s_tot[c][k];
#pragma unroll 8
    for (int t = t1 - 1; t >= t0; --t) {
        run += src[static_cast<int64_t>(t) * r] / static_cast<float>(t + 1);
        dst[static_cast<int64_t>(t) * r] = run;
    }
}

// ---------------------------------------------------------------- tensor-core GEMMs
// Split an fp32 value into a bf16 high part and a bf16 residual.
__device__ __forceinline__ void split_bf16(float v, uint16_t &hi, uint16_t &lo) {
    hi = f32_to_bf16_bits(v);
    lo = f32_to_bf16_bits(v - bf16_bits_to_f32(hi));
}

// dx[t, c] (+)= sum_j u[t, j] Wd[j, c] and dWd[j, c] += sum_t u[t, j] x[t, c] in one
// pass over the tokens, so that x is read once and dx written once: CTA = 128
// columns x kDxdwSteps steps of 64 tokens, 4 warps. The next step's x tile (bf16 x:
// cp.async into the other of two buffers) and raw fp32 u tile are in flight while a
// step computes; per step u is split into bf16 high and residual parts in shared
// memory; dx goes out through a shared fp32 tile (the step's x buffer, once read)
// as 16-B vectors; the dWd partial sums stay in registers across the steps and
// leave by fp32 reductions at the end.
constexpr int kDxdwSteps = 4;
template <int R>
struct DxdwSmem {
    static constexpr int kTok = 64, kCols = 128;
    static constexpr int kUStride = R * 2 + 16, kWStride = kCols * 2 + 16, kXStride = kCols * 2 + 16;
    static constexpr int kHalf = kCols / 2, kOS = kHalf + 4;
    static constexpr int kU = kTok * kUStride, kW = R * kWStride, kX = kTok * kXStride, kOut = kTok * kOS * 4;
    static constexpr int kURaw = kTok * R * 4;
    static_assert(kOut <= kX, "the dx staging tile reuses an x buffer");
    static constexpr int kBytes = 2 * kU + kW + 2 * kX + kURaw;
};

template <int R, int XDT, int DXDT>
__global__ void __launch_bounds__(128, 3)
route_bwd_dxdw_mma_kernel(const float *__restrict__ u, const uint16_t *__restrict__ w_down,
                          const typename Elem<XDT>::T *__restrict__ x, int64_t ntok, int d,
                          typename Elem<DXDT>::T *__restrict__ dx, int accumulate, float *__restrict__ dw_down) {
    using L = DxdwSmem<R>;
    constexpr int kTok = L::kTok, kCols = L::kCols, MT = R / 16;
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char *sUh = smem;
    unsigned char *sUl = smem + L::kU;
    unsigned char *sW = smem + 2 * L::kU;
    unsigned char *sXb = sW + L::kW;                                   // [2][kX]
    float *sURaw = reinterpret_cast<float *>(sXb + 2 * L::kX);         // [kTok][R]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c0 = blockIdx.x * kCols;
    for (int i = tid; i < R * (kCols / 8); i += 128) {
        const int j = i / (kCols / 8), ch = i % (kCols / 8);
        const int c = c0 + ch * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (c < d) v = *reinterpret_cast<const uint4 *>(w_down + static_cast<int64_t>(j) * d + c);
        *reinterpret_cast<uint4 *>(sW + j * L::kWStride + ch * 16) = v;
    }
    auto step_tok0 = [&](int st) { return (static_cast<int64_t>(blockIdx.y) * kDxdwSteps + st) * kTok; };
    // cp.async of step st's raw u tile (and, for bf16 x, its x tile into buffer st & 1)
    auto prefetch = [&](int st) {
        const int64_t tok0 = step_tok0(st);
        if (st < kDxdwSteps && tok0 < ntok) {
            const uint32_t su = smem_u32(sURaw);
            for (int i = tid; i < kTok * R / 4; i += 128) {   // 16-B pieces of a contiguous tile
                const int64_t t = tok0 + (i * 4) / R;
                const bool ok = t < ntok;
                cp_async16(su + i * 16, ok ? u + tok0 * R + i * 4 : u, ok ? 16 : 0);
            }
            if (XDT == MOM_BF16) {
                const uint32_t sx = smem_u32(sXb + (st & 1) * L::kX);
                for (int i = tid; i < kTok * (kCols / 8); i += 128) {
                    const int tl = i / (kCols / 8), ch = i % (kCols / 8);
                    const int64_t t = tok0 + tl;
                    const int c = c0 + ch * 8;
                    const bool ok = t < ntok && c < d;
                    const uint16_t *src = reinterpret_cast<const uint16_t *>(x) + (ok ? t * d + c : 0);
                    cp_async16(sx + tl * L::kXStride + ch * 16, src, ok ? 16 : 0);
                }
            }
        }
        cp_async_commit();
    };
    float accw[MT][4][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) accw[m][n][0] = accw[m][n][1] = accw[m][n][2] = accw[m][n][3] = 0.0f;
    const int g = lane >> 2, q2 = (lane & 3) * 2;
    prefetch(0);
    for (int st = 0; st < kDxdwSteps; ++st) {
        const int64_t tok0 = step_tok0(st);
        if (tok0 >= ntok) break;
        unsigned char *sX = sXb + (st & 1) * L::kX;
        cp_async_wait<0>();
        __syncthreads();   // step st's tiles landed; step st-1's readers of sU / its x buffer are done
        for (int i = tid; i < kTok * R; i += 128) {
            const int tl = i / R, j = i % R;
            uint16_t hi, lo;
            split_bf16(sURaw[i], hi, lo);
            *reinterpret_cast<uint16_t *>(sUh + tl * L::kUStride + j * 2) = hi;
            *reinterpret_cast<uint16_t *>(sUl + tl * L::kUStride + j * 2) = lo;
        }
        if (XDT != MOM_BF16) {
            for (int i = tid; i < kTok * (kCols / 8); i += 128) {
                const int tl = i / (kCols / 8), ch = i % (kCols / 8);
                const int64_t t = tok0 + tl;
                const int c = c0 + ch * 8;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (t < ntok && c < d) {
                    const float *xf = reinterpret_cast<const float *>(x) + t * d + c;
                    v.x = pack_bf16x2(xf[0], xf[1]);
                    v.y = pack_bf16x2(xf[2], xf[3]);
                    v.z = pack_bf16x2(xf[4], xf[5]);
                    v.w = pack_bf16x2(xf[6], xf[7]);
                }
                *reinterpret_cast<uint4 *>(sX + tl * L::kXStride + ch * 16) = v;
            }
        }
        __syncthreads();   // sU (and an fp32 x tile) ready; the raw u buffer and the other x buffer are free
        prefetch(st + 1);
        // dx tile: warp = 16 tokens x 128 columns
        float acc[kCols / 8][4];
#pragma unroll
        for (int n = 0; n < kCols / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < R / 16; ++ks) {
            uint32_t ah[4], al[4];
            const uint32_t aoff = (warp * 16 + (lane & 15)) * L::kUStride + (ks * 16 + (lane >> 4) * 8) * 2;
            ldmatrix_x4(ah, smem_u32(sUh) + aoff);
            ldmatrix_x4(al, smem_u32(sUl) + aoff);
#pragma unroll
            for (int p = 0; p < kCols / 16; ++p) {
                uint32_t bfr[4];
                const uint32_t boff = (ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * L::kWStride +
                                      (p * 16 + (lane >> 4) * 8) * 2;
                ldmatrix_x4_trans(bfr, smem_u32(sW) + boff);
                mma_bf16_16816(acc[2 * p], ah, bfr[0], bfr[1]);
                mma_bf16_16816(acc[2 * p + 1], ah, bfr[2], bfr[3]);
                mma_bf16_16816(acc[2 * p], al, bfr[0], bfr[1]);
                mma_bf16_16816(acc[2 * p + 1], al, bfr[2], bfr[3]);
            }
        }
        // dWd partial: warp = 32 columns x R ranks, over the step's 64 tokens
#pragma unroll
        for (int ks = 0; ks < kTok / 16; ++ks) {
            uint32_t bfr[2][4];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const uint32_t boff = (ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * L::kXStride +
                                      (warp * 32 + p * 16 + (lane >> 4) * 8) * 2;
                ldmatrix_x4_trans(bfr[p], smem_u32(sX) + boff);
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                uint32_t ah[4], al[4];
                const uint32_t aoff = (ks * 16 + (lane & 7) + (lane >> 4) * 8) * L::kUStride +
                                      (m * 16 + ((lane >> 3) & 1) * 8) * 2;
                ldmatrix_x4_trans(ah, smem_u32(sUh) + aoff);
                ldmatrix_x4_trans(al, smem_u32(sUl) + aoff);
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    mma_bf16_16816(accw[m][2 * p], ah, bfr[p][0], bfr[p][1]);
                    mma_bf16_16816(accw[m][2 * p + 1], ah, bfr[p][2], bfr[p][3]);
                    mma_bf16_16816(accw[m][2 * p], al, bfr[p][0], bfr[p][1]);
                    mma_bf16_16816(accw[m][2 * p + 1], al, bfr[p][2], bfr[p][3]);
                }
            }
        }
        // dx out: stage the fp32 tile 64 columns at a time in this step's x buffer
        // (every warp has finished reading it), then 16-B vectors
        float *sOut = reinterpret_cast<float *>(sX);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            __syncthreads();
#pragma unroll
            for (int n = 0; n < L::kHalf / 8; ++n)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row = warp * 16 + g + h * 8;
                    sOut[row * L::kOS + n * 8 + q2] = acc[half * (L::kHalf / 8) + n][2 * h];
                    sOut[row * L::kOS + n * 8 + q2 + 1] = acc[half * (L::kHalf / 8) + n][2 * h + 1];
                }
            __syncthreads();
            for (int i = tid; i < kTok * (L::kHalf / 4); i += 128) {
                const int row = i / (L::kHalf / 4), c4 = (i % (L::kHalf / 4)) * 4;
                const int64_t t = tok0 + row;
                const int c = c0 + half * L::kHalf + c4;
                if (t >= ntok || c >= d) continue;
                float v[4] = {sOut[row * L::kOS + c4], sOut[row * L::kOS + c4 + 1], sOut[row * L::kOS + c4 + 2],
                              sOut[row * L::kOS + c4 + 3]};
                if (DXDT == MOM_BF16) {
                    uint2 *pp = reinterpret_cast<uint2 *>(reinterpret_cast<uint16_t *>(dx) + t * d + c);
                    if (accumulate) {
                        const uint2 o = *pp;
                        v[0] += __uint_as_float(o.x << 16);
                        v[1] += __uint_as_float(o.x & 0xFFFF0000u);
                        v[2] += __uint_as_float(o.y << 16);
                        v[3] += __uint_as_float(o.y & 0xFFFF0000u);
                    }
                    *pp = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
                } else {
                    float4 *pp = reinterpret_cast<float4 *>(reinterpret_cast<float *>(dx) + t * d + c);
                    if (accumulate) {
                        const float4 o = *pp;
                        v[0] += o.x; v[1] += o.y; v[2] += o.z; v[3] += o.w;
                    }
                    *pp = make_float4(v[0], v[1], v[2], v[3]);
                }
            }
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            const int c = c0 + warp * 32 + n * 8 + q2;
            if (c >= d) continue;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = m * 16 + g + h * 8;
                red_add_v2(dw_down + static_cast<int64_t>(j) * d + c, accw[m][n][2 * h], accw[m][n][2 * h + 1]);
            }
        }
}

// fp32 router (parity configurations): SIMT fp32 FMA versions.
constexpr int kDxTokens = 16;
template <int CDT, int DXDT>
__global__ void __launch_bounds__(256)
route_bwd_dx_simt_kernel(const float *__restrict__ u, const typename Elem<CDT>::T *__restrict__ w_down,
                         int64_t ntok, int d, int r, typename Elem<DXDT>::T *__restrict__ dx, int accumulate) {
    __shared__ float sU[kDxTokens * kMaxRankB];
    const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * kDxTokens;
    for (int i = threadIdx.x; i < kDxTokens * r; i += blockDim.x) {
        const int64_t t = tok0 + i / r;
        sU[i] = t < ntok ? u[t * r + (i % r)] : 0.0f;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        for (int tl = 0; tl < kDxTokens; ++tl) {
            const int64_t t = tok0 + tl;
            if (t >= ntok) break;
            float acc = 0.0f;
            for (int j = 0; j < r; ++j)
                acc = fmaf(sU[tl * r + j], Elem<CDT>::load(w_down, static_cast<int64_t>(j) * d + c), acc);
            if (accumulate) acc += Elem<DXDT>::load(dx, t * d + c);
            Elem<DXDT>::store(dx, t * d + c, acc);
        }
    }
}

constexpr int kDwTok = 256;
constexpr int kDwCols = 64;
template <int XDT>
__global__ void __launch_bounds__(256)
route_bwd_dwdown_simt_kernel(const float *__restrict__ u, const typename Elem<XDT>::T *__restrict__ x,
                             int64_t ntok, int d, int r, float *__restrict__ dw_down) {
    __shared__ float sU[32 * kMaxRankB];
    __shared__ float sX[32 * kDwCols];
    const int c0 = blockIdx.x * kDwCols;
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * kDwTok;
    const int tid = threadIdx.x;
    const int cl = tid % kDwCols;
    const int jg = tid / kDwCols;
    float acc[kMaxRankB / 4];
    for (int i = 0; i < kMaxRankB / 4; ++i) acc[i] = 0.0f;
    for (int tb = 0; tb < kDwTok; tb += 32) {
        __syncthreads();
        for (int i = tid; i < 32 * r; i += 256) {
            const int64_t t = t0 + tb + i / r;
            sU[i] = t < ntok ? u[t * r + i % r] : 0.0f;
        }
        for (int i = tid; i < 32 * kDwCols; i += 256) {
            const int64_t t = t0 + tb + i / kDwCols;
            const int c = c0 + i % kDwCols;
            sX[i] = (t < ntok && c < d) ? Elem<XDT>::load(x, t * d + c) : 0.0f;
        }
        __syncthreads();
        for (int tt = 0; tt < 32; ++tt) {
            const float xv = sX[tt * kDwCols + cl];
            for (int j = jg, i = 0; j < r; j += 4, ++i) acc[i] = fmaf(sU[tt * r + j], xv, acc[i]);
        }
    }
    const int c = c0 + cl;
    if (c < d)
        for (int j = jg, i = 0; j < r; j += 4, ++i) atomicAdd(dw_down + static_cast<int64_t>(j) * d + c, acc[i]);
}

// ---------------------------------------------------------------- launcher
cudaError_t launch_route_bwd(const void *x, int xdt, int B, int S, int d, const void *w_down,
                             const void *w_up, int cdt, int r, int nb, int top, const float *probs,
                             const void *top_idx, int idx64, const float *gates, const void *act,
                             const float *dlog_gates, const float *dgates, const float *dprobs,
                             void *dx, int dxdt, int accumulate, float *dw_down, float *dw_up,
                             float *ws_dlogits, float *ws_dz, float *ws_u, cudaStream_t st) {
    const int64_t ntok = static_cast<int64_t>(B) * S;
    cudaError_t e;
    if ((e = cudaMemsetAsync(dw_down, 0, sizeof(float) * r * d, st)) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(dw_up, 0, sizeof(float) * nb * r, st)) != cudaSuccess) return e;
    if (ntok == 0) return cudaSuccess;
    {
        const int warps = 8;
        const int grid = static_cast<int>((ntok + warps - 1) / warps);
        if (cdt == MOM_BF16)
            route_bwd_token_kernel<MOM_BF16><<<grid, warps * 32, 0, st>>>(
                ntok, r, nb, top, probs, top_idx, idx64, gates, static_cast<const uint16_t *>(act),
                static_cast<const uint16_t *>(w_up), dlog_gates, dgates, dprobs, ws_dlogits, ws_dz);
        else
            route_bwd_token_kernel<MOM_F32><<<grid, warps * 32, 0, st>>>(
                ntok, r, nb, top, probs, top_idx, idx64, gates, static_cast<const float *>(act),
                static_cast<const float *>(w_up), dlog_gates, dgates, dprobs, ws_dlogits, ws_dz);
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    {   // dWu = dlogits^T act
        const int64_t nwarps = 148 * 8;
        const int64_t per_warp = std::max<int64_t>(4, (ntok + nwarps - 1) / nwarps);
        const int grid = static_cast<int>((ntok + per_warp * 8 - 1) / (per_warp * 8));
#define MOM_DWUP(NBV)                                                                                      \
    if (nb <= NBV) {                                                                                       \
        if (cdt == MOM_BF16)                                                                               \
            route_bwd_dwup_kernel<MOM_BF16, NBV><<<grid, 256, 0, st>>>(                                     \
                ws_dlogits, static_cast<const uint16_t *>(act), ntok, r, nb, per_warp, dw_up);             \
        else                                                                                               \
            route_bwd_dwup_kernel<MOM_F32, NBV><<<grid, 256, 0, st>>>(                                      \
                ws_dlogits, static_cast<const float *>(act), ntok, r, nb, per_warp, dw_up);                \
    } else
        MOM_DWUP(8) MOM_DWUP(16) {
            const int64_t per_cta = 256;
            dim3 g2((nb * r + 255) / 256, static_cast<unsigned>((ntok + per_cta - 1) / per_cta));
            if (cdt == MOM_BF16)
                route_bwd_dwup_any_kernel<MOM_BF16><<<g2, 256, 0, st>>>(
                    ws_dlogits, static_cast<const uint16_t *>(act), ntok, r, nb, per_cta, dw_up);
            else
                route_bwd_dwup_any_kernel<MOM_F32><<<g2, 256, 0, st>>>(
                    ws_dlogits, static_cast<const float *>(act), ntok, r, nb, per_cta, dw_up);
        }
#undef MOM_DWUP
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    route_bwd_revscan_kernel<<<dim3((r + kRsCols - 1) / kRsCols, B), 1024, 0, st>>>(ws_dz, ws_u, S, r);
    count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // the tensor-core pass stores dx and reads x and u in 16-B vectors
    const bool tc = cdt == MOM_BF16 && (r == 32 || r == 64) && d % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(dx) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(ws_u) & 15) == 0;
    if (tc) {
        dim3 grid((d + 127) / 128, static_cast<unsigned>((ntok + 64 * kDxdwSteps - 1) / (64 * kDxdwSteps)));
#define MOM_DXDW(R, X, D)                                                                                   \
    if (r == R && xdt == X && dxdt == D) {                                                                 \
        const int smem = DxdwSmem<R>::kBytes;                                                               \
        e = cudaFuncSetAttribute(route_bwd_dxdw_mma_kernel<R, X, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 smem);                                                                     \
        if (e != cudaSuccess) return e;                                                                     \
        route_bwd_dxdw_mma_kernel<R, X, D><<<grid, 128, smem, st>>>(                                        \
            ws_u, static_cast<const uint16_t *>(w_down), static_cast<const typename Elem<X>::T *>(x), ntok, d, \
            static_cast<typename Elem<D>::T *>(dx), accumulate, dw_down);                                  \
    }
        MOM_DXDW(32, MOM_BF16, MOM_BF16)
        MOM_DXDW(32, MOM_BF16, MOM_F32)
        MOM_DXDW(32, MOM_F32, MOM_BF16)
        MOM_DXDW(32, MOM_F32, MOM_F32)
        MOM_DXDW(64, MOM_BF16, MOM_BF16)
        MOM_DXDW(64, MOM_BF16, MOM_F32)
        MOM_DXDW(64, MOM_F32, MOM_BF16)
        MOM_DXDW(64, MOM_F32, MOM_F32)
#undef MOM_DXDW
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    } else {
        const int grid = static_cast<int>((ntok + kDxTokens - 1) / kDxTokens);
#define MOM_DX_CASE(C, X)                                                                         \
    if (cdt == C && dxdt == X)                                                                    \
        route_bwd_dx_simt_kernel<C, X><<<grid, 256, 0, st>>>(                                     \
            ws_u, static_cast<const typename Elem<C>::T *>(w_down), ntok, d, r,                  \
            static_cast<typename Elem<X>::T *>(dx), accumulate);
        MOM_DX_CASE(MOM_BF16, MOM_BF16)
        MOM_DX_CASE(MOM_BF16, MOM_F32)
        MOM_DX_CASE(MOM_F32, MOM_BF16)
        MOM_DX_CASE(MOM_F32, MOM_F32)
#undef MOM_DX_CASE
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        dim3 grid2((d + kDwCols - 1) / kDwCols, static_cast<unsigned>((ntok + kDwTok - 1) / kDwTok));
        if (xdt == MOM_BF16)
            route_bwd_dwdown_simt_kernel<MOM_BF16><<<grid2, 256, 0, st>>>(
                ws_u, static_cast<const uint16_t *>(x), ntok, d, r, dw_down);
        else
            route_bwd_dwdown_simt_kernel<MOM_F32><<<grid2, 256, 0, st>>>(
                ws_u, static_cast<const float *>(x), ntok, d, r, dw_down);
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace mom
