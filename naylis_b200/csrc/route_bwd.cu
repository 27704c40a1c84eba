// Router backward: the autograd of model.py:186-220 (prefix mean -> bf16/fp32
// router_down -> tanh -> router_up -> softmax / top-k / gate softmax).
//
//   token     per token: gate-softmax and probs-softmax adjoints -> dlogits;
//             da = dlogits . Wu; dz = da * (1 - act^2)
//   revscan   u[b,t,:] = sum_{s>=t} dz[b,s,:] / (s+1): the adjoint of the prefix
//             mean, done in rank-r space (r = 32) instead of d-space (d = 1024)
//   dx        dx = u . Wd                   (N x r) . (r x d)
//   dwdown    dWd = u^T . x                 (r x N) . (N x d), split over tokens
//   dwup      dWu = dlogits^T . act         (nb x N) . (N x r)
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
template <int CDT>
__global__ void route_bwd_token_kernel(int64_t ntok, int r, int nb, int top,
                                       const float *__restrict__ probs, const void *__restrict__ top_idx,
                                       int idx64, const float *__restrict__ gates,
                                       const typename Elem<CDT>::T *__restrict__ act,
                                       const typename Elem<CDT>::T *__restrict__ w_up,
                                       const float *__restrict__ dlog_gates,
                                       const float *__restrict__ dgates,
                                       const float *__restrict__ dprobs, float *__restrict__ dlogits,
                                       float *__restrict__ dz) {
    const int lane = threadIdx.x & 31;
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
        float da = 0.0f;
        for (int e = 0; e < nb; ++e) {
            const float dle = __shfl_sync(0xffffffffu, e < 32 ? dl0 : dl1, e & 31);
            if (j < r) da = fmaf(dle, Elem<CDT>::load(w_up, static_cast<int64_t>(e) * r + j), da);
        }
        if (j < r) {
            const float a = Elem<CDT>::load(act, t * r + j);
            dz[t * r + j] = da * (1.0f - a * a);
        }
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
    if (k == 0) {   // suffix scan over the chunks of column c
        float run = 0.0f;
        for (int kk = kRsChunks - 1; kk >= 0; --kk) {
            const float v = s_tot[c][kk];
            s_tot[c][kk] = run;   // exclusive: sum of the chunks after kk
            run += v;
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

// dx[t, c] (+)= sum_j u[t, j] * Wd[j, c]; CTA tile 64 tokens x 128 columns, 4 warps.
template <int R, int DXDT>
__global__ void __launch_bounds__(128)
route_bwd_dx_mma_kernel(const float *__restrict__ u, const uint16_t *__restrict__ w_down, int64_t ntok,
                        int d, typename Elem<DXDT>::T *__restrict__ dx, int accumulate) {
    constexpr int kTok = 64, kCols = 128;
    constexpr int kUStride = R * 2 + 16;        // bytes per token row (padded)
    constexpr int kWStride = kCols * 2 + 16;    // bytes per rank row (padded)
    // one buffer: [u hi | u lo | Wd] while computing, the fp32 output tile after
    __shared__ __align__(16) unsigned char sBuf[2 * kTok * kUStride + R * kWStride];
    unsigned char *sUh = sBuf;
    unsigned char *sUl = sBuf + kTok * kUStride;
    unsigned char *sW = sBuf + 2 * kTok * kUStride;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * kTok;
    const int c0 = blockIdx.y * kCols;
    for (int i = tid; i < kTok * R; i += 128) {
        const int tl = i / R, j = i % R;
        const int64_t t = tok0 + tl;
        const float val = t < ntok ? u[t * R + j] : 0.0f;
        uint16_t hi, lo;
        split_bf16(val, hi, lo);
        *reinterpret_cast<uint16_t *>(sUh + tl * kUStride + j * 2) = hi;
        *reinterpret_cast<uint16_t *>(sUl + tl * kUStride + j * 2) = lo;
    }
    for (int i = tid; i < R * (kCols / 8); i += 128) {
        const int j = i / (kCols / 8), ch = i % (kCols / 8);
        const int c = c0 + ch * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (c < d) v = *reinterpret_cast<const uint4 *>(w_down + static_cast<int64_t>(j) * d + c);
        *reinterpret_cast<uint4 *>(sW + j * kWStride + ch * 16) = v;
    }
    __syncthreads();
    float acc[kCols / 8][4];
#pragma unroll
    for (int n = 0; n < kCols / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < R / 16; ++ks) {
        uint32_t ah[4], al[4];
        const uint32_t aoff = (warp * 16 + (lane & 15)) * kUStride + (ks * 16 + (lane >> 4) * 8) * 2;
        ldmatrix_x4(ah, smem_u32(sUh) + aoff);
        ldmatrix_x4(al, smem_u32(sUl) + aoff);
#pragma unroll
        for (int p = 0; p < kCols / 16; ++p) {
            uint32_t bfr[4];
            const uint32_t boff = (ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kWStride +
                                  (p * 16 + (lane >> 4) * 8) * 2;
            ldmatrix_x4_trans(bfr, smem_u32(sW) + boff);
            mma_bf16_16816(acc[2 * p], ah, bfr[0], bfr[1]);
            mma_bf16_16816(acc[2 * p + 1], ah, bfr[2], bfr[3]);
            mma_bf16_16816(acc[2 * p], al, bfr[0], bfr[1]);
            mma_bf16_16816(acc[2 * p + 1], al, bfr[2], bfr[3]);
        }
    }
    // stage the fp32 tile in shared memory (reusing the operand buffers), 64
    // columns at a time, then write whole 16-B vectors of dx
    float *sOut = reinterpret_cast<float *>(sBuf);               // [kTok][kHalf + 4] fp32
    constexpr int kHalf = kCols / 2, kOS = kHalf + 4;
    static_assert(kTok * kOS * 4 <= 2 * kTok * kUStride + R * kWStride, "staging buffer");
    const int g = lane >> 2, q2 = (lane & 3) * 2;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        __syncthreads();
#pragma unroll
        for (int n = 0; n < kHalf / 8; ++n)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = warp * 16 + g + h * 8;
                sOut[row * kOS + n * 8 + q2] = acc[half * (kHalf / 8) + n][2 * h];
                sOut[row * kOS + n * 8 + q2 + 1] = acc[half * (kHalf / 8) + n][2 * h + 1];
            }
        __syncthreads();
        for (int i = threadIdx.x; i < kTok * (kHalf / 4); i += 128) {
            const int row = i / (kHalf / 4), c4 = (i % (kHalf / 4)) * 4;
            const int64_t t = tok0 + row;
            const int c = c0 + half * kHalf + c4;
            if (t >= ntok || c >= d) continue;
            float v[4] = {sOut[row * kOS + c4], sOut[row * kOS + c4 + 1], sOut[row * kOS + c4 + 2],
                          sOut[row * kOS + c4 + 3]};
            if (DXDT == MOM_BF16) {
                uint2 *p = reinterpret_cast<uint2 *>(reinterpret_cast<uint16_t *>(dx) + t * d + c);
                if (accumulate) {
                    const uint2 o = *p;
                    v[0] += __uint_as_float(o.x << 16);
                    v[1] += __uint_as_float(o.x & 0xFFFF0000u);
                    v[2] += __uint_as_float(o.y << 16);
                    v[3] += __uint_as_float(o.y & 0xFFFF0000u);
                }
                *p = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
            } else {
                float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(dx) + t * d + c);
                if (accumulate) {
                    const float4 o = *p;
                    v[0] += o.x; v[1] += o.y; v[2] += o.z; v[3] += o.w;
                }
                *p = make_float4(v[0], v[1], v[2], v[3]);
            }
        }
    }
}

// dWd[j, c] += sum_{t in chunk} u[t, j] * x[t, c]; CTA: 128 columns x 256 tokens,
// 4 warps x 32 columns, all R rows; fp32 atomics across token chunks.
template <int R, int XDT>
__global__ void __launch_bounds__(128)
route_bwd_dwdown_mma_kernel(const float *__restrict__ u, const typename Elem<XDT>::T *__restrict__ x,
                            int64_t ntok, int d, float *__restrict__ dw_down) {
    constexpr int kTok = 64;                    // tokens per smem step
    constexpr int kSteps = 4;                   // 256 tokens per CTA
    constexpr int kCols = 128;
    constexpr int kUStride = R * 2 + 16;
    constexpr int kXStride = kCols * 2 + 16;
    constexpr int MT = R / 16;
    __shared__ __align__(16) unsigned char sUh[kTok * kUStride];
    __shared__ __align__(16) unsigned char sUl[kTok * kUStride];
    __shared__ __align__(16) unsigned char sX[kTok * kXStride];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c0 = blockIdx.x * kCols;
    float acc[MT][4][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) acc[m][n][0] = acc[m][n][1] = acc[m][n][2] = acc[m][n][3] = 0.0f;
    for (int st = 0; st < kSteps; ++st) {
        const int64_t tok0 = (static_cast<int64_t>(blockIdx.y) * kSteps + st) * kTok;
        if (tok0 >= ntok) break;
        __syncthreads();
        for (int i = tid; i < kTok * R; i += 128) {
            const int tl = i / R, j = i % R;
            const int64_t t = tok0 + tl;
            const float val = t < ntok ? u[t * R + j] : 0.0f;
            uint16_t hi, lo;
            split_bf16(val, hi, lo);
            *reinterpret_cast<uint16_t *>(sUh + tl * kUStride + j * 2) = hi;
            *reinterpret_cast<uint16_t *>(sUl + tl * kUStride + j * 2) = lo;
        }
        for (int i = tid; i < kTok * (kCols / 8); i += 128) {
            const int tl = i / (kCols / 8), ch = i % (kCols / 8);
            const int64_t t = tok0 + tl;
            const int c = c0 + ch * 8;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (t < ntok && c < d) {
                if (XDT == MOM_BF16) {
                    v = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(x) + t * d + c);
                } else {
                    const float *xf = reinterpret_cast<const float *>(x) + t * d + c;
                    v.x = pack_bf16x2(xf[0], xf[1]);
                    v.y = pack_bf16x2(xf[2], xf[3]);
                    v.z = pack_bf16x2(xf[4], xf[5]);
                    v.w = pack_bf16x2(xf[6], xf[7]);
                }
            }
            *reinterpret_cast<uint4 *>(sX + tl * kXStride + ch * 16) = v;
        }
        __syncthreads();
#pragma unroll
        for (int ks = 0; ks < kTok / 16; ++ks) {
            uint32_t bfr[2][4];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const uint32_t boff = (ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kXStride +
                                      (warp * 32 + p * 16 + (lane >> 4) * 8) * 2;
                ldmatrix_x4_trans(bfr[p], smem_u32(sX) + boff);
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                uint32_t ah[4], al[4];
                const uint32_t aoff = (ks * 16 + (lane & 7) + (lane >> 4) * 8) * kUStride +
                                      (m * 16 + ((lane >> 3) & 1) * 8) * 2;
                ldmatrix_x4_trans(ah, smem_u32(sUh) + aoff);
                ldmatrix_x4_trans(al, smem_u32(sUl) + aoff);
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    mma_bf16_16816(acc[m][2 * p], ah, bfr[p][0], bfr[p][1]);
                    mma_bf16_16816(acc[m][2 * p + 1], ah, bfr[p][2], bfr[p][3]);
                    mma_bf16_16816(acc[m][2 * p], al, bfr[p][0], bfr[p][1]);
                    mma_bf16_16816(acc[m][2 * p + 1], al, bfr[p][2], bfr[p][3]);
                }
            }
        }
    }
    const int g = lane >> 2, q2 = (lane & 3) * 2;
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            const int c = c0 + warp * 32 + n * 8 + q2;
            if (c >= d) continue;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = m * 16 + g + h * 8;
                red_add_v2(dw_down + static_cast<int64_t>(j) * d + c, acc[m][n][2 * h], acc[m][n][2 * h + 1]);
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

// dWu[e, j] += sum_t dlogits[t, e] * act[t, j]; CTA = 256 tokens staged in smem.
template <int CDT>
__global__ void __launch_bounds__(256)
route_bwd_dwup_kernel(const float *__restrict__ dlogits, const typename Elem<CDT>::T *__restrict__ act,
                      int64_t ntok, int r, int nb, float *__restrict__ dw_up) {
    constexpr int kT = 64;
    __shared__ float sL[kT * kMaxNbB];
    __shared__ float sA[kT * kMaxRankB];
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * 256;
    float acc[32];
    const int nout = nb * r;
    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
    for (int tb = 0; tb < 256; tb += kT) {
        __syncthreads();
        for (int i = threadIdx.x; i < kT * nb; i += 256) {
            const int64_t t = t0 + tb + i / nb;
            sL[i] = t < ntok ? dlogits[t * nb + i % nb] : 0.0f;
        }
        for (int i = threadIdx.x; i < kT * r; i += 256) {
            const int64_t t = t0 + tb + i / r;
            sA[i] = t < ntok ? Elem<CDT>::load(act, t * r + i % r) : 0.0f;
        }
        __syncthreads();
        for (int o = threadIdx.x, oi = 0; o < nout; o += 256, ++oi) {
            const int e = o / r, j = o % r;
            float a = acc[oi];
            for (int tt = 0; tt < kT; ++tt) a = fmaf(sL[tt * nb + e], sA[tt * r + j], a);
            acc[oi] = a;
        }
    }
    for (int o = threadIdx.x, oi = 0; o < nout; o += 256, ++oi) atomicAdd(dw_up + o, acc[oi]);
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
    route_bwd_revscan_kernel<<<dim3((r + kRsCols - 1) / kRsCols, B), 1024, 0, st>>>(ws_dz, ws_u, S, r);
    count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // the tensor-core pair stores dx and reads x in 16-B vectors
    const bool tc = cdt == MOM_BF16 && (r == 32 || r == 64) && d % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(dx) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (tc) {
        dim3 grid(static_cast<unsigned>((ntok + 63) / 64), (d + 127) / 128);
#define MOM_DX_TC(R, X)                                                                              \
    if (r == R && dxdt == X)                                                                         \
        route_bwd_dx_mma_kernel<R, X><<<grid, 128, 0, st>>>(ws_u, static_cast<const uint16_t *>(w_down), \
                                                            ntok, d, static_cast<typename Elem<X>::T *>(dx), \
                                                            accumulate);
        MOM_DX_TC(32, MOM_BF16)
        MOM_DX_TC(32, MOM_F32)
        MOM_DX_TC(64, MOM_BF16)
        MOM_DX_TC(64, MOM_F32)
#undef MOM_DX_TC
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        dim3 grid2((d + 127) / 128, static_cast<unsigned>((ntok + 255) / 256));
#define MOM_DW_TC(R, X)                                                                              \
    if (r == R && xdt == X)                                                                          \
        route_bwd_dwdown_mma_kernel<R, X><<<grid2, 128, 0, st>>>(                                    \
            ws_u, static_cast<const typename Elem<X>::T *>(x), ntok, d, dw_down);
        MOM_DW_TC(32, MOM_BF16)
        MOM_DW_TC(32, MOM_F32)
        MOM_DW_TC(64, MOM_BF16)
        MOM_DW_TC(64, MOM_F32)
#undef MOM_DW_TC
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
    {
        const int grid = static_cast<int>((ntok + 255) / 256);
        if (cdt == MOM_BF16)
            route_bwd_dwup_kernel<MOM_BF16><<<grid, 256, 0, st>>>(
                ws_dlogits, static_cast<const uint16_t *>(act), ntok, r, nb, dw_up);
        else
            route_bwd_dwup_kernel<MOM_F32><<<grid, 256, 0, st>>>(
                ws_dlogits, static_cast<const float *>(act), ntok, r, nb, dw_up);
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace mom
