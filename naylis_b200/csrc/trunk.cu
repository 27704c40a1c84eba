// Fused bf16 kernels for the decoder trunk around the MoM read (the caller
// BASELINE config 3 trains): rotary embedding of the fused q/k/v projection and
// the SwiGLU gate, forward and backward, each one pass over HBM.
//
// Numerics follow what the reference's trunk computes under bf16 autocast
// (transformers' Llama: apply_rotary_pos_emb and LlamaMLP, as wired by
// model.py:280-348 of the reference):
//   RoPE     q, k come out of the projection in bf16; the rotation runs in fp32
//            with fp32 cos / sin (t * cos + rotate_half(t) * sin, each product
//            rounded, then the sum), and attention receives the result rounded
//            to bf16. Backward: dt = dout * cos + (rotate_half^T of dout * sin),
//            in fp32 from the bf16 attention gradient, rounded to bf16.
//   SwiGLU   a = bf16(silu(g)) with silu(x) = x / (1 + exp(-x)) in fp32, then
//            h = bf16(a * u). Backward: da = bf16(dh * u), du = bf16(dh * a),
//            dg = bf16(da * s * (1 + g * (1 - s))) with s = 1 / (1 + exp(-g)).
// No fused multiply-add is allowed to merge the rounded steps (explicit _rn
// intrinsics).
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace mom {
namespace {

__device__ __forceinline__ float bf(uint16_t b) { return bf16_bits_to_f32(b); }
__device__ __forceinline__ uint16_t tobf(float f) { return f32_to_bf16_bits(f); }

// Forward. qkv: (B*S, 3*H*hd) bf16, rows = tokens, columns [q | k | v], each H
// heads of hd. cos/sin: (S, hd) fp32. Out: q, k, v as (B, S, H, hd) bf16 (the
// token-major layout attention takes as a (B, H, S, hd) view).
// One thread per (token, head, pair i < hd/2): dims i and i + hd/2.
__global__ void __launch_bounds__(256)
rope_qkv_fwd_kernel(const uint16_t *__restrict__ qkv, const float *__restrict__ cosv, const float *__restrict__ sinv,
                    int B, int S, int H, int hd, uint16_t *__restrict__ q, uint16_t *__restrict__ k,
                    uint16_t *__restrict__ v) {
    const int half = hd / 2;
    const int64_t total = static_cast<int64_t>(B) * S * H * half;
    const int64_t d3 = 3LL * H * hd;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(i % half);
        const int64_t th = i / half;
        const int h = static_cast<int>(th % H);
        const int64_t tok = th / H;
        const int s = static_cast<int>(tok % S);
        const uint16_t *row = qkv + tok * d3 + static_cast<int64_t>(h) * hd;
        const float c1 = cosv[static_cast<int64_t>(s) * hd + p], c2 = cosv[static_cast<int64_t>(s) * hd + p + half];
        const float s1 = sinv[static_cast<int64_t>(s) * hd + p], s2 = sinv[static_cast<int64_t>(s) * hd + p + half];
        const int64_t o = (tok * H + h) * hd;
#pragma unroll
        for (int w = 0; w < 2; ++w) {   // q, then k
            const uint16_t *src = row + static_cast<int64_t>(w) * H * hd;
            const float x1 = bf(src[p]), x2 = bf(src[p + half]);
            // out[p] = x1*cos - x2*sin ; out[p+half] = x2*cos + x1*sin
            const float y1 = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(-x2, s1));
            const float y2 = __fadd_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s2));
            uint16_t *dst = (w == 0 ? q : k) + o;
            dst[p] = tobf(y1);
            dst[p + half] = tobf(y2);
        }
        const uint16_t *vs = row + 2LL * H * hd;
        v[o + p] = vs[p];
        v[o + p + half] = vs[p + half];
    }
}

// Backward: dq, dk, dv (B, S, H, hd) bf16 -> dqkv (B*S, 3*H*hd) bf16.
__global__ void __launch_bounds__(256)
rope_qkv_bwd_kernel(const uint16_t *__restrict__ dq, const uint16_t *__restrict__ dk, const uint16_t *__restrict__ dv,
                    const float *__restrict__ cosv, const float *__restrict__ sinv, int B, int S, int H, int hd,
                    uint16_t *__restrict__ dqkv) {
    const int half = hd / 2;
    const int64_t total = static_cast<int64_t>(B) * S * H * half;
    const int64_t d3 = 3LL * H * hd;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(i % half);
        const int64_t th = i / half;
        const int h = static_cast<int>(th % H);
        const int64_t tok = th / H;
        const int s = static_cast<int>(tok % S);
        uint16_t *row = dqkv + tok * d3 + static_cast<int64_t>(h) * hd;
        const float c1 = cosv[static_cast<int64_t>(s) * hd + p], c2 = cosv[static_cast<int64_t>(s) * hd + p + half];
        const float s1 = sinv[static_cast<int64_t>(s) * hd + p], s2 = sinv[static_cast<int64_t>(s) * hd + p + half];
        const int64_t o = (tok * H + h) * hd;
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint16_t *g = (w == 0 ? dq : dk) + o;
            const float g1 = bf(g[p]), g2 = bf(g[p + half]);
            // dx1 = g1*cos1 + g2*sin2 ; dx2 = g2*cos2 - g1*sin1
            const float d1 = __fadd_rn(__fmul_rn(g1, c1), __fmul_rn(g2, s2));
            const float d2 = __fadd_rn(__fmul_rn(g2, c2), -__fmul_rn(g1, s1));
            uint16_t *dst = row + static_cast<int64_t>(w) * H * hd;
            dst[p] = tobf(d1);
            dst[p + half] = tobf(d2);
        }
        uint16_t *dvd = row + 2LL * H * hd;
        dvd[p] = dv[o + p];
        dvd[p + half] = dv[o + p + half];
    }
}

__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// gu: (N, 2f) bf16 rows [g | u] -> h (N, f) bf16. Two columns per thread.
__global__ void __launch_bounds__(256)
swiglu_fwd_kernel(const uint32_t *__restrict__ gu, int64_t N, int f, uint32_t *__restrict__ h) {
    const int fp = f / 2;
    const int64_t total = N * fp;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / fp;
        const int c = static_cast<int>(i - t * fp);
        const uint32_t gw = gu[t * 2 * fp + c], uw = gu[t * 2 * fp + fp + c];
        float r[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float g = j ? __uint_as_float(gw & 0xFFFF0000u) : __uint_as_float(gw << 16);
            const float u = j ? __uint_as_float(uw & 0xFFFF0000u) : __uint_as_float(uw << 16);
            const float a = bf(tobf(silu_f(g)));
            r[j] = __fmul_rn(a, u);
        }
        h[t * fp + c] = pack_bf16x2(r[0], r[1]);
    }
}

// dh (N, f) bf16, gu (N, 2f) -> dgu (N, 2f) bf16 rows [dg | du].
__global__ void __launch_bounds__(256)
swiglu_bwd_kernel(const uint32_t *__restrict__ dh, const uint32_t *__restrict__ gu, int64_t N, int f,
                  uint32_t *__restrict__ dgu) {
    const int fp = f / 2;
    const int64_t total = N * fp;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / fp;
        const int c = static_cast<int>(i - t * fp);
        const uint32_t gw = gu[t * 2 * fp + c], uw = gu[t * 2 * fp + fp + c], dw = dh[t * fp + c];
        float dg[2], du[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float g = j ? __uint_as_float(gw & 0xFFFF0000u) : __uint_as_float(gw << 16);
            const float u = j ? __uint_as_float(uw & 0xFFFF0000u) : __uint_as_float(uw << 16);
            const float d = j ? __uint_as_float(dw & 0xFFFF0000u) : __uint_as_float(dw << 16);
            const float a = bf(tobf(silu_f(g)));
            const float da = bf(tobf(__fmul_rn(d, u)));
            du[j] = __fmul_rn(d, a);
            const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
            dg[j] = __fmul_rn(__fmul_rn(da, sg), __fadd_rn(1.0f, __fmul_rn(g, __fsub_rn(1.0f, sg))));
        }
        dgu[t * 2 * fp + c] = pack_bf16x2(dg[0], dg[1]);
        dgu[t * 2 * fp + fp + c] = pack_bf16x2(du[0], du[1]);
    }
}

int grid_of(int64_t work) { return static_cast<int>(std::min<int64_t>((work + 255) / 256, 148 * 16)); }

// ---- 16-byte forms of the same kernels (8 bf16 per access), used when the
// widths are multiples of 8 and the rows 16-byte aligned; same arithmetic.
__device__ __forceinline__ void unpack8(uint4 w, float (&f)[8]) {
    const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(a[i] << 16);
        f[2 * i + 1] = __uint_as_float(a[i] & 0xFFFF0000u);
    }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
}

// (token, head, group of 8 pairs) of flat item i = (tok * H + h) * ng + p / 8, with 32-bit
// unsigned divisions when the index fits (a 64-bit division costs several times as many
// instructions, and these kernels do little else per item)
__device__ __forceinline__ void rope_index(int64_t i, bool small, int ng, int H, int S, int &p, int &h,
                                           int64_t &tok, int &s) {
    if (small) {
        const uint32_t u = static_cast<uint32_t>(i), th = u / static_cast<uint32_t>(ng);
        const uint32_t t = th / static_cast<uint32_t>(H);
        p = static_cast<int>(u - th * static_cast<uint32_t>(ng)) * 8;
        h = static_cast<int>(th - t * static_cast<uint32_t>(H));
        tok = t;
        s = static_cast<int>(t % static_cast<uint32_t>(S));
    } else {
        const int64_t th = i / ng;
        p = static_cast<int>(i - th * ng) * 8;
        tok = th / H;
        h = static_cast<int>(th - tok * H);
        s = static_cast<int>(tok % S);
    }
}

// one thread per (token, head, 8 pairs)
__global__ void __launch_bounds__(256)
rope_qkv_fwd_v8_kernel(const uint16_t *__restrict__ qkv, const float *__restrict__ cosv, const float *__restrict__ sinv,
                       int B, int S, int H, int hd, uint16_t *__restrict__ q, uint16_t *__restrict__ k,
                       uint16_t *__restrict__ v) {
    const int half = hd / 2, ng = half / 8;
    const int64_t total = static_cast<int64_t>(B) * S * H * ng;
    const bool small = total <= 0xFFFFFFFFLL;   // the index fits 32 bits: cheaper divisions
    const int64_t d3 = 3LL * H * hd;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int p, h, s;
        int64_t tok;
        rope_index(i, small, ng, H, S, p, h, tok, s);
        const uint16_t *row = qkv + tok * d3 + static_cast<int64_t>(h) * hd;
        const float *cs = cosv + static_cast<int64_t>(s) * hd, *sn = sinv + static_cast<int64_t>(s) * hd;
        float c1[8], c2[8], s1[8], s2[8];
#pragma unroll
        for (int j = 0; j < 8; j += 4) {
            *reinterpret_cast<float4 *>(c1 + j) = *reinterpret_cast<const float4 *>(cs + p + j);
            *reinterpret_cast<float4 *>(c2 + j) = *reinterpret_cast<const float4 *>(cs + p + half + j);
            *reinterpret_cast<float4 *>(s1 + j) = *reinterpret_cast<const float4 *>(sn + p + j);
            *reinterpret_cast<float4 *>(s2 + j) = *reinterpret_cast<const float4 *>(sn + p + half + j);
        }
        const int64_t o = (tok * H + h) * hd;
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint16_t *src = row + static_cast<int64_t>(w) * H * hd;
            float x1[8], x2[8], y1[8], y2[8];
            unpack8(*reinterpret_cast<const uint4 *>(src + p), x1);
            unpack8(*reinterpret_cast<const uint4 *>(src + p + half), x2);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                y1[j] = __fadd_rn(__fmul_rn(x1[j], c1[j]), __fmul_rn(-x2[j], s1[j]));
                y2[j] = __fadd_rn(__fmul_rn(x2[j], c2[j]), __fmul_rn(x1[j], s2[j]));
            }
            uint16_t *dst = (w == 0 ? q : k) + o;
            *reinterpret_cast<uint4 *>(dst + p) = pack8(y1);
            *reinterpret_cast<uint4 *>(dst + p + half) = pack8(y2);
        }
        const uint16_t *vs = row + 2LL * H * hd;
        *reinterpret_cast<uint4 *>(v + o + p) = *reinterpret_cast<const uint4 *>(vs + p);
        *reinterpret_cast<uint4 *>(v + o + p + half) = *reinterpret_cast<const uint4 *>(vs + p + half);
    }
}

__global__ void __launch_bounds__(256)
rope_qkv_bwd_v8_kernel(const uint16_t *__restrict__ dq, const uint16_t *__restrict__ dk,
                       const uint16_t *__restrict__ dv, const float *__restrict__ cosv,
                       const float *__restrict__ sinv, int B, int S, int H, int hd, uint16_t *__restrict__ dqkv) {
    const int half = hd / 2, ng = half / 8;
    const int64_t total = static_cast<int64_t>(B) * S * H * ng;
    const bool small = total <= 0xFFFFFFFFLL;   // the index fits 32 bits: cheaper divisions
    const int64_t d3 = 3LL * H * hd;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int p, h, s;
        int64_t tok;
        rope_index(i, small, ng, H, S, p, h, tok, s);
        uint16_t *row = dqkv + tok * d3 + static_cast<int64_t>(h) * hd;
        const float *cs = cosv + static_cast<int64_t>(s) * hd, *sn = sinv + static_cast<int64_t>(s) * hd;
        float c1[8], c2[8], s1[8], s2[8];
#pragma unroll
        for (int j = 0; j < 8; j += 4) {
            *reinterpret_cast<float4 *>(c1 + j) = *reinterpret_cast<const float4 *>(cs + p + j);
            *reinterpret_cast<float4 *>(c2 + j) = *reinterpret_cast<const float4 *>(cs + p + half + j);
            *reinterpret_cast<float4 *>(s1 + j) = *reinterpret_cast<const float4 *>(sn + p + j);
            *reinterpret_cast<float4 *>(s2 + j) = *reinterpret_cast<const float4 *>(sn + p + half + j);
        }
        const int64_t o = (tok * H + h) * hd;
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint16_t *g = (w == 0 ? dq : dk) + o;
            float g1[8], g2[8], d1[8], d2[8];
            unpack8(*reinterpret_cast<const uint4 *>(g + p), g1);
            unpack8(*reinterpret_cast<const uint4 *>(g + p + half), g2);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                d1[j] = __fadd_rn(__fmul_rn(g1[j], c1[j]), __fmul_rn(g2[j], s2[j]));
                d2[j] = __fadd_rn(__fmul_rn(g2[j], c2[j]), -__fmul_rn(g1[j], s1[j]));
            }
            uint16_t *dst = row + static_cast<int64_t>(w) * H * hd;
            *reinterpret_cast<uint4 *>(dst + p) = pack8(d1);
            *reinterpret_cast<uint4 *>(dst + p + half) = pack8(d2);
        }
        uint16_t *dvd = row + 2LL * H * hd;
        *reinterpret_cast<uint4 *>(dvd + p) = *reinterpret_cast<const uint4 *>(dv + o + p);
        *reinterpret_cast<uint4 *>(dvd + p + half) = *reinterpret_cast<const uint4 *>(dv + o + p + half);
    }
}

// 8 columns per thread
// The flat index i = t * fv + c of a grid-stride loop, advanced by the grid's
// thread count without a 64-bit division per step (SwiGLU is issue-bound: the
// division cost about as many instructions as the arithmetic of a vector).
struct RowWalk {
    int64_t t, dt;
    int c, dc, fv;
    __device__ RowWalk(int64_t i0, int64_t stride, int fv_) : fv(fv_) {
        t = i0 / fv;
        c = static_cast<int>(i0 - t * fv);
        dt = stride / fv;
        dc = static_cast<int>(stride - dt * fv);
    }
    __device__ __forceinline__ void next() {
        t += dt;
        c += dc;
        if (c >= fv) { c -= fv; ++t; }
    }
};

__device__ __forceinline__ uint4 swiglu8(uint4 gw, uint4 uw) {
    float g[8], u[8], r[8];
    unpack8(gw, g);
    unpack8(uw, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __fmul_rn(bf(tobf(silu_f(g[j]))), u[j]);
    return pack8(r);
}

// Two vectors per round, both loaded before either is computed.
__global__ void __launch_bounds__(256)
swiglu_fwd_v8_kernel(const uint4 *__restrict__ gu, int64_t N, int f, uint4 *__restrict__ h) {
    const int fv = f / 8;
    RowWalk w(static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x,
              static_cast<int64_t>(gridDim.x) * blockDim.x, fv);
    while (w.t < N) {
        const int64_t t0 = w.t;
        const int c0 = w.c;
        w.next();
        const int64_t t1 = w.t;
        const int c1 = w.c;
        const bool two = t1 < N;
        const uint4 g0 = gu[t0 * 2 * fv + c0], u0 = gu[t0 * 2 * fv + fv + c0];
        uint4 g1 = make_uint4(0, 0, 0, 0), u1 = g1;
        if (two) {
            g1 = gu[t1 * 2 * fv + c1];
            u1 = gu[t1 * 2 * fv + fv + c1];
        }
        h[t0 * fv + c0] = swiglu8(g0, u0);
        if (two) h[t1 * fv + c1] = swiglu8(g1, u1);
        w.next();
    }
}

__device__ __forceinline__ void swiglu_bwd8(uint4 gw, uint4 uw, uint4 dw, uint4 &dgw, uint4 &duw) {
    float g[8], u[8], d[8], dg[8], du[8];
    unpack8(gw, g);
    unpack8(uw, u);
    unpack8(dw, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        // one exp per element: silu(g) = g / (1 + e^-g), sigmoid = 1 / (1 + e^-g)
        const float den = __fadd_rn(1.0f, expf(-g[j]));
        const float a = bf(tobf(__fdiv_rn(g[j], den)));
        const float da = bf(tobf(__fmul_rn(d[j], u[j])));
        du[j] = __fmul_rn(d[j], a);
        const float sg = __fdiv_rn(1.0f, den);
        dg[j] = __fmul_rn(__fmul_rn(da, sg), __fadd_rn(1.0f, __fmul_rn(g[j], __fsub_rn(1.0f, sg))));
    }
    dgw = pack8(dg);
    duw = pack8(du);
}

__global__ void __launch_bounds__(256)
swiglu_bwd_v8_kernel(const uint4 *__restrict__ dh, const uint4 *__restrict__ gu, int64_t N, int f,
                     uint4 *__restrict__ dgu) {
    const int fv = f / 8;
    RowWalk w(static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x,
              static_cast<int64_t>(gridDim.x) * blockDim.x, fv);
    while (w.t < N) {
        const int64_t t0 = w.t;
        const int c0 = w.c;
        w.next();
        const int64_t t1 = w.t;
        const int c1 = w.c;
        const bool two = t1 < N;
        const uint4 g0 = gu[t0 * 2 * fv + c0], u0 = gu[t0 * 2 * fv + fv + c0], d0 = dh[t0 * fv + c0];
        uint4 g1 = make_uint4(0, 0, 0, 0), u1 = g1, d1 = g1;
        if (two) {
            g1 = gu[t1 * 2 * fv + c1];
            u1 = gu[t1 * 2 * fv + fv + c1];
            d1 = dh[t1 * fv + c1];
        }
        uint4 dg, du;
        swiglu_bwd8(g0, u0, d0, dg, du);
        dgu[t0 * 2 * fv + c0] = dg;
        dgu[t0 * 2 * fv + fv + c0] = du;
        if (two) {
            swiglu_bwd8(g1, u1, d1, dg, du);
            dgu[t1 * 2 * fv + c1] = dg;
            dgu[t1 * 2 * fv + fv + c1] = du;
        }
        w.next();
    }
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ------------------------------------------------------------------ residual add + RMSNorm
// x_new = x + scale * delta (the sublayer's output added to the fp32 residual
// stream; scale is a device scalar or absent), then the Llama RMSNorm of x_new:
// y = w * (x_new * rsqrt(mean(x_new^2) + eps)), returned as bf16 (the next GEMM's
// input) and, when asked, as fp32 (the MoM router's input). A warp per token;
// each lane holds NV vectors of 4 columns (columns 4*lane + 128*j), and every
// load of a token is issued before any of its values is used (the loads, not
// the arithmetic, bound this kernel). r = rsqrt(...) is saved per token.
constexpr int kNormWarps = 8;

template <int DDT>   // delta: 0 none, 1 bf16, 2 fp32
__device__ __forceinline__ float4 load_delta4(const void *delta, int64_t i) {
    if (DDT == 1) {
        const uint2 w = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(delta) + i);
        return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u),
                           __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xFFFF0000u));
    }
    if (DDT == 2) return *reinterpret_cast<const float4 *>(static_cast<const float *>(delta) + i);
    return make_float4(0.f, 0.f, 0.f, 0.f);
}

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
__device__ __forceinline__ float4 bf4(const uint16_t *p) {
    const uint2 w = *reinterpret_cast<const uint2 *>(p);
    return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u), __uint_as_float(w.y << 16),
                       __uint_as_float(w.y & 0xFFFF0000u));
}
__device__ __forceinline__ void stbf4(uint16_t *p, float4 v) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

template <int DDT, int NV>
__global__ void __launch_bounds__(32 * kNormWarps)
add_rmsnorm_fwd_kernel(const float *__restrict__ x, const void *__restrict__ delta, const float *__restrict__ dscale,
                       const float *__restrict__ w, int64_t N, int d, float eps, float *__restrict__ x_out,
                       uint16_t *__restrict__ y16, float *__restrict__ y32, float *__restrict__ rstd) {
    const int lane = threadIdx.x & 31;
    const float sc = (DDT != 0 && dscale) ? *dscale : 1.0f;
    float4 wv[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) wv[j] = ld4(w + 4 * lane + 128 * j);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kNormWarps + (threadIdx.x >> 5); t < N;
         t += static_cast<int64_t>(gridDim.x) * kNormWarps) {
        const int64_t base = t * d + 4 * lane;
        float4 a[NV], b[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            a[j] = ld4(x + base + 128 * j);
            b[j] = load_delta4<DDT>(delta, base + 128 * j);
        }
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            if (DDT != 0) {
                float4 dd = b[j];
                if (dscale) dd = make_float4(__fmul_rn(sc, dd.x), __fmul_rn(sc, dd.y), __fmul_rn(sc, dd.z),
                                             __fmul_rn(sc, dd.w));
                a[j] = make_float4(__fadd_rn(a[j].x, dd.x), __fadd_rn(a[j].y, dd.y), __fadd_rn(a[j].z, dd.z),
                                   __fadd_rn(a[j].w, dd.w));
            }
            st4(x_out + base + 128 * j, a[j]);
            ss = __fmaf_rn(a[j].x, a[j].x, ss);
            ss = __fmaf_rn(a[j].y, a[j].y, ss);
            ss = __fmaf_rn(a[j].z, a[j].z, ss);
            ss = __fmaf_rn(a[j].w, a[j].w, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(d)), eps));
        if (lane == 0) rstd[t] = r;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const float4 yv = make_float4(__fmul_rn(wv[j].x, __fmul_rn(a[j].x, r)), __fmul_rn(wv[j].y, __fmul_rn(a[j].y, r)),
                                          __fmul_rn(wv[j].z, __fmul_rn(a[j].z, r)), __fmul_rn(wv[j].w, __fmul_rn(a[j].w, r)));
            stbf4(y16 + base + 128 * j, yv);
            if (y32) st4(y32 + base + 128 * j, yv);
        }
    }
}

// Named barrier `id` (1..15) over `nthreads` threads of the CTA.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

// Backward of add_rmsnorm. dy = dy16 (+ dy32), g = dy * w, xh = x_new * r:
//   d(x_new) = dx_in + r * (g - xh * mean(g * xh))      (dx_in: the residual's own gradient)
//   dx = d(x_new), d(delta) = scale * d(x_new), dw += dy * xh, dscale += sum d(x_new) * delta
// SPLIT warps share a token, each holding d / SPLIT columns (NV vectors of 4 per
// lane): with SPLIT = 2 the registers a lane needs halve and twice as many warps
// are resident to cover the loads' latency; the two partial sums of g * xh meet
// in shared memory behind a named barrier of the warp pair (double-buffered by
// token parity, so a warp one token ahead never overwrites a value its partner
// has yet to read) and both warps add them in the same order.
// dw and dscale are kept per lane across the warp's tokens, reduced per CTA in
// shared memory and added to global memory with one atomic each.
template <int DDT, int NV, int SPLIT>
__global__ void __launch_bounds__(32 * kNormWarps)
add_rmsnorm_bwd_kernel(const float *__restrict__ x_new, const float *__restrict__ rstd, const float *__restrict__ w,
                       const void *__restrict__ delta, const float *__restrict__ dscale_in,
                       const uint16_t *__restrict__ dy16, const float *__restrict__ dy32,
                       const float *__restrict__ dx_in, int64_t N, int d, float *__restrict__ dx,
                       void *__restrict__ ddelta, float *__restrict__ dw, float *__restrict__ dscale) {
    static_assert(SPLIT == 1 || SPLIT == 2, "one or two warps per token");
    constexpr int kGroups = kNormWarps / SPLIT;     // tokens in flight per CTA
    extern __shared__ float sdw[];                  // [d] + [1] + partial dots [kGroups][2][SPLIT]
    float *sdot = sdw + d + 1;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = warp / SPLIT, part = warp % SPLIT;
    const int col0 = part * (d / SPLIT) + 4 * lane;
    for (int c = threadIdx.x; c <= d; c += blockDim.x) sdw[c] = 0.0f;
    __syncthreads();
    const float sc = (DDT != 0 && dscale_in) ? *dscale_in : 1.0f;
    float4 wv[NV], aw[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        wv[j] = ld4(w + col0 + 128 * j);
        aw[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float acc_s = 0.0f;
    int slot = 0;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kGroups + grp; t < N;
         t += static_cast<int64_t>(gridDim.x) * kGroups) {
        const int64_t base = t * d + col0;
        const float r = rstd[t];
        float4 xv[NV], gv[NV], rv[NV], dl[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int64_t o = base + 128 * j;
            xv[j] = ld4(x_new + o);
            gv[j] = dy16 ? bf4(dy16 + o) : make_float4(0.f, 0.f, 0.f, 0.f);
            rv[j] = dy32 ? ld4(dy32 + o) : make_float4(0.f, 0.f, 0.f, 0.f);
            dl[j] = dx_in ? ld4(dx_in + o) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float dot = 0.0f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            float4 dyv = make_float4(gv[j].x + rv[j].x, gv[j].y + rv[j].y, gv[j].z + rv[j].z, gv[j].w + rv[j].w);
            const float4 xh = make_float4(xv[j].x * r, xv[j].y * r, xv[j].z * r, xv[j].w * r);
            aw[j].x = fmaf(dyv.x, xh.x, aw[j].x); aw[j].y = fmaf(dyv.y, xh.y, aw[j].y);
            aw[j].z = fmaf(dyv.z, xh.z, aw[j].z); aw[j].w = fmaf(dyv.w, xh.w, aw[j].w);
            gv[j] = make_float4(dyv.x * wv[j].x, dyv.y * wv[j].y, dyv.z * wv[j].z, dyv.w * wv[j].w);
            xv[j] = xh;
            dot = fmaf(gv[j].x, xh.x, fmaf(gv[j].y, xh.y, fmaf(gv[j].z, xh.z, fmaf(gv[j].w, xh.w, dot))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (SPLIT == 2) {
            float *pd = sdot + (grp * 2 + slot) * 2;
            if (lane == 0) pd[part] = dot;
            named_bar_sync(1 + grp, 64);
            dot = pd[0] + pd[1];
            slot ^= 1;
        }
        const float mean = dot / static_cast<float>(d);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int64_t o = base + 128 * j;
            const float4 gx = make_float4(fmaf(r, gv[j].x - xv[j].x * mean, dl[j].x),
                                          fmaf(r, gv[j].y - xv[j].y * mean, dl[j].y),
                                          fmaf(r, gv[j].z - xv[j].z * mean, dl[j].z),
                                          fmaf(r, gv[j].w - xv[j].w * mean, dl[j].w));
            st4(dx + o, gx);
            if (DDT != 0) {
                const float4 dd = dscale_in ? make_float4(sc * gx.x, sc * gx.y, sc * gx.z, sc * gx.w) : gx;
                if (dscale) {
                    const float4 dv = load_delta4<DDT>(delta, o);
                    acc_s = fmaf(gx.x, dv.x, fmaf(gx.y, dv.y, fmaf(gx.z, dv.z, fmaf(gx.w, dv.w, acc_s))));
                }
                if (DDT == 1) stbf4(static_cast<uint16_t *>(ddelta) + o, dd);
                else st4(static_cast<float *>(ddelta) + o, dd);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int c = col0 + 128 * j;
        atomicAdd(&sdw[c], aw[j].x);
        atomicAdd(&sdw[c + 1], aw[j].y);
        atomicAdd(&sdw[c + 2], aw[j].z);
        atomicAdd(&sdw[c + 3], aw[j].w);
    }
    if (DDT != 0 && dscale) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc_s += __shfl_xor_sync(0xffffffffu, acc_s, o);
        if (lane == 0) atomicAdd(&sdw[d], acc_s);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < d; c += blockDim.x) atomicAdd(dw + c, sdw[c]);
    if (DDT != 0 && dscale && threadIdx.x == 0) atomicAdd(dscale, sdw[d]);
}

// ---------------------------------------------------------------- LM-head cross-entropy
// The reference's loss (model.py:539-551): the LM head's logits (R, V) as the
// bf16 autocast GEMM leaves them, upcast to fp32, cross_entropy(reduction="sum")
// over the rows whose label is not ignore_index, divided by their count (the
// division stays in torch). Forward, one CTA per row: each thread keeps a running
// (max m, sum s of e^(x - m)) over 16-byte vectors of the row, the CTA combines
// them, lse = m + ln(s), row loss = lse - x[label] (0 on ignored rows, NaN when
// the label is outside [0, V)). The row is read once; the fp32 log-softmax torch
// materialises (and its cast) are never formed. Backward: dlogits =
// bf16((e^(x - lse) - [j == label]) * g) with g the gradient of the sum, 0 on
// ignored rows (what torch's log-softmax / nll backward and the cast to the
// GEMM's bf16 give).
constexpr int kXentThreads = 256;

__device__ __forceinline__ void xent_merge(float &m, float &s, float m2, float s2) {
    const float mm = fmaxf(m, m2);
    if (mm == -INFINITY) return;   // both empty
    s = s * exp2f((m - mm) * kLog2e) + s2 * exp2f((m2 - mm) * kLog2e);
    m = mm;
}

__device__ __forceinline__ void xent_add(float &m, float &s, const float (&x)[8]) {
    float mx = x[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, x[i]);
    if (mx > m) {
        s = (m == -INFINITY) ? 0.0f : s * exp2f((m - mx) * kLog2e);
        m = mx;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) s += exp2f((x[i] - m) * kLog2e);
}

template <bool kVec>
__global__ void __launch_bounds__(kXentThreads)
xent_fwd_kernel(const uint16_t *__restrict__ logits, const int64_t *__restrict__ labels, int64_t R, int V,
                int64_t ignore_index, float *__restrict__ row_loss, float *__restrict__ lse_out) {
    __shared__ float sm[kXentThreads / 32], ss[kXentThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
        const uint16_t *row = logits + r * V;
        float m = -INFINITY, s = 0.0f;
        if constexpr (kVec) {
            const uint4 *rv = reinterpret_cast<const uint4 *>(row);
            const int nv = V / 8;
            int j = threadIdx.x;
            // two vectors in flight per thread
            for (; j + kXentThreads < nv; j += 2 * kXentThreads) {
                const uint4 a = __ldcs(rv + j), b = __ldcs(rv + j + kXentThreads);
                float xa[8], xb[8];
                unpack8(a, xa);
                unpack8(b, xb);
                xent_add(m, s, xa);
                xent_add(m, s, xb);
            }
            if (j < nv) {
                float xa[8];
                unpack8(__ldcs(rv + j), xa);
                xent_add(m, s, xa);
            }
        } else {
            for (int j = threadIdx.x; j < V; j += kXentThreads) {
                const float x = bf(row[j]);
                if (x > m) {
                    s = (m == -INFINITY) ? 0.0f : s * exp2f((m - x) * kLog2e);
                    m = x;
                }
                s += exp2f((x - m) * kLog2e);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
            xent_merge(m, s, m2, s2);
        }
        if (lane == 0) {
            sm[warp] = m;
            ss[warp] = s;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float M = sm[0], Ssum = ss[0];
            for (int w = 1; w < kXentThreads / 32; ++w) xent_merge(M, Ssum, sm[w], ss[w]);
            const float l = M + logf(Ssum);
            const int64_t lab = labels[r];
            float loss = 0.0f;
            if (lab != ignore_index) loss = (lab >= 0 && lab < V) ? l - bf(row[lab]) : __int_as_float(0x7fc00000);
            row_loss[r] = loss;
            lse_out[r] = l;
        }
        __syncthreads();
    }
}

template <bool kVec>
__global__ void __launch_bounds__(kXentThreads)
xent_bwd_kernel(const uint16_t *__restrict__ logits, const int64_t *__restrict__ labels,
                const float *__restrict__ lse, const float *__restrict__ grad, int64_t R, int V, int64_t ignore_index,
                uint16_t *__restrict__ dlogits) {
    const float g = *grad;
    for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
        const int64_t lab = labels[r];
        const bool ignored = lab == ignore_index;
        const bool bad = !ignored && (lab < 0 || lab >= V);
        const float l = lse[r];
        const uint16_t *row = logits + r * V;
        uint16_t *drow = dlogits + r * V;
        auto grad_of = [&](float x, int j) -> float {
            if (ignored) return 0.0f;
            if (bad) return __int_as_float(0x7fc00000);
            // x - lse first (exact when they are close, where p - 1 cancels), then the exponential
            const float p = exp2f((x - l) * kLog2e);
            return (j == lab ? p - 1.0f : p) * g;
        };
        if constexpr (kVec) {
            const uint4 *rv = reinterpret_cast<const uint4 *>(row);
            uint4 *dv = reinterpret_cast<uint4 *>(drow);
            const int nv = V / 8;
            for (int j = threadIdx.x; j < nv; j += kXentThreads) {
                float x[8];
                unpack8(__ldcs(rv + j), x);
                uint32_t o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    o[i] = static_cast<uint32_t>(tobf(grad_of(x[2 * i], 8 * j + 2 * i))) |
                           (static_cast<uint32_t>(tobf(grad_of(x[2 * i + 1], 8 * j + 2 * i + 1))) << 16);
                __stcs(dv + j, make_uint4(o[0], o[1], o[2], o[3]));
            }
        } else {
            for (int j = threadIdx.x; j < V; j += kXentThreads) drow[j] = tobf(grad_of(bf(row[j]), j));
        }
    }
}

}  // namespace

cudaError_t launch_rope_qkv_fwd(const void *qkv, const float *cosv, const float *sinv, int B, int S, int H, int hd,
                                void *q, void *k, void *v, cudaStream_t st) {
    const int64_t work = static_cast<int64_t>(B) * S * H * (hd / 2);
    if (work == 0) return cudaSuccess;
    if (hd % 16 == 0 && al16(qkv) && al16(q) && al16(k) && al16(v) && al16(cosv) && al16(sinv)) {
        rope_qkv_fwd_v8_kernel<<<grid_of(work / 8), 256, 0, st>>>(
            static_cast<const uint16_t *>(qkv), cosv, sinv, B, S, H, hd, static_cast<uint16_t *>(q),
            static_cast<uint16_t *>(k), static_cast<uint16_t *>(v));
        count_launch();
        return cudaGetLastError();
    }
    rope_qkv_fwd_kernel<<<grid_of(work), 256, 0, st>>>(static_cast<const uint16_t *>(qkv), cosv, sinv, B, S, H, hd,
                                                       static_cast<uint16_t *>(q), static_cast<uint16_t *>(k),
                                                       static_cast<uint16_t *>(v));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_rope_qkv_bwd(const void *dq, const void *dk, const void *dv, const float *cosv, const float *sinv,
                                int B, int S, int H, int hd, void *dqkv, cudaStream_t st) {
    const int64_t work = static_cast<int64_t>(B) * S * H * (hd / 2);
    if (work == 0) return cudaSuccess;
    if (hd % 16 == 0 && al16(dq) && al16(dk) && al16(dv) && al16(dqkv) && al16(cosv) && al16(sinv)) {
        rope_qkv_bwd_v8_kernel<<<grid_of(work / 8), 256, 0, st>>>(
            static_cast<const uint16_t *>(dq), static_cast<const uint16_t *>(dk), static_cast<const uint16_t *>(dv),
            cosv, sinv, B, S, H, hd, static_cast<uint16_t *>(dqkv));
        count_launch();
        return cudaGetLastError();
    }
    rope_qkv_bwd_kernel<<<grid_of(work), 256, 0, st>>>(static_cast<const uint16_t *>(dq),
                                                       static_cast<const uint16_t *>(dk),
                                                       static_cast<const uint16_t *>(dv), cosv, sinv, B, S, H, hd,
                                                       static_cast<uint16_t *>(dqkv));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_swiglu_fwd(const void *gu, int64_t N, int f, void *h, cudaStream_t st) {
    const int64_t work = N * (f / 2);
    if (work == 0) return cudaSuccess;
    if (f % 8 == 0 && al16(gu) && al16(h)) {
        swiglu_fwd_v8_kernel<<<grid_of(work / 4), 256, 0, st>>>(static_cast<const uint4 *>(gu), N, f,
                                                                 static_cast<uint4 *>(h));
        count_launch();
        return cudaGetLastError();
    }
    swiglu_fwd_kernel<<<grid_of(work), 256, 0, st>>>(static_cast<const uint32_t *>(gu), N, f,
                                                     static_cast<uint32_t *>(h));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_swiglu_bwd(const void *dh, const void *gu, int64_t N, int f, void *dgu, cudaStream_t st) {
    const int64_t work = N * (f / 2);
    if (work == 0) return cudaSuccess;
    if (f % 8 == 0 && al16(dh) && al16(gu) && al16(dgu)) {
        swiglu_bwd_v8_kernel<<<grid_of(work / 4), 256, 0, st>>>(static_cast<const uint4 *>(dh),
                                                                 static_cast<const uint4 *>(gu), N, f,
                                                                 static_cast<uint4 *>(dgu));
        count_launch();
        return cudaGetLastError();
    }
    swiglu_bwd_kernel<<<grid_of(work), 256, 0, st>>>(static_cast<const uint32_t *>(dh),
                                                     static_cast<const uint32_t *>(gu), N, f,
                                                     static_cast<uint32_t *>(dgu));
    count_launch();
    return cudaGetLastError();
}

// d = 128, 256, 512, 1024 or 2048: d / 128 vectors of 4 columns per lane in registers.
cudaError_t launch_add_rmsnorm_fwd(const float *x, const void *delta, int ddt, const float *dscale, const float *w,
                                   int64_t N, int d, float eps, float *x_out, void *y16, float *y32, float *rstd,
                                   cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    if (d % 128 || d > 2048 || ddt < 0 || ddt > 2) return cudaErrorInvalidValue;
    const int blocks = static_cast<int>(std::min<int64_t>((N + kNormWarps - 1) / kNormWarps, 148 * 8));
    auto out16 = static_cast<uint16_t *>(y16);
    const int nv = d / 128;
#define MOM_NORM_F(DDT, NVV)                                                                                   \
    add_rmsnorm_fwd_kernel<DDT, NVV><<<blocks, 32 * kNormWarps, 0, st>>>(x, delta, dscale, w, N, d, eps, x_out, \
                                                                         out16, y32, rstd)
#define MOM_NORM_FD(NVV) \
    if (ddt == 0) MOM_NORM_F(0, NVV); else if (ddt == 1) MOM_NORM_F(1, NVV); else MOM_NORM_F(2, NVV);
    if (nv == 8) { MOM_NORM_FD(8) } else if (nv == 16) { MOM_NORM_FD(16) } else if (nv == 4) { MOM_NORM_FD(4) }
    else if (nv == 2) { MOM_NORM_FD(2) } else if (nv == 1) { MOM_NORM_FD(1) } else { return cudaErrorInvalidValue; }
#undef MOM_NORM_FD
#undef MOM_NORM_F
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_add_rmsnorm_bwd(const float *x_new, const float *rstd, const float *w, const void *delta, int ddt,
                                   const float *dscale_in, const void *dy16, const float *dy32, const float *dx_in,
                                   int64_t N, int d, float *dx, void *ddelta, float *dw, float *dscale,
                                   cudaStream_t st) {
    if (d % 128 || d > 2048 || ddt < 0 || ddt > 2) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * d, st);
    if (e == cudaSuccess && dscale) e = cudaMemsetAsync(dscale, 0, sizeof(float), st);
    if (e != cudaSuccess) return e;
    if (N == 0) return cudaSuccess;
    auto g16 = static_cast<const uint16_t *>(dy16);
    const int nv = d / 128;
    // one resident wave: every CTA zeroes, reduces and flushes its dw partials once,
    // so the fewer CTAs (the more tokens per warp) the less of that per token
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
#define MOM_NORM_B(DDT, NVV, SP)                                                                                 \
    do {                                                                                                       \
        const size_t smem = sizeof(float) * (d + 1 + 2 * kNormWarps);                                          \
        int per_sm = 1;                                                                                        \
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, add_rmsnorm_bwd_kernel<DDT, NVV, SP>,           \
                                                      32 * kNormWarps, smem);                                  \
        const int64_t groups = (N + kNormWarps / SP - 1) / (kNormWarps / SP);                                  \
        const int blocks = static_cast<int>(std::min<int64_t>(groups, static_cast<int64_t>(sms) * std::max(per_sm, 1))); \
        add_rmsnorm_bwd_kernel<DDT, NVV, SP><<<blocks, 32 * kNormWarps, smem, st>>>(                          \
            x_new, rstd, w, delta, dscale_in, g16, dy32, dx_in, N, d, dx, ddelta, dw, dscale);                 \
    } while (0)
#define MOM_NORM_BD(NVV, SP) \
    if (ddt == 0) MOM_NORM_B(0, NVV, SP); else if (ddt == 1) MOM_NORM_B(1, NVV, SP); else MOM_NORM_B(2, NVV, SP);
    // d >= 1024: a warp pair per token (NV / 2 vectors per lane)
    if (nv == 8) { MOM_NORM_BD(4, 2) } else if (nv == 16) { MOM_NORM_BD(8, 2) } else if (nv == 4) { MOM_NORM_BD(4, 1) }
    else if (nv == 2) { MOM_NORM_BD(2, 1) } else if (nv == 1) { MOM_NORM_BD(1, 1) } else { return cudaErrorInvalidValue; }
#undef MOM_NORM_BD
#undef MOM_NORM_B
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_xent_fwd(const void *logits, const int64_t *labels, int64_t R, int V, int64_t ignore_index,
                            float *row_loss, float *lse, cudaStream_t st) {
    if (R == 0) return cudaSuccess;
    const int grid = static_cast<int>(std::min<int64_t>(R, 148 * 64));
    auto lg = static_cast<const uint16_t *>(logits);
    if (V % 8 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0)
        xent_fwd_kernel<true><<<grid, kXentThreads, 0, st>>>(lg, labels, R, V, ignore_index, row_loss, lse);
    else
        xent_fwd_kernel<false><<<grid, kXentThreads, 0, st>>>(lg, labels, R, V, ignore_index, row_loss, lse);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_xent_bwd(const void *logits, const int64_t *labels, const float *lse, const float *grad, int64_t R,
                            int V, int64_t ignore_index, void *dlogits, cudaStream_t st) {
    if (R == 0) return cudaSuccess;
    const int grid = static_cast<int>(std::min<int64_t>(R, 148 * 64));
    auto lg = static_cast<const uint16_t *>(logits);
    auto dl = static_cast<uint16_t *>(dlogits);
    if (V % 8 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (reinterpret_cast<uintptr_t>(dlogits) & 15) == 0)
        xent_bwd_kernel<true><<<grid, kXentThreads, 0, st>>>(lg, labels, lse, grad, R, V, ignore_index, dl);
    else
        xent_bwd_kernel<false><<<grid, kXentThreads, 0, st>>>(lg, labels, lse, grad, R, V, ignore_index, dl);
    count_launch();
    return cudaGetLastError();
}

}  // namespace mom
