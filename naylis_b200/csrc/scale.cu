// ReZero output scale of the MoM layer, fused: model.py:239 (`self.mom_scale * out`).
//
// Under autocast `out` (the o_proj result) is bf16 and mom_scale a (1,) fp32
// parameter, so the product is fp32. Forward: y = s * o (one pass). Backward:
// d_o = s * g rounded to o's dtype and d_s = sum(g * o), in one pass over g
// and o instead of the mul / cast / mul / reduce kernels autograd would run.
#include "common.cuh"
#include "launch.h"

namespace mom {

// kVec: the arrays are aligned for 4-element vectors (16 B fp32, 8 B bf16);
// otherwise every element takes the scalar tail loop.
template <int ODT, bool kVec>
__global__ void __launch_bounds__(256)
scale_fwd_kernel(const typename Elem<ODT>::T *__restrict__ o, const float *__restrict__ scale, int64_t n,
                 float *__restrict__ y) {
    const float s = *scale;
    const int64_t n4 = kVec ? n / 4 : 0;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float4 v;
        if (ODT == MOM_BF16) {
            const uint2 raw = reinterpret_cast<const uint2 *>(o)[i];
            v = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u),
                            __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xFFFF0000u));
        } else {
            v = reinterpret_cast<const float4 *>(o)[i];
        }
        reinterpret_cast<float4 *>(y)[i] = make_float4(s * v.x, s * v.y, s * v.z, s * v.w);
    }
    for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = s * Elem<ODT>::load(o, i);
}

// elements 4i .. 4i+3 of a 16-B aligned array as fp32
template <int DT>
__device__ __forceinline__ void load4(const typename Elem<DT>::T *p, int64_t i, float (&v)[4]) {
    if (DT == MOM_BF16) {
        const uint2 raw = reinterpret_cast<const uint2 *>(p)[i];
        v[0] = __uint_as_float(raw.x << 16);
        v[1] = __uint_as_float(raw.x & 0xFFFF0000u);
        v[2] = __uint_as_float(raw.y << 16);
        v[3] = __uint_as_float(raw.y & 0xFFFF0000u);
    } else {
        const float4 f = reinterpret_cast<const float4 *>(p)[i];
        v[0] = f.x;
        v[1] = f.y;
        v[2] = f.z;
        v[3] = f.w;
    }
}

template <int ODT, int GDT, bool kVec>
__global__ void __launch_bounds__(256)
scale_bwd_kernel(const typename Elem<GDT>::T *__restrict__ g, const typename Elem<ODT>::T *__restrict__ o,
                 const float *__restrict__ scale, int64_t n, typename Elem<ODT>::T *__restrict__ d_o,
                 float *__restrict__ d_scale) {
    const float s = *scale;
    float acc = 0.0f;
    const int64_t n4 = kVec ? n / 4 : 0;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        // four elements per thread, as one 16-B (fp32) or 8-B (bf16) vector per operand
        float gv[4], ov[4];
        load4<GDT>(g, i, gv);
        load4<ODT>(o, i, ov);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc = fmaf(gv[k], ov[k], acc);
        if (ODT == MOM_BF16) {
            uint2 w;
            w.x = pack_bf16x2(s * gv[0], s * gv[1]);
            w.y = pack_bf16x2(s * gv[2], s * gv[3]);
            reinterpret_cast<uint2 *>(d_o)[i] = w;
        } else {
            reinterpret_cast<float4 *>(d_o)[i] = make_float4(s * gv[0], s * gv[1], s * gv[2], s * gv[3]);
        }
    }
    for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float gv = Elem<GDT>::load(g, i), ov = Elem<ODT>::load(o, i);
        acc = fmaf(gv, ov, acc);
        Elem<ODT>::store(d_o, i, s * gv);
    }
    __shared__ float red[8];
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        v = warp_sum(v);
        if (threadIdx.x == 0) atomicAdd(d_scale, v);
    }
}

static int scale_grid(int64_t n) {
    const int64_t want = (n / 4 + 255) / 256;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 148 * 8)));
}

static bool vec_ok(const void *p, int dt) {
    return (reinterpret_cast<uintptr_t>(p) & (dt == MOM_BF16 ? 7u : 15u)) == 0;
}

cudaError_t launch_scale_fwd(const void *o, int odt, const float *scale, int64_t n, float *y, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const bool v = vec_ok(o, odt) && vec_ok(y, MOM_F32);
    if (odt == MOM_BF16) {
        if (v) scale_fwd_kernel<MOM_BF16, true><<<scale_grid(n), 256, 0, st>>>(static_cast<const uint16_t *>(o), scale, n, y);
        else scale_fwd_kernel<MOM_BF16, false><<<scale_grid(n), 256, 0, st>>>(static_cast<const uint16_t *>(o), scale, n, y);
    } else {
        if (v) scale_fwd_kernel<MOM_F32, true><<<scale_grid(n), 256, 0, st>>>(static_cast<const float *>(o), scale, n, y);
        else scale_fwd_kernel<MOM_F32, false><<<scale_grid(n), 256, 0, st>>>(static_cast<const float *>(o), scale, n, y);
    }
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_scale_bwd(const void *g, int gdt, const void *o, int odt, const float *scale, int64_t n,
                             void *d_o, float *d_scale, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(d_scale, 0, sizeof(float), st);
    if (e != cudaSuccess || n == 0) return e;
    const bool v = vec_ok(g, gdt) && vec_ok(o, odt) && vec_ok(d_o, odt);
#define MOM_SB(O, G)                                                                                   \
    if (odt == O && gdt == G) {                                                                        \
        if (v)                                                                                         \
            scale_bwd_kernel<O, G, true><<<scale_grid(n), 256, 0, st>>>(                               \
                static_cast<const typename Elem<G>::T *>(g), static_cast<const typename Elem<O>::T *>(o), scale, \
                n, static_cast<typename Elem<O>::T *>(d_o), d_scale);                                  \
        else                                                                                           \
            scale_bwd_kernel<O, G, false><<<scale_grid(n), 256, 0, st>>>(                              \
                static_cast<const typename Elem<G>::T *>(g), static_cast<const typename Elem<O>::T *>(o), scale, \
                n, static_cast<typename Elem<O>::T *>(d_o), d_scale);                                  \
    }
    MOM_SB(MOM_BF16, MOM_F32)
    MOM_SB(MOM_BF16, MOM_BF16)
    MOM_SB(MOM_F32, MOM_F32)
    MOM_SB(MOM_F32, MOM_BF16)
#undef MOM_SB
    count_launch();
    return cudaGetLastError();
}

// Gumbel noise of the router (model.py:209-213 of the reference:
// noise_scale * -log(-log(u + 1e-9) + 1e-9) on torch.rand draws u), as one pass
// instead of the add / log / neg / add / log / neg / mul kernels the expression
// runs as torch ops. Each step is the same fp32 operation torch's kernel does
// (an fp32 add of the float constant, logf, negation, one fp32 multiply), in
// the same order, so the result is bit-identical. out may alias u.
__device__ __forceinline__ float gumbel_of(float u, float scale) {
    const float a = -logf(u + 1e-9f);
    return scale * -logf(a + 1e-9f);
}

__global__ void __launch_bounds__(256)
gumbel_kernel(const float *u, int64_t n, float scale, float *out, bool vec) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (vec) {
        const int64_t n4 = n / 4;
        for (int64_t i = i0; i < n4; i += stride) {
            float4 v = reinterpret_cast<const float4 *>(u)[i];
            v.x = gumbel_of(v.x, scale);
            v.y = gumbel_of(v.y, scale);
            v.z = gumbel_of(v.z, scale);
            v.w = gumbel_of(v.w, scale);
            reinterpret_cast<float4 *>(out)[i] = v;
        }
        done = n4 * 4;
    }
    for (int64_t i = done + i0; i < n; i += stride) out[i] = gumbel_of(u[i], scale);
}

cudaError_t launch_gumbel(const float *u, int64_t n, float scale, float *out, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const bool v = vec_ok(u, MOM_F32) && vec_ok(out, MOM_F32);
    gumbel_kernel<<<scale_grid(n), 256, 0, st>>>(u, n, scale, out, v);
    count_launch();
    return cudaGetLastError();
}

// dK, dV (L, n) fp32 -> [dK | dV] (L, 2n) bf16 (round to nearest even) in one pass:
// the read's backward accumulates dK / dV in fp32 and the bank projections' backward
// reads them side by side as one bf16 operand. 16-byte loads, 8-byte stores.
__global__ void __launch_bounds__(256)
kv_pack_kernel(const float4 *__restrict__ dk, const float4 *__restrict__ dv, int64_t L, int n4,
               uint2 *__restrict__ out) {
    const int64_t total = L * 2 * n4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = i / (2 * n4);
        const int c = static_cast<int>(i - row * 2 * n4);
        const float4 v = c < n4 ? dk[row * n4 + c] : dv[row * n4 + (c - n4)];
        out[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    }
}

cudaError_t launch_kv_pack(const float *dk, const float *dv, int64_t L, int64_t n, void *out, cudaStream_t st) {
    if (L == 0 || n == 0) return cudaSuccess;
    if (n % 4 || !vec_ok(dk, MOM_F32) || !vec_ok(dv, MOM_F32) || (reinterpret_cast<uintptr_t>(out) & 7))
        return cudaErrorInvalidValue;
    kv_pack_kernel<<<scale_grid(L * 2 * n), 256, 0, st>>>(reinterpret_cast<const float4 *>(dk),
                                                         reinterpret_cast<const float4 *>(dv), L,
                                                         static_cast<int>(n / 4), static_cast<uint2 *>(out));
    count_launch();
    return cudaGetLastError();
}

}  // namespace mom
