// AdamW over many fp32 parameter tensors in one launch, writing each updated
// parameter's bf16 copy in the same pass.
//
// The reference trains with torch's AdamW (pretrain.py's HF Trainer, optim
// "adamw_torch"; decoupled weight decay). Per element, in fp32, as torch's
// fused implementation orders it:
//   p = p * (1 - lr * wd)
//   m = beta1 * m + (1 - beta1) * g
//   v = beta2 * v + (1 - beta2) * g * g
//   p = p - (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps)
// with bc1 = 1 - beta1^step, bc2 = 1 - beta2^step. The bf16 copy (round to
// nearest even) is what the next forward's bf16 GEMMs read, so the per-step cast
// of every weight under autocast goes away.
//
// Work list: a device table of tensors {p, g, m, v, p16 (may be null), n} and a
// list of (tensor, chunk) pairs, kOptChunk elements per chunk; one CTA per
// pair, 16-byte accesses where the tensor's pointers allow.
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace mom {

namespace {
__device__ __forceinline__ float adamw_elem(float p, float g, float &m, float &v, float decay, float b1, float b2,
                                            float step_size, float inv_bc2_sqrt, float eps) {
    p = p * decay;
    m = fmaf(b1, m, (1.0f - b1) * g);
    v = fmaf(b2, v, (1.0f - b2) * g * g);
    const float denom = sqrtf(v) * inv_bc2_sqrt + eps;
    return p - step_size * (m / denom);
}

__global__ void __launch_bounds__(kOptThreads)
adamw_multi_kernel(const OptTensor *__restrict__ tensors, const int2 *__restrict__ chunks, float lr, float b1,
                   float b2, float eps, float wd, float bc1, float bc2) {
    const int2 c = chunks[blockIdx.x];
    const OptTensor t = tensors[c.x];
    const int64_t lo = static_cast<int64_t>(c.y) * kOptChunk;
    const int64_t hi = min(t.n, lo + kOptChunk);
    const float decay = 1.0f - lr * wd;
    const float step_size = lr / bc1;
    const float inv_bc2_sqrt = 1.0f / sqrtf(bc2);
    const bool vec = ((reinterpret_cast<uintptr_t>(t.p) | reinterpret_cast<uintptr_t>(t.g) |
                       reinterpret_cast<uintptr_t>(t.m) | reinterpret_cast<uintptr_t>(t.v)) & 15) == 0 &&
                     (t.p16 == nullptr || (reinterpret_cast<uintptr_t>(t.p16) & 7) == 0) && (lo & 3) == 0;
    if (vec) {
        const int64_t nv = (hi - lo) / 4;
        for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) {
            const int64_t e = lo + 4 * i;
            float4 p = *reinterpret_cast<const float4 *>(t.p + e);
            const float4 g = *reinterpret_cast<const float4 *>(t.g + e);
            float4 m = *reinterpret_cast<const float4 *>(t.m + e);
            float4 v = *reinterpret_cast<const float4 *>(t.v + e);
            p.x = adamw_elem(p.x, g.x, m.x, v.x, decay, b1, b2, step_size, inv_bc2_sqrt, eps);
            p.y = adamw_elem(p.y, g.y, m.y, v.y, decay, b1, b2, step_size, inv_bc2_sqrt, eps);
            p.z = adamw_elem(p.z, g.z, m.z, v.z, decay, b1, b2, step_size, inv_bc2_sqrt, eps);
            p.w = adamw_elem(p.w, g.w, m.w, v.w, decay, b1, b2, step_size, inv_bc2_sqrt, eps);
            *reinterpret_cast<float4 *>(t.p + e) = p;
            *reinterpret_cast<float4 *>(t.m + e) = m;
            *reinterpret_cast<float4 *>(t.v + e) = v;
            if (t.p16)
                *reinterpret_cast<uint2 *>(t.p16 + e) = make_uint2(pack_bf16x2(p.x, p.y), pack_bf16x2(p.z, p.w));
        }
        // the chunk's last elements when its length is not a multiple of 4
        for (int64_t e = lo + 4 * nv + threadIdx.x; e < hi; e += blockDim.x) {
            float m = t.m[e], v = t.v[e];
            const float p = adamw_elem(t.p[e], t.g[e], m, v, decay, b1, b2, step_size, inv_bc2_sqrt, eps);
            t.p[e] = p;
            t.m[e] = m;
            t.v[e] = v;
            if (t.p16) t.p16[e] = f32_to_bf16_bits(p);
        }
    } else {
        for (int64_t e = lo + threadIdx.x; e < hi; e += blockDim.x) {
            float m = t.m[e], v = t.v[e];
            const float p = adamw_elem(t.p[e], t.g[e], m, v, decay, b1, b2, step_size, inv_bc2_sqrt, eps);
            t.p[e] = p;
            t.m[e] = m;
            t.v[e] = v;
            if (t.p16) t.p16[e] = f32_to_bf16_bits(p);
        }
    }
}
}  // namespace

cudaError_t launch_adamw_multi(const OptTensor *tensors, const int2 *chunks, int64_t nchunks, float lr, float b1,
                               float b2, float eps, float wd, float bc1, float bc2, cudaStream_t st) {
    if (nchunks <= 0) return cudaSuccess;
    if (nchunks > 0x7FFFFFFF) return cudaErrorInvalidValue;
    adamw_multi_kernel<<<static_cast<unsigned>(nchunks), kOptThreads, 0, st>>>(tensors, chunks, lr, b1, b2, eps, wd,
                                                                              bc1, bc2);
    count_launch();
    return cudaGetLastError();
}

}  // namespace mom
