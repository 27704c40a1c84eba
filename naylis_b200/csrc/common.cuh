// Shared device helpers for the MoM kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/naylis_mom.h"

namespace mom {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ----------------------------------------------------------------- dtypes
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Round-to-nearest-even fp32 -> bf16, returned as the 16-bit pattern.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t *>(&h);
}

// fp32 value rounded to bf16 precision (kept as fp32).
__device__ __forceinline__ float round_bf16(float f) {
    return bf16_bits_to_f32(f32_to_bf16_bits(f));
}

template <int DT> struct Elem;
template <> struct Elem<MOM_F32> {
    using T = float;
    static __device__ __forceinline__ float load(const T *p, int64_t i) { return p[i]; }
    static __device__ __forceinline__ void store(T *p, int64_t i, float v) { p[i] = v; }
    static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Elem<MOM_BF16> {
    using T = uint16_t;
    static __device__ __forceinline__ float load(const T *p, int64_t i) {
        return bf16_bits_to_f32(p[i]);
    }
    static __device__ __forceinline__ void store(T *p, int64_t i, float v) {
        p[i] = f32_to_bf16_bits(v);
    }
    static __device__ __forceinline__ float round(float v) { return round_bf16(v); }
};

// Pack two fp32 into a bf16x2 register (lo in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// ----------------------------------------------------------------- async copy
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte cp.async global->shared; src_bytes < 16 zero-fills the remainder.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ----------------------------------------------------------------- mma.sync
// D(16x8 fp32) += A(16x16 bf16, row) * B(16x8 bf16, col)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a row-major tile whose
// rows are `row_bytes` long, XOR-swizzled on the low three chunk bits so that
// eight consecutive rows of one chunk column hit eight different bank groups.
__device__ __forceinline__ uint32_t swz(int row, int chunk, int row_bytes) {
    return static_cast<uint32_t>(row * row_bytes + ((chunk ^ (row & 7)) << 4));
}

// Vectorised fp32 reduction into global memory (sm_90+).
__device__ __forceinline__ void red_add_v2(float *p, float a, float b) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};\n" ::"l"(p), "f"(a), "f"(b)
                 : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace mom
