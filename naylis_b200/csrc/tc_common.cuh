// Blackwell (sm_100a) primitives: mbarriers with bounded waits, TMA tile
// loads, and the tcgen05 tensor-core / tensor-memory instructions, as inline
// PTX. Every wait is bounded: on timeout it records an error bit and returns
// false so the caller can unwind instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace mom {
namespace tc {

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// The same test with a suspend-time hint: the thread is suspended in hardware
// until the phase completes or `hint_ns` nanoseconds pass, so a waiting warp
// does not take issue slots from the warps still computing on its SM
// sub-partition.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Upper bound of one wait, in SM clock cycles (~1 s at 1.9 GHz): far above any
// legitimate wait in these kernels, far below a hang.
constexpr long long kWaitLimitCycles = 2000000000LL;
// Suspend hint of one try (ns): the abort flag and the time limit are checked
// between tries, so another role's abort is seen within about this time.
constexpr uint32_t kWaitSuspendNs = 200000;

// Wait for the phase of `parity` to complete. Returns false (and sets bit
// `err_bit` of *err, and *abort) on timeout or when another role aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int err_bit,
                                          volatile int *abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try_wait_suspend(bar, parity, kWaitSuspendNs)) return true;
        if (*abort) return false;
        if (clock64() - t0 > kWaitLimitCycles) {
            atomicOr(err, err_bit);
            *abort = 1;
            return false;
        }
    }
}

// Warp-uniform form of mbar_wait: every lane waits, all lanes get the same
// answer (the tcgen05.ld / named-barrier code after it must not diverge).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, int *err, int err_bit,
                                               volatile int *abort) {
    const bool ok = mbar_wait(bar, parity, err, err_bit, abort);
    return __all_sync(0xffffffffu, ok);
}

// ------------------------------------------------------------------ proxies
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Completion of this thread's earlier cp.async (non-bulk) copies.
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// ------------------------------------------------------------------ tcgen05
// Allocation is warp-collective; the TMEM base address is written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem], kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], kind::f16: A (128 x 16 bf16, row i in TMEM
// lane i, two K elements per 32-bit column, 8 columns) read from tensor memory.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: this thread gets its lane's 32 columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
// The same wait, with the destination registers of the load it completes as
// in/out operands: no use of them can be scheduled before it, also when other
// TMEM loads are issued in between (software pipelining).
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                   "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                   "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}


// 32 lanes x 16 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// 32 lanes x 8 consecutive 32-bit columns: this thread writes its lane's 8 columns.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// ------------------------------------------------------------------ misc
// Named barrier `id` (1..15) over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier with an OR-reduction of `pred` over the participating threads:
// every thread gets the same answer, so a group can agree to stop together.
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Stores one item's 128-row x 64-column bf16 tile that the softmax warps hold
// as 32 bytes per thread (row quarter*32 + lane, columns 16*grp .. +15), to the
// global rows tok of each row (tok < 0: padding, not stored); dst_col points at
// the tile's first column, ld is the row pitch in elements. The four warps of a
// lane quarter call it together (named barrier bar_id over 128 threads): each
// thread's 32 B go to a shared-memory copy of the quarter's rows (16-B chunks
// XOR-swizzled by row: conflict-free), then each warp stores 8 whole 128-B rows,
// 8 lanes per row, so a warp store touches 4 rows instead of 32. sOut holds 128
// rows x 128 B, sTok 128 ints; the caller keeps another barrier of the quarter
// between two calls.
__device__ __forceinline__ void store_tile_rows(uint4 *sOut, int *sTok, int quarter, int grp, int lane, int bar_id,
                                                uint4 v0, uint4 v1, int tok, uint16_t *dst_col, int64_t ld) {
    const int r = quarter * 32 + lane;
    uint4 *srow = sOut + r * 8;
    srow[(2 * grp) ^ (r & 7)] = v0;
    srow[(2 * grp + 1) ^ (r & 7)] = v1;
    if (grp == 0) sTok[r] = tok;
    named_bar(bar_id, 128);
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
        const int rr = quarter * 32 + grp * 8 + pass * 4 + (lane >> 3), ch = lane & 7;
        const int t = sTok[rr];
        if (t >= 0)
            reinterpret_cast<uint4 *>(dst_col + static_cast<int64_t>(t) * ld)[ch] = sOut[rr * 8 + (ch ^ (rr & 7))];
    }
}

// 2^x by the hardware approximation (PTX ex2.approx.ftz.f32); the results
// feed bf16 operands, far coarser than its error. Not volatile: a pure
// function the compiler may schedule among the TMEM loads.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// max of three fp32 values in one instruction (PTX max.f32 with three sources, sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;\n" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// ------------------------------------------------------------------ packed fp32 pairs
// Two fp32 lanes in one 64-bit register pair (PTX .f32x2 arithmetic, sm_100):
// one instruction issues both halves.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ uint64_t f2_bits(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_split(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;\n" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// 2^x for a pair of softmax arguments (x <= ~0) on the FMA pipe, so that part of
// a row's exponentials leave the MUFU unit: x = n + f with n = RN(x) taken by
// adding 1.5 * 2^23 (n lands in the low mantissa bits), f = x - n in [-1/2, 1/2],
// 2^f by a degree-3 polynomial, n added to the exponent field. The coefficients
// were fitted for this kernel (least squares on 4001 Chebyshev nodes of
// [-1/2, 1/2], relative error, Lawson reweighting toward minimax): maximum
// relative error 7.5e-5 in fp32 Horner evaluation, well below the bf16
// rounding of P. x is clamped at -126, where the result (a zero or denormal
// exponent field) is negligible next to the row maximum's 1.
__device__ __forceinline__ uint64_t ex2_poly2(uint64_t x) {
    const float2 xc = f2_split(x);
    const uint64_t xk = f2(fmaxf(xc.x, -126.0f), fmaxf(xc.y, -126.0f));
    const uint64_t shifter = f2(12582912.0f, 12582912.0f);           // 1.5 * 2^23
    const uint64_t t = add2(xk, shifter);
    const uint64_t f = sub2(xk, sub2(t, shifter));
    uint64_t p = fma2(f2(0x1.c3f76p-5f, 0x1.c3f76p-5f), f, f2(0x1.f0de1cp-3f, 0x1.f0de1cp-3f));
    p = fma2(p, f, f2(0x1.62f31ap-1f, 0x1.62f31ap-1f));
    p = fma2(p, f, f2(0x1.fff692p-1f, 0x1.fff692p-1f));
    const float2 pp = f2_split(p), tt = f2_split(t);
    return f2_bits(__float_as_uint(pp.x) + (__float_as_uint(tt.x) << 23),
                   __float_as_uint(pp.y) + (__float_as_uint(tt.y) << 23));
}
// 2^x for a pair by the hardware approximation.
__device__ __forceinline__ uint64_t ex2_pair(uint64_t x) {
    const float2 xc = f2_split(x);
    return f2(ex2(xc.x), ex2(xc.y));
}

// ------------------------------------------------------------------ descriptors
// Shared-memory matrix descriptor, 128-byte swizzle (the TMA SWIZZLE_128B
// layout: 128-B rows, 16-B chunks XOR-ed with row & 7, 8-row atoms of 1 KiB).
// sbo: byte distance between 8-row groups; lbo: byte distance between
// 64-element column groups (MN-major only; ignored for K-major).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
    d |= static_cast<uint64_t>(1) << 46;          // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;          // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: bf16 A and B, fp32 D.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
    return (1u << 4)                                   // D format: f32
           | (1u << 7)                                 // A format: bf16
           | (1u << 10)                                // B format: bf16
           | (static_cast<uint32_t>(a_mn_major) << 15)  // A major
           | (static_cast<uint32_t>(b_mn_major) << 16)  // B major
           | (static_cast<uint32_t>(N >> 3) << 17)      // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);     // M / 16
}

// ---------------------------------------------------------------- plan metadata
// The read kernels walk work items whose tile descriptor (P.tiles) and block set
// (P.keyset) sit behind two dependent global loads. A warp fetches them for 32
// items at once, item c0 + lane in lane `lane`, and broadcasts one item's fields
// with get(); a tile's permuted rows then take a single round trip, which the
// caller issues one item ahead. Sets of at most two blocks (the tensor-core
// kernels' limit) are held as (nblk, b0, b1).
struct LaneTile {
    int x = 0, y = 0, key = -1, nblk = 0, b0 = 0, b1 = 0;
    template <typename PV>
    __device__ __forceinline__ void fetch(const PV &P, int tile, int top) {
        const int4 td = P.tiles[tile];
        const int *set = P.keyset + static_cast<int64_t>(td.z) * top;
        const int s0 = set[0], s1 = top > 1 ? set[1] : -1;
        x = td.x;
        y = td.y;
        key = td.z;
        nblk = s0 < 0 ? 0 : (s1 < 0 ? 1 : 2);
        b0 = s0 < 0 ? 0 : s0;
        b1 = s1 < 0 ? 0 : s1;
    }
};
__device__ __forceinline__ int get(int v, int src) { return __shfl_sync(0xffffffffu, v, src); }

// Token of each of the 4 tile rows 4*lane .. 4*lane+3 (row rr < y), else 0:
// the four rows whose tokens a lane stages for the tile's row copies.
template <typename PV>
__device__ __forceinline__ void gather_rows(const PV &P, int x, int y, int lane, int rows[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int rr = lane * 4 + u;
        rows[u] = rr < y ? P.perm[x + rr] : 0;
    }
}

__device__ __forceinline__ int ld_shared_volatile(const int *p) { return *reinterpret_cast<const volatile int *>(p); }

// ---------------------------------------------------------------- row gathers
// A tile's Q / dO rows are scattered over the token dimension (the plan's
// permutation). They are copied with 16-B cp.async, eight lanes per 128-B row
// slice, four rows per instruction (one TMA tile::gather4 per four rows costs
// ~60 cycles of the SM's TMA unit each, which made the loader the bottleneck).
// Completion is signalled on an mbarrier with cp.async.mbarrier.arrive.noinc
// (one of the barrier's expected arrivals per lane). cp.async writes shared
// memory through the generic proxy: a consumer that feeds the tile to tcgen05.mma
// executes fence_proxy_async_smem() after its wait on that barrier.
__device__ __forceinline__ void cp_async_cg16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// The tile's 128 row tokens (gather_rows' four per lane, rows past the tile's y
// read token 0, whose results are masked or never stored) go through a 128-int
// shared buffer, so that a lane holds 4 tokens in registers instead of the 32 of
// the rows it copies.
__device__ __forceinline__ void stage_row_tokens(int *s_tok, const int rows[4], int lane) {
    __syncwarp();   // the previous tile's reads of s_tok are done
#pragma unroll
    for (int u = 0; u < 4; ++u) s_tok[lane * 4 + u] = rows[u];
    __syncwarp();
}

// Copy columns col0 .. col0+63 (bf16) of the 128 rows into a [128 x 64] tile in
// the 128-B-swizzled K-major layout (row r at r*128, 16-B chunk c at (c ^ (r & 7))*16):
// lane copies chunk lane & 7 of rows 4*i + (lane >> 3).
__device__ __forceinline__ void gather_tile_rows(uint32_t sdst, const uint16_t *src, int64_t ld, int col0,
                                                 const int *s_tok, int lane) {
    const int c = lane & 7, rs = lane >> 3;
    const uint16_t *base = src + col0 + c * 8;
#pragma unroll 8
    for (int i = 0; i < 32; ++i) {
        const int r = 4 * i + rs;
        cp_async_cg16(sdst + r * 128 + ((c ^ (r & 7)) << 4), base + static_cast<int64_t>(s_tok[r]) * ld);
    }
}

}  // namespace tc
}  // namespace mom
