// Causal router of the MoM layer: exact prefix mean, rank-r tanh bottleneck,
// softmax / top-k / gate softmax, and the backward in rank-r space.
//
// Reference semantics: model.py:169-220 (MoMLayer._prefix_mean,
// _router_logits, forward's softmax/topk/gates block).
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace mom {

// ============================================================ prefix scan
// Sequential fp32 accumulation per column is torch's CUDA cumsum
// (tensor_kernel_scan_outer_dim): no re-association reproduces its bits, so one
// thread walks each column in order with the carry in a register. The adds are
// cheap (a 4-cycle dependent chain per row); what costs is the correctly rounded
// division h = c / (t+1) and the stores. So the work is split by warp:
//   warp 0      the 32 column chains of this CTA over a stage of kSeqRows rows,
//               writing the running sums to shared memory;
//   warps 1..8  one stage behind, RN(c / (t+1)) by Markstein's correction from
//               the row's reciprocal, 4 columns of a row per thread (one 16-B
//               shared load, one 8- or 16-B store); they also form the next
//               stage's row reciprocals.
// x streams through a ring of shared-memory stages filled by cp.async, kept
// kSeqStages-1 stages ahead. (The fp64 mode is the parallel exact scan below.)
constexpr int kSeqCols = 32;       // columns per CTA (one chain lane each)
constexpr int kSeqRows = 64;       // rows per stage
constexpr int kSeqStages = 8;      // ring depth
constexpr int kSeqDivWarps = 8;
constexpr int kSeqThreads = 32 * (1 + kSeqDivWarps);
constexpr int kSeqBatch = 16;      // rows loaded into registers at a time by the chain warp

template <int XDT>
constexpr size_t seq_scan_smem() {
    return size_t(kSeqStages) * kSeqRows * kSeqCols * sizeof(typename Elem<XDT>::T) +
           2 * size_t(kSeqRows) * kSeqCols * sizeof(float) + 2 * size_t(kSeqRows) * sizeof(float);
}

__device__ __forceinline__ float div_by_count(float c, float den, float y);

template <int CDT> struct Store4;
template <> struct Store4<MOM_BF16> {
    static __device__ __forceinline__ void store(uint16_t *p, float4 v) {
        *reinterpret_cast<uint2 *>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    }
    static __device__ __forceinline__ void store1(uint16_t *p, float v) { *p = f32_to_bf16_bits(v); }
};
template <> struct Store4<MOM_F32> {
    static __device__ __forceinline__ void store(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
    static __device__ __forceinline__ void store1(float *p, float v) { *p = v; }
};

template <int XDT, int CDT>
__global__ void __launch_bounds__(kSeqThreads)
route_scan_kernel(const typename Elem<XDT>::T *__restrict__ x,
                  typename Elem<CDT>::T *__restrict__ hq, int S, int d, ScanShard sh) {
    using XT = typename Elem<XDT>::T;
    using CT = typename Elem<CDT>::T;
    constexpr int kRowBytes = kSeqCols * sizeof(XT);
    constexpr int kChunksPerRow = kRowBytes / 16;
    constexpr int kStageBytes = kSeqRows * kRowBytes;
    constexpr int kGroups = kSeqCols / 4;                 // 4-column groups per row
    extern __shared__ __align__(128) unsigned char smem[];
    float *csum = reinterpret_cast<float *>(smem + kSeqStages * kStageBytes);   // [2][kSeqRows][kSeqCols]
    float *rcp = csum + 2 * kSeqRows * kSeqCols;                                 // [2][kSeqRows]

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int c0 = blockIdx.x * kSeqCols;
    const int b = blockIdx.y;
    const XT *xb = x + static_cast<int64_t>(b) * S * d;
    CT *hb = hq + static_cast<int64_t>(b) * S * d;
    const int nstage = (S + kSeqRows - 1) / kSeqRows;
    const int valid_cols = min(kSeqCols, d - c0);
    const int valid_bytes = valid_cols * static_cast<int>(sizeof(XT));

    auto issue = [&](int s) {
        if (s < nstage) {
            const uint32_t base = smem_u32(smem + (s % kSeqStages) * kStageBytes);
            for (int i = tid; i < kSeqRows * kChunksPerRow; i += kSeqThreads) {
                const int r = i / kChunksPerRow, ch = i % kChunksPerRow;
                const int t = s * kSeqRows + r;
                int nbytes = 0;
                const XT *src = xb;
                if (t < S) {
                    nbytes = min(16, max(0, valid_bytes - ch * 16));
                    if (nbytes) src = xb + static_cast<int64_t>(t) * d + c0 + ch * (16 / sizeof(XT));
                }
                cp_async16(base + r * kRowBytes + ch * 16, src, nbytes);
            }
        }
        cp_async_commit();
    };

#pragma unroll 1
    for (int s = 0; s < kSeqStages - 1; ++s) issue(s);

    // a shard of the sequence continues from the running sum of the rows before it
    const int col = c0 + lane;
    float acc = (warp == 0 && sh.carry_in && col < d)
                    ? static_cast<const float *>(sh.carry_in)[static_cast<int64_t>(b) * d + col] : 0.0f;
    // a division thread's 4-column group and its first row in a stage
    const int dt = tid - 32;
    const int grp = dt % kGroups, row0 = dt / kGroups;
    constexpr int kRowStep = (kSeqThreads - 32) / kGroups;   // 32 rows per pass
    const bool vec_ok = 4 * grp + 4 <= valid_cols && (d % 4) == 0 &&
                        (reinterpret_cast<uintptr_t>(hq) % (4 * sizeof(CT))) == 0;
#pragma unroll 1
    for (int s = 0; s <= nstage; ++s) {
        cp_async_wait<kSeqStages - 2>();
        __syncthreads();
        issue(s + kSeqStages - 1);
        if (warp == 0) {
            if (s < nstage) {
                const XT *stage = reinterpret_cast<const XT *>(smem + (s % kSeqStages) * kStageBytes);
                float *cs = csum + (s & 1) * kSeqRows * kSeqCols;
                const int rows = min(kSeqRows, S - s * kSeqRows);
                // a batch of rows is read into registers before the adds use any of
                // them: only the 4-cycle add chain stays serial, not the loads
#pragma unroll 1
                for (int r0 = 0; r0 < rows; r0 += kSeqBatch) {
                    float v[kSeqBatch];
#pragma unroll
                    for (int j = 0; j < kSeqBatch; ++j)
                        v[j] = r0 + j < rows ? Elem<XDT>::load(stage, (r0 + j) * kSeqCols + lane) : 0.0f;
#pragma unroll
                    for (int j = 0; j < kSeqBatch; ++j) {
                        acc = r0 + j < rows ? __fadd_rn(acc, v[j]) : acc;
                        v[j] = acc;
                    }
#pragma unroll
                    for (int j = 0; j < kSeqBatch; ++j)
                        if (r0 + j < rows) cs[(r0 + j) * kSeqCols + lane] = v[j];
                }
            }
        } else {
            // the reciprocals of stage s's rows, read at the next iteration
            if (s < nstage && dt < kSeqRows)
                rcp[(s & 1) * kSeqRows + dt] = __frcp_rn(static_cast<float>(sh.t_base + s * kSeqRows + dt + 1));
            if (s > 0) {
                const int sp = s - 1;
                const float *cs = csum + (sp & 1) * kSeqRows * kSeqCols;
                const float *yv = rcp + (sp & 1) * kSeqRows;
                const int t0 = sp * kSeqRows;
                const int rows = min(kSeqRows, S - t0);
#pragma unroll
                for (int r = row0; r < kSeqRows; r += kRowStep) {
                    if (r >= rows) break;
                    const float4 c = *reinterpret_cast<const float4 *>(cs + r * kSeqCols + 4 * grp);
                    const float y = yv[r];
                    const float den = static_cast<float>(sh.t_base + t0 + r + 1);
                    const float4 h = make_float4(div_by_count(c.x, den, y), div_by_count(c.y, den, y),
                                                 div_by_count(c.z, den, y), div_by_count(c.w, den, y));
                    CT *dst = hb + static_cast<int64_t>(t0 + r) * d + c0 + 4 * grp;
                    if (vec_ok) {
                        Store4<CDT>::store(dst, h);
                    } else {
                        const float hv[4] = {h.x, h.y, h.z, h.w};
                        for (int j = 0; j < 4; ++j)
                            if (4 * grp + j < valid_cols) Store4<CDT>::store1(dst + j, hv[j]);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
    if (warp == 0 && sh.carry_out && col < d)
        static_cast<float *>(sh.carry_out)[static_cast<int64_t>(b) * d + col] = acc;
}

// ------------------------------------------------------------ fp32 scan, TMA-fed
// The same sequential fp32 chains and the same division as route_scan_kernel,
// decoupled by mbarriers instead of a CTA barrier per stage, so that the chain
// warp runs as far ahead as the ring allows:
//   warp 0      producer: each stage (kTRows rows x 32 columns of one batch row)
//               by one 3-D TMA box into a ring of kTStages slots (rows past S
//               and columns past d arrive as zeros);
//   warp 1      the 32 column chains (lane = column): running sums of a stage
//               into one of two shared fp32 buffers (row-major), then the x slot
//               goes back to the producer; full stages take an unpredicated loop
//               (one load, one add, one store per row);
//   warps 2..9  RN(c / (t+1)) by Markstein's correction from the row's
//               reciprocal, 4 columns of a row per thread (one 16-B shared load,
//               one 8- or 16-B store).
// Every wait is bounded; on a timeout the CTA stops and its rows of h are left
// as NaN (written at the end), so a stuck scan shows in the router's outputs.
constexpr int kTRows = 64;
constexpr int kTStages = 8;
constexpr int kTDivWarps = 8;
constexpr int kTThreads = 32 * (2 + kTDivWarps);

template <int XDT>
constexpr size_t tma_scan_smem() {
    return size_t(kTStages) * kTRows * kSeqCols * sizeof(typename Elem<XDT>::T) +
           2 * size_t(kTRows) * kSeqCols * sizeof(float) + 256 /*barriers*/ + 128 /*align*/;
}

template <int XDT, int CDT>
__global__ void __launch_bounds__(kTThreads)
route_scan_tma_kernel(const __grid_constant__ CUtensorMap xmap, typename Elem<CDT>::T *__restrict__ hq, int S,
                      int d, ScanShard sh) {
    using XT = typename Elem<XDT>::T;
    using CT = typename Elem<CDT>::T;
    constexpr uint32_t kStageBytes = kTRows * kSeqCols * sizeof(XT);
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
    const XT *ring = reinterpret_cast<const XT *>(smem);
    float *csum = reinterpret_cast<float *>(smem + kTStages * kStageBytes);     // [2][kTRows][32]
    uint64_t *bars = reinterpret_cast<uint64_t *>(csum + 2 * kTRows * kSeqCols);
    uint64_t *full = bars, *empty = bars + kTStages, *cfull = bars + 2 * kTStages, *cempty = cfull + 2;
    int *flags = reinterpret_cast<int *>(cempty + 2);                           // [0] error bits, [1] abort
    volatile int *abort_flag = flags + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c0 = blockIdx.x * kSeqCols, b = blockIdx.y;
    const int nstage = (S + kTRows - 1) / kTRows;
    const int valid_cols = min(kSeqCols, d - c0);
    CT *hb = hq + static_cast<int64_t>(b) * S * d;
    if (tid == 0) {
        for (int i = 0; i < kTStages; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&cfull[i], 32);
            tc::mbar_init(&cempty[i], 32 * kTDivWarps);
        }
        flags[0] = 0;
        flags[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            tc::prefetch_tensormap(&xmap);
            for (int s = 0; s < nstage; ++s) {
                const int slot = s % kTStages;
                if (s >= kTStages &&
                    !tc::mbar_wait(&empty[slot], ((s / kTStages) - 1) & 1, flags, 2, abort_flag))
                    break;
                tc::mbar_arrive_expect_tx(&full[slot], kStageBytes);
                tc::tma_load_3d(smem_u32(smem + slot * kStageBytes), &xmap, c0, s * kTRows, b, &full[slot]);
            }
            // the last copies have landed before the CTA may exit
            for (int s = max(0, nstage - kTStages); s < nstage; ++s)
                tc::mbar_wait(&full[s % kTStages], (s / kTStages) & 1, flags, 2, abort_flag);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ chain warp
        const int col = c0 + lane;
        float acc = (sh.carry_in && col < d) ? static_cast<const float *>(sh.carry_in)[static_cast<int64_t>(b) * d + col]
                                             : 0.0f;
        bool ok = true;
        for (int s = 0; s < nstage && ok; ++s) {
            const int slot = s % kTStages;
            float *cs = csum + (s & 1) * kTRows * kSeqCols + lane;              // this lane's column
            ok = tc::mbar_wait_warp(&full[slot], (s / kTStages) & 1, flags, 2, abort_flag);
            if (ok && s >= 2) ok = tc::mbar_wait_warp(&cempty[s & 1], ((s >> 1) - 1) & 1, flags, 2, abort_flag);
            if (!ok) break;
            const XT *st = ring + slot * kTRows * kSeqCols + lane;
            const int rows = min(kTRows, S - s * kTRows);
            if (rows == kTRows) {
#pragma unroll 2
                for (int r0 = 0; r0 < kTRows; r0 += kSeqBatch) {
                    float v[kSeqBatch];
#pragma unroll
                    for (int j = 0; j < kSeqBatch; ++j) v[j] = Elem<XDT>::load(st, (r0 + j) * kSeqCols);
#pragma unroll
                    for (int j = 0; j < kSeqBatch; ++j) {
                        acc = __fadd_rn(acc, v[j]);
                        cs[(r0 + j) * kSeqCols] = acc;
                    }
                }
            } else {
                for (int r = 0; r < rows; ++r) {
                    acc = __fadd_rn(acc, Elem<XDT>::load(st, r * kSeqCols));
                    cs[r * kSeqCols] = acc;
                }
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&empty[slot]);
            tc::mbar_arrive(&cfull[s & 1]);
        }
        if (ok && sh.carry_out && col < d)
            static_cast<float *>(sh.carry_out)[static_cast<int64_t>(b) * d + col] = acc;
    } else {
        // ------------------------------------------------------------ division warps
        constexpr int kGroups = kSeqCols / 4;
        constexpr int kRowStep = 32 * kTDivWarps / kGroups;
        const int dt = tid - 64;
        const int grp = dt % kGroups, row0 = dt / kGroups;
        const bool vec_ok = 4 * grp + 4 <= valid_cols && (d % 4) == 0 &&
                            (reinterpret_cast<uintptr_t>(hq) % (4 * sizeof(CT))) == 0;
        for (int s = 0; s < nstage; ++s) {
            if (!tc::mbar_wait_warp(&cfull[s & 1], (s >> 1) & 1, flags, 2, abort_flag)) break;
            const float *cs = csum + (s & 1) * kTRows * kSeqCols;
            const int t0 = s * kTRows;
            const int rows = min(kTRows, S - t0);
#pragma unroll
            for (int r = row0; r < kTRows; r += kRowStep) {
                if (r >= rows) break;
                const float4 c = *reinterpret_cast<const float4 *>(cs + r * kSeqCols + 4 * grp);
                const float den = static_cast<float>(sh.t_base + t0 + r + 1);
                const float y = __frcp_rn(den);
                const float4 h = make_float4(div_by_count(c.x, den, y), div_by_count(c.y, den, y),
                                             div_by_count(c.z, den, y), div_by_count(c.w, den, y));
                CT *dst = hb + static_cast<int64_t>(t0 + r) * d + c0 + 4 * grp;
                if (vec_ok) {
                    Store4<CDT>::store(dst, h);
                } else {
                    const float hv[4] = {h.x, h.y, h.z, h.w};
                    for (int j = 0; j < 4; ++j)
                        if (4 * grp + j < valid_cols) Store4<CDT>::store1(dst + j, hv[j]);
                }
            }
            tc::mbar_arrive(&cempty[s & 1]);
        }
    }
    __syncthreads();
    if (flags[0]) {
        // a wait gave up: this CTA's columns of h become NaN
        const float nanv = __int_as_float(0x7fc00000);
        for (int i = tid; i < S * kSeqCols; i += blockDim.x) {
            const int t = i / kSeqCols, c = i % kSeqCols;
            if (c < valid_cols) Store4<CDT>::store1(hb + static_cast<int64_t>(t) * d + c0 + c, nanv);
        }
    }
}

// ------------------------------------------------------------ parallel exact fp64 scan
// Sequential fp64 accumulation (the CPU cumsum) is re-association-proof when
// no partial sum rounds. Every element is an integer multiple of its ulp, so
// with e_min the smallest ulp exponent of a column's non-zero elements, every
// partial sum of any subset of them is a multiple of 2^e_min bounded by
// A = sum |x|; if A < 2^(52 + e_min) all of them are exactly representable in
// fp64 and ANY summation order returns the exact prefix sums — the values the
// sequential loop produces. The kernel checks that certificate per column (A
// bounded from above by fp32 sums rounded upward) and walks the column
// sequentially when it fails (tiny or huge dynamic range).
//
// CTA = 64 columns (32 pairs) x 32 chunks of the sequence (1024 threads):
//   phase 1  chunk sums, upper bounds of the sums of |x|, min ulp exponent
//   phase 2  per column: exclusive scan of the chunk sums, certificate
//   phase 3  each chunk re-walks its rows from its carry and writes h.
// Rows are read kScanBatch at a time into registers before any of them is
// used, so every warp keeps that many row loads in flight.
constexpr int kScanBatch = 8;

template <int XDT>
__device__ __forceinline__ int ulp_exponent(float v) {
    const uint32_t bits = __float_as_uint(v);
    const int e = static_cast<int>((bits >> 23) & 0xFF);
    return (e == 0 ? 1 : e) - 127 - (XDT == MOM_BF16 ? 7 : 23);
}

// Two adjacent columns per thread (one 4-byte bf16 pair or 8-byte fp32 pair per row).
template <int XDT> struct Pair;
template <> struct Pair<MOM_BF16> {
    static __device__ __forceinline__ float2 load(const uint16_t *p) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    }
};
template <> struct Pair<MOM_F32> {
    static __device__ __forceinline__ float2 load(const float *p) { return *reinterpret_cast<const float2 *>(p); }
};
template <int CDT> struct PairStore;
template <> struct PairStore<MOM_BF16> {
    static __device__ __forceinline__ void store(uint16_t *p, float a, float b) {
        *reinterpret_cast<uint32_t *>(p) = pack_bf16x2(a, b);
    }
};
template <> struct PairStore<MOM_F32> {
    static __device__ __forceinline__ void store(float *p, float a, float b) {
        *reinterpret_cast<float2 *>(p) = make_float2(a, b);
    }
};

// RN(c / den) for den = t + 1, a positive integer below 2^24, given y = RN(1 / den).
// Markstein's correction step (P. Markstein, "Computation of elementary functions
// on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with q0
// within one ulp of c/den, the remainder c - den*q0 is exact in one fma and
// q0 + remainder*y rounded once is the correctly rounded quotient. It holds while
// the quotient is a normal number, so zero, tiny, infinite and NaN c take the
// IEEE division instead. Division never lands exactly on a rounding midpoint,
// so no tie case arises.
// The IEEE division for the rare operands outside the fast path, kept out of
// line: inlined, the compiler may evaluate it under a predicate for every
// element (measured: ~45 instructions per element in the scan instead of ~10).
__device__ __noinline__ float div_ieee(float c, float den) { return __fdiv_rn(c, den); }

__device__ __forceinline__ float div_by_count(float c, float den, float y) {
    const uint32_t e = (__float_as_uint(c) >> 23) & 0xFFu;
    const float q0 = __fmul_rn(c, y);
    const float r = __fmaf_rn(-q0, den, c);
    float q = __fmaf_rn(r, y, q0);
    if (e - 25u >= 229u) q = div_ieee(c, den);   // zero, tiny (|c| < 2^-102), Inf or NaN
    return q;
}

template <int XDT, int CDT>
__global__ void __launch_bounds__(1024)
route_scan_par_kernel(const typename Elem<XDT>::T *__restrict__ x, typename Elem<CDT>::T *__restrict__ hq,
                      int S, int d, ScanShard sh) {
    __shared__ double s_sum[64][33];
    __shared__ float s_abs[64][33];
    __shared__ int s_emin[64][33];
    __shared__ int s_cert[64];
    const int c2 = threadIdx.x & 31, k = threadIdx.x >> 5;    // column pair, chunk
    const int b = blockIdx.y;
    const int col = blockIdx.x * 64 + 2 * c2;
    const int len = (S + 31) / 32;
    const int t0 = k * len, t1 = min(S, t0 + len);
    const bool live = col < d;                                   // d % 8 == 0: pairs are whole
    // lanes past d read (and never write) column pair 0, so that every lane of a
    // warp runs the same loop and can take part in its shuffles
    const int64_t cofs = static_cast<int64_t>(b) * S * d + (live ? col : 0);
    const typename Elem<XDT>::T *xc = x + cofs;
    typename Elem<CDT>::T *hc = hq + cofs;
    double sum0 = 0.0, sum1 = 0.0;
    float as0 = 0.0f, as1 = 0.0f;
    // e_min from the smallest non-zero magnitude (finite values: the smallest
    // magnitude has the smallest exponent field): a running unsigned min of
    // |bits| - 1, where zero wraps to 0xFFFFFFFF and never wins
    uint32_t mn0 = 0xFFFFFFFFu, mn1 = 0xFFFFFFFFu;
    auto take = [&](float2 v) {
        sum0 = __dadd_rn(sum0, static_cast<double>(v.x));
        sum1 = __dadd_rn(sum1, static_cast<double>(v.y));
        as0 = __fadd_ru(as0, fabsf(v.x));
        as1 = __fadd_ru(as1, fabsf(v.y));
        mn0 = min(mn0, (__float_as_uint(v.x) & 0x7FFFFFFFu) - 1u);
        mn1 = min(mn1, (__float_as_uint(v.y) & 0x7FFFFFFFu) - 1u);
    };
    {
        int t = t0;
        for (; t + kScanBatch <= t1; t += kScanBatch) {
            float2 v[kScanBatch];
#pragma unroll
            for (int u = 0; u < kScanBatch; ++u) v[u] = Pair<XDT>::load(xc + static_cast<int64_t>(t + u) * d);
#pragma unroll
            for (int u = 0; u < kScanBatch; ++u) take(v[u]);
        }
        for (; t < t1; ++t) take(Pair<XDT>::load(xc + static_cast<int64_t>(t) * d));
    }
    s_sum[2 * c2][k] = sum0;
    s_sum[2 * c2 + 1][k] = sum1;
    s_abs[2 * c2][k] = as0;
    s_abs[2 * c2 + 1][k] = as1;
    auto em_of = [](uint32_t mn) -> int {   // ulp exponent of the smallest non-zero element
        return mn == 0xFFFFFFFFu ? (1 << 20) : ulp_exponent<XDT>(__uint_as_float(mn + 1u));
    };
    s_emin[2 * c2][k] = em_of(mn0);
    s_emin[2 * c2 + 1][k] = em_of(mn1);
    __syncthreads();
    // a shard of the sequence: carry [0][b][col] = the sum of the rows before it,
    // [1][b][col] = the whole sequence's certificate (so every shard decides alike)
    const double *cin = static_cast<const double *>(sh.carry_in);
    const int64_t bd = static_cast<int64_t>(gridDim.y) * d;
    if (threadIdx.x < 64) {                                      // one thread per column
        const int cc = threadIdx.x;
        const int ccol = blockIdx.x * 64 + cc;
        const int64_t ci = static_cast<int64_t>(b) * d + ccol;
        double run = (cin && ccol < d) ? cin[ci] : 0.0, at = 0.0;
        int em = 1 << 20;
        for (int kk = 0; kk < 32; ++kk) {
            const double v = s_sum[cc][kk];
            s_sum[cc][kk] = run;
            run = __dadd_rn(run, v);
            at = __dadd_ru(at, static_cast<double>(s_abs[cc][kk]));   // stays an upper bound of A
            em = min(em, s_emin[cc][kk]);
        }
        // all zero -> trivially exact; else A < 2^(52 + e_min)
        s_cert[cc] = cin ? (ccol < d && cin[bd + ci] != 0.0)
                         : ((em == (1 << 20)) || (em > -1000 && at < ldexp(1.0, 52 + em)));
    }
    __syncthreads();
    const bool fast = live && s_cert[2 * c2] && s_cert[2 * c2 + 1];
    {
        double r0 = s_sum[2 * c2][k], r1 = s_sum[2 * c2 + 1][k];
        auto emit = [&](int t, float2 v, float y) {
            r0 = __dadd_rn(r0, static_cast<double>(v.x));
            r1 = __dadd_rn(r1, static_cast<double>(v.y));
            const float den = static_cast<float>(sh.t_base + t + 1);
            if (fast)
                PairStore<CDT>::store(hc + static_cast<int64_t>(t) * d, div_by_count(__double2float_rn(r0), den, y),
                                      div_by_count(__double2float_rn(r1), den, y));
        };
        int t = t0;
        for (; t + kScanBatch <= t1; t += kScanBatch) {
            float2 v[kScanBatch];
#pragma unroll
            for (int u = 0; u < kScanBatch; ++u) v[u] = Pair<XDT>::load(xc + static_cast<int64_t>(t + u) * d);
            // lane u < kScanBatch holds 1/(t + 1 + u) for the whole warp
            const float yl = __frcp_rn(static_cast<float>(sh.t_base + t + 1 + (c2 & (kScanBatch - 1))));
#pragma unroll
            for (int u = 0; u < kScanBatch; ++u) emit(t + u, v[u], __shfl_sync(0xffffffffu, yl, u));
        }
        for (; t < t1; ++t)
            emit(t, Pair<XDT>::load(xc + static_cast<int64_t>(t) * d),
                 __frcp_rn(static_cast<float>(sh.t_base + t + 1)));
        // the last chunk ends at row S - 1: its running sums are the shard's exact end state
        if (fast && k == 31 && sh.carry_out) {
            double *co = static_cast<double *>(sh.carry_out) + static_cast<int64_t>(b) * d + col;
            co[0] = r0;
            co[1] = r1;
            co[bd] = 1.0;
            co[bd + 1] = 1.0;
        }
    }
    if (live && !fast && k == 0) {
        // a certificate failed: both columns of the pair walk sequentially
        const int64_t ci = static_cast<int64_t>(b) * d + col;
        double a0 = cin ? cin[ci] : 0.0, a1 = cin ? cin[ci + 1] : 0.0;
        for (int t = 0; t < S; ++t) {
            const float2 v = Pair<XDT>::load(xc + static_cast<int64_t>(t) * d);
            a0 = __dadd_rn(a0, static_cast<double>(v.x));
            a1 = __dadd_rn(a1, static_cast<double>(v.y));
            const float den = static_cast<float>(sh.t_base + t + 1);
            PairStore<CDT>::store(hc + static_cast<int64_t>(t) * d, __fdiv_rn(__double2float_rn(a0), den),
                                  __fdiv_rn(__double2float_rn(a1), den));
        }
        if (sh.carry_out) {
            double *co = static_cast<double *>(sh.carry_out) + ci;
            co[0] = a0;
            co[1] = a1;
            co[bd] = s_cert[2 * c2] ? 1.0 : 0.0;
            co[bd + 1] = s_cert[2 * c2 + 1] ? 1.0 : 0.0;
        }
    }
}

// Per-shard totals for a sequence split across ranks: the par kernel's phase 1
// over the shard's rows, reduced per column (the sum is exact whenever the whole
// sequence's certificate holds, since the shard's elements are a subset).
template <int XDT>
__global__ void __launch_bounds__(1024)
route_scan_stats_kernel(const typename Elem<XDT>::T *__restrict__ x, int S, int d, double *__restrict__ stats) {
    __shared__ double s_sum[64][33];
    __shared__ float s_abs[64][33];
    __shared__ int s_emin[64][33];
    const int c2 = threadIdx.x & 31, k = threadIdx.x >> 5;
    const int b = blockIdx.y;
    const int col = blockIdx.x * 64 + 2 * c2;
    const int len = (S + 31) / 32;
    const int t0 = k * len, t1 = min(S, t0 + len);
    const bool live = col < d;
    const typename Elem<XDT>::T *xc = x + static_cast<int64_t>(b) * S * d + (live ? col : 0);
    double sum0 = 0.0, sum1 = 0.0;
    float as0 = 0.0f, as1 = 0.0f;
    uint32_t mn0 = 0xFFFFFFFFu, mn1 = 0xFFFFFFFFu;
    for (int t = t0; t < t1; ++t) {
        const float2 v = Pair<XDT>::load(xc + static_cast<int64_t>(t) * d);
        sum0 = __dadd_rn(sum0, static_cast<double>(v.x));
        sum1 = __dadd_rn(sum1, static_cast<double>(v.y));
        as0 = __fadd_ru(as0, fabsf(v.x));
        as1 = __fadd_ru(as1, fabsf(v.y));
        mn0 = min(mn0, (__float_as_uint(v.x) & 0x7FFFFFFFu) - 1u);
        mn1 = min(mn1, (__float_as_uint(v.y) & 0x7FFFFFFFu) - 1u);
    }
    auto em_of = [](uint32_t mn) -> int {
        return mn == 0xFFFFFFFFu ? (1 << 20) : ulp_exponent<XDT>(__uint_as_float(mn + 1u));
    };
    s_sum[2 * c2][k] = sum0;
    s_sum[2 * c2 + 1][k] = sum1;
    s_abs[2 * c2][k] = as0;
    s_abs[2 * c2 + 1][k] = as1;
    s_emin[2 * c2][k] = em_of(mn0);
    s_emin[2 * c2 + 1][k] = em_of(mn1);
    __syncthreads();
    const int cc = threadIdx.x;
    const int ccol = blockIdx.x * 64 + cc;
    if (cc < 64 && ccol < d) {
        double run = 0.0, at = 0.0;
        int em = 1 << 20;
        for (int kk = 0; kk < 32; ++kk) {
            run = __dadd_rn(run, s_sum[cc][kk]);
            at = __dadd_ru(at, static_cast<double>(s_abs[cc][kk]));
            em = min(em, s_emin[cc][kk]);
        }
        const int64_t bd = static_cast<int64_t>(gridDim.y) * d, i = static_cast<int64_t>(b) * d + ccol;
        stats[i] = run;
        stats[bd + i] = at;
        stats[2 * bd + i] = static_cast<double>(em);
    }
}

__global__ void __launch_bounds__(256)
route_shard_carry_kernel(const double *__restrict__ all, int W, int rank, int64_t bd, double *__restrict__ carry,
                         int *__restrict__ uncertified) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < bd;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        double run = 0.0, at = 0.0;
        int em = 1 << 20;
        for (int j = 0; j < W; ++j) {
            const double *st = all + static_cast<int64_t>(j) * 3 * bd;
            if (j < rank) run = __dadd_rn(run, st[i]);
            at = __dadd_ru(at, st[bd + i]);                 // stays an upper bound of A
            em = min(em, static_cast<int>(st[2 * bd + i]));
        }
        const bool cert = (em == (1 << 20)) || (em > -1000 && at < ldexp(1.0, 52 + em));
        carry[i] = run;
        carry[bd + i] = cert ? 1.0 : 0.0;
        if (!cert) atomicAdd(uncertified, 1);
    }
}

// ============================================================ router head
// Per token: z = round(hq . Wd^T), act = round(tanh z), logits = round(act . Wu^T),
// then softmax, top-k (value desc; torch's CUDA order on ties) and the gate softmax.
constexpr int kHeadTokens = 64;   // tokens per CTA
constexpr int kHeadThreads = 128; // 4 warps x 16 tokens (mma path)
constexpr int kHeadKC = 64;       // d-columns per pipeline step
constexpr int kHeadStages = 4;    // cp.async ring depth of the tensor-core head (3 steps in flight)
constexpr int kMaxNb = 64;
constexpr int kMaxRank = 128;

// Epilogue shared by both head variants: sA holds act (fp32 values already
// rounded to the compute dtype) for kHeadTokens tokens x r. W_up is staged in
// shared memory as fp32 (rows padded to r + 1 floats: the warp's 8 blocks hit 8
// banks), the logits are the same sequential fp32 FMA chains over j as the
// reference's linear, fully unrolled when the rank is a compile-time R. Per
// token: top-k on the logits (+ noise), then the softmax with one exp per logit.
// Order of the selected top-k as torch's CUDA topk returns it when selected
// values are equal (measured on B200 against torch.topk for 8 / 16 / 32 blocks,
// k = 1..8, fp32 and bf16, by an exhaustive comparison over recorded outputs).
// torch gathers the selection as (values above the k-th value, in index order)
// then (values equal to it, in index order), and sorts that list with a
// 32-wide bitonic network (Batcher) whose compare-exchange, descending, also
// exchanges equal keys; unused slots sort to the end. The network is run here
// on the same list, so ties come out in the same order. Only tokens with equal
// selected values take this path (about 1 % of tokens with bf16 logits).
__device__ __noinline__ void torch_cuda_topk_order(const float *lg, const float *noise_row, int nb, int top,
                                                   uint64_t taken, float *vals, int *idxs) {
    constexpr int P = 32;
    float key[P];
    int val[P];
    bool ok[P];
    const float kth = vals[top - 1];
    int n = 0;
    for (int pass = 0; pass < 2; ++pass)
        for (int e = 0; e < nb; ++e) {
            if (!((taken >> e) & 1ull)) continue;
            const float v = noise_row ? lg[e] + noise_row[e] : lg[e];
            if (pass == 0 ? v > kth : v == kth) { key[n] = v; val[n] = e; ok[n] = true; ++n; }
        }
    for (int i = n; i < P; ++i) { key[i] = 0.0f; val[i] = -1; ok[i] = false; }
    auto cmpx = [&](int a, int b, bool dir) {
        const bool greater = ok[a] && ok[b] && key[a] > key[b];
        const bool swap = greater || !ok[b];
        if (swap == dir) {
            const float tk = key[a]; key[a] = key[b]; key[b] = tk;
            const int tv = val[a]; val[a] = val[b]; val[b] = tv;
            const bool to = ok[a]; ok[a] = ok[b]; ok[b] = to;
        }
    };
    for (int size = 2; size < P; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1)
            for (int i = 0; i < P / 2; ++i) {
                const int pos = 2 * i - (i & (stride - 1));
                cmpx(pos, pos + stride, (i & (size >> 1)) != 0);
            }
    for (int stride = P >> 1; stride > 0; stride >>= 1)
        for (int i = 0; i < P / 2; ++i) {
            const int pos = 2 * i - (i & (stride - 1));
            cmpx(pos, pos + stride, false);
        }
    for (int k = 0; k < top; ++k) { vals[k] = key[k]; idxs[k] = val[k]; }
}

template <int CDT, int R>
__device__ void head_epilogue(const float *sA, float *sLogit, float *sWu, const typename Elem<CDT>::T *w_up,
                              int r_rt, int nb, int top, int64_t tok0, int64_t ntok,
                              const float *__restrict__ noise, float *__restrict__ probs,
                              void *__restrict__ top_idx, int idx64, float *__restrict__ gates,
                              float *__restrict__ log_gates) {
    const int r = R > 0 ? R : r_rt;
    const int ws = r + 1;
    const int tid = threadIdx.x;
    for (int i = tid; i < nb * r; i += blockDim.x) sWu[(i / r) * ws + i % r] = Elem<CDT>::load(w_up, i);
    __syncthreads();
    for (int i = tid; i < kHeadTokens * nb; i += blockDim.x) {
        const int tl = i / nb, e = i % nb;
        const float *a = sA + tl * r, *w = sWu + e * ws;
        float acc = 0.0f;
        if (R > 0) {
#pragma unroll
            for (int j = 0; j < R; ++j) acc = __fmaf_rn(a[j], w[j], acc);
        } else {
            for (int j = 0; j < r; ++j) acc = __fmaf_rn(a[j], w[j], acc);
        }
        sLogit[tl * nb + e] = Elem<CDT>::round(acc);
    }
    __syncthreads();
    if (tid < kHeadTokens && tok0 + tid < ntok) {
        const int64_t t = tok0 + tid;
        float *lg = sLogit + tid * nb;
        float m = -INFINITY;
        for (int e = 0; e < nb; ++e) m = fmaxf(m, lg[e]);
        // top-k by repeated selection: strictly greater wins, so among equal
        // values the lower block ids are the ones selected at the k-th boundary.
        // the selected values and ids stay in registers: every loop over them is
        // unrolled over the compile-time bound kMaxTop
        float vals[kMaxTop];
        int idxs[kMaxTop];
        uint64_t taken = 0;
#pragma unroll
        for (int k = 0; k < kMaxTop; ++k) {
            vals[k] = -INFINITY;
            idxs[k] = 0;
            if (k < top) {
                float best = -INFINITY;
                int bi = -1;
                for (int e = 0; e < nb; ++e) {
                    if ((taken >> e) & 1ull) continue;
                    const float v = noise ? lg[e] + noise[t * nb + e] : lg[e];
                    if (bi < 0 || v > best) { best = v; bi = e; }
                }
                taken |= 1ull << bi;
                vals[k] = best;
                idxs[k] = bi;
            }
        }
        // Output order as torch's CUDA topk gives it (the reference's eager
        // router on the GPU, model.py:214). Distinct values come out by value
        // descending whatever the method; only equal selected values need care.
        bool tied = false;
#pragma unroll
        for (int a = 1; a < kMaxTop; ++a) tied |= a < top && vals[a] == vals[a - 1];
        if (tied && top <= 3) {
            // for k <= 3 torch's network lists each run of equal values by
            // descending id: the selection has them ascending, so reverse the run
            if (top == 3 && vals[0] == vals[1] && vals[1] == vals[2]) {
                const int x = idxs[0]; idxs[0] = idxs[2]; idxs[2] = x;
            } else if (vals[0] == vals[1]) {
                const int x = idxs[0]; idxs[0] = idxs[1]; idxs[1] = x;
            } else if (top == 3 && vals[1] == vals[2]) {
                const int x = idxs[1]; idxs[1] = idxs[2]; idxs[2] = x;
            }
        } else if (tied) {
            // top >= 4 with equal selected values: the network, on copies in local memory
            float tv[kMaxTop];
            int ti[kMaxTop];
#pragma unroll
            for (int k = 0; k < kMaxTop; ++k) { tv[k] = vals[k]; ti[k] = idxs[k]; }
            torch_cuda_topk_order(lg, noise ? noise + t * nb : nullptr, nb, top, taken, tv, ti);
#pragma unroll
            for (int k = 0; k < kMaxTop; ++k) { vals[k] = tv[k]; idxs[k] = ti[k]; }
        }
        // softmax over the clean logits, exp once per logit (in place)
        float ssum = 0.0f;
        for (int e = 0; e < nb; ++e) {
            const float x = expf(lg[e] - m);
            lg[e] = x;
            ssum += x;
        }
        for (int e = 0; e < nb; ++e) probs[t * nb + e] = lg[e] / ssum;
        float gm = vals[0];
#pragma unroll
        for (int k = 1; k < kMaxTop; ++k) gm = k < top ? fmaxf(gm, vals[k]) : gm;
        float ex[kMaxTop];
        float gs = 0.0f;
#pragma unroll
        for (int k = 0; k < kMaxTop; ++k) {
            ex[k] = k < top ? expf(vals[k] - gm) : 0.0f;
            gs += ex[k];
        }
#pragma unroll
        for (int k = 0; k < kMaxTop; ++k) {
            if (k < top) {
                const float g = ex[k] / gs;
                gates[t * top + k] = g;
                if (log_gates) log_gates[t * top + k] = logf(fmaxf(g, 1e-9f));
                if (idx64) reinterpret_cast<int64_t *>(top_idx)[t * top + k] = idxs[k];
                else reinterpret_cast<int32_t *>(top_idx)[t * top + k] = idxs[k];
            }
        }
    }
}

// bf16 compute dtype: z on the tensor cores (bf16 x bf16 products are exact in
// fp32; fp32 accumulation), r must be 32 or 64 here.
template <int RANK>
__global__ void __launch_bounds__(kHeadThreads)
route_head_bf16_kernel(const uint16_t *__restrict__ hq, const uint16_t *__restrict__ w_down,
                       const uint16_t *__restrict__ w_up, int64_t ntok, int d, int nb, int top,
                       const float *__restrict__ noise, float *__restrict__ probs,
                       void *__restrict__ top_idx, int idx64, float *__restrict__ gates,
                       float *__restrict__ log_gates, uint16_t *__restrict__ act) {
    constexpr int kRowB = kHeadKC * 2;                   // 128 B per smem row
    constexpr int kHqBytes = kHeadTokens * kRowB;        // 8 KB
    constexpr int kWBytes = RANK * kRowB;                // 4/8 KB
    constexpr int kStage = kHqBytes + kWBytes;
    constexpr int NT = RANK / 8;                          // n-tiles of 8
    extern __shared__ __align__(128) unsigned char smem[];
    float *sA = reinterpret_cast<float *>(smem + kHeadStages * kStage);
    float *sLogit = sA + kHeadTokens * RANK;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * kHeadTokens;
    const int nchunk = d / kHeadKC;

    auto issue = [&](int c) {
        if (c < nchunk) {
            const uint32_t base = smem_u32(smem + (c % kHeadStages) * kStage);
            for (int i = tid; i < kHeadTokens * 8; i += kHeadThreads) {
                const int row = i >> 3, ch = i & 7;
                const int64_t t = tok0 + row;
                const bool ok = t < ntok;
                const uint16_t *src = ok ? hq + t * d + c * kHeadKC + ch * 8 : hq;
                cp_async16(base + swz(row, ch, kRowB), src, ok ? 16 : 0);
            }
            for (int i = tid; i < RANK * 8; i += kHeadThreads) {
                const int row = i >> 3, ch = i & 7;
                cp_async16(base + kHqBytes + swz(row, ch, kRowB),
                           w_down + static_cast<int64_t>(row) * d + c * kHeadKC + ch * 8, 16);
            }
        }
        cp_async_commit();
    };

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

#pragma unroll
    for (int c = 0; c < kHeadStages - 1; ++c) issue(c);
#pragma unroll 1
    for (int c = 0; c < nchunk; ++c) {
        cp_async_wait<kHeadStages - 2>();
        __syncthreads();   // step c landed for all threads; step c-1's buffer is no longer read
        issue(c + kHeadStages - 1);
        const uint32_t sq = smem_u32(smem + (c % kHeadStages) * kStage);
        const uint32_t sw = sq + kHqBytes;
#pragma unroll
        for (int ks = 0; ks < kHeadKC / 16; ++ks) {
            uint32_t a[4];
            const int arow = warp * 16 + (lane & 15);
            ldmatrix_x4(a, sq + swz(arow, ks * 2 + (lane >> 4), kRowB));
#pragma unroll
            for (int j = 0; j < NT; j += 2) {
                uint32_t bfr[4];
                const int brow = j * 8 + (lane & 7) + ((lane >> 4) << 3);
                ldmatrix_x4(bfr, sw + swz(brow, ks * 2 + ((lane >> 3) & 1), kRowB));
                mma_bf16_16816(acc[j], a, bfr[0], bfr[1]);
                mma_bf16_16816(acc[j + 1], a, bfr[2], bfr[3]);
            }
        }
    }
    cp_async_wait<0>();

    // z -> act, kept as fp32 values rounded to bf16
    const int g = lane >> 2, q2 = (lane & 3) * 2;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = warp * 16 + g + h * 8;
            const int col = j * 8 + q2;
            const float a0 = round_bf16(tanhf(round_bf16(acc[j][2 * h])));
            const float a1 = round_bf16(tanhf(round_bf16(acc[j][2 * h + 1])));
            sA[row * RANK + col] = a0;
            sA[row * RANK + col + 1] = a1;
            const int64_t t = tok0 + row;
            if (act && t < ntok) {
                *reinterpret_cast<uint32_t *>(act + t * RANK + col) = pack_bf16x2(a0, a1);
            }
        }
    }
    __syncthreads();
    // the cp.async ring is idle now: W_up goes there
    head_epilogue<MOM_BF16, RANK>(sA, sLogit, reinterpret_cast<float *>(smem), w_up, RANK, nb, top, tok0, ntok,
                                  noise, probs, top_idx, idx64, gates, log_gates);
}

// Generic SIMT head (fp32 compute dtype, or any rank): fp32 FMA accumulation.
template <int CDT>
__global__ void __launch_bounds__(kHeadThreads)
route_head_simt_kernel(const typename Elem<CDT>::T *__restrict__ hq,
                       const typename Elem<CDT>::T *__restrict__ w_down,
                       const typename Elem<CDT>::T *__restrict__ w_up, int64_t ntok, int d, int r,
                       int nb, int top, const float *__restrict__ noise, float *__restrict__ probs,
                       void *__restrict__ top_idx, int idx64, float *__restrict__ gates,
                       float *__restrict__ log_gates, typename Elem<CDT>::T *__restrict__ act) {
    extern __shared__ __align__(128) unsigned char smem[];
    float *sA = reinterpret_cast<float *>(smem);
    float *sLogit = sA + kHeadTokens * r;
    float *sH = sLogit + kHeadTokens * kMaxNb;         // kHeadTokens x kHeadKC
    float *sW = sH + kHeadTokens * kHeadKC;             // r x kHeadKC
    const int tid = threadIdx.x;
    const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * kHeadTokens;
    // thread -> (token tl, ranks j = jr, jr + 2, ...)
    const int tl = tid >> 1, jr = tid & 1;
    float acc[kMaxRank / 2];
    for (int j = 0; j < kMaxRank / 2; ++j) acc[j] = 0.0f;
    for (int c0 = 0; c0 < d; c0 += kHeadKC) {
        const int kc = min(kHeadKC, d - c0);
        __syncthreads();
        for (int i = tid; i < kHeadTokens * kHeadKC; i += blockDim.x) {
            const int row = i / kHeadKC, cc = i % kHeadKC;
            const int64_t t = tok0 + row;
            sH[i] = (t < ntok && cc < kc) ? Elem<CDT>::load(hq, t * d + c0 + cc) : 0.0f;
        }
        for (int i = tid; i < r * kHeadKC; i += blockDim.x) {
            const int row = i / kHeadKC, cc = i % kHeadKC;
            sW[i] = cc < kc ? Elem<CDT>::load(w_down, static_cast<int64_t>(row) * d + c0 + cc) : 0.0f;
        }
        __syncthreads();
        for (int jj = 0, j = jr; j < r; j += 2, ++jj) {
            float a = acc[jj];
            for (int cc = 0; cc < kc; ++cc) a = __fmaf_rn(sH[tl * kHeadKC + cc], sW[j * kHeadKC + cc], a);
            acc[jj] = a;
        }
    }
    for (int jj = 0, j = jr; j < r; j += 2, ++jj) {
        const float a = Elem<CDT>::round(tanhf(Elem<CDT>::round(acc[jj])));
        sA[tl * r + j] = a;
        const int64_t t = tok0 + tl;
        if (act && t < ntok) Elem<CDT>::store(act, t * r + j, a);
    }
    __syncthreads();
    // sH and sW (contiguous, nb x (r + 1) floats fit) are idle now: W_up goes there
    head_epilogue<CDT, 0>(sA, sLogit, sH, w_up, r, nb, top, tok0, ntok, noise, probs, top_idx, idx64,
                       gates, log_gates);
}

// ============================================================ host launchers
template <int XDT, int CDT>
static cudaError_t launch_scan_t(const void *x, void *hq, int B, int S, int d, cudaStream_t st,
                                 const ScanShard &sh) {
    using XT = typename Elem<XDT>::T;
    const size_t smem = seq_scan_smem<XDT>();
    auto k = route_scan_kernel<XDT, CDT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((d + kSeqCols - 1) / kSeqCols, B);
    k<<<grid, kSeqThreads, smem, st>>>(static_cast<const XT *>(x),
                                       static_cast<typename Elem<CDT>::T *>(hq), S, d, sh); count_launch();
    return cudaGetLastError();
}

// 3-D tensor map over x (B, S, d) with a box of 32 columns x kTRows rows of one
// batch row; false when TMA cannot address x (alignment) or the driver entry
// point is missing, and the cp.async kernel is used instead.
static bool make_scan_map(CUtensorMap *map, const void *x, int xdt, int B, int S, int d) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    const uint64_t es = xdt == MOM_F32 ? 4 : 2;
    if (!fn || (reinterpret_cast<uintptr_t>(x) % 16) != 0 || (static_cast<uint64_t>(d) * es) % 16 != 0) return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * es, static_cast<cuuint64_t>(S) * d * es};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(kSeqCols), static_cast<cuuint32_t>(kTRows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType ty = xdt == MOM_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    return fn(map, ty, 3, const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int XDT, int CDT>
static cudaError_t launch_scan_tma_t(const CUtensorMap &map, void *hq, int B, int S, int d, cudaStream_t st,
                                     const ScanShard &sh) {
    const size_t smem = tma_scan_smem<XDT>();
    auto k = route_scan_tma_kernel<XDT, CDT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((d + kSeqCols - 1) / kSeqCols, B);
    k<<<grid, kTThreads, smem, st>>>(map, static_cast<typename Elem<CDT>::T *>(hq), S, d, sh);
    count_launch();
    return cudaGetLastError();
}

template <int XDT, int CDT>
static cudaError_t launch_scan_par_t(const void *x, void *hq, int B, int S, int d, cudaStream_t st,
                                     const ScanShard &sh) {
    dim3 grid((d + 63) / 64, B);
    route_scan_par_kernel<XDT, CDT><<<grid, 1024, 0, st>>>(static_cast<const typename Elem<XDT>::T *>(x),
                                                          static_cast<typename Elem<CDT>::T *>(hq), S, d, sh);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_route_scan(const void *x, int xdt, void *hq, int cdt, int B, int S, int d,
                              int mode, cudaStream_t st, const ScanShard &sh) {
    if (mode == MOM_SCAN_FP64) {
        if (xdt == MOM_BF16 && cdt == MOM_BF16) return launch_scan_par_t<MOM_BF16, MOM_BF16>(x, hq, B, S, d, st, sh);
        if (xdt == MOM_BF16 && cdt == MOM_F32) return launch_scan_par_t<MOM_BF16, MOM_F32>(x, hq, B, S, d, st, sh);
        if (xdt == MOM_F32 && cdt == MOM_BF16) return launch_scan_par_t<MOM_F32, MOM_BF16>(x, hq, B, S, d, st, sh);
        if (xdt == MOM_F32 && cdt == MOM_F32) return launch_scan_par_t<MOM_F32, MOM_F32>(x, hq, B, S, d, st, sh);
        return cudaErrorInvalidValue;
    }
    if (mode != MOM_SCAN_FP32) return cudaErrorInvalidValue;
    CUtensorMap map;
    if (S > 0 && B > 0 && d > 0 && (xdt == MOM_BF16 || xdt == MOM_F32) && (cdt == MOM_BF16 || cdt == MOM_F32) &&
        make_scan_map(&map, x, xdt, B, S, d)) {
        if (xdt == MOM_BF16 && cdt == MOM_BF16) return launch_scan_tma_t<MOM_BF16, MOM_BF16>(map, hq, B, S, d, st, sh);
        if (xdt == MOM_F32 && cdt == MOM_BF16) return launch_scan_tma_t<MOM_F32, MOM_BF16>(map, hq, B, S, d, st, sh);
        if (xdt == MOM_F32 && cdt == MOM_F32) return launch_scan_tma_t<MOM_F32, MOM_F32>(map, hq, B, S, d, st, sh);
        return launch_scan_tma_t<MOM_BF16, MOM_F32>(map, hq, B, S, d, st, sh);
    }
    if (xdt == MOM_BF16 && cdt == MOM_BF16) return launch_scan_t<MOM_BF16, MOM_BF16>(x, hq, B, S, d, st, sh);
    if (xdt == MOM_F32 && cdt == MOM_BF16) return launch_scan_t<MOM_F32, MOM_BF16>(x, hq, B, S, d, st, sh);
    if (xdt == MOM_F32 && cdt == MOM_F32) return launch_scan_t<MOM_F32, MOM_F32>(x, hq, B, S, d, st, sh);
    if (xdt == MOM_BF16 && cdt == MOM_F32) return launch_scan_t<MOM_BF16, MOM_F32>(x, hq, B, S, d, st, sh);
    return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ aux-loss statistics
// The reference's load-balancing aux loss and router logs per MoM layer
// (model.py:476-517) from the stashed probs (N, nb) fp32 and top_idx (N, top):
//   frac_e = (tokens that selected block e) / N, mean_e = sum_t probs[t, e] / N,
//   aux = nb * sum_e frac_e * mean_e, entropy = -sum_t sum_e p log(max(p, 1e-9)) / N,
//   dead = (blocks no token selected) / nb.
// Two launches with a fixed reduction order (deterministic): each CTA of the
// first owns a contiguous token range, thread j takes block e = j % nb of tokens
// j / nb, j / nb + per, ...; it writes its partial sums [sum_e (nb) | sel_e (nb)
// | entropy] to the workspace. One CTA then adds the partials, a warp per column.
// out = [aux, entropy, dead, frac_0 .. frac_{nb-1}] (frac is what the backward needs).
constexpr int kAuxThreads = 256;

template <bool kI64>
__global__ void __launch_bounds__(kAuxThreads)
router_aux_part_kernel(const float *__restrict__ probs, const void *__restrict__ top_idx, int64_t N, int nb, int top,
                       int64_t tok_per_cta, float *__restrict__ part) {
    __shared__ float s_sum[kAuxThreads], s_sel[kAuxThreads], s_ent[kAuxThreads];
    const int per = kAuxThreads / nb;              // tokens per pass
    const int j = threadIdx.x;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * tok_per_cta;
    const int64_t t1 = min(N, t0 + tok_per_cta);
    float psum = 0.0f, sel = 0.0f, ent = 0.0f;
    if (j < per * nb) {
        const int e = j % nb;
#pragma unroll 4
        for (int64_t t = t0 + j / nb; t < t1; t += per) {
            const float p = probs[t * nb + e];
            psum += p;
            ent -= p * logf(fmaxf(p, 1e-9f));
            bool hit = false;
            for (int k = 0; k < top; ++k) {
                const int64_t id = kI64 ? static_cast<const int64_t *>(top_idx)[t * top + k]
                                        : static_cast<const int32_t *>(top_idx)[t * top + k];
                hit |= id == e;
            }
            sel += hit ? 1.0f : 0.0f;
        }
    }
    s_sum[j] = psum;
    s_sel[j] = sel;
    s_ent[j] = ent;
    __syncthreads();
    float *mine = part + static_cast<int64_t>(blockIdx.x) * (2 * nb + 1);
    if (j < nb) {
        float a = 0.0f, c = 0.0f;
        for (int g = 0; g < per; ++g) {
            a += s_sum[g * nb + j];
            c += s_sel[g * nb + j];
        }
        mine[j] = a;
        mine[nb + j] = c;
    }
    if (j == 0) {
        float en = 0.0f;
        for (int i = 0; i < per * nb; ++i) en += s_ent[i];
        mine[2 * nb] = en;
    }
}

// One warp per column of the partials ([sum_e | sel_e | entropy], 2 nb + 1 of
// them): lane l adds parts l, l + 32, ... and the warp combines its lanes by a
// fixed shuffle tree, so the order, and the result, are the same every run.
constexpr int kAuxFinalThreads = 1024;

__global__ void __launch_bounds__(kAuxFinalThreads)
router_aux_final_kernel(const float *__restrict__ part, int nparts, int64_t N, int nb, float *__restrict__ out) {
    __shared__ float s_col[2 * kAuxThreads + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ncols = 2 * nb + 1;
    for (int col = warp; col < ncols; col += kAuxFinalThreads / 32) {
        float a = 0.0f;
        for (int g = lane; g < nparts; g += 32) a += part[static_cast<int64_t>(g) * ncols + col];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) s_col[col] = a;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float inv = 1.0f / static_cast<float>(N);
        float aux = 0.0f;
        int dead = 0;
        for (int e = 0; e < nb; ++e) {
            const float frac = s_col[nb + e] * inv;
            aux += frac * (s_col[e] * inv);
            dead += s_col[nb + e] == 0.0f;
            out[3 + e] = frac;
        }
        out[0] = static_cast<float>(nb) * aux;
        out[1] = s_col[2 * nb] * inv;
        out[2] = static_cast<float>(dead) / static_cast<float>(nb);
    }
}

int64_t router_aux_parts(int64_t N, int nb) {
    const int per = std::max(1, kAuxThreads / nb);
    // about 4 passes of `per` tokens per CTA, at most 296 CTAs
    return std::max<int64_t>(1, std::min<int64_t>(296, (N + 4 * per - 1) / (4 * per)));
}

size_t router_aux_workspace_size(int64_t N, int nb) {
    return sizeof(float) * static_cast<size_t>(router_aux_parts(N, nb)) * (2 * nb + 1);
}

cudaError_t launch_router_aux(const float *probs, const void *top_idx, bool idx64, int64_t N, int nb, int top,
                              float *ws, float *out, cudaStream_t st) {
    if (nb < 1 || nb > kAuxThreads || N < 1) return cudaErrorInvalidValue;
    const int64_t parts = router_aux_parts(N, nb);
    const int64_t tok = (N + parts - 1) / parts;
    if (idx64)
        router_aux_part_kernel<true><<<static_cast<int>(parts), kAuxThreads, 0, st>>>(probs, top_idx, N, nb, top,
                                                                                      tok, ws);
    else
        router_aux_part_kernel<false><<<static_cast<int>(parts), kAuxThreads, 0, st>>>(probs, top_idx, N, nb, top,
                                                                                       tok, ws);
    count_launch();
    router_aux_final_kernel<<<1, kAuxFinalThreads, 0, st>>>(ws, static_cast<int>(parts), N, nb, out);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_route_shard_stats(const void *x, int xdt, int B, int S, int d, double *stats, cudaStream_t st) {
    dim3 grid((d + 63) / 64, B);
    if (xdt == MOM_BF16)
        route_scan_stats_kernel<MOM_BF16><<<grid, 1024, 0, st>>>(static_cast<const uint16_t *>(x), S, d, stats);
    else if (xdt == MOM_F32)
        route_scan_stats_kernel<MOM_F32><<<grid, 1024, 0, st>>>(static_cast<const float *>(x), S, d, stats);
    else
        return cudaErrorInvalidValue;
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_route_shard_carry(const double *stats_all, int W, int rank, int B, int d, double *carry,
                                     int *uncertified, cudaStream_t st) {
    const int64_t bd = static_cast<int64_t>(B) * d;
    cudaError_t e = cudaMemsetAsync(uncertified, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((bd + 255) / 256, 148 * 8)));
    route_shard_carry_kernel<<<grid, 256, 0, st>>>(stats_all, W, rank, bd, carry, uncertified);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_route_head(const void *hq, const void *w_down, const void *w_up, int cdt,
                              int64_t ntok, int d, int r, int nb, int top, const float *noise,
                              float *probs, void *top_idx, int idx64, float *gates,
                              float *log_gates, void *act, cudaStream_t st) {
    const int grid = static_cast<int>((ntok + kHeadTokens - 1) / kHeadTokens);
    if (cdt == MOM_BF16 && (r == 32 || r == 64) && d % kHeadKC == 0) {
        const size_t smem = kHeadStages * (kHeadTokens + r) * kHeadKC * 2 +
                            (kHeadTokens * r + kHeadTokens * kMaxNb) * sizeof(float);
        if (r == 32) {
            auto k = route_head_bf16_kernel<32>;
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            k<<<grid, kHeadThreads, smem, st>>>(
                static_cast<const uint16_t *>(hq), static_cast<const uint16_t *>(w_down),
                static_cast<const uint16_t *>(w_up), ntok, d, nb, top, noise, probs, top_idx, idx64,
                gates, log_gates, static_cast<uint16_t *>(act)); count_launch();
        } else {
            auto k = route_head_bf16_kernel<64>;
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            k<<<grid, kHeadThreads, smem, st>>>(
                static_cast<const uint16_t *>(hq), static_cast<const uint16_t *>(w_down),
                static_cast<const uint16_t *>(w_up), ntok, d, nb, top, noise, probs, top_idx, idx64,
                gates, log_gates, static_cast<uint16_t *>(act)); count_launch();
        }
        return cudaGetLastError();
    }
    const size_t smem = (kHeadTokens * r + kHeadTokens * kMaxNb + kHeadTokens * kHeadKC + r * kHeadKC) * sizeof(float);
    if (cdt == MOM_BF16) {
        auto k = route_head_simt_kernel<MOM_BF16>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<grid, kHeadThreads, smem, st>>>(
            static_cast<const uint16_t *>(hq), static_cast<const uint16_t *>(w_down),
            static_cast<const uint16_t *>(w_up), ntok, d, r, nb, top, noise, probs, top_idx, idx64,
            gates, log_gates, static_cast<uint16_t *>(act)); count_launch();
    } else {
        auto k = route_head_simt_kernel<MOM_F32>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<grid, kHeadThreads, smem, st>>>(
            static_cast<const float *>(hq), static_cast<const float *>(w_down),
            static_cast<const float *>(w_up), ntok, d, r, nb, top, noise, probs, top_idx, idx64,
            gates, log_gates, static_cast<float *>(act)); count_launch();
    }
    return cudaGetLastError();
}

}  // namespace mom
