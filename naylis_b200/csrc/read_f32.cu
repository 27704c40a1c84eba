// Gated memory read in fp32 (forward and backward), for fp32 activations:
// the reference's fp32 semantics (mom_kernels/reference.py:14-61; its fp32 read
// is held to 1e-5 against an independent implementation, tests/test_parity.py
// :138-188) computed with fp32 FMA throughout, no tensor-core rounding.
//
// It runs on the block-split plan (mom_bucket_split): rows are (token, k)
// pairs grouped into tiles of <= 128 rows that read the same one block, and a
// block a token picked twice is one live row carrying the sum of its
// log-gates (the reference's one-hot bias sums them), the later picks dead.
//
//   forward   CTA per (tile, head), a row per thread (two threads per row at
//             head_dim 128, 64 dimensions each; head_dim 16 / 32 / 64 / 128): the block's K / V staged in
//             shared memory 32 slots at a time, online softmax in registers;
//             each row writes its normalised output and log-sum-exp.
//   combine   per (token, head) over its live rows: lse = logsumexp_k lse_k,
//             out = sum_k exp(lse_k - lse) out_k.
//   backward  delta = <dO, O> per (token, head); then
//             row kernel   (tile, head), a row per thread: p = exp(s - lse) with
//                          the token's full lse, dp = dO.V, dS = p (dp - delta),
//                          dQ += dS K (fp32 atomics into the token's dq row),
//                          the gate gradient sum dS (atomics over heads, into
//                          every pick of the block);
//             slot kernel  (tile, head), a slot per 2 (4) threads of 32
//                          dimensions: dK += dS q, dV += p dO over the tile's
//                          rows staged in shared memory, one fp32 atomic per
//                          element and tile at the end.
// The exponentials are expf / logf (not the log2-domain approximations of the
// bf16 kernels). Sum orders differ from the reference's; the results agree to
// ~1e-6 relative.
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace mom {
namespace {

constexpr int kRows = 128;     // plan tile rows
constexpr int kSlotStep = 32;  // K / V slots staged per step (forward and row kernels)
constexpr int kRowStep = 16;   // rows staged per step (slot kernel)

__device__ __forceinline__ int64_t idx_at(const void *idx, int idx64, int64_t i) {
    return idx64 ? static_cast<const int64_t *>(idx)[i] : static_cast<const int32_t *>(idx)[i];
}

// For token t: bit k set if pick k repeats the block of an earlier pick;
// first[k] = the earliest pick of pick k's block.
__device__ __forceinline__ uint32_t dup_picks(const void *idx, int idx64, int64_t t, int top, int (&first)[kMaxTop]) {
    int64_t b[kMaxTop];
    for (int k = 0; k < top; ++k) b[k] = idx_at(idx, idx64, t * top + k);
    uint32_t dead = 0;
    for (int k = 0; k < top; ++k) {
        int f = k;
        for (int j = k - 1; j >= 0; --j)
            if (b[j] == b[k]) f = j;
        first[k] = f;
        if (f != k) dead |= 1u << k;
    }
    return dead;
}

template <int HD>
__device__ __forceinline__ void stage_kv(float (*sK)[HD], float (*sV)[HD], const float *k, const float *v,
                                         int64_t slot0, int n, int64_t ld, int h) {
    constexpr int kVec = HD / 4;
    for (int i = threadIdx.x; i < kSlotStep * kVec; i += blockDim.x) {
        const int s = i / kVec, c = i % kVec;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
        if (s < n) {
            const int64_t off = (slot0 + s) * ld + static_cast<int64_t>(h) * HD + 4 * c;
            a = *reinterpret_cast<const float4 *>(k + off);
            b = *reinterpret_cast<const float4 *>(v + off);
        }
        *reinterpret_cast<float4 *>(&sK[s][4 * c]) = a;
        *reinterpret_cast<float4 *>(&sV[s][4 * c]) = b;
    }
}

// The plan row of this thread: its (token, pick), block, bias and whether it
// is live (a real row whose pick is the first of its block).
struct RowInfo {
    int64_t t;
    int k;
    float bias;
    bool live;
};

__device__ __forceinline__ RowInfo row_info(const PlanView &P, int row, bool in_tile, int top, const void *idx,
                                            int idx64) {
    RowInfo ri{0, 0, 0.0f, false};
    if (!in_tile) return ri;
    const int pair = P.perm[row];
    ri.t = pair / top;
    ri.k = pair - static_cast<int>(ri.t) * top;
    ri.bias = P.rowbias[row];
    int first[kMaxTop];
    ri.live = !((dup_picks(idx, idx64, ri.t, top, first) >> ri.k) & 1);
    return ri;
}

// Threads per row and dimensions per thread of the row kernels: 64 dimensions
// a thread (two threads a row at head_dim 128).
template <int HD> struct RowSplit {
    static constexpr int TPR = HD > 64 ? HD / 64 : 1;
    static constexpr int D = HD / TPR;
};

template <int HD>
__global__ void __launch_bounds__(kRows * RowSplit<HD>::TPR)
read_f32_fwd_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int H,
                    int bs, int top, float scale, PlanView P, const void *__restrict__ idx, int idx64,
                    float *__restrict__ o_rows, float *__restrict__ lse_rows) {
    constexpr int TPR = RowSplit<HD>::TPR;   // threads per row
    constexpr int D = RowSplit<HD>::D;       // dimensions per thread
    __shared__ __align__(16) float sK[kSlotStep][HD];
    __shared__ __align__(16) float sV[kSlotStep][HD];
    const int tile = blockIdx.x;
    if (tile >= *P.ntiles) return;
    const int h = blockIdx.y;
    const int4 td = P.tiles[tile];
    const int blk = P.keyset[td.z];
    const int rr = threadIdx.x / TPR, part = threadIdx.x % TPR;
    const int row = td.x + rr;
    const RowInfo ri = row_info(P, row, rr < td.y, top, idx, idx64);
    const int64_t ld = static_cast<int64_t>(H) * HD;
    float qv[D], o[D];
    const float *qrow = q + ri.t * ld + static_cast<int64_t>(h) * HD + part * D;
#pragma unroll
    for (int i = 0; i < D; i += 4) {
        const float4 a = rr < td.y ? *reinterpret_cast<const float4 *>(qrow + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        qv[i] = a.x; qv[i + 1] = a.y; qv[i + 2] = a.z; qv[i + 3] = a.w;
        o[i] = o[i + 1] = o[i + 2] = o[i + 3] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    for (int c0 = 0; c0 < bs; c0 += kSlotStep) {
        const int n = min(kSlotStep, bs - c0);
        __syncthreads();
        stage_kv<HD>(sK, sV, k, v, static_cast<int64_t>(blk) * bs + c0, n, ld, h);
        __syncthreads();
        for (int s = 0; s < n; ++s) {
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < D; ++i) dot = fmaf(qv[i], sK[s][part * D + i], dot);
            if (TPR == 2) dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            const float x = fmaf(dot, scale, ri.bias);
            if (x > m) {
                const float corr = expf(m - x);
                l *= corr;
#pragma unroll
                for (int i = 0; i < D; ++i) o[i] *= corr;
                m = x;
            }
            const float p = expf(x - m);
            l += p;
#pragma unroll
            for (int i = 0; i < D; ++i) o[i] = fmaf(p, sV[s][part * D + i], o[i]);
        }
    }
    if (rr < td.y) {
        const float inv = 1.0f / l;
        float *orow = o_rows + (static_cast<int64_t>(row) * H + h) * HD + part * D;
#pragma unroll
        for (int i = 0; i < D; i += 4) *reinterpret_cast<float4 *>(orow + i) =
            make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
        if (part == 0) lse_rows[static_cast<int64_t>(row) * H + h] = m + logf(l);
    }
}

// Per (token, head): the union of the token's live rows. A pick outside
// [0, nb) has no row in the plan (the bucketing drops it and reports it), so
// it counts as dead here too.
__global__ void __launch_bounds__(256)
read_f32_combine_kernel(const float *__restrict__ o_rows, const float *__restrict__ lse_rows,
                        const int *__restrict__ iperm, const void *__restrict__ idx, int idx64, int64_t N, int top,
                        int nb, int H, int hd, float *__restrict__ out, float *__restrict__ lse) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < N * H;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / H;
        const int h = static_cast<int>(i - t * H);
        int first[kMaxTop];
        uint32_t dead = dup_picks(idx, idx64, t, top, first);
        for (int kk = 0; kk < top; ++kk) {
            const int64_t b = idx_at(idx, idx64, t * top + kk);
            if (b < 0 || b >= nb) dead |= 1u << kk;
        }
        float mx = -INFINITY;
        for (int kk = 0; kk < top; ++kk)
            if (!((dead >> kk) & 1)) mx = fmaxf(mx, lse_rows[static_cast<int64_t>(iperm[t * top + kk]) * H + h]);
        float sum = 0.0f;
        for (int kk = 0; kk < top; ++kk)
            if (!((dead >> kk) & 1)) sum += expf(lse_rows[static_cast<int64_t>(iperm[t * top + kk]) * H + h] - mx);
        const float L = mx + logf(sum);
        float *orow = out + (t * H + h) * hd;
        for (int d = 0; d < hd; d += 4) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int kk = 0; kk < top; ++kk) {
                if ((dead >> kk) & 1) continue;
                const int64_t r = iperm[t * top + kk];
                const float a = expf(lse_rows[r * H + h] - L);
                const float4 x = *reinterpret_cast<const float4 *>(o_rows + (r * H + h) * hd + d);
                acc.x = fmaf(a, x.x, acc.x); acc.y = fmaf(a, x.y, acc.y);
                acc.z = fmaf(a, x.z, acc.z); acc.w = fmaf(a, x.w, acc.w);
            }
            *reinterpret_cast<float4 *>(orow + d) = acc;
        }
        lse[t * H + h] = L;
    }
}

__global__ void __launch_bounds__(256)
read_f32_delta_kernel(const float *__restrict__ out, const float *__restrict__ dout, int64_t NH, int hd,
                      float *__restrict__ delta) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < NH;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float *a = out + i * hd, *b = dout + i * hd;
        float s = 0.0f;
        for (int d = 0; d < hd; ++d) s = fmaf(a[d], b[d], s);
        delta[i] = s;
    }
}

template <int HD>
__global__ void __launch_bounds__(kRows * RowSplit<HD>::TPR)
read_f32_bwd_row_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                        const float *__restrict__ dout, const float *__restrict__ lse,
                        const float *__restrict__ delta, int H, int bs, int top, float scale, PlanView P,
                        const void *__restrict__ idx, int idx64, float *__restrict__ dq,
                        float *__restrict__ dlog_gates) {
    constexpr int TPR = RowSplit<HD>::TPR;
    constexpr int D = RowSplit<HD>::D;
    __shared__ __align__(16) float sK[kSlotStep][HD];
    __shared__ __align__(16) float sV[kSlotStep][HD];
    const int tile = blockIdx.x;
    if (tile >= *P.ntiles) return;
    const int h = blockIdx.y;
    const int4 td = P.tiles[tile];
    const int blk = P.keyset[td.z];
    const int rr = threadIdx.x / TPR, part = threadIdx.x % TPR;
    const int row = td.x + rr;
    const RowInfo ri = row_info(P, row, rr < td.y, top, idx, idx64);
    const int64_t ld = static_cast<int64_t>(H) * HD;
    const int64_t off = ri.t * ld + static_cast<int64_t>(h) * HD + part * D;
    float qv[D], gv[D], acc[D];
#pragma unroll
    for (int i = 0; i < D; i += 4) {
        const float4 a = ri.live ? *reinterpret_cast<const float4 *>(q + off + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 b = ri.live ? *reinterpret_cast<const float4 *>(dout + off + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        qv[i] = a.x; qv[i + 1] = a.y; qv[i + 2] = a.z; qv[i + 3] = a.w;
        gv[i] = b.x; gv[i + 1] = b.y; gv[i + 2] = b.z; gv[i + 3] = b.w;
        acc[i] = acc[i + 1] = acc[i + 2] = acc[i + 3] = 0.0f;
    }
    const float L = ri.live ? lse[ri.t * H + h] : 0.0f;
    const float dl = ri.live ? delta[ri.t * H + h] : 0.0f;
    float dsum = 0.0f;
    for (int c0 = 0; c0 < bs; c0 += kSlotStep) {
        const int n = min(kSlotStep, bs - c0);
        __syncthreads();
        stage_kv<HD>(sK, sV, k, v, static_cast<int64_t>(blk) * bs + c0, n, ld, h);
        __syncthreads();
        for (int s = 0; s < n; ++s) {
            float dot = 0.0f, dp = 0.0f;
#pragma unroll
            for (int i = 0; i < D; ++i) {
                dot = fmaf(qv[i], sK[s][part * D + i], dot);
                dp = fmaf(gv[i], sV[s][part * D + i], dp);
            }
            if (TPR == 2) {
                dot += __shfl_xor_sync(0xffffffffu, dot, 1);
                dp += __shfl_xor_sync(0xffffffffu, dp, 1);
            }
            const float p = expf(fmaf(dot, scale, ri.bias) - L);
            const float ds = p * (dp - dl);
            dsum += ds;
#pragma unroll
            for (int i = 0; i < D; ++i) acc[i] = fmaf(ds, sK[s][part * D + i], acc[i]);
        }
    }
    if (!ri.live) return;
    float *dqrow = dq + off;
#pragma unroll
    for (int i = 0; i < D; ++i) atomicAdd(dqrow + i, acc[i] * scale);
    if (part == 0) {
        // d bias / d log_gate = 1 for every pick of this block (a repeated pick's
        // log-gate is part of the live row's bias)
        int first[kMaxTop];
        dup_picks(idx, idx64, ri.t, top, first);
        for (int kk = 0; kk < top; ++kk)
            if (first[kk] == ri.k) atomicAdd(dlog_gates + ri.t * top + kk, dsum);
    }
}

template <int HD>
__global__ void __launch_bounds__(256)
read_f32_bwd_slot_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                         const float *__restrict__ dout, const float *__restrict__ lse,
                         const float *__restrict__ delta, int H, int bs, int top, float scale, PlanView P,
                         const void *__restrict__ idx, int idx64, float *__restrict__ dk_acc,
                         float *__restrict__ dv_acc) {
    constexpr int D = HD < 32 ? HD : 32;   // dimensions per thread
    constexpr int TPS = HD / D;            // threads per slot (1, 2 or 4, within one warp)
    constexpr int kSlots = 256 / TPS;      // slots per pass
    __shared__ __align__(16) float sQ[kRowStep][HD];
    __shared__ __align__(16) float sG[kRowStep][HD];
    __shared__ float sBias[kRowStep], sL[kRowStep], sD[kRowStep];
    __shared__ int sLive[kRowStep];
    const int tile = blockIdx.x;
    if (tile >= *P.ntiles) return;
    const int h = blockIdx.y;
    const int4 td = P.tiles[tile];
    const int blk = P.keyset[td.z];
    const int64_t ld = static_cast<int64_t>(H) * HD;
    const int js = threadIdx.x / TPS, part = threadIdx.x % TPS;
    for (int j0 = 0; j0 < bs; j0 += kSlots) {
        const int j = j0 + js;
        const bool slot_ok = j < bs;
        const int64_t soff = (static_cast<int64_t>(blk) * bs + (slot_ok ? j : 0)) * ld + static_cast<int64_t>(h) * HD +
                             part * D;
        float kv[D], vv[D], dkv[D], dvv[D];
#pragma unroll
        for (int i = 0; i < D; ++i) {
            kv[i] = slot_ok ? k[soff + i] : 0.0f;
            vv[i] = slot_ok ? v[soff + i] : 0.0f;
            dkv[i] = dvv[i] = 0.0f;
        }
        for (int r0 = 0; r0 < td.y; r0 += kRowStep) {
            const int nr = min(kRowStep, td.y - r0);
            __syncthreads();
            if (threadIdx.x < kRowStep) {
                const int rr = threadIdx.x;
                const RowInfo ri = row_info(P, td.x + r0 + rr, rr < nr, top, idx, idx64);
                sLive[rr] = ri.live ? 1 : 0;
                sBias[rr] = ri.bias;
                sL[rr] = ri.live ? lse[ri.t * H + h] : 0.0f;
                sD[rr] = ri.live ? delta[ri.t * H + h] : 0.0f;
            }
            for (int i = threadIdx.x; i < kRowStep * (HD / 4); i += blockDim.x) {
                const int rr = i / (HD / 4), c = i % (HD / 4);
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
                if (rr < nr) {
                    const int64_t t = P.perm[td.x + r0 + rr] / top;
                    const int64_t o = t * ld + static_cast<int64_t>(h) * HD + 4 * c;
                    a = *reinterpret_cast<const float4 *>(q + o);
                    b = *reinterpret_cast<const float4 *>(dout + o);
                }
                *reinterpret_cast<float4 *>(&sQ[rr][4 * c]) = a;
                *reinterpret_cast<float4 *>(&sG[rr][4 * c]) = b;
            }
            __syncthreads();
            for (int rr = 0; rr < nr; ++rr) {
                if (!sLive[rr]) continue;
                float dot = 0.0f, dp = 0.0f;
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    dot = fmaf(kv[i], sQ[rr][part * D + i], dot);
                    dp = fmaf(vv[i], sG[rr][part * D + i], dp);
                }
#pragma unroll
                for (int w = 1; w < TPS; w <<= 1) {
                    dot += __shfl_xor_sync(0xffffffffu, dot, w);
                    dp += __shfl_xor_sync(0xffffffffu, dp, w);
                }
                const float p = expf(fmaf(dot, scale, sBias[rr]) - sL[rr]);
                const float ds = p * (dp - sD[rr]);
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    dkv[i] = fmaf(ds, sQ[rr][part * D + i], dkv[i]);
                    dvv[i] = fmaf(p, sG[rr][part * D + i], dvv[i]);
                }
            }
        }
        if (slot_ok) {
            const int64_t o = (static_cast<int64_t>(blk) * bs + j) * ld + static_cast<int64_t>(h) * HD + part * D;
#pragma unroll
            for (int i = 0; i < D; ++i) {
                atomicAdd(dk_acc + o + i, dkv[i] * scale);
                atomicAdd(dv_acc + o + i, dvv[i]);
            }
        }
    }
}

int blocks_for(int64_t work, int per) {
    return static_cast<int>(std::min<int64_t>((work + per - 1) / per, 148 * 32));
}

}  // namespace

cudaError_t launch_read_f32_fwd(const float *q, const float *k, const float *v, int64_t N, int H, int hd, int nb,
                                int bs, int top, const PlanLayout &L, const PlanView &P, const void *idx, int idx64,
                                const int *iperm, float *o_rows, float *lse_rows, float *out, float *lse,
                                cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));
    dim3 grid(static_cast<unsigned>(L.max_tiles), H);
    switch (hd) {
#define MOM_F32_FWD(HDV)                                                                                        \
    case HDV:                                                                                                    \
        read_f32_fwd_kernel<HDV><<<grid, kRows * RowSplit<HDV>::TPR, 0, st>>>(q, k, v, H, bs, top, scale, P, idx, \
                                                                              idx64, o_rows, lse_rows);          \
        break;
        MOM_F32_FWD(16) MOM_F32_FWD(32) MOM_F32_FWD(64) MOM_F32_FWD(128)
#undef MOM_F32_FWD
        default:
            return cudaErrorInvalidValue;
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    read_f32_combine_kernel<<<blocks_for(N * H, 256), 256, 0, st>>>(o_rows, lse_rows, iperm, idx, idx64, N, top, nb,
                                                                    H, hd, out, lse);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_read_f32_bwd(const float *q, const float *k, const float *v, const float *out, const float *dout,
                                const float *lse, int64_t N, int H, int hd, int bs, int top, const PlanLayout &L,
                                const PlanView &P, const void *idx, int idx64, float *delta, float *dq,
                                float *dk_acc, float *dv_acc, float *dlog_gates, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));
    read_f32_delta_kernel<<<blocks_for(N * H, 256), 256, 0, st>>>(out, dout, N * H, hd, delta);
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    dim3 grid(static_cast<unsigned>(L.max_tiles), H);
    switch (hd) {
#define MOM_F32_BWD(HDV)                                                                                           \
    case HDV:                                                                                                       \
        read_f32_bwd_row_kernel<HDV><<<grid, kRows * RowSplit<HDV>::TPR, 0, st>>>(                                   \
            q, k, v, dout, lse, delta, H, bs, top, scale, P, idx, idx64, dq, dlog_gates);                            \
        count_launch();                                                                                              \
        read_f32_bwd_slot_kernel<HDV><<<grid, 256, 0, st>>>(q, k, v, dout, lse, delta, H, bs, top, scale, P, idx,   \
                                                            idx64, dk_acc, dv_acc);                                  \
        break;
        MOM_F32_BWD(16) MOM_F32_BWD(32) MOM_F32_BWD(64) MOM_F32_BWD(128)
#undef MOM_F32_BWD
        default:
            return cudaErrorInvalidValue;
    }
    count_launch();
    return cudaGetLastError();
}

}  // namespace mom
