// Gated memory read, backward.
//
// Reference semantics: mom_kernels/triton_gpu.py:143-409 (delta, dq + dlog_gates,
// dk/dv kernels, _MomReadFunction.backward) — same decomposition
// (P rebuilt from the saved log-sum-exp, dS = P (dP - delta)), but every tile
// touches only the blocks its tokens selected:
//
//   read_bwd_dq_kernel    one CTA per token tile, all heads in turn:
//                         delta = rowsum(O*dO), dQ = dS K * scale, and the gate
//                         gradient dlog_gates = sum over heads and the block's
//                         slots of dS, reduced in registers (no atomics) from
//                         per-block fp32 sums of P*dP and P, so that it does not
//                         inherit the rounding of the bf16 output used for delta.
//   read_bwd_dkdv_kernel  one CTA per (block, 64-slot chunk, head, split): walks
//                         the tiles whose set contains the block, accumulates
//                         dK = dS^T Q * scale and dV = P^T dO in registers and
//                         adds them to the fp32 accumulators once.
#include "common.cuh"
#include "launch.h"
#include "read_common.cuh"

namespace mom {

constexpr int kMaxTopBwd = 8;

template <int HD>
__global__ void __launch_bounds__(kReadThreads)
read_bwd_dq_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                   const uint16_t *__restrict__ v, const uint16_t *__restrict__ o,
                   const uint16_t *__restrict__ dout, const float *__restrict__ lse, int H, int bs,
                   int top, float scale, float scale_log2, PlanView P, uint16_t *__restrict__ dq,
                   float *__restrict__ dlog_gates, float *__restrict__ ws_delta) {
    constexpr int kRowB = HD * 2;
    constexpr int kChunks = HD / 8;
    constexpr int kTileBytes = kTileM * kRowB;
    constexpr int kKVBytes = kSlotChunk * kRowB;
    constexpr int NTS = kSlotChunk / 8;
    constexpr int NTO = HD / 8;
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char *sQ = smem;
    unsigned char *sdO = sQ + kTileBytes;
    unsigned char *sO = sdO + kTileBytes;
    unsigned char *sKV = sO + kTileBytes;                          // [2][K|V]
    int *sTok = reinterpret_cast<int *>(sKV + 4 * kKVBytes);
    float *sBias = reinterpret_cast<float *>(sTok + kTileM);      // [kTileM][top], log2 units
    float *sLse = sBias + kTileM * top;                            // log2 units
    float *sDelta = sLse + kTileM;

    const int tile = blockIdx.x;
    if (tile >= *P.ntiles) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int4 td = P.tiles[tile];
    const int row0 = td.x, nrows = td.y;
    const int *set = P.keyset + static_cast<int64_t>(td.z) * top;
    const int64_t ld = static_cast<int64_t>(H) * HD;
    const int g = lane >> 2, q2 = (lane & 3) * 2;

    for (int i = tid; i < kTileM; i += kReadThreads) sTok[i] = i < nrows ? P.perm[row0 + i] : -1;
    for (int i = tid; i < kTileM * top; i += kReadThreads) {
        const int r = i / top;
        sBias[i] = r < nrows ? P.rowbias[static_cast<int64_t>(row0) * top + i] * kLog2e : 0.0f;
    }
    int nblk = 0;
    while (nblk < top && set[nblk] >= 0) ++nblk;
    const int cpb = (bs + kSlotChunk - 1) / kSlotChunk;
    const int nchunk = nblk * cpb;

    // gate-gradient accumulators for rows g and g+8, over all heads
    float dbacc[2][kMaxTopBwd];
#pragma unroll
    for (int jj = 0; jj < kMaxTopBwd; ++jj) dbacc[0][jj] = dbacc[1][jj] = 0.0f;

#pragma unroll 1
    for (int h = 0; h < H; ++h) {
        __syncthreads();
        for (int i = tid; i < kTileM * kChunks; i += kReadThreads) {
            const int r = i / kChunks, ch = i % kChunks;
            const int tok = sTok[r];
            const int64_t off = tok >= 0 ? tok * ld + h * HD + ch * 8 : 0;
            const int64_t offq = tok >= 0 ? (tok / P.rows_per_q) * ld + h * HD + ch * 8 : 0;
            const int nbytes = tok >= 0 ? 16 : 0;
            cp_async16(smem_u32(sQ) + swz(r, ch, kRowB), q + offq, nbytes);
            cp_async16(smem_u32(sdO) + swz(r, ch, kRowB), dout + off, nbytes);
            cp_async16(smem_u32(sO) + swz(r, ch, kRowB), o + offq, nbytes);
        }
        cp_async_commit();
        auto issue = [&](int c) {
            if (c < nchunk) {
                const int j = c / cpb, cc = c % cpb;
                const int valid = min(kSlotChunk, bs - cc * kSlotChunk);
                const int64_t slot0 = static_cast<int64_t>(set[j]) * bs + cc * kSlotChunk;
                const uint32_t sk = smem_u32(sKV + (c & 1) * 2 * kKVBytes);
                const uint32_t sv = sk + kKVBytes;
                for (int i = tid; i < kSlotChunk * kChunks; i += kReadThreads) {
                    const int r = i / kChunks, ch = i % kChunks;
                    const bool ok = r < valid;
                    const int64_t off = ok ? (slot0 + r) * ld + h * HD + ch * 8 : 0;
                    cp_async16(sk + swz(r, ch, kRowB), k + off, ok ? 16 : 0);
                    cp_async16(sv + swz(r, ch, kRowB), v + off, ok ? 16 : 0);
                }
            }
            cp_async_commit();
        };
        issue(0);
        cp_async_wait<1>();
        __syncthreads();
        // delta = rowsum(O * dO) (2 threads per row), lse in log2 units
        {
            const int r = tid >> 1, half = tid & 1;
            float acc = 0.0f;
#pragma unroll
            for (int ch = half * (kChunks / 2); ch < (half + 1) * (kChunks / 2); ++ch) {
                const uint4 a = *reinterpret_cast<const uint4 *>(sO + swz(r, ch, kRowB));
                const uint4 b = *reinterpret_cast<const uint4 *>(sdO + swz(r, ch, kRowB));
                const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    acc = fmaf(__uint_as_float(av[e] << 16), __uint_as_float(bv[e] << 16), acc);
                    acc = fmaf(__uint_as_float(av[e] & 0xFFFF0000u), __uint_as_float(bv[e] & 0xFFFF0000u), acc);
                }
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            const int tok = sTok[r];
            if (half == 0) {
                sDelta[r] = tok >= 0 ? acc : 0.0f;
                sLse[r] = tok >= 0 ? lse[static_cast<int64_t>(h) * P.n + row0 + r] * kLog2e : INFINITY;
                if (tok >= 0) ws_delta[static_cast<int64_t>(h) * P.n + row0 + r] = acc;
            }
        }
        __syncthreads();
        uint32_t qf[HD / 16][4], df[HD / 16][4];
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t off = swz(warp * 16 + (lane & 15), ks * 2 + (lane >> 4), kRowB);
            ldmatrix_x4(qf[ks], smem_u32(sQ) + off);
            ldmatrix_x4(df[ks], smem_u32(sdO) + off);
        }
        const int r0 = warp * 16 + g;
        const float lse0 = sLse[r0], lse1 = sLse[r0 + 8];
        const float dl0 = sDelta[r0], dl1 = sDelta[r0 + 8];
        float dqa[NTO][4];
#pragma unroll
        for (int j = 0; j < NTO; ++j) dqa[j][0] = dqa[j][1] = dqa[j][2] = dqa[j][3] = 0.0f;
        // per block j: A_j = sum P*dP and B_j = sum P over the block's slots
        // (fp32); the gate gradient is A_j - delta * B_j with delta = sum_j A_j,
        // which cancels exactly when a row reads a single block.
        float dba[2][kMaxTopBwd], dbb[2][kMaxTopBwd];
#pragma unroll
        for (int jj = 0; jj < kMaxTopBwd; ++jj) dba[0][jj] = dba[1][jj] = dbb[0][jj] = dbb[1][jj] = 0.0f;

#pragma unroll 1
        for (int c = 0; c < nchunk; ++c) {
            issue(c + 1);
            cp_async_wait<1>();
            __syncthreads();
            const int j = c / cpb, cc = c % cpb;
            const int valid = min(kSlotChunk, bs - cc * kSlotChunk);
            const uint32_t sk = smem_u32(sKV + (c & 1) * 2 * kKVBytes);
            const uint32_t sv = sk + kKVBytes;
            float s[NTS][4], dp[NTS][4];
#pragma unroll
            for (int n = 0; n < NTS; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
                for (int n = 0; n < NTS; n += 2) {
                    const uint32_t off = swz(n * 8 + (lane & 7) + ((lane >> 4) << 3),
                                             ks * 2 + ((lane >> 3) & 1), kRowB);
                    uint32_t b[4];
                    ldmatrix_x4(b, sk + off);
                    mma_bf16_16816(s[n], qf[ks], b[0], b[1]);
                    mma_bf16_16816(s[n + 1], qf[ks], b[2], b[3]);
                    ldmatrix_x4(b, sv + off);
                    mma_bf16_16816(dp[n], df[ks], b[0], b[1]);
                    mma_bf16_16816(dp[n + 1], df[ks], b[2], b[3]);
                }
            }
            const float bias0 = sBias[r0 * top + j], bias1 = sBias[(r0 + 8) * top + j];
            float pa0 = 0.0f, pa1 = 0.0f, pb0 = 0.0f, pb1 = 0.0f;
            uint32_t dsf[NTS / 2][4];
#pragma unroll
            for (int n = 0; n < NTS; ++n) {
                float ds[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int col = n * 8 + q2 + (e & 1);
                    const bool hi = e >= 2;
                    const float p = col < valid
                        ? exp2f(fmaf(s[n][e], scale_log2, hi ? bias1 : bias0) - (hi ? lse1 : lse0))
                        : 0.0f;
                    ds[e] = p * (dp[n][e] - (hi ? dl1 : dl0));
                    if (hi) { pa1 = fmaf(p, dp[n][e], pa1); pb1 += p; }
                    else    { pa0 = fmaf(p, dp[n][e], pa0); pb0 += p; }
                }
                dsf[n >> 1][(n & 1) * 2 + 0] = pack_bf16x2(ds[0], ds[1]);
                dsf[n >> 1][(n & 1) * 2 + 1] = pack_bf16x2(ds[2], ds[3]);
            }
#pragma unroll
            for (int jj = 0; jj < kMaxTopBwd; ++jj)
                if (jj == j) { dba[0][jj] += pa0; dba[1][jj] += pa1; dbb[0][jj] += pb0; dbb[1][jj] += pb1; }
            // dQ += dS K
#pragma unroll
            for (int kk = 0; kk < NTS / 2; ++kk) {
                const uint32_t a[4] = {dsf[kk][0], dsf[kk][1], dsf[kk][2], dsf[kk][3]};
#pragma unroll
                for (int jn = 0; jn < NTO; jn += 2) {
                    uint32_t b[4];
                    ldmatrix_x4_trans(b, sk + swz(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                                  jn + (lane >> 4), kRowB));
                    mma_bf16_16816(dqa[jn], a, b[0], b[1]);
                    mma_bf16_16816(dqa[jn + 1], a, b[2], b[3]);
                }
            }
            __syncthreads();
        }
        cp_async_wait<0>();
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float sa = 0.0f, sb = 0.0f;
#pragma unroll
            for (int jj = 0; jj < kMaxTopBwd; ++jj) {
                dba[r][jj] += __shfl_xor_sync(0xffffffffu, dba[r][jj], 1);
                dba[r][jj] += __shfl_xor_sync(0xffffffffu, dba[r][jj], 2);
                dbb[r][jj] += __shfl_xor_sync(0xffffffffu, dbb[r][jj], 1);
                dbb[r][jj] += __shfl_xor_sync(0xffffffffu, dbb[r][jj], 2);
                sa += dba[r][jj];
                sb += dbb[r][jj];
            }
            // a plan over (token, k) rows reads one block per row: its gate term
            // needs the whole token's delta (from the combined O), not the block's
            const float delta_row = P.rows_per_q > 1 ? (r == 0 ? dl0 : dl1) : (sb > 0.0f ? sa / sb : 0.0f);
#pragma unroll
            for (int jj = 0; jj < kMaxTopBwd; ++jj) dbacc[r][jj] += fmaf(-delta_row, dbb[r][jj], dba[r][jj]);
        }
        // dQ * scale -> stage in sQ (no longer read) -> 16-B stores
        __syncthreads();
#pragma unroll
        for (int jn = 0; jn < NTO; ++jn) {
            *reinterpret_cast<uint32_t *>(sQ + swz(r0, jn, kRowB) + q2 * 2) =
                pack_bf16x2(dqa[jn][0] * scale, dqa[jn][1] * scale);
            *reinterpret_cast<uint32_t *>(sQ + swz(r0 + 8, jn, kRowB) + q2 * 2) =
                pack_bf16x2(dqa[jn][2] * scale, dqa[jn][3] * scale);
        }
        __syncthreads();
        for (int i = tid; i < kTileM * kChunks; i += kReadThreads) {
            const int r = i / kChunks, ch = i % kChunks;
            const int tok = sTok[r];
            if (tok >= 0)
                *reinterpret_cast<uint4 *>(dq + tok * ld + h * HD + ch * 8) =
                    *reinterpret_cast<const uint4 *>(sQ + swz(r, ch, kRowB));
        }
    }
    // gate gradient in the caller's top order
    if ((lane & 3) == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int row = warp * 16 + g + r * 8;
            const int tok = sTok[row];
            if (tok < 0) continue;
            const uint32_t kmap = P.rowkmap[row0 + row];
            for (int kk = 0; kk < top; ++kk) {
                const int jsel = (kmap >> (4 * kk)) & 0xF;
                float val = 0.0f;
#pragma unroll
                for (int jj = 0; jj < kMaxTopBwd; ++jj)
                    if (jj == jsel) val = dbacc[r][jj];
                dlog_gates[static_cast<int64_t>(tok) * top + kk] = val;
            }
        }
    }
}

template <int HD>
__global__ void __launch_bounds__(kDkvThreads)
read_bwd_dkdv_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                     const uint16_t *__restrict__ v, const uint16_t *__restrict__ dout,
                     const float *__restrict__ lse, const float *__restrict__ ws_delta, int H, int bs,
                     int top, int cpb, int nsplit, int max_tiles, float scale, float scale_log2,
                     PlanView P, float *__restrict__ dk_acc, float *__restrict__ dv_acc) {
    constexpr int kRowB = HD * 2;
    constexpr int kChunks = HD / 8;
    constexpr int kTileBytes = kTileM * kRowB;
    constexpr int NTT = kDkvSub / 8;       // token n-tiles per compute sub-tile
    constexpr int NTO = HD / 8;
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char *sK = smem;
    unsigned char *sV = sK + kSlotChunk * kRowB;
    unsigned char *sT = sV + kSlotChunk * kRowB;                   // [2][Q|dO]
    int *sTok = reinterpret_cast<int *>(sT + 4 * kTileBytes);      // [2][kTileM]
    float *sBias = reinterpret_cast<float *>(sTok + 2 * kTileM);   // [2][kTileM] log2 units
    float *sLse = sBias + 2 * kTileM;                              // [2][kTileM] log2 units
    float *sDelta = sLse + 2 * kTileM;                             // [2][kTileM]

    const int blk = blockIdx.x / cpb, cc = blockIdx.x % cpb;
    const int h = blockIdx.y, split = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, q2 = (lane & 3) * 2;
    const int64_t ld = static_cast<int64_t>(H) * HD;
    const int valid = min(kSlotChunk, bs - cc * kSlotChunk);
    const int64_t slot0 = static_cast<int64_t>(blk) * bs + cc * kSlotChunk;
    const int count = P.blkcount[blk];
    const int *list = P.blktiles + static_cast<int64_t>(blk) * max_tiles;
    const int ntile = count > split ? (count - split + nsplit - 1) / nsplit : 0;
    if (ntile == 0) return;

    for (int i = tid; i < kSlotChunk * kChunks; i += kDkvThreads) {
        const int r = i / kChunks, ch = i % kChunks;
        const bool ok = r < valid;
        const int64_t off = ok ? (slot0 + r) * ld + h * HD + ch * 8 : 0;
        cp_async16(smem_u32(sK) + swz(r, ch, kRowB), k + off, ok ? 16 : 0);
        cp_async16(smem_u32(sV) + swz(r, ch, kRowB), v + off, ok ? 16 : 0);
    }
    cp_async_commit();

    // metadata + gathers of the i-th tile of this CTA into buffer i & 1
    auto stage = [&](int i) {
        if (i < ntile) {
            const int buf = i & 1;
            const int tile = list[split + i * nsplit];
            const int4 td = P.tiles[tile];
            const int *set = P.keyset + static_cast<int64_t>(td.z) * top;
            int jb = 0;
            while (jb < top - 1 && set[jb] != blk) ++jb;   // the list only holds tiles whose set has blk
            for (int r = tid; r < kTileM; r += kDkvThreads) {
                const int tok = r < td.y ? P.perm[td.x + r] : -1;
                sTok[buf * kTileM + r] = tok;
                sBias[buf * kTileM + r] = tok >= 0 ? P.rowbias[static_cast<int64_t>(td.x + r) * top + jb] * kLog2e : 0.0f;
                sLse[buf * kTileM + r] = tok >= 0 ? lse[static_cast<int64_t>(h) * P.n + td.x + r] * kLog2e : INFINITY;
                sDelta[buf * kTileM + r] = tok >= 0 ? ws_delta[static_cast<int64_t>(h) * P.n + td.x + r] : 0.0f;
            }
            __syncthreads();
            const uint32_t sq = smem_u32(sT + buf * 2 * kTileBytes);
            const uint32_t sd = sq + kTileBytes;
            for (int e = tid; e < kTileM * kChunks; e += kDkvThreads) {
                const int r = e / kChunks, ch = e % kChunks;
                const int tok = sTok[buf * kTileM + r];
                const int64_t off = tok >= 0 ? tok * ld + h * HD + ch * 8 : 0;
                const int64_t offq = tok >= 0 ? (tok / P.rows_per_q) * ld + h * HD + ch * 8 : 0;
                cp_async16(sq + swz(r, ch, kRowB), q + offq, tok >= 0 ? 16 : 0);
                cp_async16(sd + swz(r, ch, kRowB), dout + off, tok >= 0 ? 16 : 0);
            }
        }
        cp_async_commit();
    };
    stage(0);

    float dka[NTO][4], dva[NTO][4];
#pragma unroll
    for (int j = 0; j < NTO; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) dka[j][e] = dva[j][e] = 0.0f;

#pragma unroll 1
    for (int i = 0; i < ntile; ++i) {
        stage(i + 1);
        cp_async_wait<1>();
        __syncthreads();
        const int buf = i & 1;
        const uint32_t sq = smem_u32(sT + buf * 2 * kTileBytes);
        const uint32_t sd = sq + kTileBytes;
        const float *bias = sBias + buf * kTileM;
        const float *lsev = sLse + buf * kTileM;
        const float *delt = sDelta + buf * kTileM;
        for (int r0 = 0; r0 < kTileM; r0 += kDkvSub) {
            float s[NTT][4], dp[NTT][4];
    #pragma unroll
            for (int n = 0; n < NTT; ++n)
    #pragma unroll
                for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.0f;
    #pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                uint32_t kf[4], vf[4];
                const uint32_t aoff = swz(warp * 16 + (lane & 15), ks * 2 + (lane >> 4), kRowB);
                ldmatrix_x4(kf, smem_u32(sK) + aoff);
                ldmatrix_x4(vf, smem_u32(sV) + aoff);
    #pragma unroll
                for (int n = 0; n < NTT; n += 2) {
                    const uint32_t off = swz(r0 + n * 8 + (lane & 7) + ((lane >> 4) << 3),
                                             ks * 2 + ((lane >> 3) & 1), kRowB);
                    uint32_t b[4];
                    ldmatrix_x4(b, sq + off);
                    mma_bf16_16816(s[n], kf, b[0], b[1]);
                    mma_bf16_16816(s[n + 1], kf, b[2], b[3]);
                    ldmatrix_x4(b, sd + off);
                    mma_bf16_16816(dp[n], vf, b[0], b[1]);
                    mma_bf16_16816(dp[n + 1], vf, b[2], b[3]);
                }
            }
            uint32_t pf[NTT / 2][4], dsf[NTT / 2][4];
    #pragma unroll
            for (int n = 0; n < NTT; ++n) {
                float p[4], ds[4];
    #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int col = r0 + n * 8 + q2 + (e & 1);
                    p[e] = exp2f(fmaf(s[n][e], scale_log2, bias[col]) - lsev[col]);
                    ds[e] = p[e] * (dp[n][e] - delt[col]);
                }
                pf[n >> 1][(n & 1) * 2 + 0] = pack_bf16x2(p[0], p[1]);
                pf[n >> 1][(n & 1) * 2 + 1] = pack_bf16x2(p[2], p[3]);
                dsf[n >> 1][(n & 1) * 2 + 0] = pack_bf16x2(ds[0], ds[1]);
                dsf[n >> 1][(n & 1) * 2 + 1] = pack_bf16x2(ds[2], ds[3]);
            }
    #pragma unroll
            for (int kk = 0; kk < NTT / 2; ++kk) {
                const uint32_t ap[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
                const uint32_t as[4] = {dsf[kk][0], dsf[kk][1], dsf[kk][2], dsf[kk][3]};
    #pragma unroll
                for (int jn = 0; jn < NTO; jn += 2) {
                    const uint32_t off = swz(r0 + kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                             jn + (lane >> 4), kRowB);
                    uint32_t b[4];
                    ldmatrix_x4_trans(b, sd + off);
                    mma_bf16_16816(dva[jn], ap, b[0], b[1]);
                    mma_bf16_16816(dva[jn + 1], ap, b[2], b[3]);
                    ldmatrix_x4_trans(b, sq + off);
                    mma_bf16_16816(dka[jn], as, b[0], b[1]);
                    mma_bf16_16816(dka[jn + 1], as, b[2], b[3]);
                }
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int sl = warp * 16 + g + r * 8;
        if (sl >= valid) continue;
        float *dkr = dk_acc + (slot0 + sl) * ld + h * HD;
        float *dvr = dv_acc + (slot0 + sl) * ld + h * HD;
#pragma unroll
        for (int jn = 0; jn < NTO; ++jn) {
            red_add_v2(dkr + jn * 8 + q2, dka[jn][2 * r] * scale, dka[jn][2 * r + 1] * scale);
            red_add_v2(dvr + jn * 8 + q2, dva[jn][2 * r], dva[jn][2 * r + 1]);
        }
    }
}

template <int HD>
static cudaError_t launch_bwd_t(const void *q, const void *k, const void *v, const void *out,
                                const void *dout, const float *lse, int H, int nb, int bs, int top,
                                const PlanLayout &L, const PlanView &P, void *dq, float *dk_acc,
                                float *dv_acc, float *dlog_gates, float *ws_delta, cudaStream_t st) {
    const float scale = 1.0f / sqrtf(static_cast<float>(HD));
    const float scale_log2 = scale * kLog2e;
    cudaError_t e;
    {
        const size_t smem = 3 * kTileM * HD * 2 + 4 * kSlotChunk * HD * 2 + kTileM * sizeof(int) +
                            kTileM * top * sizeof(float) + 2 * kTileM * sizeof(float);
        auto kern = read_bwd_dq_kernel<HD>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        kern<<<static_cast<unsigned>(L.max_tiles), kReadThreads, smem, st>>>(
            static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
            static_cast<const uint16_t *>(v), static_cast<const uint16_t *>(out),
            static_cast<const uint16_t *>(dout), lse, H, bs, top, scale, scale_log2, P,
            static_cast<uint16_t *>(dq), dlog_gates, ws_delta); count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    {
        const int cpb = (bs + kSlotChunk - 1) / kSlotChunk;
        const int base = nb * cpb * H;
        const int nsplit = std::max(1, std::min(16, (4 * 148 * 2 + base - 1) / base));
        const size_t smem = 2 * kSlotChunk * HD * 2 + 4 * kTileM * HD * 2 + 2 * kTileM * sizeof(int) +
                            6 * kTileM * sizeof(float);
        auto kern = read_bwd_dkdv_kernel<HD>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        dim3 grid(nb * cpb, H, nsplit);
        kern<<<grid, kDkvThreads, smem, st>>>(
            static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
            static_cast<const uint16_t *>(v), static_cast<const uint16_t *>(dout), lse, ws_delta, H,
            bs, top, cpb, nsplit, static_cast<int>(L.max_tiles), scale, scale_log2, P, dk_acc, dv_acc); count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_read_bwd(const void *q, const void *q_rows, const void *k, const void *v, const void *out,
                            const void *dout, const float *lse, int B, int S, int H, int hd,
                            int nb, int bs, int top, const PlanLayout &L, const PlanView &P,
                            void *dq, float *dk_acc, float *dv_acc, float *dlog_gates,
                            float *ws_delta, void *do_rows, cudaStream_t st, const float *row_w,
                            const int *iperm) {
    const size_t kv_bytes = sizeof(float) * static_cast<size_t>(nb) * bs * H * hd;
    cudaError_t e = cudaMemsetAsync(dk_acc, 0, kv_bytes, st);
    if (e != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(dv_acc, 0, kv_bytes, st)) != cudaSuccess) return e;
    const int64_t N = static_cast<int64_t>(B) * S;
    if ((e = cudaMemsetAsync(dlog_gates, 0, sizeof(float) * N * top, st)) != cudaSuccess) return e;
    if (L.max_tiles == 0) return cudaSuccess;
    // tensor-core kernels for 128-slot blocks with head_dim 64 (top <= 2) or
    // head_dim 128 (top 1: block-split plans); other geometries take the
    // warp-level mma kernels below
    const bool tc = read_bwd_tc_supported(hd, bs, top, q_rows, k, v, dout, H);
    // weighted rows are formed only by the row copy of the tensor-core path
    if (row_w && (!tc || !do_rows)) return cudaErrorInvalidValue;
    if (tc) {
        // delta = <dO, O> per plan row and head, and dO in plan order when there is
        // room for it (every tile's rows are then one TMA box)
        e = (row_w && iperm)
                ? launch_split_row_delta(dout, out, row_w, iperm, L.N / P.rows_per_q, P.rows_per_q, H, hd, do_rows,
                                         ws_delta, st)
                : launch_row_delta(dout, out, L.N, H, hd, P.perm, do_rows, ws_delta, st, P.rows_per_q, row_w);
        if (e != cudaSuccess) return e;
        if (do_rows)
            return launch_read_bwd_tc(q_rows, k, v, do_rows, true, lse, hd, H, nb, top, L, P, dq, dk_acc, dv_acc,
                                      dlog_gates, ws_delta, st);
        return launch_read_bwd_tc(q_rows, k, v, dout, false, lse, hd, H, nb, top, L, P, dq, dk_acc, dv_acc,
                                  dlog_gates, ws_delta, st);
    }
    if (hd == 64)
        return launch_bwd_t<64>(q, k, v, out, dout, lse, H, nb, bs, top, L, P, dq, dk_acc, dv_acc,
                                dlog_gates, ws_delta, st);
    if (hd == 128)
        return launch_bwd_t<128>(q, k, v, out, dout, lse, H, nb, bs, top, L, P, dq, dk_acc, dv_acc,
                                 dlog_gates, ws_delta, st);
    return cudaErrorInvalidValue;
}

}  // namespace mom
