// Gated memory read, backward, on the tensor cores (tcgen05 + TMA + TMEM).
//
// Reference semantics: mom_kernels/triton_gpu.py:143-409 (P rebuilt from the
// saved log-sum-exp, dS = P (dP - delta), dq = dS k * scale, dk = dS^T q *
// scale, dv = P^T do, dlog_gates = per-block sums of dS over slots and heads).
// Specialised like read_fwd_tc.cu: 128-slot blocks; head_dim 64 with top <= 2,
// head_dim 128 with one block per row (block-split plans).
// Q and dO are read in routing-plan row order (q_rows from the forward, dO
// copied by the row kernel that also forms delta = <dO, O> per row and head),
// so every tile is one 2-D TMA box; the no-workspace entry gathers dO's rows
// from token order with cp.async instead (kDoRows = false).
//
// read_bwd_dq_tc_kernel — item = (128-token tile, head), persistent CTAs over
// contiguous runs of items ordered head-major, so consecutive items usually
// share their block set and head and reuse the K/V tiles in shared memory.
//   warp 0     loader: Q, dO tiles; K, V blocks by TMA when the run changes
//   warps 1, 2 MMA issuers: S = Q K^T (TMEM cols 0-255) and dP = dO V^T
//              (cols 256-511), then dQ over block 0 / block 1 (TS form, dS
//              from TMEM) into cols 256-319 / 320-383 (head_dim 128: S 0-127,
//              dP then the one 128-column dQ at 256-383)
//   warps 3-18 softmax, one pass: P = exp2(S*scale + bias - lse), dS = P (dP -
//              delta) as bf16 over the S columns already read; the exact row
//              sums of P dP and P per block for the gate gradient (fp32 atomics
//              over heads); then dQ -> global
// read_bwd_dkdv_tc_kernel — each CTA an equal contiguous share of the (block,
// head, tile) units, walked as segments of one (block, head); a tile's tokens
// in steps of 64
//   warp 0     loader: K_b, V_b once per item (TMA); per tile Q, dO and the
//              tile's per-token bias - lse and delta into shared memory
//   warp 1     MMA: S^T = K_b Q^T, dP^T = V_b dO^T into one of three step
//              buffers (TMEM cols 128*b, +64; two buffers at head_dim 128)
//   warp 2     MMA: dK += dS^T Q, dV += P^T dO (TS form) into cols 384 / 448
//              (head_dim 128: 256 / 384, 128 columns each)
//   warps 3-18 P^T, dS^T (one slot row per thread) -> bf16 in TMEM over the
//              step buffer; at the end of the item dK * scale, dV -> fp32
//              reductions into global.
// Every wait is bounded; a timeout sets bit 1 of the plan's error word.
#include <cudaTypedefs.h>

#include "launch.h"
#include "tc_common.cuh"

namespace mom {

namespace {
constexpr int kBS = 128;
constexpr int kTM = 128;
constexpr int kSoftWarps = 16;                 // 4 per SM sub-partition
constexpr int kSoftThreads = kSoftWarps * 32;
constexpr uint32_t kBoxBytes = 128 * 128;      // one TMA box: 128 rows x 64 bf16 columns (128-B swizzle)
constexpr uint32_t kTmemCols = 512;
// Rows of Q / dO / K / V are 64-column TMA boxes side by side (kBoxBytes apart):
// one box at head_dim 64, two at head_dim 128.
template <int HD> struct Geo {
    static constexpr int kBoxes = HD / 64;
    static constexpr uint32_t kRowTile = kTM * HD * 2;   // 128 rows x HD bf16
    // K / V / Q / dO as the MN-major B operand (N = HD): N-atoms of 64 columns
    // kBoxBytes apart (head_dim 64 has one atom; its value is what the validated
    // kernels used)
    __host__ __device__ static constexpr uint32_t kLbo(uint32_t hd64_value) { return HD == 64 ? hd64_value : kBoxBytes; }
};
// K-step kk of an MMA whose K dimension is head_dim: +32 B within a 64-column
// box (+2 in the descriptor's address field), +kBoxBytes (+1024) per box
__device__ __forceinline__ uint64_t hd_step(int kk) { return 1024u * (kk >> 2) + 2u * (kk & 3); }

struct DqBars {
    uint64_t full[2], empty[2], kv_full, kv_empty, s_full, ds_full, dq_full, dq_free, drain;
    uint32_t tmem_base;
    int abort;
    // per stage: blocks loaded | (K/V reload << 8) | (blocks of the set << 12); written
    // before the stage's barrier
    int meta[2];
    int tok[128];     // the loader's row tokens of the tile being copied
};
static_assert(sizeof(DqBars) <= 1024, "barrier block");
// head_dim 64: sets of up to two blocks; head_dim 128: one block per row (the
// block-split plan), so K / V hold one block and dQ is one 128-column sum.
template <int HD> struct Dq {
    static constexpr int kMaxBlk = HD == 64 ? 2 : 1;
    static constexpr uint32_t kRowTile = Geo<HD>::kRowTile;
    static constexpr uint32_t kBlkBytes = kBS * HD * 2;
    static constexpr uint32_t kStage = 2 * kRowTile;                       // Q + dO
    static constexpr uint32_t kKV = 2 * kMaxBlk * kBlkBytes;               // K blocks + V blocks
    static constexpr uint32_t kScratch = 2 * 2 * 4 * kTM * 4               // [2 items][P.dP | P][4 groups][128] fp32
                                         + kTM * 64 * 2 + kTM * 4;         // 64 dQ columns staged, tokens
    static constexpr uint32_t kSmem = 2 * kStage + kKV + kScratch + 1024 + 1024;
    static_assert(kSmem <= 227 * 1024, "shared memory");
};
// warp 0 loader, warps 1 and 2 MMA issuers (warp 1: S, then dQ over block 0;
// warp 2: dP, then dQ over block 1; warp 1 owns TMEM), warps 3-18 softmax.
// TMEM: S at columns 0..255 (dS written back over it as bf16, the A operand of
// dQ), dP at 256..511, the two dQ partial sums at 256..319 and 320..383 once
// dP has been consumed.
constexpr int kDqThreads = 96 + kSoftThreads;
}  // namespace

// ============================================================================ dQ
// kDoRows: dO in plan order (one TMA box per tile, like Q); else dO in token
// order, its rows gathered with cp.async.
template <int HD, bool kDoRows>
__global__ void __launch_bounds__(kDqThreads, 1)
read_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                      const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_do,
                      const uint16_t *__restrict__ dout,
                      const float *__restrict__ lse, int H, int top, float scale, float scale_log2, PlanView P,
                      uint16_t *__restrict__ dq, float *__restrict__ dlog_gates, float *__restrict__ ws_delta) {
    using C = Dq<HD>;
    constexpr int kHD = HD;
    constexpr uint32_t kRowTile = C::kRowTile, kDqStage = C::kStage, kDqKV = C::kKV, kDqScratch = C::kScratch;
    constexpr uint32_t kBlkBytes = C::kBlkBytes;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char *sbase = smem_raw + (base - raw);
    const uint32_t sKV = base + 2 * kDqStage;
    const uint32_t sK = sKV, sV = sKV + C::kMaxBlk * kBlkBytes;
    float *sPart = reinterpret_cast<float *>(sbase + 2 * kDqStage + kDqKV);
    uint4 *sOut = reinterpret_cast<uint4 *>(sPart + 2 * 2 * 4 * kTM);      // [128 rows][8 x 16 B]
    int *sTok = reinterpret_cast<int *>(sOut + kTM * 8);
    DqBars *bars = reinterpret_cast<DqBars *>(sbase + 2 * kDqStage + kDqKV + kDqScratch);
    volatile int *abort_flag = &bars->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = *P.ntiles;
    const int nitems = ntiles * H;
    const int per = (nitems + gridDim.x - 1) / gridDim.x;
    const int it0 = blockIdx.x * per, it1 = min(nitems, it0 + per);
    const int64_t ld = static_cast<int64_t>(H) * kHD;

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            // the loader's arrive with the TMA bytes (+ 32 lanes' dO cp.async when gathering)
            tc::mbar_init(&bars->full[s], kDoRows ? 1 : 33);
            tc::mbar_init(&bars->empty[s], 2);   // both MMA warps read the stage
        }
        tc::mbar_init(&bars->kv_full, 1);
        tc::mbar_init(&bars->kv_empty, 2);   // both MMA warps
        tc::mbar_init(&bars->s_full, 2);
        tc::mbar_init(&bars->ds_full, kSoftThreads);
        tc::mbar_init(&bars->dq_full, 2);
        tc::mbar_init(&bars->dq_free, kSoftThreads);
        tc::mbar_init(&bars->drain, 2);
        bars->abort = 0;
    }
    if (warp == 1) {
        tc::tmem_alloc(&bars->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    // item -> (tile, head); items are head-major so runs of one CTA share (set, head)
    auto item_tile = [&](int item) { return item % ntiles; };
    auto item_head = [&](int item) { return item / ntiles; };
    const int nmine = max(0, it1 - it0);

    if (warp == 0) {
        // ------------------------------------------------------------ loader
        // Tile metadata 32 items at a time (one per lane), the Q / dO rows of item
        // i+1 read while item i waits for its stage. Per stage the loader posts the
        // block count and whether K/V change (a new (set, head) run) in shared
        // memory before the stage's barrier; Q / dO go first, then, on a change,
        // K/V once the MMAs of the previous run are done with them (kv_empty,
        // committed by the MMA warp when it meets the change).
        tc::LaneTile lt;
        int mh = 0, mreload = 0, prev_key = -1, prev_h = -1;
        int rows[4];
        int nreload = 0, last_full = -1;
        for (int i = 0; i < nmine; ++i) {
            const int s = i & 1, j = i >> 1, src = i & 31;
            if (src == 0) {
                const int item = it0 + i + lane;
                if (item < it1) {
                    lt.fetch(P, item_tile(item), top);
                    mh = item_head(item);
                }
                int pk = __shfl_up_sync(0xffffffffu, lt.key, 1), ph = __shfl_up_sync(0xffffffffu, mh, 1);
                if (lane == 0) {
                    pk = prev_key;
                    ph = prev_h;
                }
                mreload = (lt.key != pk || mh != ph) ? 1 : 0;
                prev_key = tc::get(lt.key, 31);
                prev_h = tc::get(mh, 31);
                if (!kDoRows) tc::gather_rows(P, tc::get(lt.x, 0), tc::get(lt.y, 0), lane, rows);
            }
            const int x0 = tc::get(lt.x, src);
            const int h = tc::get(mh, src), nblk = tc::get(lt.nblk, src);
            const int b0 = tc::get(lt.b0, src), b1 = tc::get(lt.b1, src);
            const int reload = tc::get(mreload, src);
            if (!tc::mbar_wait_warp(&bars->empty[s], (j & 1) ^ 1, P.err, 2, abort_flag)) break;
            const int nload = nblk > 0 ? nblk : 1;
            const uint32_t sQ = base + s * kDqStage, sD = sQ + kRowTile;
            if (!kDoRows) {
                tc::stage_row_tokens(bars->tok, rows, lane);
#pragma unroll
                for (int c = 0; c < Geo<HD>::kBoxes; ++c)
                    tc::gather_tile_rows(sD + c * kBoxBytes, dout, ld, h * kHD + 64 * c, bars->tok, lane);
                tc::cp_async_arrive_noinc(&bars->full[s]);
            }
            if (lane == 0) {
                bars->meta[s] = nload | (reload << 8) | (nblk << 12);   // released by the arrive below
                tc::mbar_arrive_expect_tx(&bars->full[s], kDoRows ? 2 * kRowTile : kRowTile);
#pragma unroll
                for (int c = 0; c < Geo<HD>::kBoxes; ++c) {
                    tc::tma_load_2d(sQ + c * kBoxBytes, &tmap_q, h * kHD + 64 * c, x0, &bars->full[s]);
                    if (kDoRows)
                        tc::tma_load_2d(sD + c * kBoxBytes, &tmap_do, h * kHD + 64 * c, x0, &bars->full[s]);
                }
            }
            __syncwarp();
            last_full = i;
            if (!kDoRows && src < 31 && i + 1 < nmine)
                tc::gather_rows(P, tc::get(lt.x, src + 1), tc::get(lt.y, src + 1), lane, rows);
            if (reload) {
                if (nreload > 0 && !tc::mbar_wait_warp(&bars->kv_empty, (nreload - 1) & 1, P.err, 2, abort_flag)) break;
                if (lane == 0) {
                    tc::mbar_arrive_expect_tx(&bars->kv_full, 2 * nload * kBlkBytes);
                    for (int jb = 0; jb < nload; ++jb) {
                        const int blk = nblk > 0 ? (jb == 0 ? b0 : b1) : 0;
#pragma unroll
                        for (int c = 0; c < Geo<HD>::kBoxes; ++c) {
                            tc::tma_load_2d(sK + jb * kBlkBytes + c * kBoxBytes, &tmap_k, h * kHD + 64 * c,
                                            blk * kBS, &bars->kv_full);
                            tc::tma_load_2d(sV + jb * kBlkBytes + c * kBoxBytes, &tmap_v, h * kHD + 64 * c,
                                            blk * kBS, &bars->kv_full);
                        }
                    }
                }
                __syncwarp();
                ++nreload;
            }
        }
        if (last_full >= 0) tc::mbar_wait_warp(&bars->full[last_full & 1], (last_full >> 1) & 1, P.err, 2, abort_flag);
        if (nreload > 0) tc::mbar_wait_warp(&bars->kv_full, (nreload - 1) & 1, P.err, 2, abort_flag);
        tc::cp_async_wait_all();
    } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------------------ MMA issuers
        // warp 1: S = Q K^T, then dQ_0 = dS[:, block 0] K_0; warp 2: dP = dO V^T, then
        // dQ_1 = dS[:, block 1] K_1 (dS read from TMEM). Two issuers, because one
        // thread issues a tcgen05.mma only every ~100 cycles.
        const bool wa = warp == 1;
        const uint32_t idesc_dq = tc::idesc_bf16_f32(kTM, kHD, false, true);
        const uint64_t bk0 = tc::smem_desc_sw128(sK + (wa ? 0 : kBlkBytes), Geo<HD>::kLbo(4 * kRowTile), 1024);
        int nreload = 0;
        for (int i = 0; i < nmine; ++i) {
            const int s = i & 1, j = i >> 1;
            if (!tc::mbar_wait_warp(&bars->full[s], j & 1, P.err, 2, abort_flag)) break;
            tc::fence_proxy_async_smem();   // dO rows may have come through cp.async (generic proxy)
            const int meta = tc::ld_shared_volatile(&bars->meta[s]);
            const int nload = meta & 0xFF, nblk = (meta >> 12) & 0xF;
            if ((meta >> 8) & 1) {
                // a new (set, head) run: the previous run's K/V are free once every
                // MMA this warp issued so far has completed
                if (i > 0 && lane == 0) tc::mma_commit(&bars->kv_empty);
                __syncwarp();
                if (!tc::mbar_wait_warp(&bars->kv_full, nreload & 1, P.err, 2, abort_flag)) break;
                ++nreload;
            }
            // S / dP overwrite TMEM columns that dQ(i-1) used: wait for its epilogue
            if (i > 0 && !tc::mbar_wait_warp(&bars->dq_free, (i - 1) & 1, P.err, 2, abort_flag)) break;
            tc::tc_fence_after();
            if (lane == 0) {
                const uint32_t idesc_s = tc::idesc_bf16_f32(kTM, nload * kBS, false, false);
                const uint32_t sA = base + s * kDqStage + (wa ? 0 : kRowTile);   // Q or dO
                const uint64_t da = tc::smem_desc_sw128(sA, 16, 1024);
                const uint64_t db = tc::smem_desc_sw128(wa ? sK : sV, 16, 1024);
#pragma unroll
                for (int kk = 0; kk < kHD / 16; ++kk)
                    tc::mma_bf16_ss(tmem + (wa ? 0 : 256), da + hd_step(kk), db + hd_step(kk), idesc_s, kk > 0);
                tc::mma_commit(&bars->s_full);
                tc::mma_commit(&bars->empty[s]);
            }
            __syncwarp();
            if (!tc::mbar_wait_warp(&bars->ds_full, i & 1, P.err, 2, abort_flag)) break;
            tc::tc_fence_after();
            if (lane == 0) {
                if (nblk > (wa ? 0 : 1) && (wa || C::kMaxBlk > 1)) {
#pragma unroll
                    for (int k8 = 0; k8 < 8; ++k8) {   // the block's 128 slots, 16 per step
                        const int kk = (wa ? 0 : 8) + k8;
                        tc::mma_bf16_ts(tmem + (wa ? 256 : 320), tmem + 64 * (kk >> 2) + 8 * (kk & 3),
                                        bk0 + 128 * k8, idesc_dq, k8 > 0);
                    }
                }
                tc::mma_commit(&bars->dq_full);
            }
            __syncwarp();
        }
        if (lane == 0) tc::mma_commit(&bars->drain);
        __syncwarp();
        tc::mbar_wait_warp(&bars->drain, 0, P.err, 2, abort_flag);
    } else {
        // ------------------------------------------------------------ softmax-backward
        // 16 warps: warp & 3 = TMEM lane quarter (token rows), grp = (warp-3) >> 2 the
        // 64-column group of the 256 S / dP columns (block grp >> 1). Partial sums of
        // P*dP and P per group meet in shared memory under named barrier 1 + quarter,
        // which is also where the four warps of a quarter agree to stop on a timeout.
        const int quarter = warp & 3;
        const int grp = (warp - 3) >> 2;
        const int jb = grp >> 1;
        const int r = quarter * 32 + lane;
        const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        const int bar_id = 1 + quarter;
        bool dead = false;
        // per-item row metadata: tile fields 32 items at a time (one per lane),
        // this thread's row (token, bias, lse, caller-slot map) one item ahead
        struct Meta { int x, nblk, h, tok; float bias, lse2, dlt; uint32_t kmap; };
        tc::LaneTile lt;
        int mh = 0;
        auto fetch = [&](int src, Meta &m) {
            m.x = tc::get(lt.x, src);
            const int y = tc::get(lt.y, src);
            m.nblk = tc::get(lt.nblk, src);
            m.h = tc::get(mh, src);
            const bool in = r < y;
            m.tok = in ? P.perm[m.x + r] : -1;
            m.bias = (in && jb < m.nblk) ? P.rowbias[static_cast<int64_t>(m.x + r) * top + jb] * kLog2e : 0.0f;
            m.lse2 = in ? lse[static_cast<int64_t>(m.h) * P.n + m.x + r] * kLog2e : INFINITY;
            m.dlt = in ? ws_delta[static_cast<int64_t>(m.h) * P.n + m.x + r] : 0.0f;
            m.kmap = (in && grp == 0) ? P.rowkmap[m.x + r] : 0u;
        };
        Meta cur, nxt;
        for (int i = 0; i < nmine; ++i) {
            const int src = i & 31;
            if (src == 0) {
                const int item = it0 + i + lane;
                if (item < it1) {
                    lt.fetch(P, item_tile(item), top);
                    mh = item_head(item);
                }
                fetch(0, cur);
            } else {
                cur = nxt;   // prefetched during item i-1
            }
            if (src < 31 && i + 1 < nmine) fetch(src + 1, nxt);
            const int h = cur.h, nblk = cur.nblk, tok = cur.tok;
            const float bias = cur.bias, lse2 = cur.lse2;
            if (!dead && !tc::mbar_wait_warp(&bars->s_full, i & 1, P.err, 2, abort_flag)) dead = true;
            tc::tc_fence_after();
            // warp-uniform: the tcgen05.ld below are warp-collective. Padding rows
            // (tok < 0) have lse2 = +inf and get P = 0 from the same code.
            const bool live = jb < nblk && !dead;
            // one pass over this thread's 64 columns, 16 at a time: P = exp2(s*scale + bias
            // - lse), dS = P (dP - delta) with delta = <dO, O> (the row kernel's), written
            // back to TMEM as bf16 over S values already read (chunk c's 16 slots packed
            // into columns grp*64 + 8c .. +7: the A operand of dQ); partial sums of P*dP
            // and P for the gate gradient
            float pa = 0.0f, pb = 0.0f;
            if (live) {
                const float bj = bias - lse2, dlt = cur.dlt;
                const uint64_t sc2 = tc::f2(scale_log2, scale_log2), bj2 = tc::f2(bj, bj), dl2 = tc::f2(dlt, dlt);
                uint64_t pa2 = tc::f2(0.0f, 0.0f), pb2 = pa2;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int col0 = grp * 64 + c * 16;
                    uint32_t sv[16], dv[16];
                    tc::tmem_ld16(trow + col0, sv);
                    tc::tmem_ld16(trow + 256 + col0, dv);
                    tc::tmem_ld_wait_regs(sv);
                    tc::tmem_ld_wait_regs(dv);
                    uint32_t ok[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        // column pairs: 2 of 8 by the FMA-pipe polynomial, the rest by MUFU
                        const uint64_t x2 = tc::fma2(tc::f2_bits(sv[2 * e], sv[2 * e + 1]), sc2, bj2);
                        const uint64_t p2 = (e & 3) == 1 ? tc::ex2_poly2(x2) : tc::ex2_pair(x2);
                        const uint64_t d2 = tc::f2_bits(dv[2 * e], dv[2 * e + 1]);
                        pa2 = tc::fma2(p2, d2, pa2);
                        pb2 = tc::add2(pb2, p2);
                        const float2 ds = tc::f2_split(tc::mul2(p2, tc::sub2(d2, dl2)));
                        ok[e] = pack_bf16x2(ds.x, ds.y);
                    }
                    tc::tmem_st8(trow + grp * 64 + c * 8, ok);
                }
                tc::tmem_st_wait();
                const float2 a = tc::f2_split(pa2), bsum = tc::f2_split(pb2);
                pa = a.x + a.y;
                pb = bsum.x + bsum.y;
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&bars->ds_full);
            // exact row term sum_j P*dP for the gate gradient, off the MMAs' path
            float *part = sPart + (i & 1) * (2 * 4 * kTM);
            part[grp * kTM + r] = pa;
            part[(4 + grp) * kTM + r] = pb;
            dead = tc::named_bar_or(bar_id, 128, dead);
            if (dead) break;
            // a plan over (token, k) rows reads one block per row: its gate term
            // needs the whole token's delta (the row kernel's, from the combined O)
            const bool pseudo = P.rows_per_q > 1;
            const float delta = pseudo ? cur.dlt : part[r] + part[kTM + r] + part[2 * kTM + r] + part[3 * kTM + r];
            // gate gradient (sum over heads by fp32 atomics). A set of one block gets
            // none: its gates shift all of the token's scores alike, which the
            // softmax cancels, so the gradient is exactly zero (dlog_gates is zeroed
            // before the kernels run).
            if (grp == 0 && tok >= 0 && (nblk > 1 || pseudo)) {
                // per block of the set: A = sum P*dP, B = sum P (selected by value, not by
                // a dynamically indexed array, which would live in local memory)
                const float A0 = part[r] + part[kTM + r], A1 = part[2 * kTM + r] + part[3 * kTM + r];
                const float B0 = part[4 * kTM + r] + part[5 * kTM + r], B1 = part[6 * kTM + r] + part[7 * kTM + r];
                const uint32_t kmap = cur.kmap;
                for (int kk = 0; kk < top; ++kk) {
                    const int jsel = (kmap >> (4 * kk)) & 0xF;
                    if (jsel < nblk && jsel < 2)
                        atomicAdd(dlog_gates + static_cast<int64_t>(tok) * top + kk,
                                  fmaf(-delta, jsel ? B1 : B0, jsel ? A1 : A0));
                }
            }
            // epilogue: 16 of the 64 dQ columns, dQ_0 + dQ_1 (the set's blocks) * scale ->
            // global through shared memory; the quarter's four warps agree first (the
            // store's barrier needs all of them)
            bool bad = !tc::mbar_wait_warp(&bars->dq_full, i & 1, P.err, 2, abort_flag);
            if (tc::named_bar_or(bar_id, 128, bad)) {
                dead = true;
                break;
            }
            tc::tc_fence_after();
            // head_dim 64: dQ_0 + dQ_1 (the set's blocks) at 256 / 320; head_dim 128:
            // columns 16g.. and 64+16g.. of the one dQ at 256
            uint32_t a0[16], a1[16];
            tc::tmem_ld16(trow + 256 + grp * 16, a0);          // both in one round trip
            tc::tmem_ld16(trow + 320 + grp * 16, a1);
            tc::tmem_ld_wait_regs(a0);
            tc::tmem_ld_wait_regs(a1);
            tc::tc_fence_before();
            tc::mbar_arrive(&bars->dq_free);
            auto pack16 = [&](const float (&o)[16], uint4 &v0, uint4 &v1) {
                v0.x = pack_bf16x2(o[0] * scale, o[1] * scale);
                v0.y = pack_bf16x2(o[2] * scale, o[3] * scale);
                v0.z = pack_bf16x2(o[4] * scale, o[5] * scale);
                v0.w = pack_bf16x2(o[6] * scale, o[7] * scale);
                v1.x = pack_bf16x2(o[8] * scale, o[9] * scale);
                v1.y = pack_bf16x2(o[10] * scale, o[11] * scale);
                v1.z = pack_bf16x2(o[12] * scale, o[13] * scale);
                v1.w = pack_bf16x2(o[14] * scale, o[15] * scale);
            };
            float o[16];
            uint4 v0, v1;
            if constexpr (HD == 64) {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    o[e] = (nblk > 0 ? __uint_as_float(a0[e]) : 0.0f) + (nblk > 1 ? __uint_as_float(a1[e]) : 0.0f);
                pack16(o, v0, v1);
                tc::store_tile_rows(sOut, sTok, quarter, grp, lane, bar_id, v0, v1, tok, dq + h * kHD, ld);
            } else {
#pragma unroll
                for (int e = 0; e < 16; ++e) o[e] = nblk > 0 ? __uint_as_float(a0[e]) : 0.0f;
                pack16(o, v0, v1);
                tc::store_tile_rows(sOut, sTok, quarter, grp, lane, bar_id, v0, v1, tok, dq + h * kHD, ld);
                tc::named_bar(bar_id, 128);   // the staging rows are read out before they are rewritten
#pragma unroll
                for (int e = 0; e < 16; ++e) o[e] = nblk > 0 ? __uint_as_float(a1[e]) : 0.0f;
                pack16(o, v0, v1);
                tc::store_tile_rows(sOut, sTok, quarter, grp, lane, bar_id, v0, v1, tok, dq + h * kHD + 64, ld);
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// ============================================================================ dK / dV
namespace {
constexpr int kDkvMaxStages = 4;
// warp 0 loader, warp 1 S^T / dP^T MMAs (and TMEM owner), warp 2 dK / dV MMAs,
// warps 3-18 softmax + epilogue: one thread issues a tcgen05.mma only every
// ~100 cycles, so the two GEMM pairs get an issuing warp each.
constexpr int kDkvThreads = 96 + kSoftThreads;
struct DkvBars {
    uint64_t full[kDkvMaxStages], empty[kDkvMaxStages], kv_full, kv_empty, s_full[3], pds_full[3], buf_free[3],
        acc_full, acc_free, drain;
    uint32_t tmem_base;
    int abort;
    int tok[128];     // the loader's row tokens of the tile being copied
};
static_assert(sizeof(DkvBars) <= 1024, "barrier block");
constexpr uint32_t kMetaBytes = 2 * kTM * 4;                     // bias2 - lse2, delta
// A tile's 128 tokens go through the MMAs and the softmax in two steps of 64.
// TMEM: step buffer b (= step % kBufs) at column 128*b holds S^T [128 slots x 64
// tokens] in columns +0..63 and dP^T in +64..127; the softmax overwrites them in
// place with bf16 P^T and dS^T (softmax group g's 16 tokens packed into the first
// 8 of its 16 columns), the A operands of dV += P^T dO and dK += dS^T Q. dK is
// accumulated at columns kAccCol.., dV at kAccCol + HD... head_dim 64: three
// buffers (0..383), dK / dV at 384 / 448, four Q / dO stages; the S^T / dP^T
// MMAs of step s+2 run while the softmax works on step s+1 and the dK / dV MMAs
// of step s still read their buffer. head_dim 128: the two 128-column
// accumulators at 256 / 384 leave room for two buffers, and shared memory for
// two stages.
constexpr int kHalf = 64;
template <int HD> struct Dkv {
    static constexpr int kStages = HD == 64 ? 4 : 2;
    static constexpr int kBufs = HD == 64 ? 3 : 2;
    static constexpr uint32_t kAccCol = HD == 64 ? 384 : 256;
    static constexpr uint32_t kRowTile = Geo<HD>::kRowTile;
    static constexpr uint32_t kKvTile = kBS * HD * 2;                 // one block of K or V
    static constexpr uint32_t kStage = 2 * kRowTile;                  // Q + dO
    static constexpr uint32_t kSmem = 2 * kKvTile + kStages * kStage + kStages * kMetaBytes + 1024 + 1024;
    static_assert(kSmem <= 227 * 1024, "shared memory");
    static_assert(kStages <= kDkvMaxStages && kBufs <= 3 && kAccCol + 2 * HD <= kTmemCols, "layout");
};
}  // namespace

template <int HD, bool kDoRows>
__global__ void __launch_bounds__(kDkvThreads, 1)
read_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                        const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_do,
                        const uint16_t *__restrict__ dout,
                        const float *__restrict__ lse, const float *__restrict__ ws_delta, int H, int nb, int top,
                        int max_tiles, float scale, float scale_log2, PlanView P,
                        float *__restrict__ dk_acc, float *__restrict__ dv_acc) {
    using C = Dkv<HD>;
    constexpr int kHD = HD, kDkvStages = C::kStages, kBufs = C::kBufs;
    constexpr uint32_t kRowTile = C::kRowTile, kKvTile = C::kKvTile, kDkvStage = C::kStage, kAccCol = C::kAccCol;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char *sbase = smem_raw + (base - raw);
    const uint32_t sK = base, sV = base + kKvTile;
    const uint32_t sStage = base + 2 * kKvTile;                  // [stages][Q | dO]
    float *meta = reinterpret_cast<float *>(sbase + 2 * kKvTile + kDkvStages * kDkvStage);   // [stages][2][128]
    DkvBars *bars = reinterpret_cast<DkvBars *>(reinterpret_cast<unsigned char *>(meta) + kDkvStages * kMetaBytes);
    volatile int *abort_flag = &bars->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t ld = static_cast<int64_t>(H) * kHD;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kDkvStages; ++s) {
            // per lane: the arrive after its metadata stores (lane 0's carries the TMA
            // bytes), + its dO cp.async when gathering
            tc::mbar_init(&bars->full[s], kDoRows ? 32 : 64);
            tc::mbar_init(&bars->empty[s], 1);
        }
        tc::mbar_init(&bars->kv_full, 1);
        tc::mbar_init(&bars->kv_empty, 1);
        for (int b = 0; b < kBufs; ++b) {
            tc::mbar_init(&bars->s_full[b], 1);
            tc::mbar_init(&bars->pds_full[b], kSoftThreads);
            tc::mbar_init(&bars->buf_free[b], 1);
        }
        tc::mbar_init(&bars->acc_full, 1);
        tc::mbar_init(&bars->acc_free, kSoftThreads);
        tc::mbar_init(&bars->drain, 2);
        bars->abort = 0;
    }
    if (warp == 1) {
        tc::tmem_alloc(&bars->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    // Work split: the sequence of (block, head, tile of the block's list) units,
    // block-major, cut into gridDim.x equal contiguous ranges. A CTA walks its
    // range as segments of one (block, head) (K_b, V_b loaded once, dK / dV
    // accumulated in TMEM and reduced into global at the segment's end); a
    // (block, head) cut between two CTAs is reduced by both.
    int64_t units = 0;
    for (int b = 0; b < nb; ++b) units += static_cast<int64_t>(P.blkcount[b]) * H;
    const int64_t u_begin = units * blockIdx.x / gridDim.x, u_end = units * (blockIdx.x + 1) / gridDim.x;
    struct Seg { int blk, h, t0, nt; };
    // next segment of [u, u_end); advances u
    auto next_seg = [&](int64_t &u, Seg &sg) -> bool {
        if (u >= u_end) return false;
        int64_t base = 0;
        int blk = 0;
        for (; blk < nb - 1; ++blk) {
            const int64_t span = static_cast<int64_t>(P.blkcount[blk]) * H;
            if (u < base + span) break;
            base += span;
        }
        const int cnt = P.blkcount[blk];
        const int64_t rem = u - base;
        sg.blk = blk;
        sg.h = static_cast<int>(rem / cnt);
        sg.t0 = static_cast<int>(rem % cnt);
        const int64_t end = min(u_end, base + static_cast<int64_t>(sg.h + 1) * cnt);
        sg.nt = static_cast<int>(end - u);
        u = end;
        return true;
    };

    if (warp == 0) {
        // ------------------------------------------------------------ loader
        // Per segment: the tile list entry, tile descriptor and the block's position
        // in the tile's set for 32 tiles at a time (one per lane); per tile the
        // row tokens, gate bias, lse and delta (one round trip) are loaded right
        // after the previous tile's copies were issued.
        const int64_t ld = static_cast<int64_t>(H) * kHD;
        int g = 0, nkv = 0, last = -1;         // g: global tile-step counter of this CTA
        int cx = 0, cy = 0, cjb = 0;           // this lane's tile of the current chunk
        int rows[4];
        float mcomb[4], mdelta[4];
        auto fetch_rows = [&](int src, int h) {
            const int x = tc::get(cx, src), y = tc::get(cy, src), jb = tc::get(cjb, src);
            if (!kDoRows) tc::gather_rows(P, x, y, lane, rows);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                // lse and delta are stored in plan-row order: no dependence on perm
                const int rr = lane * 4 + u;
                const bool ok = rr < y;
                const int64_t prow = static_cast<int64_t>(h) * P.n + x + rr;
                // the token's exponent offset bias - lse (log2 units); -inf for padding rows
                mcomb[u] = ok ? P.rowbias[static_cast<int64_t>(x + rr) * top + jb] * kLog2e - lse[prow] * kLog2e
                              : -INFINITY;
                mdelta[u] = ok ? ws_delta[prow] : 0.0f;
            }
        };
        int64_t u = u_begin;
        Seg sg;
        while (next_seg(u, sg)) {
            const int blk = sg.blk, h = sg.h, nt = sg.nt;
            // K_b, V_b: every S^T / dP^T MMA of the previous segment has completed (kv_empty)
            if (nkv > 0 && !tc::mbar_wait_warp(&bars->kv_empty, (nkv - 1) & 1, P.err, 2, abort_flag)) break;
            if (lane == 0) {
                tc::mbar_arrive_expect_tx(&bars->kv_full, 2 * kKvTile);
#pragma unroll
                for (int c = 0; c < Geo<HD>::kBoxes; ++c) {
                    tc::tma_load_2d(sK + c * kBoxBytes, &tmap_k, h * kHD + 64 * c, blk * kBS, &bars->kv_full);
                    tc::tma_load_2d(sV + c * kBoxBytes, &tmap_v, h * kHD + 64 * c, blk * kBS, &bars->kv_full);
                }
            }
            ++nkv;
            const int *list = P.blktiles + static_cast<int64_t>(blk) * max_tiles;
            bool stop = false;
            for (int t = 0; t < nt; ++t, ++g) {
                const int src = t & 31;
                if (src == 0) {
                    if (t + lane < nt) {
                        const int tile = list[sg.t0 + t + lane];
                        const int4 td = P.tiles[tile];
                        cx = td.x;
                        cy = td.y;
                        cjb = (top > 1 && P.keyset[static_cast<int64_t>(td.z) * top] != blk) ? 1 : 0;
                    }
                    fetch_rows(0, h);
                }
                const int s = g % kDkvStages, j = g / kDkvStages;
                if (!tc::mbar_wait_warp(&bars->empty[s], (j & 1) ^ 1, P.err, 2, abort_flag)) { stop = true; break; }
                float *mb = meta + s * 2 * kTM;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int rr = lane * 4 + u;
                    mb[rr] = mcomb[u];
                    mb[kTM + rr] = mdelta[u];
                }
                const uint32_t sQ = sStage + s * kDkvStage, sD = sQ + kRowTile;
                const int x0 = tc::get(cx, src);
                if (!kDoRows) {
                    tc::stage_row_tokens(bars->tok, rows, lane);
#pragma unroll
                    for (int c = 0; c < Geo<HD>::kBoxes; ++c)
                        tc::gather_tile_rows(sD + c * kBoxBytes, dout, ld, h * kHD + 64 * c, bars->tok, lane);
                    tc::cp_async_arrive_noinc(&bars->full[s]);
                }
                if (lane == 0) {
                    tc::mbar_arrive_expect_tx(&bars->full[s], kDoRows ? 2 * kRowTile : kRowTile);
#pragma unroll
                    for (int c = 0; c < Geo<HD>::kBoxes; ++c) {
                        tc::tma_load_2d(sQ + c * kBoxBytes, &tmap_q, h * kHD + 64 * c, x0, &bars->full[s]);
                        if (kDoRows)
                            tc::tma_load_2d(sD + c * kBoxBytes, &tmap_do, h * kHD + 64 * c, x0, &bars->full[s]);
                    }
                } else {
                    tc::mbar_arrive(&bars->full[s]);
                }
                last = g;
                if (src < 31 && t + 1 < nt) fetch_rows(src + 1, h);
            }
            if (stop || *abort_flag) break;
        }
        if (last >= 0) tc::mbar_wait_warp(&bars->full[last % kDkvStages], (last / kDkvStages) & 1, P.err, 2, abort_flag);
        if (nkv > 0) tc::mbar_wait_warp(&bars->kv_full, (nkv - 1) & 1, P.err, 2, abort_flag);
        tc::cp_async_wait_all();
    } else if (warp == 1) {
        // ------------------------------------------------------------ S^T / dP^T MMAs
        // Per step (64 tokens of a tile): S^T = K_b Q^T and dP^T = V_b dO^T into the
        // step's TMEM buffer, once the dK / dV MMAs of the step two before have
        // read that buffer (buf_free); they run while the softmax works on the
        // previous step.
        const uint32_t idesc_s = tc::idesc_bf16_f32(kBS, kHalf, false, false);
        const uint64_t dk0 = tc::smem_desc_sw128(sK, 16, 1024), dv0 = tc::smem_desc_sw128(sV, 16, 1024);
        int g = 0, hs = 0, nkv = 0;       // g: tile (stage) counter, hs: step counter
        bool stop = false;
        int64_t u = u_begin;
        Seg sg;
        while (!stop && next_seg(u, sg)) {
            const int nt = sg.nt;
            if (!tc::mbar_wait_warp(&bars->kv_full, nkv & 1, P.err, 2, abort_flag)) break;
            for (int t = 0; t < nt && !stop; ++t, ++g) {
                if (!tc::mbar_wait_warp(&bars->full[g % kDkvStages], (g / kDkvStages) & 1, P.err, 2, abort_flag)) {
                    stop = true;
                    break;
                }
                tc::fence_proxy_async_smem();   // dO rows may have come through cp.async (generic proxy)
                for (int half = 0; half < 2; ++half, ++hs) {
                    const int b = hs % kBufs, use = hs / kBufs;   // buffer, and its use count
                    if (use > 0 &&
                        !tc::mbar_wait_warp(&bars->buf_free[b], (use - 1) & 1, P.err, 2, abort_flag)) {
                        stop = true;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sQ = sStage + (g % kDkvStages) * kDkvStage + half * (kHalf * 128);
                    const uint64_t dq0 = tc::smem_desc_sw128(sQ, 16, 1024);
                    const uint64_t dd0 = tc::smem_desc_sw128(sQ + kRowTile, 16, 1024);
                    const uint32_t tb = tmem + b * 128;
                    if (lane == 0) {
#pragma unroll
                        for (int kk = 0; kk < kHD / 16; ++kk) {
                            tc::mma_bf16_ss(tb, dk0 + hd_step(kk), dq0 + hd_step(kk), idesc_s, kk > 0);
                            tc::mma_bf16_ss(tb + kHalf, dv0 + hd_step(kk), dd0 + hd_step(kk), idesc_s, kk > 0);
                        }
                        tc::mma_commit(&bars->s_full[b]);
                    }
                    __syncwarp();
                }
            }
            if (stop) break;
            if (lane == 0) tc::mma_commit(&bars->kv_empty);   // K_b, V_b free once these complete
            __syncwarp();
            ++nkv;
        }
        if (lane == 0) tc::mma_commit(&bars->drain);
        __syncwarp();
        tc::mbar_wait_warp(&bars->drain, 0, P.err, 2, abort_flag);
    } else if (warp == 2) {
        // ------------------------------------------------------------ dK / dV MMAs
        // dV += P^T dO and dK += dS^T Q per step, P^T / dS^T read from TMEM.
        const uint32_t idesc_acc = tc::idesc_bf16_f32(kBS, kHD, false, true);
        int g = 0, hs = 0, nkv = 0;
        bool stop = false;
        int64_t u = u_begin;
        Seg sg;
        while (!stop && next_seg(u, sg)) {
            const int nt = sg.nt;
            for (int t = 0; t < nt && !stop; ++t, ++g) {
                // the stage's Q / dO (acquired directly; the stage is released by this warp)
                if (!tc::mbar_wait_warp(&bars->full[g % kDkvStages], (g / kDkvStages) & 1, P.err, 2, abort_flag)) {
                    stop = true;
                    break;
                }
                tc::fence_proxy_async_smem();
                for (int half = 0; half < 2; ++half, ++hs) {
                    const bool last = (t + 1 == nt) && half == 1;
                    const int b = hs % kBufs, use = hs / kBufs;
                    if (!tc::mbar_wait_warp(&bars->pds_full[b], use & 1, P.err, 2, abort_flag)) {
                        stop = true;
                        break;
                    }
                    // the accumulators are reset by the segment's first step; the
                    // epilogue of the previous segment must have read them
                    if (t == 0 && half == 0 && nkv > 0 &&
                        !tc::mbar_wait_warp(&bars->acc_free, (nkv - 1) & 1, P.err, 2, abort_flag)) {
                        stop = true;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sQ = sStage + (g % kDkvStages) * kDkvStage + half * (kHalf * 128);
                    const uint64_t bq = tc::smem_desc_sw128(sQ, Geo<HD>::kLbo(2 * kRowTile), 1024);
                    const uint64_t bd = tc::smem_desc_sw128(sQ + kRowTile, Geo<HD>::kLbo(2 * kRowTile), 1024);
                    const uint32_t tb = tmem + b * 128;
                    if (lane == 0) {
#pragma unroll
                        for (int kk = 0; kk < kHalf / 16; ++kk) {   // +16 rows (2048 B) per K step
                            const uint32_t acc = (t > 0 || half > 0 || kk > 0) ? 1u : 0u;
                            tc::mma_bf16_ts(tmem + kAccCol, tb + kHalf + kk * 16, bq + 128 * kk, idesc_acc, acc);
                            tc::mma_bf16_ts(tmem + kAccCol + kHD, tb + kk * 16, bd + 128 * kk, idesc_acc, acc);
                        }
                        tc::mma_commit(&bars->buf_free[b]);
                        if (half == 1) tc::mma_commit(&bars->empty[g % kDkvStages]);
                        if (last) tc::mma_commit(&bars->acc_full);
                    }
                    __syncwarp();
                }
            }
            ++nkv;
        }
        if (lane == 0) tc::mma_commit(&bars->drain);
        __syncwarp();
        tc::mbar_wait_warp(&bars->drain, 0, P.err, 2, abort_flag);
    } else {
        // ------------------------------------------------------------ P^T, dS^T, epilogue
        // 16 warps: warp & 3 = TMEM lane quarter (slot rows), (warp-3) >> 2 = the
        // 16-token group of a 64-token step this thread handles; no cross-thread
        // reduction.
        const int quarter = warp & 3;
        const int grp = (warp - 3) >> 2;
        const int r = quarter * 32 + lane;                       // slot row within the block
        const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        int g = 0, hs = 0, nkv = 0;
        bool stop = false;
        int64_t u = u_begin;
        Seg sg;
        while (!stop && next_seg(u, sg)) {
            const int blk = sg.blk, h = sg.h, nt = sg.nt;
            for (int t = 0; t < nt && !stop; ++t, ++g) {
                const int s = g % kDkvStages;
                // the loader's per-token metadata of this stage (acquire it directly)
                if (!tc::mbar_wait_warp(&bars->full[s], (g / kDkvStages) & 1, P.err, 2, abort_flag)) {
                    stop = true;
                    break;
                }
                const float *mb = meta + s * 2 * kTM;
                for (int half = 0; half < 2; ++half, ++hs) {
                    const int b = hs % kBufs, use = hs / kBufs;
                    if (!tc::mbar_wait_warp(&bars->s_full[b], use & 1, P.err, 2, abort_flag)) {
                        stop = true;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t tb = trow + b * 128 + grp * 16;
                    uint32_t sv[16], dv[16];
                    tc::tmem_ld16(tb, sv);
                    tc::tmem_ld16(tb + kHalf, dv);
                    tc::tmem_ld_wait();
                    const int col0 = half * kHalf + grp * 16;        // token within the tile
                    // the 16 tokens' offsets and deltas: 16-B shared loads
                    float cb[16], dl[16];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 a = reinterpret_cast<const float4 *>(mb + col0)[u];
                        const float4 d = reinterpret_cast<const float4 *>(mb + kTM + col0)[u];
                        cb[4 * u] = a.x, cb[4 * u + 1] = a.y, cb[4 * u + 2] = a.z, cb[4 * u + 3] = a.w;
                        dl[4 * u] = d.x, dl[4 * u + 1] = d.y, dl[4 * u + 2] = d.z, dl[4 * u + 3] = d.w;
                    }
                    const uint64_t sc2 = tc::f2(scale_log2, scale_log2);
                    uint32_t pk[8], dk[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const uint64_t x2 = tc::fma2(tc::f2_bits(sv[2 * e], sv[2 * e + 1]), sc2,
                                                     tc::f2(cb[2 * e], cb[2 * e + 1]));
                        const uint64_t p2 = tc::ex2_pair(x2);
                        const float2 p = tc::f2_split(p2);
                        const float2 ds = tc::f2_split(tc::mul2(
                            p2, tc::sub2(tc::f2_bits(dv[2 * e], dv[2 * e + 1]), tc::f2(dl[2 * e], dl[2 * e + 1]))));
                        pk[e] = pack_bf16x2(p.x, p.y);
                        dk[e] = pack_bf16x2(ds.x, ds.y);
                    }
                    // in place: these columns' S^T / dP^T values are already in registers
                    tc::tmem_st8(tb, pk);
                    tc::tmem_st8(tb + kHalf, dk);
                    tc::tmem_st_wait();
                    tc::tc_fence_before();
                    tc::mbar_arrive(&bars->pds_full[b]);
                }
            }
            if (stop) break;
            // epilogue of the segment: 16 columns of dK and of dV per 64-column box
            // and thread -> fp32 reductions
            if (!tc::mbar_wait_warp(&bars->acc_full, nkv & 1, P.err, 2, abort_flag)) break;
            tc::tc_fence_after();
            uint32_t kr[Geo<HD>::kBoxes][16], vr[Geo<HD>::kBoxes][16];
#pragma unroll
            for (int c = 0; c < Geo<HD>::kBoxes; ++c) {
                tc::tmem_ld16(trow + kAccCol + 64 * c + grp * 16, kr[c]);
                tc::tmem_ld16(trow + kAccCol + kHD + 64 * c + grp * 16, vr[c]);
            }
            tc::tmem_ld_wait();
            tc::tc_fence_before();
            tc::mbar_arrive(&bars->acc_free);
            ++nkv;
#pragma unroll
            for (int cb = 0; cb < Geo<HD>::kBoxes; ++cb) {
                float *dkr = dk_acc + (static_cast<int64_t>(blk) * kBS + r) * ld + h * kHD + 64 * cb + grp * 16;
                float *dvr = dv_acc + (static_cast<int64_t>(blk) * kBS + r) * ld + h * kHD + 64 * cb + grp * 16;
#pragma unroll
                for (int c = 0; c < 16; c += 2) {
                    red_add_v2(dkr + c, __uint_as_float(kr[cb][c]) * scale, __uint_as_float(kr[cb][c + 1]) * scale);
                    red_add_v2(dvr + c, __uint_as_float(vr[cb][c]), __uint_as_float(vr[cb][c + 1]));
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------ host side
bool make_bf16_map(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows);
int device_sm_count();

bool read_bwd_tc_supported(int hd, int bs, int top, const void *q, const void *k, const void *v,
                           const void *dout, int H) {
    // head_dim 64 with sets of up to two blocks, head_dim 128 with one block per row
    return read_fwd_tc_supported(hd, bs, top, q, k, v, H) && (reinterpret_cast<uintptr_t>(dout) % 16) == 0;
}

template <int HD, bool kDoRows>
static cudaError_t launch_bwd_tc_t(const CUtensorMap &mk, const CUtensorMap &mv, const CUtensorMap &mq,
                                   const CUtensorMap &md, const uint16_t *dout, const float *lse, int H, int nb,
                                   int top, const PlanLayout &L, const PlanView &P, void *dq, float *dk_acc,
                                   float *dv_acc, float *dlog_gates, float *ws_delta, cudaStream_t st) {
    const float scale = 1.0f / sqrtf(static_cast<float>(HD));
    const float scale_log2 = scale * kLog2e;
    const int sms = device_sm_count();
    constexpr uint32_t dq_smem = Dq<HD>::kSmem, dkv_smem = Dkv<HD>::kSmem;
    cudaError_t e = cudaFuncSetAttribute(read_bwd_dq_tc_kernel<HD, kDoRows>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dq_smem);
    if (e != cudaSuccess) return e;
    const int64_t items = L.max_tiles * H;
    const int grid = static_cast<int>(std::min<int64_t>(items, sms));
    read_bwd_dq_tc_kernel<HD, kDoRows><<<grid, kDqThreads, dq_smem, st>>>(
        mk, mv, mq, md, dout, lse, H, top, scale, scale_log2, P, static_cast<uint16_t *>(dq), dlog_gates, ws_delta);
    count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    e = cudaFuncSetAttribute(read_bwd_dkdv_tc_kernel<HD, kDoRows>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)dkv_smem);
    if (e != cudaSuccess) return e;
    // one CTA per SM, each over an equal share of the (block, head, tile) units
    read_bwd_dkdv_tc_kernel<HD, kDoRows><<<sms, kDkvThreads, dkv_smem, st>>>(
        mk, mv, mq, md, dout, lse, ws_delta, H, nb, top, static_cast<int>(L.max_tiles), scale, scale_log2,
        P, dk_acc, dv_acc);
    count_launch();
    return cudaGetLastError();
}

template <int HD>
static cudaError_t launch_read_bwd_tc_hd(const void *q_rows, const void *k, const void *v, const void *do_src,
                                         bool do_is_rows, const float *lse, int H, int nb, int top,
                                         const PlanLayout &L, const PlanView &P, void *dq, float *dk_acc,
                                         float *dv_acc, float *dlog_gates, float *ws_delta, cudaStream_t st) {
    CUtensorMap mk, mv, mq, md;
    const uint64_t rows = static_cast<uint64_t>(nb) * kBS, cols = static_cast<uint64_t>(H) * HD;
    if (!make_bf16_map(&mk, k, rows, cols, kBS) || !make_bf16_map(&mv, v, rows, cols, kBS) ||
        !make_bf16_map(&mq, q_rows, static_cast<uint64_t>(L.N), cols, kTM))
        return cudaErrorInvalidValue;
    const uint16_t *do16 = static_cast<const uint16_t *>(do_src);
    if (do_is_rows) {
        if (!make_bf16_map(&md, do_src, static_cast<uint64_t>(L.N), cols, kTM)) return cudaErrorInvalidValue;
        return launch_bwd_tc_t<HD, true>(mk, mv, mq, md, do16, lse, H, nb, top, L, P, dq, dk_acc, dv_acc,
                                         dlog_gates, ws_delta, st);
    }
    md = mq;   // unused by the gathering variant
    return launch_bwd_tc_t<HD, false>(mk, mv, mq, md, do16, lse, H, nb, top, L, P, dq, dk_acc, dv_acc, dlog_gates,
                                      ws_delta, st);
}

cudaError_t launch_read_bwd_tc(const void *q_rows, const void *k, const void *v, const void *do_src,
                               bool do_is_rows, const float *lse, int hd, int H, int nb, int top,
                               const PlanLayout &L, const PlanView &P, void *dq, float *dk_acc, float *dv_acc,
                               float *dlog_gates, float *ws_delta, cudaStream_t st) {
    if (hd == 64)
        return launch_read_bwd_tc_hd<64>(q_rows, k, v, do_src, do_is_rows, lse, H, nb, top, L, P, dq, dk_acc,
                                         dv_acc, dlog_gates, ws_delta, st);
    if (hd == 128 && top == 1)
        return launch_read_bwd_tc_hd<128>(q_rows, k, v, do_src, do_is_rows, lse, H, nb, top, L, P, dq, dk_acc,
                                          dv_acc, dlog_gates, ws_delta, st);
    return cudaErrorInvalidValue;
}

}  // namespace mom
