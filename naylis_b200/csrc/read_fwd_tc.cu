// Gated memory read, forward, on the 5th-generation tensor cores (tcgen05).
//
// Same math as read_fwd.cu (reference: mom_kernels/reference.py:39-61 with the
// bias of :14-29, triton_gpu.py:64-141), specialised for the shapes of the
// Naylis configurations: 128-slot blocks; head_dim 64 with at most two blocks
// per routing set (top-2), or head_dim 128 with one block per row (the
// block-split plan of top-k routing with many blocks). A work item is (tile of
// <= 128 tokens sharing one block set, head); CTAs are persistent over items.
//
// Warp roles (608 threads):
//   warp 0     loader: the tile's 128 Q rows by TMA (SWIZZLE_128B boxes of 128
//              rows x 64) into a 4-stage ring, from Q's copy in routing-plan row
//              order (q_rows), where a tile's rows are contiguous; the set's K, V
//              blocks into K/V buffers (two at head_dim 64, one at 128) once per
//              run of items with the same (set, head); tile metadata 32 items at
//              a time (one per lane)
//   warp 1     TMEM owner; S[128 x 256] = Q K^T into TMEM, then O_0 = P[:, block 0] V_0
//   warp 2     O_1 = P[:, block 1] V_1 (one thread issues a tcgen05.mma only every
//              ~100 cycles: the two PV halves get an issuing warp each)
//   warps 3-18 softmax (one TMEM lane = one token row per thread; four warps per
//              lane quarter, 64 score columns each): row max, exp2, row sum, P as
//              bf16 into TMEM (the A operand of PV); the rows' max, sum and token
//              go to the epilogue through a two-item ring in shared memory
//   warps 19-22 epilogue, one per TMEM lane quarter, one item behind the softmax:
//              (O_0 + O_1) / l -> shared memory -> global as whole 128-B rows,
//              log-sum-exp -> global. O is read out of TMEM first and released
//              (o_free) before the stores, so PV(i+1) does not wait for them.
// TMEM: S at columns 0..255, P (bf16 pairs) at 256..383, O_0 / O_1 at 384 / 448
// (head_dim 128: S 0..127, P 256..319, O 384..511).
// P has its own columns so that S(i+1) is issued as soon as the softmax has read
// S(i), overlapping PV(i); the softmax writes P(i+1) once PV(i) is done
// (pv_done), PV(i+1) writes O once the epilogue warps have read O(i) (o_free),
// and the softmax of i+1 runs while the epilogue of i stores.
// All waits are bounded (tc::mbar_wait); a timeout sets bit 1 of the plan's
// error word and every role unwinds.
#include <cudaTypedefs.h>

#include "launch.h"
#include "tc_common.cuh"

namespace mom {

namespace {
constexpr int kBS = 128;
constexpr int kTM = 128;                       // token rows per tile (TMEM lanes)
constexpr int kSoftWarps = 16;                 // 4 per SM sub-partition
constexpr int kSoftThreads = kSoftWarps * 32;
constexpr int kEpiWarp0 = 3 + kSoftWarps;       // first epilogue warp (warp & 3 = its lane quarter)
constexpr int kEpiThreads = 4 * 32;
constexpr int kThreads = 96 + kSoftThreads + kEpiThreads;   // loader + 2 MMA issuers + softmax + epilogue
constexpr uint32_t kBoxBytes = 128 * 128;      // one TMA box: 128 rows x 64 bf16 columns (128-B swizzle)
constexpr uint32_t kOutBytes = kTM * 64 * 2;   // 64 output columns of the tile, staged for coalesced stores
// row max / sums [4][128]; O staging [128 rows][128 B]; the epilogue ring: two
// items of {row max, row sum, token} [128] and {head, blocks, first plan row}
constexpr uint32_t kRingItemBytes = 3 * kTM * 4 + 16;
constexpr uint32_t kScratchBytes = 8 * kTM * 4 + kOutBytes + 2 * kRingItemBytes;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kPCol = 256;                // P: group g's 64 slots at 256 + 32g (bf16 pairs)
constexpr uint32_t kOCol = 384;                // head_dim 64: O_0 at 384, O_1 at 448; head_dim 128: O at 384

// head_dim 64: sets of up to two blocks (S 256 columns, two O halves).
// head_dim 128: one block per row (the block-split plan): S 128, O 128 columns.
// Rows of Q / K / V are 64-column TMA boxes side by side (kBoxBytes apart).
template <int HD>
struct Fwd {
    static constexpr int kHD = HD;
    static constexpr int kMaxBlk = HD == 64 ? 2 : 1;
    static constexpr int kBoxes = HD / 64;
    static constexpr uint32_t kQBytes = kTM * HD * 2;
    static constexpr uint32_t kBlkBytes = kBS * HD * 2;     // one 128-slot block of K or V
    // Q tiles in a ring of kQStages; the set's K and V blocks in kKvBufs buffers,
    // loaded once per run of items with the same (set, head)
    static constexpr int kQStages = 4;
    static constexpr int kKvBufs = HD == 64 ? 2 : 1;
    static constexpr uint32_t kKvBytes = 2 * kMaxBlk * kBlkBytes;   // K blocks + V blocks
    static constexpr uint32_t kRingBytes = kQStages * kQBytes + kKvBufs * kKvBytes;
    static constexpr uint32_t kSmemBytes = kRingBytes + kScratchBytes + 1024 /*barriers*/ + 1024 /*align*/;
    // V as the MN-major B operand of PV: N-atoms of 64 columns kBoxBytes apart
    // (head_dim 64 has one atom; its value is what the validated kernel used)
    static constexpr uint32_t kVLbo = HD == 64 ? 2 * kBlkBytes : kBoxBytes;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

struct Bars {
    uint64_t q_full[4], q_empty[4], kv_full[2], kv_empty[2], s_full, p_full, pv_done, o_full, o_free, drain,
        s_issued, stats_full[2], stats_free[2];
    uint32_t tmem_base;
    int abort;
    // per Q stage: blocks loaded | (blocks of the set << 8) | (new K/V load << 16);
    // written before the stage's barrier
    int meta[4];
};
static_assert(sizeof(Bars) <= 1024, "barrier block");
}  // namespace

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
read_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                   const __grid_constant__ CUtensorMap tmap_q, int H, int top, float scale_log2, PlanView P,
                   uint16_t *__restrict__ out, float *__restrict__ lse) {
    using C = Fwd<HD>;
    constexpr int kHD = C::kHD, kQStages = C::kQStages, kKvBufs = C::kKvBufs;
    constexpr uint32_t kQBytes = C::kQBytes, kBlkBytes = C::kBlkBytes, kKvBytes = C::kKvBytes;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char *sbase = smem_raw + (base - raw);
    const uint32_t kvbase = base + kQStages * kQBytes;                 // [kKvBufs][K blocks | V blocks]
    float *sMax = reinterpret_cast<float *>(sbase + C::kRingBytes);     // [4][128]
    float *sSum = sMax + 4 * kTM;                                        // [4][128]
    uint4 *sOut = reinterpret_cast<uint4 *>(sSum + 4 * kTM);            // [128 rows][8 x 16 B], swizzled
    // epilogue ring, item parity p: eM[p][128], eL[p][128], eTok[p][128], eInfo[p][4]
    unsigned char *sRing = reinterpret_cast<unsigned char *>(sOut + kTM * 8);
    auto eM = [&](int p) { return reinterpret_cast<float *>(sRing + p * kRingItemBytes); };
    auto eL = [&](int p) { return eM(p) + kTM; };
    auto eTok = [&](int p) { return reinterpret_cast<int *>(eM(p) + 2 * kTM); };
    auto eInfo = [&](int p) { return eTok(p) + kTM; };
    Bars *bars = reinterpret_cast<Bars *>(sbase + C::kRingBytes + kScratchBytes);
    volatile int *abort_flag = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = *P.ntiles;
    const int nitems = ntiles * H;
    // items of this CTA: a contiguous run it0 + i, i < nmine, ordered head-major
    // (item = head * ntiles + tile), so that consecutive items usually share
    // their block set and head: a stage keeps its K/V blocks when they repeat
    const int per = (nitems + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
    const int it0 = static_cast<int>(blockIdx.x) * per;
    const int nmine = max(0, min(nitems, it0 + per) - it0);
    auto item_tile = [&](int item) { return item % ntiles; };
    auto item_head = [&](int item) { return item / ntiles; };
    const int64_t ld = static_cast<int64_t>(H) * kHD;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kQStages; ++s) {
            tc::mbar_init(&bars->q_full[s], 1);
            tc::mbar_init(&bars->q_empty[s], 2);    // both MMA warps release a stage (meta is read by both)
        }
        for (int b = 0; b < kKvBufs; ++b) {
            tc::mbar_init(&bars->kv_full[b], 1);
            // the warps whose MMAs read K/V: warp 1 (S, PV of block 0), warp 2 (PV of block 1)
            tc::mbar_init(&bars->kv_empty[b], C::kMaxBlk > 1 ? 2 : 1);
        }
        tc::mbar_init(&bars->o_full, 2);
        tc::mbar_init(&bars->o_free, kEpiThreads);
        for (int p = 0; p < 2; ++p) {
            tc::mbar_init(&bars->stats_full[p], kSoftThreads);
            tc::mbar_init(&bars->stats_free[p], kEpiThreads);
        }
        tc::mbar_init(&bars->s_full, 1);
        tc::mbar_init(&bars->p_full, kSoftThreads);
        tc::mbar_init(&bars->pv_done, 2);
        tc::mbar_init(&bars->drain, 2);
        tc::mbar_init(&bars->s_issued, 1);
        bars->abort = 0;
    }
    if (warp == 1) {
        tc::tmem_alloc(&bars->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tc::prefetch_tensormap(&tmap_k);
        tc::prefetch_tensormap(&tmap_v);
        tc::prefetch_tensormap(&tmap_q);
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ loader
        // Per item: its Q tile into the next ring stage, with the stage's meta; when
        // the (set, head) changes, then the set's K/V blocks into the next K/V buffer
        // once the MMAs that read that buffer's previous load are done (kv_empty).
        // Q and meta go first: the MMA warps release a K/V buffer when they meet the
        // item that starts the next load.
        tc::LaneTile lt;
        int issued = 0, nkv = 0, cur_kv = -1;
        for (int i = 0; i < nmine; ++i) {
            const int item = it0 + i;
            const int s = i % kQStages, j = i / kQStages, src = i & 31;
            if (src == 0 && i + lane < nmine) lt.fetch(P, item_tile(item + lane), top);
            const int x0 = tc::get(lt.x, src);
            const int nblk = tc::get(lt.nblk, src), b0 = tc::get(lt.b0, src), b1 = tc::get(lt.b1, src);
            if (!tc::mbar_wait_warp(&bars->q_empty[s], (j & 1) ^ 1, P.err, 2, abort_flag)) break;
            const int h = item_head(item);
            const int nload = nblk > 0 ? nblk : 1;
            const uint32_t sQ = base + s * kQBytes;
            const int kv = tc::get(lt.key, src) * H + h;
            const bool reload = kv != cur_kv;
            cur_kv = kv;
            if (lane == 0) {
                bars->meta[s] = nload | (nblk << 8) | (reload ? 1 << 16 : 0);   // released by the arrive below
                tc::mbar_arrive_expect_tx(&bars->q_full[s], kQBytes);
                // the tile's rows x0 .. x0+127 (rows past the tile are never stored)
#pragma unroll
                for (int c = 0; c < C::kBoxes; ++c)
                    tc::tma_load_2d(sQ + c * kBoxBytes, &tmap_q, h * kHD + 64 * c, x0, &bars->q_full[s]);
            }
            __syncwarp();
            issued = i + 1;
            if (reload) {
                const int b = nkv % kKvBufs, u = nkv / kKvBufs;
                if (u > 0 && !tc::mbar_wait_warp(&bars->kv_empty[b], (u - 1) & 1, P.err, 2, abort_flag)) break;
                const uint32_t sK = kvbase + b * kKvBytes, sV = sK + C::kMaxBlk * kBlkBytes;
                if (lane == 0) {
                    tc::mbar_arrive_expect_tx(&bars->kv_full[b], 2 * nload * kBlkBytes);
                    for (int jb = 0; jb < nload; ++jb) {
                        const int blk = nblk > 0 ? (jb == 0 ? b0 : b1) : 0;
#pragma unroll
                        for (int c = 0; c < C::kBoxes; ++c) {
                            tc::tma_load_2d(sK + jb * kBlkBytes + c * kBoxBytes, &tmap_k, h * kHD + 64 * c,
                                            blk * kBS, &bars->kv_full[b]);
                            tc::tma_load_2d(sV + jb * kBlkBytes + c * kBoxBytes, &tmap_v, h * kHD + 64 * c,
                                            blk * kBS, &bars->kv_full[b]);
                        }
                    }
                }
                __syncwarp();
                ++nkv;
            }
        }
        // make sure no TMA write is still in flight when the CTA retires
        if (issued > 0) {
            const int i = issued - 1;
            tc::mbar_wait_warp(&bars->q_full[i % kQStages], (i / kQStages) & 1, P.err, 2, abort_flag);
        }
        if (nkv > 0)
            tc::mbar_wait_warp(&bars->kv_full[(nkv - 1) % kKvBufs], ((nkv - 1) / kKvBufs) & 1, P.err, 2, abort_flag);
    } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------------------ MMA issuers
        // Warp 1 issues S(i+1) as soon as the softmax has read S(i) (p_full of i),
        // ahead of its half of PV(i); warp 2 issues the other half only after that
        // (s_issued), so S(i+1) runs first on the tensor pipe and the softmax of i+1
        // starts while PV(i) still runs. K/V loads: each warp counts the loads it has
        // switched to (nkv); load n sits in buffer n % kKvBufs. A warp releases a
        // buffer (kv_empty) after its last MMA that reads it. With one buffer, the
        // item that starts a new load has its S issued after PV of the item before
        // (both read the buffer), so warp 1 then issues PV(i) first.
        const bool wa = warp == 1;
        const uint32_t idesc_o = tc::idesc_bf16_f32(kTM, kHD, false, true);
        int nkv = 0;
        // wait for item i's Q stage; its meta
        auto stage_meta = [&](int i, int &meta) -> bool {
            if (!tc::mbar_wait_warp(&bars->q_full[i % kQStages], (i / kQStages) & 1, P.err, 2, abort_flag))
                return false;
            meta = tc::ld_shared_volatile(&bars->meta[i % kQStages]);
            return true;
        };
        // the next K/V load has landed (this warp's nkv-th switch)
        auto kv_switch = [&]() -> bool {
            const int n = nkv++;
            return tc::mbar_wait_warp(&bars->kv_full[n % kKvBufs], (n / kKvBufs) & 1, P.err, 2, abort_flag);
        };
        // warp 1: S(i) = Q K^T into TMEM columns 0..255, K from buffer kb
        auto issue_s = [&](int i, int meta, int kb) {
            const int nload = meta & 0xFF;
            const uint32_t sQ = base + (i % kQStages) * kQBytes;
            const uint32_t sK = kvbase + kb * kKvBytes;
            tc::tc_fence_after();
            if (lane == 0) {
                const uint32_t idesc_s = tc::idesc_bf16_f32(kTM, nload * kBS, false, false);
                const uint64_t ad = tc::smem_desc_sw128(sQ, 16, 1024), bd = tc::smem_desc_sw128(sK, 16, 1024);
#pragma unroll
                for (int kk = 0; kk < kHD / 16; ++kk) {
                    // +32 B per K step within a 64-column box (+2 in the address field),
                    // +kBoxBytes (+1024) to the next box
                    const uint64_t step = 1024u * (kk >> 2) + 2u * (kk & 3);
                    tc::mma_bf16_ss(tmem, ad + step, bd + step, idesc_s, kk > 0);
                }
                tc::mma_commit(&bars->s_full);
            }
            __syncwarp();
        };
        // PV of item i's block (warp 1: block 0, warp 2: block 1), V from buffer kb
        auto issue_pv = [&](int i, int nblk, int kb) {
            tc::tc_fence_after();
            if (lane == 0) {
                if (nblk > (wa ? 0 : 1) && (wa || C::kMaxBlk > 1)) {
                    const uint32_t sV = kvbase + kb * kKvBytes + C::kMaxBlk * kBlkBytes;
                    const uint64_t bv = tc::smem_desc_sw128(sV + (wa ? 0 : kBlkBytes), C::kVLbo, 1024);
#pragma unroll
                    for (int k8 = 0; k8 < 8; ++k8) {   // the block's 128 slots, 16 per step
                        const int kk = (wa ? 0 : 8) + k8;
                        tc::mma_bf16_ts(tmem + kOCol + (wa ? 0 : kHD), tmem + kPCol + 32 * (kk >> 2) + 8 * (kk & 3),
                                        bv + 128 * k8, idesc_o, k8 > 0);
                    }
                }
                tc::mma_commit(&bars->o_full);
                tc::mma_commit(&bars->q_empty[i % kQStages]);
                tc::mma_commit(&bars->pv_done);
            }
            __syncwarp();
        };
        auto release = [&](int kb) {
            if (lane == 0) tc::mma_commit(&bars->kv_empty[kb]);
            __syncwarp();
        };
        if (wa) {
            int meta_next = 0, kb_next = 0;
            bool ok = nmine > 0 && stage_meta(0, meta_next) && kv_switch();
            if (ok) {
                kb_next = (nkv - 1) % kKvBufs;
                issue_s(0, meta_next, kb_next);
            }
            for (int i = 0; ok && i < nmine; ++i) {
                const int meta_i = meta_next, kb_i = kb_next;
                // P(i) written to TMEM (and S(i) read) by the softmax
                if (!tc::mbar_wait_warp(&bars->p_full, i & 1, P.err, 2, abort_flag)) break;
                const bool next = i + 1 < nmine;
                if (next && !stage_meta(i + 1, meta_next)) break;
                const bool sw = next && ((meta_next >> 16) & 1);
                const bool pv_first = sw && kKvBufs == 1;
                if (next && !pv_first) {
                    if (sw && !kv_switch()) break;
                    kb_next = (nkv - 1) % kKvBufs;
                    issue_s(i + 1, meta_next, kb_next);
                }
                if (!pv_first) {
                    // S(i+1) is in the tensor pipe ahead of both PV halves of i
                    if (lane == 0) tc::mbar_arrive(&bars->s_issued);
                    __syncwarp();
                }
                // O read by the epilogue of i-1
                if (i > 0 && !tc::mbar_wait_warp(&bars->o_free, (i - 1) & 1, P.err, 2, abort_flag)) break;
                issue_pv(i, (meta_i >> 8) & 0xFF, kb_i);
                if (sw) release(kb_i);   // this warp's last MMA on item i's K/V load
                if (pv_first) {
                    if (!kv_switch()) break;
                    kb_next = (nkv - 1) % kKvBufs;
                    issue_s(i + 1, meta_next, kb_next);
                    if (lane == 0) tc::mbar_arrive(&bars->s_issued);
                    __syncwarp();
                }
            }
        } else {
            int kb = 0;
            for (int i = 0; i < nmine; ++i) {
                int meta = 0;
                if (!stage_meta(i, meta)) break;
                if (C::kMaxBlk > 1 && ((meta >> 16) & 1)) {
                    // a new K/V load: PV(i-1), this warp's last read of the previous one, is issued
                    if (i > 0) release(kb);
                    if (!kv_switch()) break;
                    kb = (nkv - 1) % kKvBufs;
                }
                if (!tc::mbar_wait_warp(&bars->p_full, i & 1, P.err, 2, abort_flag)) break;
                if (!tc::mbar_wait_warp(&bars->s_issued, i & 1, P.err, 2, abort_flag)) break;
                if (i > 0 && !tc::mbar_wait_warp(&bars->o_free, (i - 1) & 1, P.err, 2, abort_flag)) break;
                issue_pv(i, (meta >> 8) & 0xFF, kb);
            }
        }
        // drain: every MMA this thread issued has completed before TMEM is freed
        if (lane == 0) tc::mma_commit(&bars->drain);
        __syncwarp();
        tc::mbar_wait_warp(&bars->drain, 0, P.err, 2, abort_flag);
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------------ softmax
        // 16 warps: warp & 3 is the TMEM lane quarter (hardware rule), (warp-3) >> 2
        // the 64-column group of the 256 score columns (block = group >> 1). The
        // four warps of one lane quarter exchange partial row max / sum through
        // shared memory under named barrier 1 + quarter.
        const int quarter = warp & 3;
        const int grp = (warp - 3) >> 2;
        const int jb = grp >> 1;
        const int r = quarter * 32 + lane;
        const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        const int bar_id = 1 + quarter;
        // per-item row metadata: tile fields for 32 items at a time (one per lane),
        // this thread's row (token, gate bias) one item ahead, so that no global
        // load latency sits on the softmax path
        struct Meta { int nblk, tok, row; float bias; };
        tc::LaneTile lt;
        auto fetch = [&](int src, Meta &m) {
            const int x = tc::get(lt.x, src), y = tc::get(lt.y, src);
            m.nblk = tc::get(lt.nblk, src);
            m.tok = r < y ? P.perm[x + r] : -1;
            m.row = x + r;
            m.bias = (r < y && jb < m.nblk) ? P.rowbias[static_cast<int64_t>(x + r) * top + jb] * kLog2e : 0.0f;
        };
        Meta cur, nxt;
        int count = 0;
        bool dead = false;   // a bounded wait gave up: skip work, keep the barrier structure
        for (int i = 0; i < nmine; ++i) {
            const int item = it0 + i;
            const int src = i & 31;
            if (src == 0) {
                if (i + lane < nmine) lt.fetch(P, item_tile(item + lane), top);
                fetch(0, cur);
            } else {
                cur = nxt;   // prefetched during item i-1
            }
            if (src < 31 && i + 1 < nmine) fetch(src + 1, nxt);
            const int h = item_head(item), nblk = cur.nblk, tok = cur.tok;
            const float bias = cur.bias;
            if (!dead && !tc::mbar_wait_warp(&bars->s_full, i & 1, P.err, 2, abort_flag)) dead = true;
            const bool live = jb < nblk && !dead;
            tc::tc_fence_after();
            // pass 1: partial row maximum over this thread's 64 columns
            float mpart = -INFINITY;
            if (live) {
                float mx = -INFINITY;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t v[32];
                    tc::tmem_ld32(trow + grp * 64 + c * 32, v);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; e += 2) mx = tc::fmax3(mx, __uint_as_float(v[e]), __uint_as_float(v[e + 1]));
                }
                mpart = fmaf(mx, scale_log2, bias);
            }
            sMax[grp * kTM + r] = mpart;
            tc::named_bar(bar_id, 128);
            float m = sMax[r];
#pragma unroll
            for (int g = 1; g < 4; ++g) m = fmaxf(m, sMax[g * kTM + r]);
            const float mref = (m == -INFINITY) ? 0.0f : m;
            // P(i-1) must have been consumed by PV(i-1) before P(i) overwrites it
            if (!dead && i > 0 && !tc::mbar_wait_warp(&bars->pv_done, (i - 1) & 1, P.err, 2, abort_flag))
                dead = true;
            tc::tc_fence_after();
            // pass 2: p = 2^(s*scale + bias - m) -> bf16 P into TMEM (group grp's 64 slots
            // at kPCol + 32*grp, chunk c at +16c), partial row sum
            float lpart = 0.0f;
            if (live && !dead) {
                const float bj = bias - mref;
                const uint64_t sc2 = tc::f2(scale_log2, scale_log2), bj2 = tc::f2(bj, bj);
                uint64_t l2 = tc::f2(0.0f, 0.0f);
                // chunk c: 16 score columns -> 8 bf16 pairs of P at kPCol + 32*grp + 8c
                auto chunk = [&](const uint32_t (&v)[16], int c) {
                    uint32_t pk[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        // column pairs: 3 of 8 by the FMA-pipe polynomial, the rest by MUFU
                        const uint64_t x2 = tc::fma2(tc::f2_bits(v[2 * e], v[2 * e + 1]), sc2, bj2);
                        const uint64_t p2 = (e & 1) && e < 7 ? tc::ex2_poly2(x2) : tc::ex2_pair(x2);
                        l2 = tc::add2(l2, p2);
                        const float2 p = tc::f2_split(p2);
                        pk[e] = pack_bf16x2(p.x, p.y);
                    }
                    tc::tmem_st8(trow + kPCol + grp * 32 + c * 8, pk);
                };
                // the load of chunk c+1 is in flight while chunk c is computed
                const uint32_t s0 = trow + grp * 64;
                uint32_t va[16], vb[16];
                tc::tmem_ld16(s0, va);
                tc::tmem_ld_wait_regs(va);
                tc::tmem_ld16(s0 + 16, vb);
                chunk(va, 0);
                tc::tmem_ld_wait_regs(vb);
                tc::tmem_ld16(s0 + 32, va);
                chunk(vb, 1);
                tc::tmem_ld_wait_regs(va);
                tc::tmem_ld16(s0 + 48, vb);
                chunk(va, 2);
                tc::tmem_ld_wait_regs(vb);
                chunk(vb, 3);
                tc::tmem_st_wait();
                const float2 l = tc::f2_split(l2);
                lpart = l.x + l.y;
            }
            sSum[grp * kTM + r] = lpart;
            tc::tc_fence_before();
            tc::mbar_arrive(&bars->p_full);
            // row sums of item i complete; the four warps of this lane quarter agree
            // on stopping together
            dead = tc::named_bar_or(bar_id, 128, dead);
            if (dead) break;
            // item i's rows (max, sum, token) to the epilogue warps, ring slot i & 1,
            // once the epilogue has read the slot's previous item (stats_free)
            const int ps = i & 1;
            if (grp == 0) {
                const bool ok = i < 2 || tc::mbar_wait_warp(&bars->stats_free[ps], ((i >> 1) - 1) & 1, P.err, 2,
                                                            abort_flag);
                if (ok) {
                    eM(ps)[r] = m;
                    eL(ps)[r] = sSum[r] + sSum[kTM + r] + sSum[2 * kTM + r] + sSum[3 * kTM + r];
                    eTok(ps)[r] = tok;
                    if (r == 0) {
                        eInfo(ps)[0] = h;
                        eInfo(ps)[1] = nblk;
                        eInfo(ps)[2] = cur.row;   // the tile's first plan row (this is row 0)
                    }
                }
            }
            tc::mbar_arrive(&bars->stats_full[ps]);
            count = i + 1;
        }
        (void)count;
    } else {
        // ------------------------------------------------------------ epilogue
        // One warp per TMEM lane quarter (warp & 3), one item behind the softmax:
        // O(i) out of TMEM (both halves of a two-block set summed), released to
        // PV(i+1) (o_free), then scaled by 1/l, packed to bf16, staged as whole
        // 128-B rows in shared memory and stored; the log-sum-exp per row.
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        uint4 *srow = sOut + r * 8;                       // this thread's staging row
        const int64_t n_rows = P.n;
        // rows quarter*32 .. +31 of the staging buffer to global, 4 rows per store
        auto store_rows = [&](int tok, uint16_t *dst_col) {
            __syncwarp();
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int rr = k * 4 + (lane >> 3), ch = lane & 7;
                const int t = __shfl_sync(0xffffffffu, tok, rr);
                const int row = quarter * 32 + rr;
                if (t >= 0 && t < n_rows)
                    reinterpret_cast<uint4 *>(dst_col + static_cast<int64_t>(t) * ld)[ch] = sOut[row * 8 + (ch ^ (row & 7))];
            }
            __syncwarp();
        };
        for (int i = 0; i < nmine; ++i) {
            const int ps = i & 1;
            if (!tc::mbar_wait_warp(&bars->stats_full[ps], (i >> 1) & 1, P.err, 2, abort_flag)) break;
            if (!tc::mbar_wait_warp(&bars->o_full, i & 1, P.err, 2, abort_flag)) break;
            const float m = eM(ps)[r], l = eL(ps)[r];
            const int tok = eTok(ps)[r];
            const int h = eInfo(ps)[0], nblk = eInfo(ps)[1], row0 = eInfo(ps)[2];
            tc::mbar_arrive(&bars->stats_free[ps]);
            if (*abort_flag || h < 0 || h >= H) break;
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            tc::tc_fence_after();
            uint16_t *dst = out + static_cast<int64_t>(h) * kHD;
            auto pack8 = [&](const float (&o)[16], int c, uint32_t (&pk)[8]) {
                (void)c;
#pragma unroll
                for (int e = 0; e < 8; ++e) pk[e] = pack_bf16x2(o[2 * e] * inv, o[2 * e + 1] * inv);
            };
            auto stage = [&](int c, const uint32_t (&pk)[8]) {
                srow[(2 * c) ^ (r & 7)] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                srow[(2 * c + 1) ^ (r & 7)] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            };
            if constexpr (HD == 64) {
                // O_0 at 384, O_1 at 448: the set's two blocks, summed
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t a0[16], a1[16];
                    tc::tmem_ld16(trow + kOCol + 16 * c, a0);
                    tc::tmem_ld16(trow + kOCol + 64 + 16 * c, a1);
                    tc::tmem_ld_wait_regs(a0);
                    tc::tmem_ld_wait_regs(a1);
                    float o[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        o[e] = (nblk > 0 ? __uint_as_float(a0[e]) : 0.0f) + (nblk > 1 ? __uint_as_float(a1[e]) : 0.0f);
                    uint32_t pk[8];
                    pack8(o, c, pk);
                    stage(c, pk);
                }
                tc::tc_fence_before();
                tc::mbar_arrive(&bars->o_free);
                store_rows(tok, dst);
            } else {
                // one O of 128 columns: the first 64 staged and stored, the second
                // kept in registers until O is released
                uint32_t hi[4][8];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t a0[16], a1[16];
                    tc::tmem_ld16(trow + kOCol + 16 * c, a0);
                    tc::tmem_ld16(trow + kOCol + 64 + 16 * c, a1);
                    tc::tmem_ld_wait_regs(a0);
                    tc::tmem_ld_wait_regs(a1);
                    float o[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] = nblk > 0 ? __uint_as_float(a0[e]) : 0.0f;
                    uint32_t pk[8];
                    pack8(o, c, pk);
                    stage(c, pk);
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] = nblk > 0 ? __uint_as_float(a1[e]) : 0.0f;
                    pack8(o, c, hi[c]);
                }
                tc::tc_fence_before();
                tc::mbar_arrive(&bars->o_free);
                store_rows(tok, dst);
#pragma unroll
                for (int c = 0; c < 4; ++c) stage(c, hi[c]);
                store_rows(tok, dst + 64);
            }
            if (tok >= 0 && row0 + r < n_rows)
                lse[static_cast<int64_t>(h) * n_rows + row0 + r] = l > 0.0f ? (m + log2f(l)) * kLn2 : -INFINITY;
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D bf16 map over a row-major [rows, cols] matrix, box = 64 columns x box_rows, 128-B swizzle.
bool make_bf16_map(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// head_dim 64 with sets of up to two blocks; head_dim 128 with one block per row
// (the block-split plan)
bool read_fwd_tc_supported(int hd, int bs, int top, const void *q, const void *k, const void *v, int H) {
    return ((hd == 64 && top >= 1 && top <= 2) || (hd == 128 && top == 1)) && bs == kBS &&
           (reinterpret_cast<uintptr_t>(k) % 16) == 0 && (reinterpret_cast<uintptr_t>(v) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(q) % 16) == 0 && (H * hd * 2) % 16 == 0 && encode_fn() != nullptr;
}

int device_sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int HD>
static cudaError_t launch_fwd_tc_t(const void *q_rows, const void *k, const void *v, int H, int nb, int top,
                                   const PlanLayout &L, const PlanView &P, void *out, float *lse, cudaStream_t st) {
    CUtensorMap mk, mv, mq;
    const uint64_t rows = static_cast<uint64_t>(nb) * kBS, cols = static_cast<uint64_t>(H) * HD;
    if (!make_bf16_map(&mk, k, rows, cols, kBS) || !make_bf16_map(&mv, v, rows, cols, kBS) ||
        !make_bf16_map(&mq, q_rows, static_cast<uint64_t>(L.N), cols, kTM))
        return cudaErrorInvalidValue;
    constexpr uint32_t smem = Fwd<HD>::kSmemBytes;
    cudaError_t e = cudaFuncSetAttribute(read_fwd_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    const int64_t items = L.max_tiles * H;
    const int grid = static_cast<int>(std::min<int64_t>(items, device_sm_count()));
    const float scale_log2 = kLog2e / sqrtf(static_cast<float>(HD));
    read_fwd_tc_kernel<HD><<<grid, kThreads, smem, st>>>(mk, mv, mq, H, top, scale_log2, P,
                                                         static_cast<uint16_t *>(out), lse);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_read_fwd_tc(const void *q_rows, const void *k, const void *v, int hd, int H, int nb, int top,
                               const PlanLayout &L, const PlanView &P, void *out, float *lse,
                               cudaStream_t st) {
    if (hd == 64) return launch_fwd_tc_t<64>(q_rows, k, v, H, nb, top, L, P, out, lse, st);
    if (hd == 128 && top == 1) return launch_fwd_tc_t<128>(q_rows, k, v, H, nb, top, L, P, out, lse, st);
    return cudaErrorInvalidValue;
}

}  // namespace mom
