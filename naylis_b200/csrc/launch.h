// Host-side launchers shared between the kernel files and the C ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mom {

// Kernels launched by this library since it was loaded (all devices/threads).
void count_launch(int n = 1);
uint64_t launches();

constexpr int kTileM = 128;       // tokens per read tile (one routing set per tile)
constexpr int kMaxKeys = 8192;    // routing sets the bucketing supports
constexpr int kBucketChunk = 256;    // tokens per bucketing chunk (one CTA)
constexpr int kMaxTop = 8;        // top_blocks the library takes

// Routing sets of size s <= top over nb blocks, ranked by the combinatorial
// number system; key = (number of sets of smaller size) + rank.
int64_t num_route_keys(int64_t nb, int64_t top);

// A shard of the sequence for the router scan: rows [t_base, t_base + S) of
// every batch row. carry_in (may be null: t_base = 0, nothing before) is the
// running state entering the shard; carry_out (may be null) receives it after
// the shard's last row. Layouts: exact fp64 mode double[2][B][d] ([0] the sum of
// the rows before, [1] 1.0 where the whole sequence's exactness certificate
// holds); fp32 mode float[B][d] (the sequential fp32 sum).
struct ScanShard {
    int64_t t_base = 0;
    const void *carry_in = nullptr;
    void *carry_out = nullptr;
};

struct PlanLayout {
    int64_t N = 0, nb = 0, top = 0, num_keys = 0, chunks = 0, max_tiles = 0;
    size_t off_err = 0, off_ntiles = 0, off_key = 0, off_hist = 0, off_keytot = 0,
           off_keybase = 0, off_keytb = 0, off_keyset = 0, off_perm = 0, off_rowbias = 0,
           off_rowkmap = 0, off_tiles = 0, off_blkcount = 0, off_blktiles = 0, total = 0;
};
PlanLayout plan_layout(int64_t N, int64_t nb, int64_t top);

// Device view of a plan (pointers into the caller's buffer).
struct PlanView {
    int64_t n;           // tokens (rows of the plan)
    int *err;            // [1]     error word (bit 0: index out of range)
    int *ntiles;         // [1]     number of tiles
    int *key;            // [N]     routing-set key of each token
    int *hist;           // [chunks][num_keys] per-chunk counts -> offsets
    int *keytot;         // [num_keys]
    int *keybase;        // [num_keys] first permuted row of each key
    int *keytb;          // [num_keys] first tile of each key
    int *keyset;         // [num_keys][top] blocks of each set, ascending, -1 padded
    int *perm;           // [N]     token of each permuted row
    float *rowbias;      // [N][top] bias of the j-th block of the row's set
    uint32_t *rowkmap;   // [N]     4 bits per caller slot k: set position j (0xF = none)
    int4 *tiles;         // [max_tiles] {first row, rows, key, 0}
    int *blkcount;       // [nb]
    int *blktiles;       // [nb][max_tiles] tiles whose set contains block b
    // Rows of q (and, in the backward, of the output O used for delta) are
    // perm[r] / rows_per_q: 1 for a plan over tokens; `top` for a plan over
    // (token, k) pairs, where every token's q row serves its `top` rows while
    // the per-row outputs, dO and dQ stay indexed by perm[r].
    int rows_per_q;
};
PlanView plan_view(void *plan, const PlanLayout &L);

cudaError_t launch_route_scan(const void *x, int xdt, void *hq, int cdt, int B, int S, int d,
                              int mode, cudaStream_t st,
                              const ScanShard &sh = ScanShard());
// Per (b, column) state of a sequence shard for the exact fp64 scan:
// stats double[3][B][d] = its sum, an upper bound of its sum of |x|, the ulp
// exponent of its smallest non-zero element (1 << 20 when all are zero).
// The aux loss, router entropy and dead-block fraction of one MoM layer from its
// router outputs; out = [aux, entropy, dead, frac_0 .. frac_{nb-1}].
size_t router_aux_workspace_size(int64_t N, int nb);
cudaError_t launch_router_aux(const float *probs, const void *top_idx, bool idx64, int64_t N, int nb, int top,
                              float *ws, float *out, cudaStream_t st);
cudaError_t launch_route_shard_stats(const void *x, int xdt, int B, int S, int d, double *stats, cudaStream_t st);
// From all shards' stats (W x [3][B][d], rank order): carry double[2][B][d] for
// shard `rank` and, in *uncertified, the number of (b, column) whose whole-
// sequence certificate fails (those need the sequential carry of the previous
// shard instead of the sum).
cudaError_t launch_route_shard_carry(const double *stats_all, int W, int rank, int B, int d, double *carry,
                                     int *uncertified, cudaStream_t st);
cudaError_t launch_route_head(const void *hq, const void *w_down, const void *w_up, int cdt,
                              int64_t ntok, int d, int r, int nb, int top, const float *noise,
                              float *probs, void *top_idx, int idx64, float *gates,
                              float *log_gates, void *act, cudaStream_t st);
cudaError_t launch_route_bwd(const void *x, int xdt, int B, int S, int d, const void *w_down,
                             const void *w_up, int cdt, int r, int nb, int top, const float *probs,
                             const void *top_idx, int idx64, const float *gates, const void *act,
                             const float *dlog_gates, const float *dgates, const float *dprobs,
                             void *dx, int dxdt, int accumulate, float *dw_down, float *dw_up,
                             float *ws_dlogits, float *ws_dz, float *ws_u, cudaStream_t st);
cudaError_t launch_scale_fwd(const void *o, int odt, const float *scale, int64_t n, float *y, cudaStream_t st);
cudaError_t launch_scale_bwd(const void *g, int gdt, const void *o, int odt, const float *scale, int64_t n,
                             void *d_o, float *d_scale, cudaStream_t st);
// out = scale * -log(-log(u + 1e-9) + 1e-9), elementwise (out may alias u).
cudaError_t launch_gumbel(const float *u, int64_t n, float scale, float *out, cudaStream_t st);
// [dk | dv] (L, 2n) bf16 from dk, dv (L, n) fp32; n % 4 == 0, 16-B aligned inputs.
cudaError_t launch_kv_pack(const float *dk, const float *dv, int64_t L, int64_t n, void *out, cudaStream_t st);
cudaError_t launch_bucket(const void *top_idx, int idx64, const float *log_gates,
                          const PlanLayout &L, const PlanView &P, cudaStream_t st);
// Row copy into routing-plan order: dst[r] = src[perm[r]] (rows of row_bytes, a multiple of 16).
// rows_per_src: dst[r] = src[perm[r] / rows_per_src] (a plan over (token, k) rows).
cudaError_t launch_permute_rows(const void *src, int64_t N, int64_t row_bytes, const int *perm, void *dst,
                                cudaStream_t st, int rows_per_src = 1);
// delta[h][r] = <dO, O> of plan row r's token and head h (fp32), dO's row copied to
// do_rows[r] when do_rows is not null.
cudaError_t launch_row_delta(const void *dout, const void *out, int64_t N, int H, int hd, const int *perm,
                             void *do_rows, float *delta, cudaStream_t st, int rows_per_out = 1,
                             const float *row_w = nullptr);
// Read forward. q is token-ordered; q_rows (N x H*hd, same dtype) receives q in
// plan order and is what the tensor-core kernels (and the backward) read.
// iperm (block-split plans, rows_per_q > 1): q_rows is filled token-major.
cudaError_t launch_read_fwd(const void *q, const void *k, const void *v, int B, int S, int H,
                            int hd, int nb, int bs, int top, const PlanLayout &L,
                            const PlanView &P, void *out, float *lse, void *q_rows, cudaStream_t st,
                            const int *iperm = nullptr);
bool read_fwd_tc_supported(int hd, int bs, int top, const void *q, const void *k, const void *v, int H);
cudaError_t launch_read_fwd_tc(const void *q_rows, const void *k, const void *v, int hd, int H, int nb, int top,
                               const PlanLayout &L, const PlanView &P, void *out, float *lse,
                               cudaStream_t st);
bool read_bwd_tc_supported(int hd, int bs, int top, const void *q, const void *k, const void *v,
                           const void *dout, int H);
// do_src: dO in plan order (do_is_rows) or token order (rows gathered by the kernels).
cudaError_t launch_read_bwd_tc(const void *q_rows, const void *k, const void *v, const void *do_src,
                               bool do_is_rows, const float *lse, int hd, int H, int nb, int top, const PlanLayout &L,
                               const PlanView &P, void *dq, float *dk_acc, float *dv_acc, float *dlog_gates,
                               float *ws_delta, cudaStream_t st);
// Block-split read (split.cu): rows are (token, k) pairs of a top-1 plan built
// over N*top rows with PlanView::rows_per_q = top.
cudaError_t launch_split_prep(const void *top_idx, int idx64, const float *log_gates, int64_t N, int top,
                              float *lg_rows, cudaStream_t st);
// weights (N*top, H) fp32: a_k = exp(lse_k - logsumexp over the token's live rows);
// out (N, H*hd) = sum_k a_k out_rows[t*top + k] (bf16).
cudaError_t launch_split_combine(const void *out_rows, const float *lse_rows, const int *perm, const void *top_idx,
                                 int idx64, int64_t N, int top, int H, int hd, float *weights, void *out,
                                 cudaStream_t st);
// iperm[perm[r]] = r over the M = N*top rows of a block-split plan.
cudaError_t launch_split_iperm(const int *perm, int64_t M, int *iperm, cudaStream_t st);
// q_rows[iperm[t*top + k]] = q[t]: q in plan order, each token's row read once.
cudaError_t launch_split_permute_q(const void *q, const int *iperm, int64_t N, int top, int64_t row_bytes,
                                   void *q_rows, cudaStream_t st);
// The tensor-core backward's row copy for a block-split plan, token-major:
// do_rows[iperm[t*top+k]] = bf16(w[t*top+k][h] dO[t]), delta per row and head.
cudaError_t launch_split_row_delta(const void *dout, const void *out, const float *weights, const int *iperm,
                                   int64_t N, int top, int H, int hd, void *do_rows, float *delta, cudaStream_t st);
cudaError_t launch_split_gate_do(const void *dout, const float *weights, int64_t N, int top, int H, int hd, void *g,
                                 cudaStream_t st);
cudaError_t launch_split_dq_sum(const void *dq_rows, const void *top_idx, int idx64, int64_t N, int top, int H,
                                int hd, void *dq, float *dlog_gates, cudaStream_t st);
// Read backward. q_rows: as filled by launch_read_fwd. do_rows: N x H*hd scratch for
// dO in plan order, or null (the tensor-core kernels then gather dO rows).
// row_w (a block-split plan on the tensor-core path, with do_rows): dout is the
// token-order dO of the combined output and row r's dO is row_w[perm[r]][h] times
// it, formed while dO is copied into plan order (no separate weighted copy).
cudaError_t launch_read_bwd(const void *q, const void *q_rows, const void *k, const void *v, const void *out,
                            const void *dout, const float *lse, int B, int S, int H, int hd,
                            int nb, int bs, int top, const PlanLayout &L, const PlanView &P,
                            void *dq, float *dk_acc, float *dv_acc, float *dlog_gates,
                            float *ws_delta, void *do_rows, cudaStream_t st, const float *row_w = nullptr,
                            const int *iperm = nullptr);

// fp32 read (read_f32.cu) on a block-split plan (rows = (token, k) pairs, PlanView
// over N*top rows with rows_per_q = top). Forward: o_rows (M x H x hd) and lse_rows
// (M x H) scratch, out (N, H, hd) and lse (N, H) token order. Backward: delta (N x H)
// scratch; dq, dk_acc, dv_acc and dlog_gates are accumulated into (zero them first).
cudaError_t launch_read_f32_fwd(const float *q, const float *k, const float *v, int64_t N, int H, int hd, int nb,
                                int bs, int top, const PlanLayout &L, const PlanView &P, const void *idx, int idx64,
                                const int *iperm, float *o_rows, float *lse_rows, float *out, float *lse,
                                cudaStream_t st);
cudaError_t launch_read_f32_bwd(const float *q, const float *k, const float *v, const float *out, const float *dout,
                                const float *lse, int64_t N, int H, int hd, int bs, int top, const PlanLayout &L,
                                const PlanView &P, const void *idx, int idx64, float *delta, float *dq,
                                float *dk_acc, float *dv_acc, float *dlog_gates, cudaStream_t st);

// Decoder trunk (trunk.cu): rotary embedding of the fused q/k/v projection output
// (B*S, 3*H*hd) bf16 into (B, S, H, hd) bf16 q / k / v, and back; SwiGLU of the fused
// gate/up output (N, 2f) bf16, and back.
cudaError_t launch_rope_qkv_fwd(const void *qkv, const float *cosv, const float *sinv, int B, int S, int H, int hd,
                                void *q, void *k, void *v, cudaStream_t st);
cudaError_t launch_rope_qkv_bwd(const void *dq, const void *dk, const void *dv, const float *cosv, const float *sinv,
                                int B, int S, int H, int hd, void *dqkv, cudaStream_t st);
cudaError_t launch_swiglu_fwd(const void *gu, int64_t N, int f, void *h, cudaStream_t st);
cudaError_t launch_swiglu_bwd(const void *dh, const void *gu, int64_t N, int f, void *dgu, cudaStream_t st);
// Residual add + RMSNorm (ddt: 0 no delta, 1 bf16, 2 fp32 delta; dscale: optional
// device scalar multiplying delta); y16 bf16 always, y32 fp32 optional; rstd per token.
cudaError_t launch_add_rmsnorm_fwd(const float *x, const void *delta, int ddt, const float *dscale, const float *w,
                                   int64_t N, int d, float eps, float *x_out, void *y16, float *y32, float *rstd,
                                   cudaStream_t st);
cudaError_t launch_add_rmsnorm_bwd(const float *x_new, const float *rstd, const float *w, const void *delta, int ddt,
                                   const float *dscale_in, const void *dy16, const float *dy32, const float *dx_in,
                                   int64_t N, int d, float *dx, void *ddelta, float *dw, float *dscale,
                                   cudaStream_t st);
// LM-head cross-entropy over bf16 logits (R, V): per-row loss (0 on ignored rows)
// and log-sum-exp; backward dlogits = bf16((softmax - onehot) * (*grad)).
// AdamW over a table of fp32 tensors (one launch), with optional bf16 copies.
struct OptTensor {
    float *p;
    const float *g;
    float *m;
    float *v;
    uint16_t *p16;   // may be null
    int64_t n;
};
constexpr int kOptChunk = 65536;   // elements per CTA
constexpr int kOptThreads = 256;
cudaError_t launch_adamw_multi(const OptTensor *tensors, const int2 *chunks, int64_t nchunks, float lr, float b1,
                               float b2, float eps, float wd, float bc1, float bc2, cudaStream_t st);
cudaError_t launch_xent_fwd(const void *logits, const int64_t *labels, int64_t R, int V, int64_t ignore_index,
                            float *row_loss, float *lse, cudaStream_t st);
cudaError_t launch_xent_bwd(const void *logits, const int64_t *labels, const float *lse, const float *grad, int64_t R,
                            int V, int64_t ignore_index, void *dlogits, cudaStream_t st);

}  // namespace mom
