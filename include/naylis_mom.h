/*
 * naylis_mom.h — C ABI of the B200 (sm_100a) Mixture-of-Memory hot path.
 *
 * Every entry point takes plain device pointers, int64 sizes, dtype enums and
 * a CUDA stream passed as `void *` (a cudaStream_t; NULL = legacy default
 * stream). No call allocates device memory, synchronises the host or throws:
 * the caller owns every buffer (workspace sizes are queried first) and each
 * call returns an `int` status (mom_status). The library holds no device
 * memory across calls.
 *
 * The entry points replace the reference's Python-level hot path; each
 * declaration names the reference interface it stands in for.
 */
#ifndef NAYLIS_MOM_H
#define NAYLIS_MOM_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOM_API __attribute__((visibility("default")))
#else
#define MOM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    MOM_OK = 0,
    MOM_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, inconsistent geometry   */
    MOM_ERR_UNSUPPORTED = 2,      /* valid request outside what the kernels implement */
    MOM_ERR_ARCH = 3,             /* current device is not sm_100                     */
    MOM_ERR_WORKSPACE = 4,        /* workspace / plan buffer smaller than required    */
    MOM_ERR_LAUNCH = 5,           /* a kernel launch failed (message has the CUDA error) */
    MOM_ERR_DEVICE_TIMEOUT = 6,   /* a bounded device-side wait gave up               */
    MOM_ERR_DEVICE_INDEX = 7      /* a kernel saw a routing index outside [0, nb)     */
} mom_status;

typedef enum { MOM_F32 = 0, MOM_BF16 = 1, MOM_I32 = 2, MOM_I64 = 3 } mom_dtype;

typedef enum {
    MOM_SCAN_FP64 = 0, /* sequential fp64 accumulation per column (torch CPU cumsum)          */
    MOM_SCAN_FP32 = 1  /* sequential fp32 accumulation per column (torch CUDA outer-dim scan) */
} mom_scan_mode;

/* Library version (major*10000 + minor*100 + patch). */
MOM_API int mom_version(void);

/* Number of kernels this library has launched since it was loaded (telemetry). */
MOM_API uint64_t mom_kernel_launches(void);

/* Message of the last failing call on this host thread ("" if none). */
MOM_API const char *mom_last_error_string(void);

/* MOM_OK when `device` is an sm_100 GPU this build has code for.
 * Stands in for mom_kernels/__init__.py:37-53 (preflight) on the native side. */
MOM_API int mom_device_check(int device);

/* ------------------------------------------------------------------ prefix mean
 * h[b,t,:] = cumsum_{i<=t} x[b,i,:] / (t+1), rounded to out_dtype (F32|BF16).
 * Replaces mom_kernels/reference.py:32-36 (prefix_mean_reference) and
 * model.py:169-176 (MoMLayer._prefix_mean); bit-exact to torch.cumsum of the
 * chosen backend (scan_mode) followed by the fp32 division. */
MOM_API int mom_prefix_mean(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d, void *out,
                    int out_dtype, int scan_mode, void *stream);

/* ------------------------------------------------------------------ router
 * Fused causal router forward. Replaces model.py:178-220
 * (MoMLayer._prefix_mean, _router_logits and the softmax / topk / gate block
 * of MoMLayer.forward); the reference keeps it inline, outside the
 * mom_kernels door.
 *
 *   h      = cumsum_t(x) / (t+1)      (exact: scan_mode picks the backend semantics)
 *   z      = round_cd(round_cd(h) . w_down^T)         w_down (r, d)
 *   act    = round_cd(tanh(z))                        saved for the backward
 *   logits = float(round_cd(act . w_up^T))            w_up (nb, r)
 *   probs  = softmax(logits)
 *   top_idx, top_vals = topk(logits + noise, top)     value desc, ties -> lower index
 *   gates  = softmax(top_vals);  log_gates = log(max(gates, 1e-9))
 *
 * x: (B,S,d) of x_dtype (F32|BF16); w_down/w_up/act of compute_dtype (F32|BF16),
 * the dtype the router linears run in (BF16 under autocast). noise: (B,S,nb)
 * fp32 or NULL. top_idx of idx_dtype (I32|I64). log_gates and act may be NULL.
 */
MOM_API size_t mom_route_workspace_size(int64_t B, int64_t S, int64_t d, int64_t r, int64_t nb,
                                int compute_dtype);
MOM_API int mom_route_fwd(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d,
                  const void *w_down, const void *w_up, int compute_dtype,
                  int64_t r, int64_t nb, int64_t top, const float *noise, int scan_mode,
                  float *probs, void *top_idx, int idx_dtype, float *gates,
                  float *log_gates, void *act, void *workspace, size_t workspace_bytes,
                  void *stream);

/* Sequence-sharded router forward (long-context prefill split by sequence over
 * ranks; the reference has no such split). Each rank holds rows
 * [t_base, t_base + S) of every sequence; the prefix mean at global row t
 * divides by t + 1, so t_base + S < 2^24. The results equal mom_route_fwd over
 * the whole sequence bit for bit, given the scan state entering the shard:
 *
 * scan_mode FP64, carry double[2][B][d]: [0] the sum of the earlier rows,
 *   [1] 1.0 where the whole sequence's exactness certificate holds. Recipe:
 *   mom_route_shard_stats on each shard (stats double[3][B][d]: sum, an upper
 *   bound of sum |x|, smallest ulp exponent), all-gather them in rank order
 *   (W x 3 x B x d), mom_route_shard_carry. Certified columns are exact in any
 *   order, so all shards run at once. When *uncertified > 0 (tiny or huge
 *   dynamic range) those columns need the sequential sum: run the shards in
 *   rank order, each passing its carry_out (same layout) as the next carry_in.
 * scan_mode FP32 (the sequential fp32 scan): carry float[B][d], always passed
 *   shard to shard in rank order.
 * carry_in may be NULL only for t_base = 0 in FP64 mode with a whole
 * sequence; carry_out may be NULL. Other arguments as mom_route_fwd. */
MOM_API int mom_route_shard_stats(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d,
                                  double *stats, void *stream);
MOM_API int mom_route_shard_carry(const double *stats_all, int64_t world, int64_t rank, int64_t B,
                                  int64_t d, double *carry, int *uncertified, void *stream);
MOM_API int mom_route_fwd_shard(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d,
                                const void *w_down, const void *w_up, int compute_dtype, int64_t r,
                                int64_t nb, int64_t top, const float *noise, int scan_mode,
                                int64_t t_base, const void *carry_in, void *carry_out, float *probs,
                                void *top_idx, int idx_dtype, float *gates, float *log_gates,
                                void *act, void *workspace, size_t workspace_bytes, void *stream);

/* The MoM load-balancing aux loss of one layer and its router logs
 * (NaylisLlamaModel._collect_mom_aux_loss, model.py:476-517) from the router's
 * probs (N, nb) fp32 and top_idx (N, top): out[0] = nb * sum_e frac_e * mean_e
 * (frac_e = share of tokens that selected block e, mean_e = mean of probs[:, e]),
 * out[1] = router entropy -mean_t sum_e p log(max(p, 1e-9)), out[2] = share of
 * blocks no token selected, out[3 + e] = frac_e (the gradient of out[0] w.r.t.
 * probs[t, e] is nb * frac_e / N). Deterministic (a fixed summation order); nb <= 256;
 * out holds 3 + nb floats; the workspace is mom_router_aux_workspace_size bytes. */
MOM_API size_t mom_router_aux_workspace_size(int64_t N, int64_t nb);
MOM_API int mom_router_aux(const float *probs, const void *top_idx, int idx_dtype, int64_t N, int64_t nb,
                           int64_t top, void *workspace, size_t workspace_bytes, float *out, void *stream);

/* Router backward: autograd of the block above (model.py:186-220).
 * dlog_gates (B,S,top): gradient w.r.t. log_gates, or NULL; dgates: w.r.t. gates,
 * or NULL; dprobs (B,S,nb): w.r.t. probs (the aux load-balance loss), or NULL.
 * Outputs: dx (B,S,d) of dx_dtype (F32|BF16; accumulated into when
 * accumulate_dx != 0), dw_down (r,d) fp32, dw_up (nb,r) fp32.
 * The reverse scan runs in rank-r space: dx_t = w_down^T sum_{s>=t} dz_s/(s+1). */
MOM_API size_t mom_route_bwd_workspace_size(int64_t B, int64_t S, int64_t d, int64_t r, int64_t nb);
MOM_API int mom_route_bwd(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d,
                  const void *w_down, const void *w_up, int compute_dtype, int64_t r,
                  int64_t nb, int64_t top, const float *probs, const void *top_idx,
                  int idx_dtype, const float *gates, const void *act,
                  const float *dlog_gates, const float *dgates, const float *dprobs,
                  void *dx, int dx_dtype, int accumulate_dx, float *dw_down, float *dw_up,
                  void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------ bucketing
 * Routing permutation: groups the N = B*S tokens by the SET of blocks they
 * selected, into tiles of at most tile_m tokens that all read the same blocks.
 * The reference has no counterpart (its kernels read all L slots for every
 * token, mom_kernels/triton_gpu.py:98-133); it turns the per-token hard mask
 * into block skipping. The plan is an opaque device buffer of
 * mom_plan_size() bytes, consumed by mom_read_fwd / mom_read_bwd.
 * top_idx (N, top) of idx_dtype, log_gates (N, top) fp32. */
MOM_API size_t mom_plan_size(int64_t N, int64_t nb, int64_t top);
MOM_API int mom_bucket(const void *top_idx, int idx_dtype, const float *log_gates, int64_t N,
               int64_t nb, int64_t top, void *plan, size_t plan_bytes, void *stream);

/* ------------------------------------------------------------------ memory read
 * Gated memory read forward. Replaces mom_kernels/__init__.py:87-102
 * (mom_read) -> mom_kernels/triton_gpu.py:323-356 (_MomReadFunction.forward).
 * q (B,S,H,hd) and out of dtype (BF16); k, v: the shared bank projections
 * (L, H*hd), L = nb*bs; lse (H, B*S) fp32 in routing-plan row order, saved
 * for the backward. q_rows: a caller buffer of B*S*H*hd elements of dtype,
 * 16-byte aligned, which this call fills with q's rows in routing-plan row
 * order (where every tile of the read is contiguous); pass it unchanged to
 * mom_read_bwd, like lse. `plan` comes from mom_bucket on the same routing. */
MOM_API int mom_read_fwd(const void *q, const void *k, const void *v, int dtype, int64_t B,
                 int64_t S, int64_t H, int64_t hd, int64_t nb, int64_t bs, int64_t top,
                 const void *plan, void *out, float *lse, void *q_rows, void *stream);

/* Gated memory read backward. Replaces mom_kernels/triton_gpu.py:358-409
 * (_MomReadFunction.backward). Produces dq (B,S,H,hd) of dtype, dk_acc and
 * dv_acc (L, H*hd) fp32 (overwritten), dlog_gates (B*S, top) fp32 in the
 * caller's top order (gradient w.r.t. log(max(gate, 1e-9))). q_rows as filled
 * by mom_read_fwd. The workspace holds delta (H x B*S fp32) and dO in
 * routing-plan row order (B*S x H*hd of dtype). */
MOM_API size_t mom_read_bwd_workspace_size(int64_t B, int64_t S, int64_t H, int64_t hd);
MOM_API int mom_read_bwd(const void *q, const void *k, const void *v, const void *out,
                 const void *dout, const float *lse, int dtype, int64_t B, int64_t S,
                 int64_t H, int64_t hd, int64_t nb, int64_t bs, int64_t top,
                 const void *plan, const void *q_rows, void *dq, float *dk_acc, float *dv_acc,
                 float *dlog_gates, void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------ fp32 read
 * The same read for fp32 activations (q, k, v, out, dout all fp32), computed with
 * fp32 FMA throughout: the reference's fp32 read (mom_kernels/reference.py:14-61,
 * held to 1e-5 in tests/test_parity.py:138-188), reached through the same door
 * (mom_kernels/__init__.py:87-102) when the tensors are fp32. It runs on the
 * block-split plan: build it with mom_bucket_split first (any top <= 8, repeated
 * block ids summed as the reference's bias sums them). head_dim 16, 32, 64 or
 * 128 (the reference's powers of two); any block size. lse is (B*S, H) fp32 in token order (saved for the backward).
 * Workspace: mom_read_f32_workspace_size bytes, for either call. The backward
 * zeroes and then accumulates dq (B*S x H*hd), dk, dv (L x H*hd) and dlog_gates
 * (B*S x top), all fp32. */
MOM_API size_t mom_read_f32_workspace_size(int64_t B, int64_t S, int64_t H, int64_t head_dim, int64_t top);
MOM_API int mom_read_f32_fwd(const float *q, const float *k, const float *v, int64_t B, int64_t S, int64_t H,
                             int64_t head_dim, int64_t num_blocks, int64_t block_size, int64_t top,
                             const void *top_idx, int idx_dtype, const void *plan, float *out, float *lse,
                             void *workspace, size_t workspace_bytes, void *stream);
MOM_API int mom_read_f32_bwd(const float *q, const float *k, const float *v, const float *out,
                             const float *dout, const float *lse, int64_t B, int64_t S, int64_t H,
                             int64_t head_dim, int64_t num_blocks, int64_t block_size, int64_t top,
                             const void *top_idx, int idx_dtype, const void *plan, float *dq, float *dk,
                             float *dv, float *dlog_gates, void *workspace, size_t workspace_bytes,
                             void *stream);

/* ------------------------------------------------------------------ decoder trunk
 * bf16 kernels of the trunk around the MoM layer (the caller that BASELINE
 * config 3 trains), with the rounding points of the reference's trunk under bf16
 * autocast (transformers' Llama apply_rotary_pos_emb and LlamaMLP, wired by
 * model.py:280-348).
 * mom_rope_qkv_fwd: qkv (B*S, 3*H*hd) bf16, the fused q/k/v projection output
 * ([q | k | v], H heads of hd each); cos, sin (S, hd) fp32 -> q, k with the
 * rotary embedding (fp32 math, bf16 result) and v, each (B, S, H, hd) bf16
 * (attention takes them as (B, H, S, hd) views). mom_rope_qkv_bwd: the attention
 * gradients dq, dk, dv in that (B, S, H, hd) layout -> dqkv (B*S, 3*H*hd) bf16. Replace the reference's
 * q/k/v views, apply_rotary_pos_emb and their autograd. */
MOM_API int mom_rope_qkv_fwd(const void *qkv, const float *cos, const float *sin, int64_t B, int64_t S, int64_t H,
                             int64_t head_dim, void *q, void *k, void *v, void *stream);
MOM_API int mom_rope_qkv_bwd(const void *dq, const void *dk, const void *dv, const float *cos, const float *sin,
                             int64_t B, int64_t S, int64_t H, int64_t head_dim, void *dqkv, void *stream);
/* mom_swiglu_fwd: gu (N, 2f) bf16, the fused gate/up projection output ([g | u])
 * -> h = bf16(bf16(silu(g)) * u), (N, f). mom_swiglu_bwd: dh (N, f), gu ->
 * dgu (N, 2f) = [dg | du], bf16. Replace LlamaMLP's act_fn(gate) * up and its
 * autograd. f even, buffers 4-byte aligned. */
MOM_API int mom_swiglu_fwd(const void *gu, int64_t N, int64_t f, void *h, void *stream);
MOM_API int mom_swiglu_bwd(const void *dh, const void *gu, int64_t N, int64_t f, void *dgu, void *stream);

/* mom_add_rmsnorm_fwd: the residual add before a Llama RMSNorm fused with it:
 * x_out = x + s * delta (s = *delta_scale when given, else 1; delta bf16 or fp32,
 * or NULL for no add), then y = w * (x_out * rsqrt(mean(x_out^2) + eps)) as bf16
 * (y_bf16, the next projection's input) and, when y_f32 is not NULL, fp32 (the
 * MoM router's input); rstd (N) per token for the backward. x, x_out, w fp32;
 * rows of d = 128, 256, 512, 1024 or 2048, 16-byte (fp32) / 8-byte (bf16) aligned. Replaces the reference's
 * `residual + hidden_states` and LlamaRMSNorm (model.py:319-345) and, with
 * delta_scale = mom_scale, `mom_scale * o_proj(out)` (model.py:239).
 * mom_add_rmsnorm_bwd: from dy (bf16 and/or fp32) and dx_in (the residual
 * stream's own gradient, may be NULL): dx (fp32), ddelta = s * dx in delta's
 * dtype, dw (d, zeroed then accumulated) and, when ddelta_scale is given,
 * d s = sum(dx * delta). */
MOM_API int mom_add_rmsnorm_fwd(const float *x, const void *delta, int delta_dtype, const float *delta_scale,
                                const float *w, int64_t N, int64_t d, double eps, float *x_out, void *y_bf16,
                                float *y_f32, float *rstd, void *stream);
MOM_API int mom_add_rmsnorm_bwd(const float *x_new, const float *rstd, const float *w, const void *delta,
                                int delta_dtype, const float *delta_scale, const void *dy_bf16, const float *dy_f32,
                                const float *dx_in, int64_t N, int64_t d, float *dx, void *ddelta, float *dw,
                                float *ddelta_scale, void *stream);

/* AdamW over many fp32 parameter tensors in one launch (the reference's
 * optimizer, torch.optim.AdamW with decoupled weight decay, as
 * pretrain.py's HF Trainer runs it), writing each updated parameter's bf16 copy
 * in the same pass when the table entry asks for one.
 * tensors: ntensors entries of {float *p; const float *g; float *m; float *v;
 * uint16_t *p16 (bf16 copy of p, or NULL); int64_t n} (48 bytes each, device
 * memory); chunks: nchunks {int32 tensor, int32 chunk} pairs covering every
 * tensor in chunks of 65,536 elements. step >= 1 is the step count after this
 * update (bias corrections 1 - beta^step). */
MOM_API int mom_adamw_step(const void *tensors, int64_t ntensors, const void *chunks, int64_t nchunks, double lr,
                           double beta1, double beta2, double eps, double weight_decay, int64_t step, void *stream);

/* mom_xent_fwd: the causal-LM loss of model.py:539-551 (NaylisLlamaForCausalLM:
 * cross_entropy(logits.float(), labels, reduction="sum") over the shifted rows,
 * then divided by the count of labels != ignore_index) without materialising the
 * fp32 logits: logits (R, V) bf16 as the LM head's autocast GEMM writes them,
 * labels (R) int64; row_loss (R) fp32 = logsumexp(row) - row[label] (0 where
 * label == ignore_index, NaN where the label is outside [0, V)), lse (R) fp32
 * for the backward. The caller sums row_loss and divides.
 * mom_xent_bwd: dlogits (R, V) bf16 = ((softmax(row) - onehot(label)) * *grad)
 * rounded to bf16, 0 on ignored rows; grad is a device scalar, the gradient of
 * the sum of row_loss. */
MOM_API int mom_xent_fwd(const void *logits, const int64_t *labels, int64_t R, int64_t V, int64_t ignore_index,
                         float *row_loss, float *lse, void *stream);
MOM_API int mom_xent_bwd(const void *logits, const int64_t *labels, const float *lse, const float *grad, int64_t R,
                         int64_t V, int64_t ignore_index, void *dlogits, void *stream);

/* mom_read_bwd without a workspace argument: for callers that cannot allocate
 * device memory (a plugin whose host framework's caching allocator owns the
 * device, or an FFI caller with no device allocator). It has no counterpart
 * in the reference. The delta scratch is a fixed 4 MiB device array
 * inside the library (mom_read_bwd_noalloc_max_bytes()), so B*S*H may be at
 * most 1,048,576; larger calls return MOM_ERR_WORKSPACE. It calls no
 * cudaMalloc/cudaFree. Its first call on a device looks the array's address
 * up (make that call before any stream capture). All calls share the array:
 * calls that overlap on the GPU race. Arguments and results as mom_read_bwd;
 * dO is read in token order (its rows gathered by the kernels), so nothing
 * beyond delta needs scratch. */
MOM_API size_t mom_read_bwd_noalloc_max_bytes(void);
MOM_API int mom_read_bwd_noalloc(const void *q, const void *k, const void *v, const void *out,
                                 const void *dout, const float *lse, int dtype, int64_t B,
                                 int64_t S, int64_t H, int64_t head_dim, int64_t num_blocks,
                                 int64_t block_size, int64_t top, const void *plan,
                                 const void *q_rows, void *dq, float *dk_acc, float *dv_acc,
                                 float *dlog_gates, void *stream);

/* ------------------------------------------------------------------ block-split read
 * The same read (mom_kernels/__init__.py:87-102 -> triton_gpu.py:323-409) for
 * top-k routing whose block sets are more than the set bucketing holds
 * (mom_plan_size() returns 0 there: top-4 of 32 blocks has 35,960 sets). Each
 * (token, k) pair becomes a row of a top-1 plan that reads its one block; a
 * token's rows are combined by their log-sum-exp into the softmax over the
 * union of its blocks, the reference's result. A block chosen twice by a token
 * is read once with the sum of its log-gates, as in the reference's bias.
 *
 * Plan: mom_plan_split_size() bytes, filled by mom_bucket_split from top_idx
 * (N, top) and log_gates (N, top). mom_plan_check(plan, N*top, nb, 1) reads its
 * error word. Forward: out (B,S,H,hd) of dtype; lse_rows (H, B*S*top) fp32 and
 * weights (B*S*top, H) fp32 (the rows' share of each token's softmax), both
 * saved for the backward; q_rows: B*S*top*H*hd elements of dtype, filled here;
 * workspace: the rows' outputs. Backward: as mom_read_bwd, dlog_gates (B*S, top)
 * in the caller's top order. No counterpart entry in the reference. */
MOM_API size_t mom_plan_split_size(int64_t N, int64_t nb, int64_t top);
MOM_API int mom_bucket_split(const void *top_idx, int idx_dtype, const float *log_gates, int64_t N,
                             int64_t nb, int64_t top, void *plan, size_t plan_bytes, void *stream);
MOM_API size_t mom_read_split_fwd_workspace_size(int64_t B, int64_t S, int64_t H, int64_t hd,
                                                 int64_t top);
MOM_API int mom_read_split_fwd(const void *q, const void *k, const void *v, int dtype, int64_t B,
                               int64_t S, int64_t H, int64_t hd, int64_t nb, int64_t bs, int64_t top,
                               const void *top_idx, int idx_dtype, const void *plan, void *out,
                               float *lse_rows, float *weights, void *q_rows, void *workspace,
                               size_t workspace_bytes, void *stream);
MOM_API size_t mom_read_split_bwd_workspace_size(int64_t B, int64_t S, int64_t H, int64_t hd,
                                                 int64_t top);
MOM_API int mom_read_split_bwd(const void *q, const void *k, const void *v, const void *out,
                               const void *dout, const float *lse_rows, const float *weights,
                               int dtype, int64_t B, int64_t S, int64_t H, int64_t hd, int64_t nb,
                               int64_t bs, int64_t top, const void *top_idx, int idx_dtype,
                               const void *plan, const void *q_rows, void *dq, float *dk_acc,
                               float *dv_acc, float *dlog_gates, void *workspace,
                               size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------ output scale
 * ReZero output scale of the layer, fused: y = scale[0] * o with y in fp32
 * (model.py:239, `self.mom_scale * out`: a (1,) fp32 parameter times the bf16
 * o_proj output promotes to fp32). `scale` is a device pointer to one float. */
MOM_API int mom_scale_fwd(const void *o, int o_dtype, int64_t n, const float *scale, float *y,
                          void *stream);
/* Its backward in one pass: d_o = scale[0] * g in o's dtype, d_scale[0] = sum(g * o). */
MOM_API int mom_scale_bwd(const void *g, int g_dtype, const void *o, int o_dtype, int64_t n,
                          const float *scale, void *d_o, float *d_scale, void *stream);

/* Router Gumbel noise from uniform draws u (fp32, n values; torch.rand): out =
 * noise_scale * -log(-log(u + 1e-9) + 1e-9), bit for bit the reference's
 * expression (model.py:209-213) evaluated by torch's fp32 kernels. out may be u.
 * Replaces the seven elementwise torch ops of that expression. */
MOM_API int mom_gumbel(const float *u, int64_t n, float noise_scale, float *out, void *stream);

/* The read backward's dK, dV (L, n) fp32, as mom_read_bwd leaves them, cast to bf16
 * (round to nearest even) side by side into out (L, 2n) = [dK | dV]: the gradient of
 * the bank's k and v projections (model.py:253-256, `k_proj(slots)`, `v_proj(slots)`
 * under autocast, whose dK / dV the autograd casts to bf16) laid out for one GEMM over
 * both. n % 4 == 0, dk / dv 16-byte and out 8-byte aligned. */
MOM_API int mom_kv_pack_bf16(const float *dk, const float *dv, int64_t L, int64_t n, void *out, void *stream);

/* Reads (and clears) the device error word of a plan: MOM_OK, or
 * MOM_ERR_DEVICE_INDEX when mom_bucket saw an index outside [0, nb).
 * Synchronises `stream`. */
MOM_API int mom_plan_check(const void *plan, int64_t N, int64_t nb, int64_t top, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NAYLIS_MOM_H */
