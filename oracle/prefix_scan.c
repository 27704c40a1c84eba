/*
 * ORACLE — test infrastructure only. Nothing in the product path links or
 * calls this file; tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline use it as the checker.
 *
 * CPU restatement of the causal prefix mean of the Naylis MoM router:
 *
 *     h[b, t, c] = cumsum_{i <= t}(x[b, i, c]) / (t + 1)       (fp32 result)
 *
 * Reference: model.py:169-176 (MoMLayer._prefix_mean) and
 * mom_kernels/reference.py:32-36 (prefix_mean_reference):
 *     cs = torch.cumsum(x.float(), dim=1)
 *     h  = cs / torch.arange(1, S + 1, dtype=float32)
 *
 * torch.cumsum's accumulation is backend-specific, so two modes are kept:
 *   mode 0 ("fp64"): the CPU backend. Each column is accumulated
 *     sequentially in double and every prefix is rounded to float
 *     (verified bit-identical to torch CPU cumsum for fp32 input).
 *   mode 1 ("fp32"): the CUDA backend for a non-innermost scan dimension,
 *     one thread per column with a float accumulator walking t in order
 *     (ATen/native/cuda/ScanUtils.cuh, tensor_kernel_scan_outer_dim).
 * The division is a single IEEE float division by (float)(t + 1).
 *
 * Compile with -ffp-contract=off: no fused multiply-add may appear here.
 */
#include <stdint.h>
#include <stddef.h>

/* x: (B, S, d) float, row-major. h: (B, S, d) float output. */
int oracle_prefix_mean_f32(const float *x, float *h, int64_t B, int64_t S,
                           int64_t d, int mode)
{
    if (!x || !h || B < 0 || S < 0 || d < 0 || (mode != 0 && mode != 1))
        return 1;
    for (int64_t b = 0; b < B; ++b) {
        const float *xb = x + b * S * d;
        float *hb = h + b * S * d;
        for (int64_t c = 0; c < d; ++c) {
            double acc64 = 0.0;
            float acc32 = 0.0f;
            for (int64_t t = 0; t < S; ++t) {
                float cs;
                if (mode == 0) {
                    acc64 += (double)xb[t * d + c];
                    cs = (float)acc64;
                } else {
                    acc32 += xb[t * d + c];
                    cs = acc32;
                }
                hb[t * d + c] = cs / (float)(t + 1);
            }
        }
    }
    return 0;
}

/*
 * Reverse-time companion used by the router backward oracle:
 *     u[b, t, j] = sum_{s >= t} g[b, s, j] / (s + 1)
 * accumulated in double from t = S-1 down to 0, rounded to float.
 * This is the adjoint of the prefix mean (d h_s / d x_t = 1/(s+1) for s >= t).
 */
int oracle_suffix_scaled_sum_f32(const float *g, float *u, int64_t B,
                                 int64_t S, int64_t n)
{
    if (!g || !u || B < 0 || S < 0 || n < 0)
        return 1;
    for (int64_t b = 0; b < B; ++b) {
        const float *gb = g + b * S * n;
        float *ub = u + b * S * n;
        for (int64_t j = 0; j < n; ++j) {
            double acc = 0.0;
            for (int64_t t = S - 1; t >= 0; --t) {
                acc += (double)gb[t * n + j] / (double)(t + 1);
                ub[t * n + j] = (float)acc;
            }
        }
    }
    return 0;
}
