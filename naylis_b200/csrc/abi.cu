// extern "C" entry points of libnaylis_mom.so (declared in include/naylis_mom.h).
//
// This layer validates every argument, turns CUDA errors into status codes
// with a thread-local message, and forwards to the launchers. It allocates
// nothing and never synchronises the host, except mom_plan_check, whose job
// is to read the plan's device error word.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launch.h"

namespace mom {
static std::atomic<uint64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }
uint64_t launches() { return g_launches.load(std::memory_order_relaxed); }
}  // namespace mom

namespace {

thread_local char g_err[512] = {0};

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char *where) {
    return fail(MOM_ERR_LAUNCH, "%s: %s (%s)", where, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool is_float_dtype(int dt) { return dt == MOM_F32 || dt == MOM_BF16; }
bool is_idx_dtype(int dt) { return dt == MOM_I32 || dt == MOM_I64; }
size_t dt_size(int dt) { return (dt == MOM_BF16) ? 2 : (dt == MOM_I64 ? 8 : 4); }
size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// sm_100 check of the current device, cached per device.
int check_current_device() {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    static std::mutex mu;
    static int cache[64];
    static bool init = false;
    std::lock_guard<std::mutex> lk(mu);
    if (!init) {
        for (int &c : cache) c = -1;
        init = true;
    }
    if (dev >= 0 && dev < 64 && cache[dev] >= 0)
        return cache[dev] ? MOM_OK : fail(MOM_ERR_ARCH, "device %d is not sm_100", dev);
    int major = 0, minor = 0;
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
        return cuda_fail(e, "cudaDeviceGetAttribute");
    if ((e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
        return cuda_fail(e, "cudaDeviceGetAttribute");
    const bool ok = major == 10 && minor == 0;
    if (dev >= 0 && dev < 64) cache[dev] = ok ? 1 : 0;
    return ok ? MOM_OK
              : fail(MOM_ERR_ARCH, "device %d is sm_%d%d; this library is built for sm_100a only",
                     dev, major, minor);
}

#define MOM_REQUIRE(cond, ...)                                  \
    do {                                                        \
        if (!(cond)) return fail(MOM_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)

int check_router_geometry(int64_t B, int64_t S, int64_t d, int64_t r, int64_t nb, int64_t top) {
    MOM_REQUIRE(B >= 0 && S >= 0, "B and S must be >= 0 (got %lld, %lld)", (long long)B, (long long)S);
    MOM_REQUIRE(d > 0 && d % 8 == 0, "d_model must be a positive multiple of 8 (got %lld)", (long long)d);
    MOM_REQUIRE(r > 0 && r <= 128, "router_rank must be in [1, 128] (got %lld)", (long long)r);
    MOM_REQUIRE(nb > 0 && nb <= 64, "num_blocks must be in [1, 64] (got %lld)", (long long)nb);
    MOM_REQUIRE(top > 0 && top <= 8 && top <= nb, "top_blocks must be in [1, min(8, num_blocks)] (got %lld)",
                (long long)top);
    MOM_REQUIRE(B * S < (int64_t(1) << 31), "B*S too large");
    MOM_REQUIRE(S < (int64_t(1) << 24), "sequence length too large for the fp32 divisor");
    return MOM_OK;
}

}  // namespace

extern "C" {

int mom_version(void) { return 100; }

uint64_t mom_kernel_launches(void) { return mom::launches(); }

const char *mom_last_error_string(void) { return g_err; }

int mom_device_check(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(MOM_ERR_INVALID_ARGUMENT, "no CUDA device %d", device);
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0)
        return fail(MOM_ERR_ARCH, "device %d is sm_%d%d; this library is built for sm_100a only",
                    device, major, minor);
    return MOM_OK;
}

// ------------------------------------------------------------------ prefix mean
int mom_prefix_mean(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d, void *out,
                    int out_dtype, int scan_mode, void *stream) {
    MOM_REQUIRE(B >= 0 && S >= 0 && S < (int64_t(1) << 24), "bad B, S");
    MOM_REQUIRE(d > 0 && d % 8 == 0, "d must be a positive multiple of 8 (got %lld)", (long long)d);
    MOM_REQUIRE(is_float_dtype(x_dtype) && is_float_dtype(out_dtype), "dtypes must be F32 or BF16");
    MOM_REQUIRE(scan_mode == MOM_SCAN_FP64 || scan_mode == MOM_SCAN_FP32, "unknown scan mode %d", scan_mode);
    if (B * S == 0) return MOM_OK;
    MOM_REQUIRE(x && out, "null pointer argument");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_route_scan(x, x_dtype, out, out_dtype, (int)B, (int)S, (int)d, scan_mode,
                                           static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "prefix_mean");
}

// ------------------------------------------------------------------ router
size_t mom_route_workspace_size(int64_t B, int64_t S, int64_t d, int64_t r, int64_t nb,
                                int compute_dtype) {
    (void)r;
    (void)nb;
    if (B < 0 || S < 0 || d < 0 || !is_float_dtype(compute_dtype)) return 0;
    return align256(static_cast<size_t>(B) * S * d * dt_size(compute_dtype));
}

namespace {
int route_fwd_impl(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d, const void *w_down,
                   const void *w_up, int compute_dtype, int64_t r, int64_t nb, int64_t top, const float *noise,
                   int scan_mode, float *probs, void *top_idx, int idx_dtype, float *gates, float *log_gates,
                   void *act, void *workspace, size_t workspace_bytes, const mom::ScanShard &sh, void *stream) {
    int rc = check_router_geometry(B, S, d, r, nb, top);
    if (rc) return rc;
    MOM_REQUIRE(is_float_dtype(x_dtype), "x dtype must be F32 or BF16");
    MOM_REQUIRE(is_float_dtype(compute_dtype), "compute dtype must be F32 or BF16");
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    MOM_REQUIRE(scan_mode == MOM_SCAN_FP64 || scan_mode == MOM_SCAN_FP32, "unknown scan mode %d", scan_mode);
    MOM_REQUIRE(sh.t_base >= 0 && sh.t_base + S < (int64_t(1) << 24),
                "shard offset %lld + length %lld: positions must stay below 2^24 (fp32 divisor)",
                (long long)sh.t_base, (long long)S);
    const int64_t N = B * S;
    if (N == 0) return MOM_OK;
    MOM_REQUIRE(x && w_down && w_up && probs && top_idx && gates, "null pointer argument");
    const size_t need = mom_route_workspace_size(B, S, d, r, nb, compute_dtype);
    if (workspace_bytes < need || (need && !workspace))
        return fail(MOM_ERR_WORKSPACE, "route workspace %zu < %zu bytes", workspace_bytes, need);
    if ((rc = check_current_device())) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = mom::launch_route_scan(x, x_dtype, workspace, compute_dtype, (int)B, (int)S, (int)d,
                                           scan_mode, st, sh);
    if (e != cudaSuccess) return cuda_fail(e, "route_scan");
    e = mom::launch_route_head(workspace, w_down, w_up, compute_dtype, N, (int)d, (int)r, (int)nb,
                               (int)top, noise, probs, top_idx, idx_dtype == MOM_I64, gates,
                               log_gates, act, st);
    if (e != cudaSuccess) return cuda_fail(e, "route_head");
    return MOM_OK;
}
}  // namespace

int mom_route_fwd(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d, const void *w_down,
                  const void *w_up, int compute_dtype, int64_t r, int64_t nb, int64_t top,
                  const float *noise, int scan_mode, float *probs, void *top_idx, int idx_dtype,
                  float *gates, float *log_gates, void *act, void *workspace,
                  size_t workspace_bytes, void *stream) {
    return route_fwd_impl(x, x_dtype, B, S, d, w_down, w_up, compute_dtype, r, nb, top, noise, scan_mode, probs,
                          top_idx, idx_dtype, gates, log_gates, act, workspace, workspace_bytes, mom::ScanShard(),
                          stream);
}

// ------------------------------------------------------------------ sequence shards
int mom_route_shard_stats(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d, double *stats,
                          void *stream) {
    MOM_REQUIRE(B >= 0 && S >= 0 && B * S < (int64_t(1) << 31), "bad B, S");
    MOM_REQUIRE(d > 0 && d % 8 == 0, "d_model must be a positive multiple of 8 (got %lld)", (long long)d);
    MOM_REQUIRE(is_float_dtype(x_dtype), "x dtype must be F32 or BF16");
    MOM_REQUIRE(stats && (S == 0 || x), "null pointer argument");
    int rc = check_current_device();
    if (rc) return rc;
    if (B == 0) return MOM_OK;
    // an empty shard (S = 0) reads nothing and reports sum 0, bound 0, no element
    cudaError_t e = mom::launch_route_shard_stats(x, x_dtype, (int)B, (int)S, (int)d, stats,
                                                  static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "route_shard_stats");
}

int mom_route_shard_carry(const double *stats_all, int64_t world, int64_t rank, int64_t B, int64_t d,
                          double *carry, int *uncertified, void *stream) {
    MOM_REQUIRE(world > 0 && world <= 65536 && rank >= 0 && rank < world, "bad (world, rank)");
    MOM_REQUIRE(B >= 0 && d > 0 && B * d < (int64_t(1) << 31), "bad B, d");
    MOM_REQUIRE(stats_all && carry && uncertified, "null pointer argument");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_route_shard_carry(stats_all, (int)world, (int)rank, (int)B, (int)d, carry,
                                                  uncertified, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "route_shard_carry");
}

int mom_route_fwd_shard(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d, const void *w_down,
                        const void *w_up, int compute_dtype, int64_t r, int64_t nb, int64_t top,
                        const float *noise, int scan_mode, int64_t t_base, const void *carry_in, void *carry_out,
                        float *probs, void *top_idx, int idx_dtype, float *gates, float *log_gates, void *act,
                        void *workspace, size_t workspace_bytes, void *stream) {
    MOM_REQUIRE(carry_in || t_base == 0, "a shard that does not start at row 0 needs carry_in");
    mom::ScanShard sh;
    sh.t_base = t_base;
    sh.carry_in = carry_in;
    sh.carry_out = carry_out;
    if (carry_out && B * S == 0 && B > 0 && d > 0) {   // nothing to walk: the state passes through
        MOM_REQUIRE(carry_in, "carry_out of an empty first shard: pass a zero carry_in");
        const size_t bytes = (scan_mode == MOM_SCAN_FP64 ? 2 * sizeof(double) : sizeof(float)) *
                             static_cast<size_t>(B) * d;
        cudaError_t e = cudaMemcpyAsync(carry_out, carry_in, bytes, cudaMemcpyDeviceToDevice,
                                        static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_fail(e, "route_fwd_shard");
    }
    return route_fwd_impl(x, x_dtype, B, S, d, w_down, w_up, compute_dtype, r, nb, top, noise, scan_mode, probs,
                          top_idx, idx_dtype, gates, log_gates, act, workspace, workspace_bytes, sh, stream);
}

size_t mom_route_bwd_workspace_size(int64_t B, int64_t S, int64_t d, int64_t r, int64_t nb) {
    (void)d;
    if (B < 0 || S < 0 || r < 0 || nb < 0) return 0;
    const size_t N = static_cast<size_t>(B) * S;
    return align256(N * nb * 4) + 2 * align256(N * r * 4);
}

size_t mom_router_aux_workspace_size(int64_t N, int64_t nb) {
    if (N < 1 || nb < 1 || nb > 256) return 0;
    return mom::router_aux_workspace_size(N, (int)nb);
}

int mom_router_aux(const float *probs, const void *top_idx, int idx_dtype, int64_t N, int64_t nb, int64_t top,
                   void *workspace, size_t workspace_bytes, float *out, void *stream) {
    MOM_REQUIRE(N > 0 && nb >= 1 && nb <= 256 && top >= 1 && top <= nb, "bad router geometry");
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    MOM_REQUIRE(probs && top_idx && out && workspace, "null pointer argument");
    MOM_REQUIRE(workspace_bytes >= mom::router_aux_workspace_size(N, (int)nb), "workspace too small");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_router_aux(probs, top_idx, idx_dtype == MOM_I64, N, (int)nb, (int)top,
                                           static_cast<float *>(workspace), out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "router_aux");
}

int mom_route_bwd(const void *x, int x_dtype, int64_t B, int64_t S, int64_t d, const void *w_down,
                  const void *w_up, int compute_dtype, int64_t r, int64_t nb, int64_t top,
                  const float *probs, const void *top_idx, int idx_dtype, const float *gates,
                  const void *act, const float *dlog_gates, const float *dgates,
                  const float *dprobs, void *dx, int dx_dtype, int accumulate_dx, float *dw_down,
                  float *dw_up, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_router_geometry(B, S, d, r, nb, top);
    if (rc) return rc;
    MOM_REQUIRE(is_float_dtype(x_dtype) && is_float_dtype(compute_dtype) && is_float_dtype(dx_dtype),
                "x / compute / dx dtypes must be F32 or BF16");
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    MOM_REQUIRE(x && w_down && w_up && probs && top_idx && gates && act && dx && dw_down && dw_up,
                "null pointer argument");
    const size_t need = mom_route_bwd_workspace_size(B, S, d, r, nb);
    if (workspace_bytes < need || !workspace)
        return fail(MOM_ERR_WORKSPACE, "route bwd workspace %zu < %zu bytes", workspace_bytes, need);
    if ((rc = check_current_device())) return rc;
    const size_t N = static_cast<size_t>(B) * S;
    char *ws = static_cast<char *>(workspace);
    float *dlogits = reinterpret_cast<float *>(ws);
    float *dz = reinterpret_cast<float *>(ws + align256(N * nb * 4));
    float *u = reinterpret_cast<float *>(ws + align256(N * nb * 4) + align256(N * r * 4));
    cudaError_t e = mom::launch_route_bwd(
        x, x_dtype, (int)B, (int)S, (int)d, w_down, w_up, compute_dtype, (int)r, (int)nb, (int)top,
        probs, top_idx, idx_dtype == MOM_I64, gates, act, dlog_gates, dgates, dprobs, dx, dx_dtype,
        accumulate_dx, dw_down, dw_up, dlogits, dz, u, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "route_bwd");
    return MOM_OK;
}

// ------------------------------------------------------------------ bucketing
size_t mom_plan_size(int64_t N, int64_t nb, int64_t top) {
    if (N < 0 || nb <= 0 || nb > 64 || top <= 0 || top > 8 || top > nb) return 0;
    if (mom::num_route_keys(nb, top) > mom::kMaxKeys) return 0;
    return mom::plan_layout(N, nb, top).total;
}

int mom_bucket(const void *top_idx, int idx_dtype, const float *log_gates, int64_t N, int64_t nb,
               int64_t top, void *plan, size_t plan_bytes, void *stream) {
    MOM_REQUIRE(N >= 0 && N < (int64_t(1) << 31), "token count out of range");
    MOM_REQUIRE(nb > 0 && nb <= 64 && top > 0 && top <= 8 && top <= nb, "bad (num_blocks, top)");
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    const int64_t keys = mom::num_route_keys(nb, top);
    if (keys > mom::kMaxKeys)
        return fail(MOM_ERR_UNSUPPORTED,
                    "%lld routing sets for top-%lld of %lld blocks exceed the %d the set bucketing supports",
                    (long long)keys, (long long)top, (long long)nb, mom::kMaxKeys);
    const mom::PlanLayout L = mom::plan_layout(N, nb, top);
    MOM_REQUIRE(plan, "null plan");
    if (plan_bytes < L.total) return fail(MOM_ERR_WORKSPACE, "plan %zu < %zu bytes", plan_bytes, L.total);
    MOM_REQUIRE(N == 0 || (top_idx && log_gates), "null routing tensors");
    int rc = check_current_device();
    if (rc) return rc;
    const mom::PlanView P = mom::plan_view(plan, L);
    cudaError_t e = mom::launch_bucket(top_idx, idx_dtype == MOM_I64, log_gates, L, P,
                                       static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "bucket");
    return MOM_OK;
}

// ------------------------------------------------------------------ output scale
int mom_scale_fwd(const void *o, int o_dtype, int64_t n, const float *scale, float *y, void *stream) {
    MOM_REQUIRE(n >= 0, "n must be >= 0");
    MOM_REQUIRE(is_float_dtype(o_dtype), "o dtype must be F32 or BF16");
    if (n == 0) return MOM_OK;
    MOM_REQUIRE(o && scale && y, "null pointer argument");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_scale_fwd(o, o_dtype, scale, n, y, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "scale_fwd");
}

int mom_scale_bwd(const void *g, int g_dtype, const void *o, int o_dtype, int64_t n, const float *scale,
                  void *d_o, float *d_scale, void *stream) {
    MOM_REQUIRE(n >= 0, "n must be >= 0");
    MOM_REQUIRE(is_float_dtype(o_dtype) && is_float_dtype(g_dtype), "dtypes must be F32 or BF16");
    MOM_REQUIRE(scale && d_scale && (n == 0 || (g && o && d_o)), "null pointer argument");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_scale_bwd(g, g_dtype, o, o_dtype, scale, n, d_o, d_scale,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "scale_bwd");
}

int mom_gumbel(const float *u, int64_t n, float noise_scale, float *out, void *stream) {
    MOM_REQUIRE(n >= 0, "n must be >= 0");
    if (n == 0) return MOM_OK;
    MOM_REQUIRE(u && out, "null pointer argument");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_gumbel(u, n, noise_scale, out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "gumbel");
}

int mom_kv_pack_bf16(const float *dk, const float *dv, int64_t L, int64_t n, void *out, void *stream) {
    MOM_REQUIRE(L >= 0 && n >= 0, "L and n must be >= 0");
    if (L == 0 || n == 0) return MOM_OK;
    MOM_REQUIRE(dk && dv && out, "null pointer argument");
    MOM_REQUIRE(n % 4 == 0, "n must be a multiple of 4");
    MOM_REQUIRE(((reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 7) == 0,
                "dk, dv must be 16-byte and out 8-byte aligned");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_kv_pack(dk, dv, L, n, out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "kv_pack");
}

int mom_plan_check(const void *plan, int64_t N, int64_t nb, int64_t top, void *stream) {
    MOM_REQUIRE(plan, "null plan");
    const mom::PlanLayout L = mom::plan_layout(N, nb, top);
    const mom::PlanView P = mom::plan_view(const_cast<void *>(plan), L);
    int err = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&err, P.err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "plan_check");
    if (err) {
        cudaMemsetAsync(P.err, 0, sizeof(int), st);
        if (err & 2)
            return fail(MOM_ERR_DEVICE_TIMEOUT, "a bounded device-side wait of a read kernel gave up");
        return fail(MOM_ERR_DEVICE_INDEX, "top_idx holds a block index outside [0, %lld)", (long long)nb);
    }
    return MOM_OK;
}

// ------------------------------------------------------------------ read
static int check_read_geometry(int dtype, int64_t B, int64_t S, int64_t H, int64_t hd, int64_t nb,
                               int64_t bs, int64_t top) {
    MOM_REQUIRE(dtype == MOM_BF16, "the read kernels take bf16 activations (got dtype %d)", dtype);
    MOM_REQUIRE(B >= 0 && S >= 0 && B * S < (int64_t(1) << 31), "bad B, S");
    MOM_REQUIRE(H > 0 && H <= 1024, "bad n_heads %lld", (long long)H);
    if (hd != 64 && hd != 128)
        return fail(MOM_ERR_UNSUPPORTED, "head_dim %lld: the sm_100a read kernels take 64 or 128",
                    (long long)hd);
    MOM_REQUIRE(nb > 0 && nb <= 64 && top > 0 && top <= 8 && top <= nb, "bad (num_blocks, top)");
    MOM_REQUIRE(bs > 0 && nb * bs < (int64_t(1) << 24), "bad block_size %lld", (long long)bs);
    if (mom::num_route_keys(nb, top) > mom::kMaxKeys)
        return fail(MOM_ERR_UNSUPPORTED, "top-%lld of %lld blocks: too many routing sets", (long long)top,
                    (long long)nb);
    return MOM_OK;
}

int mom_read_fwd(const void *q, const void *k, const void *v, int dtype, int64_t B, int64_t S,
                 int64_t H, int64_t hd, int64_t nb, int64_t bs, int64_t top, const void *plan,
                 void *out, float *lse, void *q_rows, void *stream) {
    int rc = check_read_geometry(dtype, B, S, H, hd, nb, bs, top);
    if (rc) return rc;
    if (B * S == 0) return MOM_OK;
    MOM_REQUIRE(q && k && v && plan && out && lse && q_rows, "null pointer argument");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(q_rows) & 15) == 0,
                "q and q_rows must be 16-byte aligned");
    if ((rc = check_current_device())) return rc;
    const mom::PlanLayout L = mom::plan_layout(B * S, nb, top);
    const mom::PlanView P = mom::plan_view(const_cast<void *>(plan), L);
    cudaError_t e = mom::launch_read_fwd(q, k, v, (int)B, (int)S, (int)H, (int)hd, (int)nb, (int)bs,
                                         (int)top, L, P, out, lse, q_rows, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "read_fwd");
    return MOM_OK;
}

size_t mom_read_bwd_workspace_size(int64_t B, int64_t S, int64_t H, int64_t hd) {
    if (B < 0 || S < 0 || H < 0 || hd < 0) return 0;
    const size_t nh = static_cast<size_t>(B) * S * H;
    return align256(nh * 4) + align256(nh * hd * 2);
}

namespace {
// Shared by mom_read_bwd and mom_read_bwd_noalloc: ws_delta holds H x B*S fp32;
// do_rows (B*S x H*hd, or null) receives dO in plan order.
int read_bwd_impl(const void *q, const void *k, const void *v, const void *out, const void *dout,
                  const float *lse, int dtype, int64_t B, int64_t S, int64_t H, int64_t hd, int64_t nb,
                  int64_t bs, int64_t top, const void *plan, const void *q_rows, void *dq, float *dk_acc,
                  float *dv_acc, float *dlog_gates, float *ws_delta, void *do_rows, void *stream) {
    int rc;
    if ((rc = check_current_device())) return rc;
    if (B * S == 0) {
        const size_t kv = sizeof(float) * static_cast<size_t>(nb) * bs * H * hd;
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        cudaError_t e = cudaMemsetAsync(dk_acc, 0, kv, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(dv_acc, 0, kv, st);
        return e == cudaSuccess ? MOM_OK : cuda_fail(e, "read_bwd");
    }
    const mom::PlanLayout L = mom::plan_layout(B * S, nb, top);
    const mom::PlanView P = mom::plan_view(const_cast<void *>(plan), L);
    cudaError_t e = mom::launch_read_bwd(q, q_rows, k, v, out, dout, lse, (int)B, (int)S, (int)H, (int)hd,
                                         (int)nb, (int)bs, (int)top, L, P, dq, dk_acc, dv_acc,
                                         dlog_gates, ws_delta, do_rows, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "read_bwd");
    return MOM_OK;
}

int check_read_bwd_args(int dtype, int64_t B, int64_t S, int64_t H, int64_t hd, int64_t nb, int64_t bs,
                        int64_t top, const void *q, const void *k, const void *v, const void *out,
                        const void *dout, const float *lse, const void *plan, const void *q_rows, void *dq,
                        float *dk_acc, float *dv_acc, float *dlog_gates) {
    int rc = check_read_geometry(dtype, B, S, H, hd, nb, bs, top);
    if (rc) return rc;
    MOM_REQUIRE(k && v && dk_acc && dv_acc, "null pointer argument");
    MOM_REQUIRE(B * S == 0 || (q && out && dout && lse && plan && q_rows && dq && dlog_gates),
                "null pointer argument");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(q_rows) & 15) == 0 && (reinterpret_cast<uintptr_t>(dout) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                "q_rows, out and dout must be 16-byte aligned");
    return MOM_OK;
}
}  // namespace

int mom_read_bwd(const void *q, const void *k, const void *v, const void *out, const void *dout,
                 const float *lse, int dtype, int64_t B, int64_t S, int64_t H, int64_t hd,
                 int64_t nb, int64_t bs, int64_t top, const void *plan, const void *q_rows, void *dq,
                 float *dk_acc, float *dv_acc, float *dlog_gates, void *workspace, size_t workspace_bytes,
                 void *stream) {
    int rc = check_read_bwd_args(dtype, B, S, H, hd, nb, bs, top, q, k, v, out, dout, lse, plan, q_rows, dq,
                                 dk_acc, dv_acc, dlog_gates);
    if (rc) return rc;
    const size_t need = mom_read_bwd_workspace_size(B, S, H, hd);
    if (workspace_bytes < need || (need && !workspace))
        return fail(MOM_ERR_WORKSPACE, "read bwd workspace %zu < %zu bytes", workspace_bytes, need);
    char *ws = static_cast<char *>(workspace);
    float *delta = reinterpret_cast<float *>(ws);
    void *do_rows = ws + align256(static_cast<size_t>(B) * S * H * 4);
    return read_bwd_impl(q, k, v, out, dout, lse, dtype, B, S, H, hd, nb, bs, top, plan, q_rows, dq, dk_acc,
                         dv_acc, dlog_gates, delta, do_rows, stream);
}

// ------------------------------------------------------------------ block-split read
// Top-k routing with more block sets than the set bucketing holds: every
// (token, k) pair is a row of a top-1 plan over B*S*top rows, read by the same
// kernels with PlanView::rows_per_q = top, then combined per token (split.cu).
namespace {
// tail of a block-split plan: the rows' log-gates (M fp32), then iperm (M int32)
size_t split_tail_offset(int64_t M, int64_t nb) { return align256(mom::plan_layout(M, nb, 1).total); }
size_t split_iperm_offset(int64_t M, int64_t nb) {
    return split_tail_offset(M, nb) + align256(static_cast<size_t>(M) * 4);
}

int check_split_geometry(int dtype, int64_t B, int64_t S, int64_t H, int64_t hd, int64_t nb, int64_t bs,
                         int64_t top) {
    MOM_REQUIRE(top > 0 && top <= mom::kMaxTop && top <= nb, "bad (num_blocks, top)");
    MOM_REQUIRE(B >= 0 && S >= 0 && B * S * top < (int64_t(1) << 31), "B*S*top too large");
    return check_read_geometry(dtype, 1, B * S * top, H, hd, nb, bs, 1);
}
}  // namespace

size_t mom_plan_split_size(int64_t N, int64_t nb, int64_t top) {
    if (N < 0 || nb <= 0 || nb > 64 || top <= 0 || top > mom::kMaxTop || top > nb) return 0;
    const int64_t M = N * top;
    if (M >= (int64_t(1) << 31)) return 0;
    return split_iperm_offset(M, nb) + align256(static_cast<size_t>(M) * 4);
}

int mom_bucket_split(const void *top_idx, int idx_dtype, const float *log_gates, int64_t N, int64_t nb,
                     int64_t top, void *plan, size_t plan_bytes, void *stream) {
    MOM_REQUIRE(N >= 0 && nb > 0 && nb <= 64 && top > 0 && top <= mom::kMaxTop && top <= nb,
                "bad (tokens, num_blocks, top)");
    MOM_REQUIRE(N * top < (int64_t(1) << 31), "token count out of range");
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    MOM_REQUIRE(plan, "null plan");
    const size_t need = mom_plan_split_size(N, nb, top);
    if (plan_bytes < need) return fail(MOM_ERR_WORKSPACE, "plan %zu < %zu bytes", plan_bytes, need);
    MOM_REQUIRE(N == 0 || (top_idx && log_gates), "null routing tensors");
    int rc = check_current_device();
    if (rc) return rc;
    const int64_t M = N * top;
    const mom::PlanLayout L = mom::plan_layout(M, nb, 1);
    const mom::PlanView P = mom::plan_view(plan, L);
    float *lg_rows = reinterpret_cast<float *>(static_cast<char *>(plan) + split_tail_offset(M, nb));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int idx64 = idx_dtype == MOM_I64;
    int *iperm = reinterpret_cast<int *>(static_cast<char *>(plan) + split_iperm_offset(M, nb));
    cudaError_t e = mom::launch_split_prep(top_idx, idx64, log_gates, N, (int)top, lg_rows, st);
    if (e == cudaSuccess) e = mom::launch_bucket(top_idx, idx64, lg_rows, L, P, st);
    if (e == cudaSuccess) e = mom::launch_split_iperm(P.perm, M, iperm, st);
    if (e != cudaSuccess) return cuda_fail(e, "bucket_split");
    return MOM_OK;
}

size_t mom_read_split_fwd_workspace_size(int64_t B, int64_t S, int64_t H, int64_t hd, int64_t top) {
    if (B < 0 || S < 0 || H < 0 || hd < 0 || top < 0) return 0;
    return align256(static_cast<size_t>(B) * S * top * H * hd * 2);
}

int mom_read_split_fwd(const void *q, const void *k, const void *v, int dtype, int64_t B, int64_t S, int64_t H,
                       int64_t hd, int64_t nb, int64_t bs, int64_t top, const void *top_idx, int idx_dtype,
                       const void *plan, void *out, float *lse_rows, float *weights, void *q_rows,
                       void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_split_geometry(dtype, B, S, H, hd, nb, bs, top);
    if (rc) return rc;
    if (B * S == 0) return MOM_OK;
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    MOM_REQUIRE(q && k && v && top_idx && plan && out && lse_rows && weights && q_rows, "null pointer argument");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(q_rows) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                "q, q_rows and out must be 16-byte aligned");
    const size_t need = mom_read_split_fwd_workspace_size(B, S, H, hd, top);
    if (workspace_bytes < need || !workspace)
        return fail(MOM_ERR_WORKSPACE, "split read fwd workspace %zu < %zu bytes", workspace_bytes, need);
    if ((rc = check_current_device())) return rc;
    const int64_t N = B * S, M = N * top;
    const mom::PlanLayout L = mom::plan_layout(M, nb, 1);
    mom::PlanView P = mom::plan_view(const_cast<void *>(plan), L);
    P.rows_per_q = (int)top;
    const int *iperm = reinterpret_cast<const int *>(static_cast<const char *>(plan) + split_iperm_offset(M, nb));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = mom::launch_read_fwd(q, k, v, 1, (int)M, (int)H, (int)hd, (int)nb, (int)bs, 1, L, P, workspace,
                                         lse_rows, q_rows, st, iperm);
    if (e == cudaSuccess)
        e = mom::launch_split_combine(workspace, lse_rows, P.perm, top_idx, idx_dtype == MOM_I64, N, (int)top, (int)H,
                                      (int)hd, weights, out, st);
    if (e != cudaSuccess) return cuda_fail(e, "read_split_fwd");
    return MOM_OK;
}

size_t mom_read_split_bwd_workspace_size(int64_t B, int64_t S, int64_t H, int64_t hd, int64_t top) {
    if (B < 0 || S < 0 || H < 0 || hd < 0 || top < 0) return 0;
    const size_t M = static_cast<size_t>(B) * S * top;
    return align256(M * H * 4) + 3 * align256(M * H * hd * 2);
}

int mom_read_split_bwd(const void *q, const void *k, const void *v, const void *out, const void *dout,
                       const float *lse_rows, const float *weights, int dtype, int64_t B, int64_t S, int64_t H,
                       int64_t hd, int64_t nb, int64_t bs, int64_t top, const void *top_idx, int idx_dtype,
                       const void *plan, const void *q_rows, void *dq, float *dk_acc, float *dv_acc,
                       float *dlog_gates, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_split_geometry(dtype, B, S, H, hd, nb, bs, top);
    if (rc) return rc;
    MOM_REQUIRE(k && v && dk_acc && dv_acc, "null pointer argument");
    MOM_REQUIRE(B * S == 0 || (q && out && dout && lse_rows && weights && top_idx && plan && q_rows && dq &&
                               dlog_gates),
                "null pointer argument");
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(q_rows) & 15) == 0 && (reinterpret_cast<uintptr_t>(dout) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 15) == 0 && (reinterpret_cast<uintptr_t>(dq) & 15) == 0,
                "q_rows, out, dout and dq must be 16-byte aligned");
    const size_t need = mom_read_split_bwd_workspace_size(B, S, H, hd, top);
    if (workspace_bytes < need || (need && !workspace))
        return fail(MOM_ERR_WORKSPACE, "split read bwd workspace %zu < %zu bytes", workspace_bytes, need);
    if ((rc = check_current_device())) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t N = B * S, M = N * top;
    if (N == 0) {
        const size_t kv = sizeof(float) * static_cast<size_t>(nb) * bs * H * hd;
        cudaError_t e = cudaMemsetAsync(dk_acc, 0, kv, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(dv_acc, 0, kv, st);
        return e == cudaSuccess ? MOM_OK : cuda_fail(e, "read_split_bwd");
    }
    const size_t rows_bytes = align256(static_cast<size_t>(M) * H * hd * 2);
    char *ws = static_cast<char *>(workspace);
    float *delta = reinterpret_cast<float *>(ws);
    char *g = ws + align256(static_cast<size_t>(M) * H * 4);
    char *dq_rows = g + rows_bytes;
    char *do_rows = dq_rows + rows_bytes;
    const mom::PlanLayout L = mom::plan_layout(M, nb, 1);
    mom::PlanView P = mom::plan_view(const_cast<void *>(plan), L);
    P.rows_per_q = (int)top;
    const int idx64 = idx_dtype == MOM_I64;
    cudaError_t e = cudaSuccess;
    if (mom::read_bwd_tc_supported((int)hd, (int)bs, 1, q_rows, k, v, dout, (int)H)) {
        // the rows' dO = weight x dO, formed by the tensor-core path's row copy
        const int *iperm = reinterpret_cast<const int *>(static_cast<const char *>(plan) + split_iperm_offset(M, nb));
        e = mom::launch_read_bwd(q, q_rows, k, v, out, dout, lse_rows, 1, (int)M, (int)H, (int)hd, (int)nb, (int)bs,
                                 1, L, P, dq_rows, dk_acc, dv_acc, dlog_gates, delta, do_rows, st, weights, iperm);
    } else {
        e = mom::launch_split_gate_do(dout, weights, N, (int)top, (int)H, (int)hd, g, st);
        if (e == cudaSuccess)
            e = mom::launch_read_bwd(q, q_rows, k, v, out, g, lse_rows, 1, (int)M, (int)H, (int)hd, (int)nb,
                                     (int)bs, 1, L, P, dq_rows, dk_acc, dv_acc, dlog_gates, delta, do_rows, st);
    }
    if (e == cudaSuccess)
        e = mom::launch_split_dq_sum(dq_rows, top_idx, idx64, N, (int)top, (int)H, (int)hd, dq, dlog_gates, st);
    if (e != cudaSuccess) return cuda_fail(e, "read_split_bwd");
    return MOM_OK;
}

// ------------------------------------------------------------------ fp32 read
namespace {
int check_f32_read(int64_t B, int64_t S, int64_t H, int64_t hd, int64_t nb, int64_t bs, int64_t top) {
    MOM_REQUIRE(B >= 0 && S >= 0 && B * S * top < (int64_t(1) << 31), "bad B, S");
    MOM_REQUIRE(H > 0 && H <= 1024, "bad n_heads %lld", (long long)H);
    if (hd != 16 && hd != 32 && hd != 64 && hd != 128)
        return fail(MOM_ERR_UNSUPPORTED, "head_dim %lld: the fp32 read takes 16, 32, 64 or 128", (long long)hd);
    MOM_REQUIRE(nb > 0 && nb <= 64 && top > 0 && top <= mom::kMaxTop && top <= nb, "bad (num_blocks, top)");
    MOM_REQUIRE(bs > 0 && nb * bs < (int64_t(1) << 24), "bad block_size %lld", (long long)bs);
    return MOM_OK;
}
bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

size_t mom_read_f32_workspace_size(int64_t B, int64_t S, int64_t H, int64_t hd, int64_t top) {
    if (B < 0 || S < 0 || H < 0 || hd < 0 || top < 0) return 0;
    const size_t M = static_cast<size_t>(B) * S * top;
    const size_t fwd = align256(M * H * hd * 4) + align256(M * H * 4);
    const size_t bwd = align256(static_cast<size_t>(B) * S * H * 4);
    return fwd > bwd ? fwd : bwd;
}

int mom_read_f32_fwd(const float *q, const float *k, const float *v, int64_t B, int64_t S, int64_t H, int64_t hd,
                     int64_t nb, int64_t bs, int64_t top, const void *top_idx, int idx_dtype, const void *plan,
                     float *out, float *lse, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_f32_read(B, S, H, hd, nb, bs, top);
    if (rc) return rc;
    if (B * S == 0) return MOM_OK;
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    MOM_REQUIRE(q && k && v && top_idx && plan && out && lse && workspace, "null pointer argument");
    MOM_REQUIRE(al16(q) && al16(k) && al16(v) && al16(out), "q, k, v and out must be 16-byte aligned");
    const size_t need = mom_read_f32_workspace_size(B, S, H, hd, top);
    if (workspace_bytes < need)
        return fail(MOM_ERR_WORKSPACE, "fp32 read fwd workspace %zu < %zu bytes", workspace_bytes, need);
    if ((rc = check_current_device())) return rc;
    const int64_t N = B * S, M = N * top;
    const mom::PlanLayout L = mom::plan_layout(M, nb, 1);
    mom::PlanView P = mom::plan_view(const_cast<void *>(plan), L);
    P.rows_per_q = (int)top;
    const int *iperm = reinterpret_cast<const int *>(static_cast<const char *>(plan) + split_iperm_offset(M, nb));
    float *o_rows = static_cast<float *>(workspace);
    float *lse_rows = reinterpret_cast<float *>(static_cast<char *>(workspace) + align256(M * H * hd * 4));
    cudaError_t e = mom::launch_read_f32_fwd(q, k, v, N, (int)H, (int)hd, (int)nb, (int)bs, (int)top, L, P, top_idx,
                                             idx_dtype == MOM_I64, iperm, o_rows, lse_rows, out, lse,
                                             static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "read_f32_fwd");
    return MOM_OK;
}

int mom_read_f32_bwd(const float *q, const float *k, const float *v, const float *out, const float *dout,
                     const float *lse, int64_t B, int64_t S, int64_t H, int64_t hd, int64_t nb, int64_t bs,
                     int64_t top, const void *top_idx, int idx_dtype, const void *plan, float *dq, float *dk,
                     float *dv, float *dlog_gates, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_f32_read(B, S, H, hd, nb, bs, top);
    if (rc) return rc;
    MOM_REQUIRE(k && v && dk && dv, "null pointer argument");
    MOM_REQUIRE(B * S == 0 || (q && out && dout && lse && top_idx && plan && dq && dlog_gates && workspace),
                "null pointer argument");
    MOM_REQUIRE(is_idx_dtype(idx_dtype), "index dtype must be I32 or I64");
    MOM_REQUIRE(B * S == 0 || (al16(q) && al16(k) && al16(v) && al16(out) && al16(dout)),
                "q, k, v, out and dout must be 16-byte aligned");
    const size_t need = mom_read_f32_workspace_size(B, S, H, hd, top);
    if (B * S > 0 && workspace_bytes < need)
        return fail(MOM_ERR_WORKSPACE, "fp32 read bwd workspace %zu < %zu bytes", workspace_bytes, need);
    if ((rc = check_current_device())) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t N = B * S, M = N * top;
    const size_t kv = sizeof(float) * static_cast<size_t>(nb) * bs * H * hd;
    cudaError_t e = cudaMemsetAsync(dk, 0, kv, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(dv, 0, kv, st);
    if (e == cudaSuccess && N > 0) e = cudaMemsetAsync(dq, 0, sizeof(float) * static_cast<size_t>(N) * H * hd, st);
    if (e == cudaSuccess && N > 0) e = cudaMemsetAsync(dlog_gates, 0, sizeof(float) * static_cast<size_t>(N) * top, st);
    if (e == cudaSuccess && N > 0) {
        const mom::PlanLayout L = mom::plan_layout(M, nb, 1);
        mom::PlanView P = mom::plan_view(const_cast<void *>(plan), L);
        P.rows_per_q = (int)top;
        e = mom::launch_read_f32_bwd(q, k, v, out, dout, lse, N, (int)H, (int)hd, (int)bs, (int)top, L, P, top_idx,
                                     idx_dtype == MOM_I64, static_cast<float *>(workspace), dq, dk, dv, dlog_gates,
                                     st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "read_f32_bwd");
    return MOM_OK;
}

// ------------------------------------------------------------------ decoder trunk
int mom_rope_qkv_fwd(const void *qkv, const float *cosv, const float *sinv, int64_t B, int64_t S, int64_t H,
                     int64_t hd, void *q, void *k, void *v, void *stream) {
    MOM_REQUIRE(B >= 0 && S >= 0 && H > 0 && hd > 0 && hd % 2 == 0 && hd <= 256, "bad rope geometry");
    MOM_REQUIRE(B * S * H * hd < (int64_t(1) << 40), "rope size out of range");
    if (B * S == 0) return MOM_OK;
    MOM_REQUIRE(qkv && cosv && sinv && q && k && v, "null pointer argument");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_rope_qkv_fwd(qkv, cosv, sinv, (int)B, (int)S, (int)H, (int)hd, q, k, v,
                                             static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "rope_qkv_fwd");
}

int mom_rope_qkv_bwd(const void *dq, const void *dk, const void *dv, const float *cosv, const float *sinv, int64_t B,
                     int64_t S, int64_t H, int64_t hd, void *dqkv, void *stream) {
    MOM_REQUIRE(B >= 0 && S >= 0 && H > 0 && hd > 0 && hd % 2 == 0 && hd <= 256, "bad rope geometry");
    if (B * S == 0) return MOM_OK;
    MOM_REQUIRE(dq && dk && dv && cosv && sinv && dqkv, "null pointer argument");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_rope_qkv_bwd(dq, dk, dv, cosv, sinv, (int)B, (int)S, (int)H, (int)hd, dqkv,
                                             static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "rope_qkv_bwd");
}

int mom_swiglu_fwd(const void *gu, int64_t N, int64_t f, void *h, void *stream) {
    MOM_REQUIRE(N >= 0 && f > 0 && f % 2 == 0 && f < (int64_t(1) << 30), "bad swiglu geometry");
    if (N == 0) return MOM_OK;
    MOM_REQUIRE(gu && h, "null pointer argument");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(gu) & 3) == 0 && (reinterpret_cast<uintptr_t>(h) & 3) == 0,
                "gu and h must be 4-byte aligned");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_swiglu_fwd(gu, N, (int)f, h, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "swiglu_fwd");
}

int mom_swiglu_bwd(const void *dh, const void *gu, int64_t N, int64_t f, void *dgu, void *stream) {
    MOM_REQUIRE(N >= 0 && f > 0 && f % 2 == 0 && f < (int64_t(1) << 30), "bad swiglu geometry");
    if (N == 0) return MOM_OK;
    MOM_REQUIRE(dh && gu && dgu, "null pointer argument");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(dh) & 3) == 0 && (reinterpret_cast<uintptr_t>(gu) & 3) == 0 &&
                    (reinterpret_cast<uintptr_t>(dgu) & 3) == 0,
                "dh, gu and dgu must be 4-byte aligned");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_swiglu_bwd(dh, gu, N, (int)f, dgu, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "swiglu_bwd");
}

namespace {
int delta_code(int delta_dtype, const void *delta) {
    if (!delta) return 0;
    if (delta_dtype == MOM_BF16) return 1;
    if (delta_dtype == MOM_F32) return 2;
    return -1;
}
}  // namespace

int mom_add_rmsnorm_fwd(const float *x, const void *delta, int delta_dtype, const float *delta_scale, const float *w,
                        int64_t N, int64_t d, double eps, float *x_out, void *y_bf16, float *y_f32, float *rstd,
                        void *stream) {
    const int ddt = delta_code(delta_dtype, delta);
    MOM_REQUIRE(ddt >= 0, "delta dtype must be F32 or BF16");
    MOM_REQUIRE(N >= 0 && (d == 128 || d == 256 || d == 512 || d == 1024 || d == 2048),
                "d must be 128, 256, 512, 1024 or 2048");
    if (N == 0) return MOM_OK;
    MOM_REQUIRE(x && w && x_out && y_bf16 && rstd, "null pointer argument");
    MOM_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(x_out) | reinterpret_cast<uintptr_t>(w) |
                  reinterpret_cast<uintptr_t>(y_f32)) & 15) == 0 && ((reinterpret_cast<uintptr_t>(y_bf16) |
                  reinterpret_cast<uintptr_t>(delta)) & 7) == 0, "rows must be 16-byte (fp32) / 8-byte (bf16) aligned");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_add_rmsnorm_fwd(x, delta, ddt, delta_scale, w, N, (int)d, static_cast<float>(eps), x_out,
                                                y_bf16, y_f32, rstd, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "add_rmsnorm_fwd");
}

int mom_add_rmsnorm_bwd(const float *x_new, const float *rstd, const float *w, const void *delta, int delta_dtype,
                        const float *delta_scale, const void *dy_bf16, const float *dy_f32, const float *dx_in,
                        int64_t N, int64_t d, float *dx, void *ddelta, float *dw, float *ddelta_scale, void *stream) {
    const int ddt = delta_code(delta_dtype, delta);
    MOM_REQUIRE(ddt >= 0, "delta dtype must be F32 or BF16");
    MOM_REQUIRE(N >= 0 && (d == 128 || d == 256 || d == 512 || d == 1024 || d == 2048),
                "d must be 128, 256, 512, 1024 or 2048");
    MOM_REQUIRE(w && dw, "null pointer argument");
    MOM_REQUIRE(N == 0 || (x_new && rstd && dx && (dy_bf16 || dy_f32) && (ddt == 0 || ddelta)),
                "null pointer argument");
    MOM_REQUIRE(!ddelta_scale || (ddt != 0 && delta_scale), "a scale gradient needs a scaled delta");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_add_rmsnorm_bwd(x_new, rstd, w, delta, ddt, delta_scale, dy_bf16, dy_f32, dx_in, N,
                                                (int)d, dx, ddelta, dw, ddelta_scale,
                                                static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "add_rmsnorm_bwd");
}

int mom_adamw_step(const void *tensors, int64_t ntensors, const void *chunks, int64_t nchunks, double lr,
                   double beta1, double beta2, double eps, double weight_decay, int64_t step, void *stream) {
    MOM_REQUIRE(ntensors >= 0 && nchunks >= 0 && step >= 1, "bad optimizer arguments");
    if (nchunks == 0) return MOM_OK;
    MOM_REQUIRE(tensors && chunks, "null pointer argument");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(tensors) & 7) == 0 && (reinterpret_cast<uintptr_t>(chunks) & 7) == 0,
                "tables must be 8-byte aligned");
    int rc = check_current_device();
    if (rc) return rc;
    const double bc1 = 1.0 - std::pow(beta1, static_cast<double>(step));
    const double bc2 = 1.0 - std::pow(beta2, static_cast<double>(step));
    cudaError_t e = mom::launch_adamw_multi(static_cast<const mom::OptTensor *>(tensors),
                                            static_cast<const int2 *>(chunks), nchunks, (float)lr, (float)beta1,
                                            (float)beta2, (float)eps, (float)weight_decay, (float)bc1, (float)bc2,
                                            static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "adamw_step");
}

int mom_xent_fwd(const void *logits, const int64_t *labels, int64_t R, int64_t V, int64_t ignore_index,
                 float *row_loss, float *lse, void *stream) {
    MOM_REQUIRE(R >= 0 && V > 0 && V < (int64_t(1) << 31), "bad cross-entropy geometry");
    if (R == 0) return MOM_OK;
    MOM_REQUIRE(logits && labels && row_loss && lse, "null pointer argument");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(logits) & 1) == 0, "logits must be 2-byte aligned");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_xent_fwd(logits, labels, R, (int)V, ignore_index, row_loss, lse,
                                         static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "xent_fwd");
}

int mom_xent_bwd(const void *logits, const int64_t *labels, const float *lse, const float *grad, int64_t R, int64_t V,
                 int64_t ignore_index, void *dlogits, void *stream) {
    MOM_REQUIRE(R >= 0 && V > 0 && V < (int64_t(1) << 31), "bad cross-entropy geometry");
    if (R == 0) return MOM_OK;
    MOM_REQUIRE(logits && labels && lse && grad && dlogits, "null pointer argument");
    MOM_REQUIRE((reinterpret_cast<uintptr_t>(logits) & 1) == 0 && (reinterpret_cast<uintptr_t>(dlogits) & 1) == 0,
                "logits and dlogits must be 2-byte aligned");
    int rc = check_current_device();
    if (rc) return rc;
    cudaError_t e = mom::launch_xent_bwd(logits, labels, lse, grad, R, (int)V, ignore_index, dlogits,
                                         static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MOM_OK : cuda_fail(e, "xent_bwd");
}

// ------------------------------------------------- read backward, no allocation
// mom_read_bwd_noalloc runs mom_read_bwd with its workspace (the per-row delta,
// H x B*S fp32) in a fixed device array of this library instead of caller
// memory. It is for callers that cannot allocate device memory: a plugin
// handed its tensors by a framework whose caching allocator has reserved the
// device (a cudaMalloc of its own would fail or sit outside that pool), or a C
// caller over FFI with no device allocator at all.
//
// The array is kNoAllocScratchBytes (4 MiB) and lives in every device's copy
// of this library's code, from when the CUDA runtime loads it on that device
// until the process exits. In host code `g_read_bwd_scratch` only names the
// symbol; its device address comes from cudaGetSymbolAddress, looked up once
// per device with that device current, on the first call made on it (make
// that first call before any stream capture), and again whenever the device's
// current context is another one than at the last look-up (after a
// cudaDeviceReset the runtime loads the module anew, at a new address). All
// calls share the one array
// and it keeps the last call's contents; nothing in it has to start at zero
// (the dQ pass writes every delta entry that the dK/dV pass reads), but calls
// that overlap on the GPU (two streams, or two threads) race on it.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
constexpr int kNoAllocMaxDevices = 64;
__device__ __align__(256) unsigned char g_read_bwd_scratch[kNoAllocScratchBytes];

// The driver's cuCtxGetCurrent, through the runtime's entry-point query (no
// link against libcuda): the context the cached address belongs to.
PFN_cuCtxGetCurrent_v4000 ctx_get_current_fn() {
    static PFN_cuCtxGetCurrent_v4000 fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        return static_cast<PFN_cuCtxGetCurrent_v4000>(nullptr);
    }();
    return fn;
}

int noalloc_scratch(void **ptr) {
    static std::mutex mu;
    static void *addr[kNoAllocMaxDevices] = {};
    static CUcontext owner[kNoAllocMaxDevices] = {};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(MOM_ERR_UNSUPPORTED, "device ordinal %d beyond %d", dev, kNoAllocMaxDevices);
    CUcontext ctx = nullptr;
    if (PFN_cuCtxGetCurrent_v4000 get = ctx_get_current_fn()) get(&ctx);
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev] || owner[dev] != ctx) {
        void *p = nullptr;
        if ((e = cudaGetSymbolAddress(&p, g_read_bwd_scratch)) != cudaSuccess)
            return cuda_fail(e, "cudaGetSymbolAddress(read bwd scratch)");
        addr[dev] = p;
        owner[dev] = ctx;
    }
    *ptr = addr[dev];
    return MOM_OK;
}
}  // namespace

size_t mom_read_bwd_noalloc_max_bytes(void) { return kNoAllocScratchBytes; }

int mom_read_bwd_noalloc(const void *q, const void *k, const void *v, const void *out, const void *dout,
                         const float *lse, int dtype, int64_t B, int64_t S, int64_t H, int64_t hd,
                         int64_t nb, int64_t bs, int64_t top, const void *plan, const void *q_rows, void *dq,
                         float *dk_acc, float *dv_acc, float *dlog_gates, void *stream) {
    int rc = check_read_geometry(dtype, B, S, H, hd, nb, bs, top);
    if (rc) return rc;
    const size_t need = align256(static_cast<size_t>(B) * S * H * 4);
    if (need > kNoAllocScratchBytes)
        return fail(MOM_ERR_WORKSPACE,
                    "mom_read_bwd_noalloc: B*S*H = %lld needs %zu bytes of scratch, over its fixed %zu "
                    "(at most %zu tokens x heads); use mom_read_bwd with a caller workspace",
                    (long long)(B * S * H), need, kNoAllocScratchBytes, kNoAllocScratchBytes / 4);
    if ((rc = check_read_bwd_args(dtype, B, S, H, hd, nb, bs, top, q, k, v, out, dout, lse, plan, q_rows, dq,
                                  dk_acc, dv_acc, dlog_gates)))
        return rc;
    if ((rc = check_current_device())) return rc;
    void *scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    // dO stays in token order (no scratch for a plan-order copy): the kernels gather its rows
    return read_bwd_impl(q, k, v, out, dout, lse, dtype, B, S, H, hd, nb, bs, top, plan, q_rows, dq, dk_acc,
                         dv_acc, dlog_gates, static_cast<float *>(scratch), nullptr, stream);
}

}  // extern "C"
