// Routing permutation: a stable counting sort of the tokens by the set of
// memory blocks they selected, cut into tiles of at most kTileM tokens that
// all read the same blocks. This is what lets the read touch only the
// selected slots (top*bs per token) instead of all L slots with a mask, as
// the reference kernels do (mom_kernels/triton_gpu.py:98-133).
//
// Four launches, no host synchronisation:
//   bucket_keys    per token: validated, sorted set -> key; per-chunk histogram
//   bucket_keyscan per key (one CTA each): offsets of the chunks within the key
//   bucket_scan    one CTA: key bases, tiles, key sets, per-block tile lists
//   bucket_scatter per token: stable rank inside its chunk -> permuted row,
//                  with the row's per-block biases and the caller-order map.
#include "common.cuh"
#include "launch.h"

namespace mom {

__host__ __device__ inline uint64_t binom(int n, int k) {
    if (k < 0 || k > n) return 0;
    if (k > n - k) k = n - k;
    uint64_t r = 1;
    for (int i = 1; i <= k; ++i) r = r * static_cast<uint64_t>(n - k + i) / static_cast<uint64_t>(i);
    return r;
}

int64_t num_route_keys(int64_t nb, int64_t top) {
    uint64_t n = 0;
    for (int s = 0; s <= top; ++s) n += binom(static_cast<int>(nb), s);
    return static_cast<int64_t>(n);
}

static size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

PlanLayout plan_layout(int64_t N, int64_t nb, int64_t top) {
    PlanLayout L;
    L.N = N;
    L.nb = nb;
    L.top = top;
    L.num_keys = num_route_keys(nb, top);
    L.chunks = (N + kBucketChunk - 1) / kBucketChunk;
    L.max_tiles = (N + kTileM - 1) / kTileM + std::min<int64_t>(N, L.num_keys);
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t at = o; o = align256(o + bytes); return at; };
    L.off_err = take(sizeof(int));
    L.off_ntiles = take(sizeof(int));
    L.off_key = take(sizeof(int) * N);
    L.off_hist = take(sizeof(int) * L.chunks * L.num_keys);
    L.off_keytot = take(sizeof(int) * L.num_keys);
    L.off_keybase = take(sizeof(int) * L.num_keys);
    L.off_keytb = take(sizeof(int) * L.num_keys);
    L.off_keyset = take(sizeof(int) * L.num_keys * top);
    L.off_perm = take(sizeof(int) * N);
    L.off_rowbias = take(sizeof(float) * N * top);
    L.off_rowkmap = take(sizeof(uint32_t) * N);
    L.off_tiles = take(sizeof(int4) * L.max_tiles);
    L.off_blkcount = take(sizeof(int) * nb);
    L.off_blktiles = take(sizeof(int) * nb * L.max_tiles);
    L.total = o;
    return L;
}

PlanView plan_view(void *plan, const PlanLayout &L) {
    char *p = static_cast<char *>(plan);
    PlanView v;
    v.n = L.N;
    v.err = reinterpret_cast<int *>(p + L.off_err);
    v.ntiles = reinterpret_cast<int *>(p + L.off_ntiles);
    v.key = reinterpret_cast<int *>(p + L.off_key);
    v.hist = reinterpret_cast<int *>(p + L.off_hist);
    v.keytot = reinterpret_cast<int *>(p + L.off_keytot);
    v.keybase = reinterpret_cast<int *>(p + L.off_keybase);
    v.keytb = reinterpret_cast<int *>(p + L.off_keytb);
    v.keyset = reinterpret_cast<int *>(p + L.off_keyset);
    v.perm = reinterpret_cast<int *>(p + L.off_perm);
    v.rowbias = reinterpret_cast<float *>(p + L.off_rowbias);
    v.rowkmap = reinterpret_cast<uint32_t *>(p + L.off_rowkmap);
    v.tiles = reinterpret_cast<int4 *>(p + L.off_tiles);
    v.blkcount = reinterpret_cast<int *>(p + L.off_blkcount);
    v.blktiles = reinterpret_cast<int *>(p + L.off_blktiles);
    v.rows_per_q = 1;
    return v;
}

// The distinct, ascending set of blocks of one token (invalid entries dropped).
struct TokenSet {
    int blk[8];
    int n;
    bool bad;
};

__device__ __forceinline__ int load_idx(const void *top_idx, int idx64, int64_t i) {
    if (idx64) {
        const int64_t v = reinterpret_cast<const int64_t *>(top_idx)[i];
        return (v < INT32_MIN || v > INT32_MAX) ? -1 : static_cast<int>(v);
    }
    return reinterpret_cast<const int32_t *>(top_idx)[i];
}

__device__ TokenSet token_set(const void *top_idx, int idx64, int64_t t, int nb, int top) {
    TokenSet s;
    s.n = 0;
    s.bad = false;
    for (int k = 0; k < top; ++k) {
        const int b = load_idx(top_idx, idx64, t * top + k);
        if (b < 0 || b >= nb) { s.bad = true; continue; }
        int pos = 0;
        bool dup = false;
        while (pos < s.n && s.blk[pos] <= b) { dup |= s.blk[pos] == b; ++pos; }
        if (dup) continue;
        for (int q = s.n; q > pos; --q) s.blk[q] = s.blk[q - 1];
        s.blk[pos] = b;
        ++s.n;
    }
    return s;
}

// Binomial coefficients C(n, k), n <= 64, k <= 8, as a shared-memory table built
// by one warp from Pascal's rule (no integer division on the token path). Values
// saturate at 2^31 - 1: every coefficient a key or its decoding uses is at most
// the number of keys (<= kMaxKeys).
constexpr int kBinomN = 65, kBinomK = 9;
__device__ void build_binom(uint32_t *tab) {
    if (threadIdx.x >= 32) return;
    const int k = threadIdx.x;
    uint32_t c = k == 0 ? 1u : 0u;   // row n = 0
    for (int n = 0; n < kBinomN; ++n) {
        if (k < kBinomK) tab[n * kBinomK + k] = c;
        const uint32_t left = __shfl_up_sync(0xffffffffu, c, 1);
        const uint64_t next = static_cast<uint64_t>(c) + (k > 0 ? left : 0u);
        c = next > 0x7FFFFFFFu ? 0x7FFFFFFFu : static_cast<uint32_t>(next);
    }
}
__device__ __forceinline__ uint32_t binom_tab(const uint32_t *tab, int n, int k) {
    return (k < 0 || k >= kBinomK || n < 0 || n >= kBinomN || k > n) ? 0u : tab[n * kBinomK + k];
}

__device__ int set_key(const TokenSet &s, int nb, const uint32_t *tab) {
    uint32_t off = 0, rank = 0;
    for (int q = 0; q < s.n; ++q) {
        off += binom_tab(tab, nb, q);
        rank += binom_tab(tab, s.blk[q], q + 1);
    }
    return static_cast<int>(off + rank);
}

__global__ void __launch_bounds__(kBucketChunk)
bucket_keys_kernel(const void *__restrict__ top_idx, int idx64, int64_t N, int nb, int top,
                   int num_keys, PlanView P) {
    extern __shared__ int s_hist[];
    __shared__ uint32_t s_binom[kBinomN * kBinomK];
    for (int i = threadIdx.x; i < num_keys; i += blockDim.x) s_hist[i] = 0;
    build_binom(s_binom);
    __syncthreads();
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kBucketChunk + threadIdx.x;
    if (t < N) {
        const TokenSet s = token_set(top_idx, idx64, t, nb, top);
        if (s.bad) atomicOr(P.err, 1);
        const int key = set_key(s, nb, s_binom);
        P.key[t] = key;
        atomicAdd(&s_hist[key], 1);
    }
    __syncthreads();
    int *h = P.hist + static_cast<int64_t>(blockIdx.x) * num_keys;
    for (int i = threadIdx.x; i < num_keys; i += blockDim.x) h[i] = s_hist[i];
}

// Exclusive block-wide scan of one value per thread (blockDim.x == 1024).
__device__ int block_exclusive_scan(int v, int *s_tmp, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) s_tmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < (blockDim.x >> 5) ? s_tmp[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += n;
        }
        s_tmp[32 + lane] = wi - w;
        if (lane == 31) s_tmp[64] = wi;
    }
    __syncthreads();
    const int res = s_tmp[32 + warp] + incl - v;
    total = s_tmp[64];
    __syncthreads();
    return res;
}

// Per key: exclusive scan of the chunks' counts -> hist[c][k] = offset of chunk c
// within key k's rows; keytot[k] = the key's token count.
__global__ void __launch_bounds__(256)
bucket_keyscan_kernel(int num_keys, int chunks, PlanView P) {
    __shared__ int s_tmp[96];
    const int k = blockIdx.x;
    int carry = 0;
    for (int c0 = 0; c0 < chunks; c0 += blockDim.x) {
        const int c = c0 + threadIdx.x;
        int *h = P.hist + static_cast<int64_t>(c) * num_keys + k;
        const int v = c < chunks ? *h : 0;
        int total;
        const int ex = block_exclusive_scan(v, s_tmp, total);
        if (c < chunks) *h = carry + ex;
        carry += total;
    }
    if (threadIdx.x == 0) P.keytot[k] = carry;
}

// One CTA: key row bases and first tiles (scans over the keys), the tiles, each
// key's block set, and per block the list of tiles that read it. Dynamic shared
// memory: per key the block mask (u64), tile count and first tile.
__global__ void __launch_bounds__(1024)
bucket_scan_kernel(int nb, int top, int num_keys, int max_tiles, PlanView P) {
    extern __shared__ __align__(8) unsigned char s_dyn[];
    uint64_t *s_mask = reinterpret_cast<uint64_t *>(s_dyn);
    int *s_nt = reinterpret_cast<int *>(s_mask + num_keys);
    int *s_tb = s_nt + num_keys;
    __shared__ int s_tmp[96];
    __shared__ uint32_t s_binom[kBinomN * kBinomK];
    build_binom(s_binom);
    __syncthreads();
    const int tid = threadIdx.x;
    const int per = (num_keys + 1023) / 1024;          // <= kMaxKeys / 1024 = 8
    const int k0 = min(num_keys, tid * per), k1 = min(num_keys, k0 + per);
    int rows = 0, tiles = 0;
    for (int k = k0; k < k1; ++k) {
        const int n = P.keytot[k];
        s_nt[k] = (n + kTileM - 1) / kTileM;
        rows += n;
        tiles += s_nt[k];
    }
    int total_rows, total_tiles;
    int row_base = block_exclusive_scan(rows, s_tmp, total_rows);
    int tile_base = block_exclusive_scan(tiles, s_tmp, total_tiles);
    for (int k = k0; k < k1; ++k) {
        const int n = P.keytot[k];
        const int nt = s_nt[k];
        P.keybase[k] = row_base;
        P.keytb[k] = tile_base;
        s_tb[k] = tile_base;
        for (int j = 0; j < nt; ++j)
            P.tiles[tile_base + j] = make_int4(row_base + j * kTileM, min(kTileM, n - j * kTileM), k, 0);
        row_base += n;
        tile_base += nt;
        // decode the key into its block set
        int sz = 0;
        uint32_t off = 0;
        while (sz < top && off + binom_tab(s_binom, nb, sz) <= static_cast<uint32_t>(k)) {
            off += binom_tab(s_binom, nb, sz);
            ++sz;
        }
        uint32_t rank = static_cast<uint32_t>(k) - off;
        int *set = P.keyset + static_cast<int64_t>(k) * top;
        for (int q = top - 1; q >= 0; --q) set[q] = -1;
        uint64_t mask = 0;
        for (int q = sz - 1; q >= 0; --q) {
            int b = q;
            while (b + 1 < nb && binom_tab(s_binom, b + 1, q + 1) <= rank) ++b;
            set[q] = b;
            mask |= uint64_t(1) << b;
            rank -= binom_tab(s_binom, b, q + 1);
        }
        s_mask[k] = mask;
    }
    if (tid == 0) *P.ntiles = total_tiles;
    __syncthreads();
    // per-block tile lists, in key order (warp per block)
    const int warp = tid >> 5, lane = tid & 31;
    for (int b = warp; b < nb; b += 32) {
        int count = 0;
        for (int kb = 0; kb < num_keys; kb += 32) {
            const int k = kb + lane;
            const int nt = (k < num_keys && ((s_mask[k] >> b) & 1)) ? s_nt[k] : 0;
            int incl = nt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            const int base = count + incl - nt;
            for (int j = 0; j < nt; ++j) P.blktiles[static_cast<int64_t>(b) * max_tiles + base + j] = s_tb[k] + j;
            count += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) P.blkcount[b] = count;
    }
}

__global__ void __launch_bounds__(kBucketChunk)
bucket_scatter_kernel(const void *__restrict__ top_idx, int idx64, const float *__restrict__ log_gates,
                      int64_t N, int nb, int top, int num_keys, PlanView P) {
    extern __shared__ int s_run[];
    for (int i = threadIdx.x; i < num_keys; i += blockDim.x) s_run[i] = 0;
    __syncthreads();
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kBucketChunk + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int key = t < N ? P.key[t] : -1;
    // everything this token needs from global memory, loaded before the rank pass
    constexpr int kMaxTopB = 8;
    int bk[kMaxTopB];
    float lgk[kMaxTopB];
    int setv[kMaxTopB];
    int base = 0;
    if (key >= 0) {
        base = P.hist[static_cast<int64_t>(blockIdx.x) * num_keys + key] + P.keybase[key];
#pragma unroll
        for (int k = 0; k < kMaxTopB; ++k) {
            bk[k] = k < top ? load_idx(top_idx, idx64, t * top + k) : -1;
            lgk[k] = k < top ? log_gates[t * top + k] : 0.0f;
            setv[k] = k < top ? P.keyset[static_cast<int64_t>(key) * top + k] : -1;
        }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const int leader = __ffs(peers) - 1;
    int pos = -1;
    for (int w = 0; w < (kBucketChunk >> 5); ++w) {   // warps in token order: a stable sort
        if (warp == w && key >= 0) {
            pos = s_run[key] + rank;
            __syncwarp(peers);
            if (lane == leader) s_run[key] += __popc(peers);
        }
        __syncthreads();
    }
    if (t >= N) return;
    pos += base;
    P.perm[pos] = static_cast<int>(t);
    uint32_t kmap = 0xFFFFFFFFu;
    float bias[kMaxTopB];
#pragma unroll
    for (int j = 0; j < kMaxTopB; ++j) bias[j] = 0.0f;
#pragma unroll
    for (int k = 0; k < kMaxTopB; ++k) {
#pragma unroll
        for (int j = 0; j < kMaxTopB; ++j) {
            if (k < top && j < top && setv[j] >= 0 && setv[j] == bk[k]) {
                bias[j] += lgk[k];
                kmap = (kmap & ~(0xFu << (4 * k))) | (static_cast<uint32_t>(j) << (4 * k));
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kMaxTopB; ++j)
        if (j < top) P.rowbias[static_cast<int64_t>(pos) * top + j] = bias[j];
    P.rowkmap[pos] = kmap;
}

cudaError_t launch_bucket(const void *top_idx, int idx64, const float *log_gates,
                          const PlanLayout &L, const PlanView &P, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(P.err, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
    if (L.N == 0) return cudaMemsetAsync(P.ntiles, 0, sizeof(int), st);
    const int nk = static_cast<int>(L.num_keys);
    const size_t smem = sizeof(int) * nk;
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(bucket_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(bucket_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    bucket_keys_kernel<<<static_cast<unsigned>(L.chunks), kBucketChunk, smem, st>>>(
        top_idx, idx64, L.N, static_cast<int>(L.nb), static_cast<int>(L.top), nk, P); count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    bucket_keyscan_kernel<<<nk, 256, 0, st>>>(nk, static_cast<int>(L.chunks), P); count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t scan_smem = static_cast<size_t>(nk) * 16;
    if (scan_smem > 48 * 1024) {
        e = cudaFuncSetAttribute(bucket_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)scan_smem);
        if (e != cudaSuccess) return e;
    }
    bucket_scan_kernel<<<1, 1024, scan_smem, st>>>(static_cast<int>(L.nb), static_cast<int>(L.top), nk,
                                                   static_cast<int>(L.max_tiles), P); count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    bucket_scatter_kernel<<<static_cast<unsigned>(L.chunks), kBucketChunk, smem, st>>>(
        top_idx, idx64, log_gates, L.N, static_cast<int>(L.nb), static_cast<int>(L.top), nk, P); count_launch();
    return cudaGetLastError();
}

}  // namespace mom
