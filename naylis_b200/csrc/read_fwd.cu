// Gated memory read, forward: for every tile of tokens that selected the same
// set of memory blocks, attend over exactly those blocks' slots with the
// per-token log-gate bias, online softmax in registers.
//
// Reference semantics: mom_kernels/reference.py:14-61 (build_gate_bias +
// mom_attention_reference) and the Triton forward
// mom_kernels/triton_gpu.py:64-141, which reads all L slots with a -1e6 mask;
// here the masked slots are never loaded (their probability is exactly 0 in
// the reference too, as finfo.min / -1e6 underflows).
#include "common.cuh"
#include "launch.h"
#include "read_common.cuh"

namespace mom {

template <int HD>
__global__ void __launch_bounds__(kReadThreads)
read_fwd_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                const uint16_t *__restrict__ v, int H, int bs, int top, float scale_log2,
                PlanView P, uint16_t *__restrict__ out, float *__restrict__ lse) {
    constexpr int kRowB = HD * 2;
    constexpr int kChunks = HD / 8;                 // 16-B chunks per row
    constexpr int kTileBytes = kTileM * kRowB;      // Q / O tile
    constexpr int kKVBytes = kSlotChunk * kRowB;    // one K or V chunk
    constexpr int NTS = kSlotChunk / 8;             // score n-tiles per chunk
    constexpr int NTO = HD / 8;                     // output n-tiles
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char *sQ = smem;
    unsigned char *sKV = smem + kTileBytes;         // [2][K|V]
    int *sTok = reinterpret_cast<int *>(sKV + 4 * kKVBytes);
    float *sBias = reinterpret_cast<float *>(sTok + kTileM);   // [kTileM][top]

    const int tile = blockIdx.x;
    if (tile >= *P.ntiles) return;
    const int h = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int4 td = P.tiles[tile];
    const int row0 = td.x, nrows = td.y;
    const int *set = P.keyset + static_cast<int64_t>(td.z) * top;
    const int64_t ld = static_cast<int64_t>(H) * HD;          // row stride of q/k/v/out

    for (int i = tid; i < kTileM; i += kReadThreads) sTok[i] = i < nrows ? P.perm[row0 + i] : -1;
    for (int i = tid; i < kTileM * top; i += kReadThreads) {
        const int r = i / top;
        sBias[i] = r < nrows ? P.rowbias[static_cast<int64_t>(row0) * top + i] * kLog2e : 0.0f;
    }
    __syncthreads();
    // Q tile (gathered rows)
    for (int i = tid; i < kTileM * kChunks; i += kReadThreads) {
        const int r = i / kChunks, ch = i % kChunks;
        const int tok = sTok[r];
        const uint16_t *src = tok >= 0 ? q + (tok / P.rows_per_q) * ld + h * HD + ch * 8 : q;
        cp_async16(smem_u32(sQ) + swz(r, ch, kRowB), src, tok >= 0 ? 16 : 0);
    }
    cp_async_commit();

    int nblk = 0;
    while (nblk < top && set[nblk] >= 0) ++nblk;
    const int cpb = (bs + kSlotChunk - 1) / kSlotChunk;     // slot chunks per block
    const int nchunk = nblk * cpb;

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

    // per-thread state: rows g and g+8 of this warp's 16
    const int g = lane >> 2, q2 = (lane & 3) * 2;
    float o[NTO][4];
#pragma unroll
    for (int j = 0; j < NTO; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};

    cp_async_wait<1>();   // Q landed (chunk 0 may be in flight)
    __syncthreads();
    uint32_t qf[HD / 16][4];
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks)
        ldmatrix_x4(qf[ks], smem_u32(sQ) + swz(warp * 16 + (lane & 15), ks * 2 + (lane >> 4), kRowB));

#pragma unroll 1
    for (int c = 0; c < nchunk; ++c) {
        issue(c + 1);
        cp_async_wait<1>();
        __syncthreads();
        const int j = c / cpb, cc = c % cpb;
        const int valid = min(kSlotChunk, bs - cc * kSlotChunk);
        const uint32_t sk = smem_u32(sKV + (c & 1) * 2 * kKVBytes);
        const uint32_t sv = sk + kKVBytes;

        float s[NTS][4];
#pragma unroll
        for (int n = 0; n < NTS; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
            for (int n = 0; n < NTS; n += 2) {
                uint32_t b[4];
                ldmatrix_x4(b, sk + swz(n * 8 + (lane & 7) + ((lane >> 4) << 3),
                                        ks * 2 + ((lane >> 3) & 1), kRowB));
                mma_bf16_16816(s[n], qf[ks], b[0], b[1]);
                mma_bf16_16816(s[n + 1], qf[ks], b[2], b[3]);
            }
        }
        // scale + bias (log2 domain), mask, online softmax
        const float bias0 = sBias[(warp * 16 + g) * top + j];
        const float bias1 = sBias[(warp * 16 + g + 8) * top + j];
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < NTS; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = n * 8 + q2 + (e & 1);
                const float bb = (e < 2) ? bias0 : bias1;
                const float val = col < valid ? fmaf(s[n][e], scale_log2, bb) : -INFINITY;
                s[n][e] = val;
                mx[e >> 1] = fmaxf(mx[e >> 1], val);
            }
        }
        float alpha[2], mref[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float mnew = fmaxf(m_r[r], mx[r]);
            mref[r] = mnew == -INFINITY ? 0.0f : mnew;
            alpha[r] = exp2f(m_r[r] - mref[r]);
            m_r[r] = mnew;
            l_r[r] *= alpha[r];
        }
#pragma unroll
        for (int jn = 0; jn < NTO; ++jn) {
            o[jn][0] *= alpha[0];
            o[jn][1] *= alpha[0];
            o[jn][2] *= alpha[1];
            o[jn][3] *= alpha[1];
        }
        uint32_t pf[NTS / 2][4];
#pragma unroll
        for (int n = 0; n < NTS; ++n) {
            const float p0 = exp2f(s[n][0] - mref[0]);
            const float p1 = exp2f(s[n][1] - mref[0]);
            const float p2 = exp2f(s[n][2] - mref[1]);
            const float p3 = exp2f(s[n][3] - mref[1]);
            l_r[0] += p0 + p1;
            l_r[1] += p2 + p3;
            pf[n >> 1][(n & 1) * 2 + 0] = pack_bf16x2(p0, p1);
            pf[n >> 1][(n & 1) * 2 + 1] = pack_bf16x2(p2, p3);
        }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < NTS / 2; ++kk) {
            const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
            for (int jn = 0; jn < NTO; jn += 2) {
                uint32_t b[4];
                ldmatrix_x4_trans(b, sv + swz(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                              jn + (lane >> 4), kRowB));
                mma_bf16_16816(o[jn], a, b[0], b[1]);
                mma_bf16_16816(o[jn + 1], a, b[2], b[3]);
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();

    // finalize: O / l, stage through shared memory, 16-B stores
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
        l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
    }
    const float inv0 = l_r[0] > 0.0f ? 1.0f / l_r[0] : 0.0f;
    const float inv1 = l_r[1] > 0.0f ? 1.0f / l_r[1] : 0.0f;
    __syncthreads();
#pragma unroll
    for (int jn = 0; jn < NTO; ++jn) {
        const int r0 = warp * 16 + g;
        const int chk = jn, within = q2 * 2;   // byte offset inside the 16-B chunk
        *reinterpret_cast<uint32_t *>(sQ + swz(r0, chk, kRowB) + within) =
            pack_bf16x2(o[jn][0] * inv0, o[jn][1] * inv0);
        *reinterpret_cast<uint32_t *>(sQ + swz(r0 + 8, chk, kRowB) + within) =
            pack_bf16x2(o[jn][2] * inv1, o[jn][3] * inv1);
    }
    if ((lane & 3) == 0) {
        const int r0 = warp * 16 + g;
        const int t0 = sTok[r0], t1 = sTok[r0 + 8];
        if (t0 >= 0) lse[static_cast<int64_t>(h) * P.n + row0 + r0] = l_r[0] > 0.0f ? (m_r[0] + log2f(l_r[0])) * kLn2 : -INFINITY;
        if (t1 >= 0) lse[static_cast<int64_t>(h) * P.n + row0 + r0 + 8] = l_r[1] > 0.0f ? (m_r[1] + log2f(l_r[1])) * kLn2 : -INFINITY;
    }
    __syncthreads();
    for (int i = tid; i < kTileM * kChunks; i += kReadThreads) {
        const int r = i / kChunks, ch = i % kChunks;
        const int tok = sTok[r];
        if (tok >= 0)
            *reinterpret_cast<uint4 *>(out + tok * ld + h * HD + ch * 8) =
                *reinterpret_cast<const uint4 *>(sQ + swz(r, ch, kRowB));
    }
}

template <int HD>
static cudaError_t launch_fwd_t(const void *q, const void *k, const void *v, int H, int bs, int top,
                                const PlanLayout &L, const PlanView &P, void *out, float *lse,
                                cudaStream_t st) {
    const size_t smem = kTileM * HD * 2 + 4 * kSlotChunk * HD * 2 + kTileM * sizeof(int) +
                        kTileM * top * sizeof(float);
    auto kern = read_fwd_kernel<HD>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const float scale_log2 = kLog2e / sqrtf(static_cast<float>(HD));
    dim3 grid(static_cast<unsigned>(L.max_tiles), H);
    kern<<<grid, kReadThreads, smem, st>>>(static_cast<const uint16_t *>(q),
                                          static_cast<const uint16_t *>(k),
                                          static_cast<const uint16_t *>(v), H, bs, top, scale_log2, P,
                                          static_cast<uint16_t *>(out), lse); count_launch();
    return cudaGetLastError();
}

cudaError_t launch_read_fwd(const void *q, const void *k, const void *v, int B, int S, int H,
                            int hd, int nb, int bs, int top, const PlanLayout &L,
                            const PlanView &P, void *out, float *lse, void *q_rows, cudaStream_t st,
                            const int *iperm) {
    (void)B; (void)S; (void)nb;
    if (L.max_tiles == 0) return cudaSuccess;
    // q in plan order, for the tensor-core kernels of this call and of the backward
    cudaError_t e = iperm ? launch_split_permute_q(q, iperm, L.N / P.rows_per_q, P.rows_per_q,
                                                   static_cast<int64_t>(H) * hd * 2, q_rows, st)
                          : launch_permute_rows(q, L.N, static_cast<int64_t>(H) * hd * 2, P.perm, q_rows, st,
                                                P.rows_per_q);
    if (e != cudaSuccess) return e;
    // the tensor-core kernel covers 128-slot blocks with head_dim 64 (top <= 2)
    // or head_dim 128 (top 1: block-split plans); other geometries take the
    // warp-level mma kernel below
    if (read_fwd_tc_supported(hd, bs, top, q_rows, k, v, H))
        return launch_read_fwd_tc(q_rows, k, v, hd, H, nb, top, L, P, out, lse, st);
    if (hd == 64) return launch_fwd_t<64>(q, k, v, H, bs, top, L, P, out, lse, st);
    if (hd == 128) return launch_fwd_t<128>(q, k, v, H, bs, top, L, P, out, lse, st);
    return cudaErrorInvalidValue;
}

}  // namespace mom
