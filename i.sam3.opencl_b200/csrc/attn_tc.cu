// SPDX-License-Identifier: Unlicense
// Fused self-attention of the PE backbone on tcgen05 tensor cores: one
// kernel replaces the reference's QK^T gemm -> softmax_rows -> P.V gemm
// sequence on a materialised fp32 score buffer (sam3_model.c:1000-1013,
// sam3_kernels.cl:637-656), for 24x24 windows (N = 576) and for global
// attention over the whole grid (N = 5184) alike.
//
// Input: bf16 qkv rows [nseq * N, 3E] (RoPE already applied to q and k by
// the QKV GEMM epilogue or by k_rope_cast_bf16), head h at column h*64.
// A CTA owns one (sequence, head) and two 128-query tiles; the two tiles
// ping-pong so the tensor core works on one tile's S = Q K^T or O += P V
// while the other tile's softmax runs.
//
//   warps 0-3  softmax of query tile 0, warps 4-7 of tile 1 (one thread per
//              query row, TMEM lanes 32*(warp%4)...): online softmax in the
//              log2 domain (ex2), P as bf16 into 128B-swizzled smem, running
//              O accumulated in registers from each tile's P.V partial.
//   warp 8     TMA producer: Q tiles once, then K/V tiles of 192 keys
//              through a 2-stage ring.
//   warp 9     TMEM owner and MMA issuer.
//
// Tensor memory (512 columns): S0 [0,192) PV0 [192,256) S1 [256,448)
// PV1 [448,512), fp32.
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>

namespace sam3 {
namespace {

constexpr int HD = 64;
constexpr int BQ = 128;
constexpr int BKV = 192;
constexpr int kThreads = 320;
constexpr int Q_BYTES = BQ * HD * 2;     // 16 KB
constexpr int KV_BYTES = BKV * HD * 2;   // 24 KB per K or V tile
constexpr int P_SUB = BQ * 64 * 2;       // 16 KB: 128 rows x 64 keys
constexpr int P_BYTES = 3 * P_SUB;       // 48 KB
constexpr int OFF_Q = 0;
constexpr int OFF_KV = 2 * Q_BYTES;                      // 2 stages x (K, V)
constexpr int OFF_P = OFF_KV + 2 * 2 * KV_BYTES;         // 2 tiles
constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr int NBAR = 1 + 2 + 2 + 2 + 2 + 2 + 1;
constexpr int SMEM_BYTES = OFF_BAR + NBAR * 8 + 16 + 1024;
static_assert(SMEM_BYTES <= 232448, "attention smem");

struct AttnArgs {
    int nseq, N, E, heads;
    float scale_log2;
    void *out;
    int *err;
};

template <bool OUT_BF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmKV, const AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars;
    uint64_t *kv_full = bars + 1;
    uint64_t *kv_empty = bars + 3;
    uint64_t *s_full = bars + 5;
    uint64_t *p_ready = bars + 7;
    uint64_t *pv_full = bars + 9;
    uint64_t *drain = bars + 11;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int nqt = (a.N + BQ - 1) / BQ;
    const int npairs = (nqt + 1) / 2;
    const int pair = blockIdx.x % npairs;
    const int head = (blockIdx.x / npairs) % a.heads;
    const int seq = blockIdx.x / (npairs * a.heads);
    const int ntile = min(2, nqt - 2 * pair);
    const int nkv = (a.N + BKV - 1) / BKV;
    const int row0 = seq * a.N;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_ready[i], 4);
            mbar_init(&pv_full[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 9) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 8) {
        if (elect_one()) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmKV);
            mbar_arrive_expect_tx(q_full, ntile * Q_BYTES);
            for (int t = 0; t < ntile; t++)
                tma_load_2d(smem + OFF_Q + t * Q_BYTES, &tmQ, q_full, head * HD,
                            row0 + (2 * pair + t) * BQ);
            int last = -1;
            for (int j = 0; j < nkv; j++) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&kv_empty[st], ph ^ 1, a.err, abort_flag))
                    break;
                uint8_t *kv = smem + OFF_KV + st * 2 * KV_BYTES;
                mbar_arrive_expect_tx(&kv_full[st], 2 * KV_BYTES);
                tma_load_2d(kv, &tmKV, &kv_full[st], a.E + head * HD, row0 + j * BKV);
                tma_load_2d(kv + KV_BYTES, &tmKV, &kv_full[st], 2 * a.E + head * HD,
                            row0 + j * BKV);
                last = j;
            }
            // Let every issued copy land before the CTA can exit.
            volatile int no_abort = 0;
            mbar_wait(q_full, 0, a.err, &no_abort);
            for (int j = last > 0 ? last - 1 : 0; j <= last; j++)
                if (j >= 0)
                    mbar_wait(&kv_full[j & 1], (j >> 1) & 1, a.err, &no_abort);
        }
    }
    else if (warp == 9) {
        if (elect_one()) {
            constexpr uint32_t idS = idesc_bf16_f32(BQ, BKV, 0, 0);
            constexpr uint32_t idPV = idesc_bf16_f32(BQ, HD, 0, 1);
            const uint32_t sQ = smem_addr(smem + OFF_Q);
            const uint32_t sKV = smem_addr(smem + OFF_KV);
            const uint32_t sP = smem_addr(smem + OFF_P);
            bool ok = mbar_wait(q_full, 0, a.err, abort_flag) &&
                      mbar_wait(&kv_full[0], 0, a.err, abort_flag);
            if (ok) {
                tc_fence_after();
                for (int t = 0; t < ntile; t++) {
                    for (int k = 0; k < HD / 16; k++)
                        tc_mma(tmem_base + t * 256, sw128_desc(sQ + t * Q_BYTES + k * 32, 16, 1024),
                               sw128_desc(sKV + k * 32, 16, 1024), idS, k != 0);
                    tc_commit(&s_full[t]);
                }
            }
            for (int j = 0; j < nkv && ok; j++) {
                const uint32_t kvj = sKV + (j & 1) * 2 * KV_BYTES;
                const uint32_t kvn = sKV + ((j + 1) & 1) * 2 * KV_BYTES;
                for (int t = 0; t < ntile; t++) {
                    if (!mbar_wait(&p_ready[t], j & 1, a.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (j + 1 < nkv) {
                        if (t == 0 &&
                            !mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, a.err,
                                       abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        for (int k = 0; k < HD / 16; k++)
                            tc_mma(tmem_base + t * 256,
                                   sw128_desc(sQ + t * Q_BYTES + k * 32, 16, 1024),
                                   sw128_desc(kvn + k * 32, 16, 1024), idS, k != 0);
                        tc_commit(&s_full[t]);
                    }
                    const uint32_t pt = sP + t * P_BYTES;
                    for (int kk = 0; kk < BKV / 16; kk++)
                        tc_mma(tmem_base + t * 256 + BKV,
                               sw128_desc(pt + (kk >> 2) * P_SUB + (kk & 3) * 32, 16, 1024),
                               sw128_desc(kvj + KV_BYTES + kk * 2048, BKV * 128, 1024), idPV,
                               kk != 0);
                    tc_commit(&pv_full[t]);
                }
                if (ok)
                    tc_commit(&kv_empty[j & 1]);
            }
            tc_commit(drain);
            volatile int no_abort = 0;
            mbar_wait(drain, 0, a.err, &no_abort);
        }
    }
    else {
        const int t = warp >> 2;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // query row within the tile
        if (t < ntile) {
            const uint32_t tS = tmem_base + ((uint32_t)(quarter * 32) << 16) + t * 256;
            const uint32_t tPV = tS + BKV;
            const uint32_t pbase = smem_addr(smem + OFF_P + t * P_BYTES) + r * 128;
            const float sl2 = a.scale_log2;
            float o[HD];
#pragma unroll
            for (int d = 0; d < HD; d++)
                o[d] = 0.0f;
            float m_run = -INFINITY, l_run = 0.0f;
            bool ok = true;
            for (int j = 0; j < nkv; j++) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, a.err, abort_flag));
                if (!ok)
                    break;
                tc_fence_after();
                const int valid = a.N - j * BKV;
                // Only a sequence's last KV tile can hold keys beyond N.
                const bool masked = valid < BKV;
                // Pass 1: row maximum of the scaled scores (64 columns per
                // TMEM round trip, four independent max chains).
                float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll 1
                for (int c = 0; c < BKV / 32; c += 2) {
                    uint32_t s[64];
                    tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(s));
                    tmem_ld32(tS + c * 32 + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
                    tmem_wait_ld();
                    if (masked) {
#pragma unroll
                        for (int e = 0; e < 64; e++)
                            if (c * 32 + e >= valid)
                                s[e] = __float_as_uint(-INFINITY);
                    }
#pragma unroll
                    for (int e = 0; e < 64; e += 4) {
                        mx0 = fmaxf(mx0, __uint_as_float(s[e]));
                        mx1 = fmaxf(mx1, __uint_as_float(s[e + 1]));
                        mx2 = fmaxf(mx2, __uint_as_float(s[e + 2]));
                        mx3 = fmaxf(mx3, __uint_as_float(s[e + 3]));
                    }
                }
                const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
                const float m_new = fmaxf(m_run, mx * sl2);
                // Fold the previous tile's P.V (relative to m_run) into O.
                if (j > 0) {
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(&pv_full[t], (j - 1) & 1, a.err, abort_flag));
                    if (!ok)
                        break;
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < 2; c++) {
                        uint32_t pv[32];
                        tmem_ld32(tPV + c * 32, pv);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; e++)
                            o[c * 32 + e] += __uint_as_float(pv[e]);
                    }
                }
                if (m_new != m_run) {  // rescale only when the maximum moved
                    const float alpha = ex2_approx(m_run - m_new);
#pragma unroll
                    for (int d = 0; d < HD; d++)
                        o[d] *= alpha;
                    l_run *= alpha;
                }
                // Pass 2: P = 2^(s * scale_log2 - m_new) as bf16 into smem
                // (K-major, 128B swizzle: 16-byte chunk q of row r at
                // chunk q ^ (r & 7)); four independent row-sum chains.
                float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f, l3 = 0.0f;
#pragma unroll 1
                for (int c = 0; c < BKV / 32; c += 2) {
                    uint32_t s[64];
                    tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(s));
                    tmem_ld32(tS + c * 32 + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
                    tmem_wait_ld();
                    float p[64];
#pragma unroll
                    for (int e = 0; e < 64; e++)
                        p[e] = ex2_approx(fmaf(__uint_as_float(s[e]), sl2, -m_new));
                    if (masked) {
#pragma unroll
                        for (int e = 0; e < 64; e++)
                            if (c * 32 + e >= valid)
                                p[e] = 0.0f;
                    }
#pragma unroll
                    for (int e = 0; e < 64; e += 4) {
                        l0 += p[e];
                        l1 += p[e + 1];
                        l2 += p[e + 2];
                        l3 += p[e + 3];
                    }
                    const uint32_t sub = pbase + (c >> 1) * P_SUB;
#pragma unroll
                    for (int q = 0; q < 8; q++)
                        st_shared_v4(sub + ((q ^ (r & 7)) << 4),
                                     pack_bf16x2(p[q * 8 + 0], p[q * 8 + 1]),
                                     pack_bf16x2(p[q * 8 + 2], p[q * 8 + 3]),
                                     pack_bf16x2(p[q * 8 + 4], p[q * 8 + 5]),
                                     pack_bf16x2(p[q * 8 + 6], p[q * 8 + 7]));
                }
                l_run += (l0 + l1) + (l2 + l3);
                m_run = m_new;
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&p_ready[t]);
            }
            if (ok)
                ok = __all_sync(0xffffffffu,
                                mbar_wait(&pv_full[t], (nkv - 1) & 1, a.err, abort_flag));
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    uint32_t pv[32];
                    tmem_ld32(tPV + c * 32, pv);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e++)
                        o[c * 32 + e] += __uint_as_float(pv[e]);
                }
                const int q = (2 * pair + t) * BQ + r;
                if (q < a.N) {
                    const float inv = 1.0f / l_run;
                    const long orow = (long)(row0 + q) * a.E + head * HD;
                    if (OUT_BF16) {
                        uint4 *dst = reinterpret_cast<uint4 *>(
                            reinterpret_cast<__nv_bfloat16 *>(a.out) + orow);
#pragma unroll
                        for (int d = 0; d < HD; d += 8) {
                            uint4 v;
                            v.x = pack_bf16x2(o[d] * inv, o[d + 1] * inv);
                            v.y = pack_bf16x2(o[d + 2] * inv, o[d + 3] * inv);
                            v.z = pack_bf16x2(o[d + 4] * inv, o[d + 5] * inv);
                            v.w = pack_bf16x2(o[d + 6] * inv, o[d + 7] * inv);
                            dst[d / 8] = v;
                        }
                    }
                    else {
                        float4 *dst = reinterpret_cast<float4 *>(
                            reinterpret_cast<float *>(a.out) + orow);
#pragma unroll
                        for (int d = 0; d < HD; d += 4)
                            dst[d / 4] = make_float4(o[d] * inv, o[d + 1] * inv,
                                                     o[d + 2] * inv, o[d + 3] * inv);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

template <bool OUT_BF16>
int launch(const CUtensorMap &tq, const CUtensorMap &tkv, const AttnArgs &a, int grid,
           cudaStream_t s)
{
    auto kern = attn_tc_kernel<OUT_BF16>;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess)
        return (int)e;
    kern<<<grid, kThreads, SMEM_BYTES, s>>>(tq, tkv, a);
    return (int)cudaGetLastError();
}

}  // namespace
}  // namespace sam3

extern "C" int k_attn_tc(const void *qkv, int nseq, int N, int E, int heads, float scale,
                         void *out, int out_bf16, int *err, k_stream s)
{
    using namespace sam3;
    if (nseq <= 0 || N <= 0 || heads <= 0 || E != heads * HD ||
        (reinterpret_cast<uintptr_t>(out) & 15))
        return K_EARG;
    const uint64_t rows = (uint64_t)nseq * N;
    CUtensorMap tq, tkv;
    if (!make_tmap_bf16(&tq, qkv, rows, 3ull * E, 3ull * E, BQ) ||
        !make_tmap_bf16(&tkv, qkv, rows, 3ull * E, 3ull * E, BKV))
        return K_ETMAP;
    AttnArgs a;
    a.nseq = nseq;
    a.N = N;
    a.E = E;
    a.heads = heads;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.err = err;
    const int nqt = (N + BQ - 1) / BQ;
    const long grid = (long)nseq * heads * ((nqt + 1) / 2);
    if (grid > 0x7fffffffL)
        return K_EARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    return out_bf16 ? launch<true>(tq, tkv, a, (int)grid, st)
                    : launch<false>(tq, tkv, a, (int)grid, st);
}
