// SPDX-License-Identifier: Unlicense
// Fused self-attention of the PE backbone on tcgen05 tensor cores: one
// kernel replaces the reference's QK^T gemm -> softmax_rows -> P.V gemm
// sequence on a materialised fp32 score buffer (sam3_model.c:1000-1013,
// sam3_kernels.cl:637-656), for 24x24 windows (N = 576) and for global
// attention over the whole grid (N = 5184) alike.
//
// Input: bf16 qkv rows [nseq * N, 3E] (RoPE already applied to q and k by
// the QKV GEMM epilogue or by k_rope_cast_bf16), head h at column h*64.
// A CTA owns one (sequence, head) and two 128-query tiles that share the
// K/V stream. KV tiles hold 96 keys (576 = 6 x 96, 5184 = 54 x 96).
//
//   warps 0-3  softmax of query tile 0, warps 4-7 of tile 1 (one thread per
//              query row; warp w reads TMEM lanes 32*(w%4)...);
//   warp 8     TMA producers: lane 0 loads Q and the K ring, lane 1 the V
//              ring (two stages each);
//   warp 9     TMEM owner and MMA issuer.
//
// Tensor memory per query tile t (512 columns in all): two S buffers of 96
// fp32 columns at t*256 and t*256+96, and the output accumulator O (64
// columns) at t*256+192. Shared memory holds two P buffers per tile. Per
// tile the MMA order is S(0) S(1) | PV(0) S(2) | PV(1) S(3) | ...: S(j+2) is
// issued as soon as P(j) is handed over, so while the softmax works on tile
// j the scores of j+1 are already in TMEM, and P(j) is written into the
// buffer P.V(j-2) has long finished reading. The softmax therefore never
// waits for the tensor core unless the tensor core is the bottleneck.
//
// Softmax per KV tile (two TMEM passes of 32-column chunks): row maximum
// with three-input max; P = 2^(s * scale * log2 e - m) with 3/4 of the
// exponentials on the MUFU unit and 1/4 on the FMA pipe (exp2_poly2); row
// sums in packed fp32; P as bf16 into a 128B-swizzled K-major tile. The
// running maximum is only raised (and O rescaled in TMEM by 2^(m_old -
// m_new)) when the tile maximum exceeds it by more than 8 in log2 units, so
// P stays <= 2^8 and most tiles skip the rescale; the final division by the
// row sum makes the result independent of the offset used.
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>

namespace sam3 {
namespace {

constexpr int HD = 64;
constexpr int BQ = 128;
constexpr int BKV = 96;
constexpr int kSoftmaxWarps = 8;  // 2 tiles x 4 lane quarters
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 32 * 10;
// Of every 8 pairs of scores, this many take the FMA-pipe exponential
// (exp2_poly2) instead of the MUFU unit: MUFU ex2 runs at 16 lanes per clock
// per SM, against 256 MMA flops per score, so about a third of the
// exponentials must move to the FMA pipe for the MUFU not to bound the loop.
constexpr int kPolyPairsPer16 = 3;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int Q_BYTES = BQ * HD * 2;     // 16 KB
constexpr int KV_BYTES = BKV * HD * 2;   // 12 KB per K or V tile
constexpr int P_SUB = BQ * 128;          // one 64-key swizzle atom: 128 rows x 128 B
constexpr int P_BYTES = 2 * P_SUB;       // keys 0-63 and 64-95 (second atom half used)
constexpr int OFF_Q = 0;
constexpr int OFF_K = 2 * Q_BYTES;               // K ring, 2 stages
constexpr int OFF_V = OFF_K + 2 * KV_BYTES;      // V ring, 2 stages
constexpr int OFF_P = OFF_V + 2 * KV_BYTES;      // [tile][buffer]
constexpr int OFF_BAR = OFF_P + 4 * P_BYTES;
// q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2][2],
// s_free[2][2], p_ready[2][2], pv_full[2][2], drain. Every barrier that a
// waiter could see advance by two phases before it looks (the softmax may
// finish KV tiles j and j+1 before the MMA warp consumes P(j)) is split per
// buffer, so consecutive uses alternate between two barriers and a parity
// wait never aliases.
constexpr int NBAR = 1 + 8 + 4 + 4 + 4 + 4 + 1;
constexpr int SMEM_BYTES = OFF_BAR + NBAR * 8 + 16 + 1024;
static_assert(SMEM_BYTES <= 232448, "attention smem");
static_assert(OFF_K % 1024 == 0 && OFF_V % 1024 == 0 && OFF_P % 1024 == 0 &&
                  KV_BYTES % 1024 == 0,
              "alignment");

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
    uint64_t *k_full = bars + 1;
    uint64_t *k_empty = k_full + 2;
    uint64_t *v_full = k_empty + 2;
    uint64_t *v_empty = v_full + 2;
    uint64_t *s_full = v_empty + 2;   // [tile * 2 + buffer]
    uint64_t *s_free = s_full + 4;    // [tile * 2 + buffer]
    uint64_t *p_ready = s_free + 4;   // [tile * 2 + buffer]
    uint64_t *pv_full = p_ready + 4;  // [tile * 2 + buffer]
    uint64_t *drain = pv_full + 4;
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
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 4; i++) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
            mbar_init(&p_ready[i], 4);
            mbar_init(&pv_full[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kProducerWarp) {
        // Two independent single-thread producers (diverged lanes).
        if (lane < 2) {
            const bool is_k = lane == 0;
            if (is_k) {
                prefetch_tmap(&tmQ);
                prefetch_tmap(&tmKV);
                mbar_arrive_expect_tx(q_full, ntile * Q_BYTES);
                for (int t = 0; t < ntile; t++)
                    tma_load_2d(smem + OFF_Q + t * Q_BYTES, &tmQ, q_full, head * HD,
                                row0 + (2 * pair + t) * BQ);
            }
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *empty = is_k ? k_empty : v_empty;
            uint8_t *ring = smem + (is_k ? OFF_K : OFF_V);
            const int col = (is_k ? a.E : 2 * a.E) + head * HD;
            int last = -1;
            for (int j = 0; j < nkv; j++) {
                const int st = j & 1;
                if (!mbar_wait(&empty[st], ((j >> 1) & 1) ^ 1, a.err, abort_flag))
                    break;
                mbar_arrive_expect_tx(&full[st], KV_BYTES);
                tma_load_2d(ring + st * KV_BYTES, &tmKV, &full[st], col, row0 + j * BKV);
                last = j;
            }
            // Let every issued copy land before the CTA can exit.
            volatile int no_abort = 0;
            if (is_k)
                mbar_wait(q_full, 0, a.err, &no_abort);
            for (int j = last - 1; j <= last; j++)
                if (j >= 0)
                    mbar_wait(&full[j & 1], (j >> 1) & 1, a.err, &no_abort);
        }
    }
    else if (warp == kMmaWarp) {
        if (elect_one()) {
            constexpr uint32_t idS = idesc_bf16_f32(BQ, BKV, 0, 0);
            constexpr uint32_t idPV = idesc_bf16_f32(BQ, HD, 0, 1);
            const uint32_t sQ = smem_addr(smem + OFF_Q);
            const uint32_t sK = smem_addr(smem + OFF_K);
            const uint32_t sV = smem_addr(smem + OFF_V);
            const uint32_t sP = smem_addr(smem + OFF_P);
            // S_t(jj) = Q_t K(jj)^T into S buffer jj % 2 (K ring stage jj % 2).
            auto issue_s = [&](int t, int jj) {
                const uint32_t kj = sK + (jj & 1) * KV_BYTES;
                for (int k = 0; k < HD / 16; k++)
                    tc_mma(tmem_base + t * 256 + (jj & 1) * BKV,
                           sw128_desc(sQ + t * Q_BYTES + k * 32, 16, 1024),
                           sw128_desc(kj + k * 32, 16, 1024), idS, k != 0);
                tc_commit(&s_full[t * 2 + (jj & 1)]);
            };
            bool ok = mbar_wait(q_full, 0, a.err, abort_flag);
            for (int jj = 0; ok && jj < 2 && jj < nkv; jj++) {
                ok = mbar_wait(&k_full[jj], 0, a.err, abort_flag);
                if (!ok)
                    break;
                tc_fence_after();
                for (int t = 0; t < ntile; t++)
                    issue_s(t, jj);
                tc_commit(&k_empty[jj]);
            }
            for (int j = 0; ok && j < nkv; j++) {
                const int b = j & 1;
                if (!mbar_wait(&v_full[b], (j >> 1) & 1, a.err, abort_flag)) {
                    ok = false;
                    break;
                }
                const uint32_t vj = sV + b * KV_BYTES;
                for (int t = 0; t < ntile; t++) {
                    if (!mbar_wait(&p_ready[t * 2 + b], (j >> 1) & 1, a.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // O_t += P_t(j) V(j), P buffer b.
                    const uint32_t pt = sP + (t * 2 + b) * P_BYTES;
                    for (int kk = 0; kk < BKV / 16; kk++)
                        tc_mma(tmem_base + t * 256 + 2 * BKV,
                               sw128_desc(pt + (kk >> 2) * P_SUB + (kk & 3) * 32, 16, 1024),
                               sw128_desc(vj + kk * 2048, BKV * 128, 1024), idPV,
                               (j | kk) != 0);
                    tc_commit(&pv_full[t * 2 + b]);
                    if (j + 2 < nkv) {
                        // S(j+2) into the buffer the softmax read S(j) from.
                        if ((t == 0 && !mbar_wait(&k_full[b], ((j + 2) >> 1) & 1, a.err,
                                                  abort_flag)) ||
                            !mbar_wait(&s_free[t * 2 + b], (j >> 1) & 1, a.err, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        issue_s(t, j + 2);
                    }
                }
                if (!ok)
                    break;
                tc_commit(&v_empty[b]);
                if (j + 2 < nkv)
                    tc_commit(&k_empty[b]);
            }
            tc_commit(drain);
            volatile int no_abort = 0;
            mbar_wait(drain, 0, a.err, &no_abort);
        }
    }
    else if (warp < kSoftmaxWarps) {
        const int t = warp >> 2;           // query tile
        const int quarter = warp & 3;      // TMEM lane quarter = rows 32q..32q+31
        const int r = quarter * 32 + lane; // query row within the tile
        if (t < ntile) {
            const uint32_t tT = tmem_base + ((uint32_t)(quarter * 32) << 16) + t * 256;
            const uint32_t tO = tT + 2 * BKV;
            const uint32_t prow = smem_addr(smem + OFF_P + t * 2 * P_BYTES) + r * 128;
            const float sl2 = a.scale_log2;
            const uint64_t sl2x2 = f2_make(sl2, sl2);
            // Warps whose 32 query rows all lie beyond N (the second half of a
            // sequence's last 128-row tile when N % 128 == 64) keep the barrier
            // protocol but skip the softmax work: their rows are never stored.
            const bool rows_live = (2 * pair + t) * BQ + quarter * 32 < a.N;
            float m_used = -INFINITY;
            uint64_t lsum0 = 0, lsum1 = 0;  // packed partial row sums
            bool ok = true;
            for (int j = 0; j < nkv; j++) {
                const int b = j & 1;
                ok = __all_sync(0xffffffffu,
                                mbar_wait(&s_full[t * 2 + b], (j >> 1) & 1, a.err, abort_flag));
                if (!ok)
                    break;
                tc_fence_after();
                // The whole 96-score row in one TMEM round trip; the S buffer
                // is handed back at once for S(j+2).
                uint32_t s[BKV];
                tmem_ld32(tT + b * BKV, *reinterpret_cast<uint32_t(*)[32]>(s));
                tmem_ld32(tT + b * BKV + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
                tmem_ld32(tT + b * BKV + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64));
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&s_free[t * 2 + b]);

                const int valid = a.N - j * BKV;
                const bool masked = valid < BKV;  // only a sequence's last tile
                bool resc = false;
                float factor = 1.0f;
                if (rows_live) {
                    if (masked) {
#pragma unroll
                        for (int e = 0; e < BKV; e++)
                            if (e >= valid)
                                s[e] = __float_as_uint(-INFINITY);
                    }
                    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                    for (int e = 0; e < BKV; e += 4) {
                        mx0 = max3f(mx0, __uint_as_float(s[e]), __uint_as_float(s[e + 1]));
                        mx1 = max3f(mx1, __uint_as_float(s[e + 2]), __uint_as_float(s[e + 3]));
                    }
                    const float m_tile = fmaxf(mx0, mx1) * sl2;
                    if (m_used == -INFINITY) {
                        m_used = m_tile;  // first tile: O is still empty
                    }
                    else if (m_tile > m_used + kRescaleThreshold) {
                        resc = true;
                        factor = ex2_approx(m_used - m_tile);
                        m_used = m_tile;
                        const uint64_t f2v = f2_make(factor, factor);
                        lsum0 = mul2(lsum0, f2v);
                        lsum1 = mul2(lsum1, f2v);
                    }
                }
                // P buffer b was last read by P.V(j-2).
                if (j >= 2) {
                    ok = __all_sync(0xffffffffu, mbar_wait(&pv_full[t * 2 + b],
                                                           ((j - 2) >> 1) & 1, a.err, abort_flag));
                    if (!ok)
                        break;
                    tc_fence_after();
                }
                if (rows_live) {
                    // P = 2^(s * scale_log2 - m_used), in place.
                    const uint64_t negm = f2_make(-m_used, -m_used);
#pragma unroll
                    for (int e = 0; e < BKV; e += 2) {
                        const uint64_t x2 = fma2(f2_make(__uint_as_float(s[e]),
                                                         __uint_as_float(s[e + 1])),
                                                 sl2x2, negm);
                        float x0, x1, p0, p1;
                        f2_split(x2, x0, x1);
                        if (((e >> 1) & 7) >= 8 - kPolyPairsPer16)
                            exp2_poly2(x0, x1, p0, p1);
                        else {
                            p0 = ex2_approx(x0);
                            p1 = ex2_approx(x1);
                        }
                        s[e] = __float_as_uint(p0);
                        s[e + 1] = __float_as_uint(p1);
                    }
                    if (masked) {
#pragma unroll
                        for (int e = 0; e < BKV; e++)
                            if (e >= valid)
                                s[e] = 0;
                    }
#pragma unroll
                    for (int e = 0; e < BKV; e += 4) {
                        lsum0 = add2(lsum0, f2_make(__uint_as_float(s[e]), __uint_as_float(s[e + 1])));
                        lsum1 = add2(lsum1,
                                     f2_make(__uint_as_float(s[e + 2]), __uint_as_float(s[e + 3])));
                    }
                    // P row as bf16, K-major 128B swizzle: 16-byte chunk q of
                    // row r at chunk position q ^ (r & 7); keys 0-63 in the
                    // first atom, 64-95 in the second.
                    const uint32_t pb = prow + b * P_BYTES;
#pragma unroll
                    for (int q = 0; q < BKV / 8; q++) {
                        const uint32_t dst = pb + (q >> 3) * P_SUB + (((q & 7) ^ (r & 7)) << 4);
                        const uint32_t *v = s + q * 8;
                        st_shared_v4(dst,
                                     pack_bf16x2(__uint_as_float(v[0]), __uint_as_float(v[1])),
                                     pack_bf16x2(__uint_as_float(v[2]), __uint_as_float(v[3])),
                                     pack_bf16x2(__uint_as_float(v[4]), __uint_as_float(v[5])),
                                     pack_bf16x2(__uint_as_float(v[6]), __uint_as_float(v[7])));
                    }
                    fence_proxy_async_smem();
                }
                // A raised maximum rescales O (after P is out of the registers), which
                // needs P.V(j-1) done; P.V(j) is only issued after p_ready below.
                if (__any_sync(0xffffffffu, resc)) {
                    const int jp = j - 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&pv_full[t * 2 + (jp & 1)],
                                                           (jp >> 1) & 1, a.err, abort_flag));
                    if (!ok)
                        break;
                    tc_fence_after();
                    const uint64_t f2v = f2_make(factor, factor);
#pragma unroll
                    for (int c = 0; c < 2; c++) {
                        uint32_t o[32];
                        tmem_ld32(tO + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            float o0, o1;
                            f2_split(mul2(f2_make(__uint_as_float(o[e]),
                                                  __uint_as_float(o[e + 1])),
                                          f2v),
                                     o0, o1);
                            o[e] = __float_as_uint(o0);
                            o[e + 1] = __float_as_uint(o1);
                        }
                        tmem_st32(tO + c * 32, o);
                    }
                    tmem_wait_st();
                }
                // P(j) is ready for the MMA.
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&p_ready[t * 2 + b]);
            }
            if (ok) {
                const int jl = nkv - 1;
                ok = __all_sync(0xffffffffu, mbar_wait(&pv_full[t * 2 + (jl & 1)],
                                                       (jl >> 1) & 1, a.err, abort_flag));
            }
            if (ok && rows_live) {
                tc_fence_after();
                uint32_t ov[64];
                tmem_ld32(tO, *reinterpret_cast<uint32_t(*)[32]>(ov));
                tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(ov + 32));
                tmem_wait_ld();
                float la, lb, lc, ld;
                f2_split(lsum0, la, lb);
                f2_split(lsum1, lc, ld);
                const float inv = 1.0f / ((la + lb) + (lc + ld));
                const int q = (2 * pair + t) * BQ + r;
                if (q < a.N) {
                    const long orow = (long)(row0 + q) * a.E + head * HD;
                    if (OUT_BF16) {
                        uint4 *dst = reinterpret_cast<uint4 *>(
                            reinterpret_cast<__nv_bfloat16 *>(a.out) + orow);
#pragma unroll
                        for (int d = 0; d < HD; d += 8) {
                            uint4 w;
                            w.x = pack_bf16x2(__uint_as_float(ov[d]) * inv,
                                              __uint_as_float(ov[d + 1]) * inv);
                            w.y = pack_bf16x2(__uint_as_float(ov[d + 2]) * inv,
                                              __uint_as_float(ov[d + 3]) * inv);
                            w.z = pack_bf16x2(__uint_as_float(ov[d + 4]) * inv,
                                              __uint_as_float(ov[d + 5]) * inv);
                            w.w = pack_bf16x2(__uint_as_float(ov[d + 6]) * inv,
                                              __uint_as_float(ov[d + 7]) * inv);
                            dst[d / 8] = w;
                        }
                    }
                    else {
                        float4 *dst = reinterpret_cast<float4 *>(
                            reinterpret_cast<float *>(a.out) + orow);
#pragma unroll
                        for (int d = 0; d < HD; d += 4)
                            dst[d / 4] = make_float4(
                                __uint_as_float(ov[d]) * inv, __uint_as_float(ov[d + 1]) * inv,
                                __uint_as_float(ov[d + 2]) * inv,
                                __uint_as_float(ov[d + 3]) * inv);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
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
