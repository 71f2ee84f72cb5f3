// SPDX-License-Identifier: Unlicense
// Fused self-attention of the PE backbone on tcgen05 tensor cores: one
// kernel replaces the reference's QK^T gemm -> softmax_rows -> P.V gemm
// sequence on a materialised fp32 score buffer (sam3_model.c:1000-1013,
// sam3_kernels.cl:637-656), for 24x24 windows (N = 576) and for global
// attention over the whole grid (N = 5184) alike.
//
// Input: bf16 qkv rows [nseq * N, 3E] (RoPE already applied to q and k by
// the QKV GEMM epilogue or by k_rope_cast_bf16), head h at column h*64.
//
// Work items are (sequence, head, 128-query tile), query tile fastest so
// that CTAs running at the same time share a head's K/V in L2. Two CTAs run
// on each SM, each persistent (CTA c takes items c, c + grid, ...) with its
// own MMA thread and K/V stream: the two pipelines drift apart in phase, so
// one CTA's softmax runs while the other's tensor-core work or loads do, and
// a short launch balances at the granularity of one tile. KV tiles hold 96
// keys (576 = 6 x 96, 5184 = 54 x 96). Rows of a tail tile beyond N (576 =
// 4.5 x 128) run through the tensor core, but their softmax work is skipped
// and nothing is stored.
//
//   warps 0-3  softmax, one thread per query row (warp w reads TMEM lanes
//              32w..32w+31);
//   warp 4     TMA producers: lane 0 loads Q (two buffers, so the next
//              item's Q arrives early) and the K ring, lane 1 the V ring
//              (three stages each);
//   warp 5     TMEM owner (256 columns) and MMA issuer.
//
// Tensor memory: two score buffers of 96 fp32 columns (S(g) in buffer g % 2,
// g counting this CTA's KV tiles across items) and the output accumulator O
// (64 columns) at column 192, reset by the first P.V of each item. The
// softmax writes P(g) as bf16 pairs into the first 48 columns of the buffer
// it read S(g) from, P.V(g) takes its A operand from there, and S(g + 2) is
// issued into the same buffer right after P.V(g) (tensor-core operations of
// one thread run in issue order): the scores of the next KV tile are always
// ready when the softmax finishes one.
//
// Softmax per KV tile, one pass: the row's 96 scores in one TMEM round
// trip; x = s * scale * log2 e - m in packed fp32; 2^x on the MUFU unit, 2
// of 8 pairs on the FMA pipe (exp2_poly2); tile sums in packed fp32; P
// packed to bf16 pairs. The offset m is the row maximum of the item's first
// KV tile and is kept for the following tiles without taking their maxima
// (a dependent 48-step chain per tile): P may then exceed 1, which bf16 and
// the fp32 sums carry without loss. A tile whose row sum reaches 2^13 (a
// score that far above the offset, or an inf) is taken again: its scores
// are reloaded from TMEM (P is only written back afterwards), m is raised to
// the tile maximum and O and the sums are rescaled by 2^(m_old - m_new)
// once the previous P.V has finished. The final division by the row sum
// makes the result independent of the offset used.
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>

namespace sam3 {
namespace {

constexpr int HD = 64;
constexpr int BQ = 128;
constexpr int BKV = 96;
constexpr int KST = 3;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kThreads = 32 * 6;
constexpr int kCtasPerSm = 2;
// Of every 8 pairs of scores, this many take the FMA-pipe exponential
// (exp2_poly2) instead of two MUFU instructions: the MUFU unit runs 16
// exponentials per clock per SM against 256 MMA flops per score.
constexpr int kPolyPairsPer8 = 2;
// A row's tile sum at or above this (some P >= 2^13, or inf / NaN) sends
// the tile through the maximum pass again with a raised offset.
constexpr float kOverflowSum = 8192.0f;
constexpr int Q_BYTES = BQ * HD * 2;
constexpr int KV_BYTES = BKV * HD * 2;
constexpr int OFF_Q = 0;                       // [buffer], one query tile each
constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
constexpr int OFF_V = OFF_K + KST * KV_BYTES;
constexpr int OFF_BAR = OFF_V + KST * KV_BYTES;
constexpr uint32_t TM_O = 2 * BKV;             // O at columns 192..255
constexpr uint32_t TM_COLS = 256;              // per CTA: two CTAs share the 512
// q_full[2], q_empty[2], k_full[KST], k_empty[KST], v_full[KST],
// v_empty[KST], s_full[2], p_ready[2], pv_full[2], drain. Score buffer b is
// refilled (S(g + 2)) only after P.V(g), which needs the softmax's p_ready(g),
// so no waiter finds a barrier two phases ahead; pv_full waits (rescale,
// item end) follow s_full(g), which already implies P.V(g - 2) is done.
constexpr int NBAR = 4 + 4 * KST + 2 + 2 + 2 + 1;
constexpr int SMEM_BYTES = OFF_BAR + NBAR * 8 + 16 + 1024;
static_assert(kCtasPerSm * SMEM_BYTES <= 232448, "two CTAs per SM");
static_assert(TM_O + HD <= TM_COLS && kCtasPerSm * TM_COLS <= 512, "tensor memory");

struct AttnArgs {
    int nseq, N, E, heads, nqt, nitems;
    float scale_log2;
    void *out;
    int *err;
};

template <bool OUT_BF16>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                 const AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars, *q_empty = q_full + 2;
    uint64_t *k_full = q_empty + 2, *k_empty = k_full + KST;
    uint64_t *v_full = k_empty + KST, *v_empty = v_full + KST;
    uint64_t *s_full = v_empty + KST, *p_ready = s_full + 2, *pv_full = p_ready + 2;
    uint64_t *drain = pv_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkv = (a.N + BKV - 1) / BKV;
    const int nmine = (int)blockIdx.x < a.nitems
                          ? (a.nitems - 1 - (int)blockIdx.x) / (int)gridDim.x + 1
                          : 0;
    const int total = nmine * nkv;
    auto coords = [&](int k, int &seq, int &head, int &qt) {
        const int item = (int)blockIdx.x + k * (int)gridDim.x;
        qt = item % a.nqt;
        head = (item / a.nqt) % a.heads;
        seq = item / (a.nqt * a.heads);
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_ready[i], 4);
            mbar_init(&pv_full[i], 1);
        }
        for (int i = 0; i < KST; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, TM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kProducerWarp) {
        if (lane < 2) {
            const bool is_k = lane == 0;
            if (is_k) {
                prefetch_tmap(&tmQ);
                prefetch_tmap(&tmKV);
            }
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *empty = is_k ? k_empty : v_empty;
            uint8_t *ring = smem + (is_k ? OFF_K : OFF_V);
            int lastq = -1, lastg = -1, st = 0, use = 0;
            bool ok = true;
            for (int k = 0; k < nmine && ok; k++) {
                int seq, head, qt;
                coords(k, seq, head, qt);
                const int row0 = seq * a.N;
                if (is_k) {
                    if (!mbar_wait(&q_empty[k & 1], ((k >> 1) & 1) ^ 1, a.err, abort_flag))
                        break;
                    mbar_arrive_expect_tx(&q_full[k & 1], Q_BYTES);
                    tma_load_2d(smem + OFF_Q + (k & 1) * Q_BYTES, &tmQ, &q_full[k & 1], head * HD,
                                row0 + qt * BQ);
                    lastq = k;
                }
                const int col = (is_k ? a.E : 2 * a.E) + head * HD;
                for (int j = 0; j < nkv; j++) {
                    if (!mbar_wait(&empty[st], (use & 1) ^ 1, a.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[st], KV_BYTES);
                    tma_load_2d(ring + st * KV_BYTES, &tmKV, &full[st], col, row0 + j * BKV);
                    lastg = k * nkv + j;
                    if (++st == KST) {
                        st = 0;
                        use++;
                    }
                }
            }
            volatile int no_abort = 0;
            for (int k = lastq - 1; k <= lastq; k++)
                if (k >= 0)
                    mbar_wait(&q_full[k & 1], (k >> 1) & 1, a.err, &no_abort);
            for (int g = lastg - (KST - 1); g <= lastg; g++)
                if (g >= 0)
                    mbar_wait(&full[g % KST], (g / KST) & 1, a.err, &no_abort);
        }
    }
    else if (warp == kMmaWarp) {
        if (elect_one() && total > 0) {
            constexpr uint32_t idS = idesc_bf16_f32(BQ, BKV, 0, 0);
            constexpr uint32_t idPV = idesc_bf16_f32(BQ, HD, 0, 1);
            const uint64_t dQ = sw128_desc(smem_addr(smem + OFF_Q), 16, 1024);
            const uint64_t dK = sw128_desc(smem_addr(smem + OFF_K), 16, 1024);
            const uint64_t dV = sw128_desc(smem_addr(smem + OFF_V), BKV * 128, 1024);
            // cursor for S (ahead) and for P.V (cur): g, kst/kph, j, k
            struct Cur {
                int g, kst, kph, j, k;
            };
            auto adv = [&](Cur &c) {
                c.g++;
                if (++c.kst == KST) {
                    c.kst = 0;
                    c.kph ^= 1;
                }
                if (++c.j == nkv) {
                    c.j = 0;
                    c.k++;
                }
            };
            auto issue_s = [&](const Cur &c) -> bool {
                if (!mbar_wait(&k_full[c.kst], c.kph, a.err, abort_flag))
                    return false;
                if (c.j == 0 && !mbar_wait(&q_full[c.k & 1], (c.k >> 1) & 1, a.err, abort_flag))
                    return false;
                tc_fence_after();
                const uint64_t qd = dQ + (uint64_t)(((c.k & 1) * Q_BYTES) >> 4);
                const uint64_t kd = dK + (uint64_t)((c.kst * KV_BYTES) >> 4);
                const uint32_t dS = tmem_base + (c.g & 1) * BKV;
#pragma unroll
                for (int kq = 0; kq < HD / 16; kq++)
                    tc_mma(dS, qd + 2 * kq, kd + 2 * kq, idS, kq != 0);
                tc_commit(&s_full[c.g & 1]);
                tc_commit(&k_empty[c.kst]);
                if (c.j == nkv - 1)
                    tc_commit(&q_empty[c.k & 1]);
                return true;
            };
            auto issue_pv = [&](const Cur &c) -> bool {
                if (!mbar_wait(&v_full[c.kst], c.kph, a.err, abort_flag))
                    return false;
                if (!mbar_wait(&p_ready[c.g & 1], (c.g >> 1) & 1, a.err, abort_flag))
                    return false;
                tc_fence_after();
                const uint64_t vd = dV + (uint64_t)((c.kst * KV_BYTES) >> 4);
                const uint32_t aP = tmem_base + (c.g & 1) * BKV;
#pragma unroll
                for (int kk = 0; kk < BKV / 16; kk++)
                    tc_mma_ts(tmem_base + TM_O, aP + kk * 8, vd + 128 * kk, idPV, (c.j | kk) != 0);
                tc_commit(&pv_full[c.g & 1]);
                tc_commit(&v_empty[c.kst]);
                return true;
            };
            Cur ahead = {0, 0, 0, 0, 0}, cur = ahead;
            bool ok = true;
            for (int i = 0; ok && i < 2 && ahead.g < total; i++) {
                ok = issue_s(ahead);
                adv(ahead);
            }
            while (ok && cur.g < total) {
                ok = issue_pv(cur);
                if (ok && ahead.g < total) {
                    ok = issue_s(ahead);
                    adv(ahead);
                }
                adv(cur);
            }
            tc_commit(drain);
            volatile int no_abort = 0;
            mbar_wait(drain, 0, a.err, &no_abort);
        }
    }
    else {  // softmax warps 0-3, warp = TMEM lane quarter
        const int quarter = warp;
        const int r = quarter * 32 + lane;
        const uint32_t tL = tmem_base + ((uint32_t)(quarter * 32) << 16);
        const uint32_t tO = tL + TM_O;
        const float sl2 = a.scale_log2;
        const uint64_t sl2x2 = f2_make(sl2, sl2);
        bool ok = true;
        int g = 0;
        for (int k = 0; k < nmine && ok; k++) {
            int seq, head, qt;
            coords(k, seq, head, qt);
            const bool rows_live = qt * BQ + quarter * 32 < a.N;
            float m_used = -INFINITY;
            uint64_t lsum0 = 0, lsum1 = 0;
            for (int j = 0; j < nkv; j++, g++) {
                const int b = g & 1;
                ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (g >> 1) & 1, a.err, abort_flag));
                if (!ok)
                    break;
                tc_fence_after();
                const uint32_t tS = tL + b * BKV;
                bool resc = false;
                float factor = 1.0f;
                if (rows_live) {
                    uint32_t s[BKV];
#pragma unroll
                    for (int c = 0; c < BKV / 32; c++)
                        tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
                    tmem_wait_ld();
                    const int valid = a.N - j * BKV;
                    if (valid < BKV) {
#pragma unroll
                        for (int e = 0; e < BKV; e++)
                            if (e >= valid)
                                s[e] = __float_as_uint(-INFINITY);
                    }
                    // Pass 0 takes the exponentials against the running
                    // offset m_used, which only the item's first tile sets
                    // from its maximum. If a value reached 2^13 (tile sum
                    // check), pass 1 reloads the scores, raises m_used to
                    // the tile maximum and takes them again.
                    uint64_t t0, t1;
#pragma unroll 1
                    for (int pass = 0;; pass++) {
                        if (m_used == -INFINITY || pass == 1) {
                            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                            for (int e = 0; e < BKV; e += 4) {
                                mx0 = max3f(mx0, __uint_as_float(s[e]), __uint_as_float(s[e + 1]));
                                mx1 = max3f(mx1, __uint_as_float(s[e + 2]), __uint_as_float(s[e + 3]));
                            }
                            const float m_tile = fmaxf(mx0, mx1) * sl2;
                            if (m_used == -INFINITY)
                                m_used = m_tile;
                            else if (m_tile > m_used) {
                                resc = true;
                                factor = ex2_approx(m_used - m_tile);
                                m_used = m_tile;
                                lsum0 = mul2(lsum0, f2_make(factor, factor));
                                lsum1 = mul2(lsum1, f2_make(factor, factor));
                            }
                        }
                        const uint64_t negm = f2_make(-m_used, -m_used);
                        t0 = 0;
                        t1 = 0;
#pragma unroll
                        for (int e = 0; e < BKV; e += 2) {
                            const uint64_t x2 = fma2(f2_make(__uint_as_float(s[e]),
                                                             __uint_as_float(s[e + 1])),
                                                     sl2x2, negm);
                            float x0, x1, p0, p1;
                            f2_split(x2, x0, x1);
                            if (((e >> 1) & 7) >= 8 - kPolyPairsPer8)
                                exp2_poly2(x0, x1, p0, p1);
                            else {
                                p0 = ex2_approx(x0);
                                p1 = ex2_approx(x1);
                            }
                            if ((e >> 1) & 1)
                                t1 = add2(t1, f2_make(p0, p1));
                            else
                                t0 = add2(t0, f2_make(p0, p1));
                            s[e >> 1] = pack_bf16x2(p0, p1);
                        }
                        float u0, u1, u2, u3;
                        f2_split(t0, u0, u1);
                        f2_split(t1, u2, u3);
                        const bool over = !(((u0 + u1) + (u2 + u3)) < kOverflowSum);
                        if (pass == 1 || !__any_sync(0xffffffffu, over))
                            break;
#pragma unroll
                        for (int c = 0; c < BKV / 32; c++)
                            tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
                        tmem_wait_ld();
                        if (valid < BKV) {
#pragma unroll
                            for (int e = 0; e < BKV; e++)
                                if (e >= valid)
                                    s[e] = __float_as_uint(-INFINITY);
                        }
                    }
                    lsum0 = add2(lsum0, t0);
                    lsum1 = add2(lsum1, t1);
                    tmem_st32(tS, *reinterpret_cast<const uint32_t(*)[32]>(s));
                    tmem_st16(tS + 32, *reinterpret_cast<const uint32_t(*)[16]>(s + 32));
                }
                if (__any_sync(0xffffffffu, resc)) {
                    const int gp = g - 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&pv_full[gp & 1], (gp >> 1) & 1, a.err,
                                                           abort_flag));
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
                            f2_split(mul2(f2_make(__uint_as_float(o[e]), __uint_as_float(o[e + 1])),
                                          f2v),
                                     o0, o1);
                            o[e] = __float_as_uint(o0);
                            o[e + 1] = __float_as_uint(o1);
                        }
                        tmem_st32(tO + c * 32, o);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&p_ready[b]);
            }
            if (!ok)
                break;
            {
                const int gl = g - 1;
                ok = __all_sync(0xffffffffu,
                                mbar_wait(&pv_full[gl & 1], (gl >> 1) & 1, a.err, abort_flag));
                if (!ok)
                    break;
            }
            if (rows_live) {
                tc_fence_after();
                uint32_t ov[64];
                tmem_ld32(tO, *reinterpret_cast<uint32_t(*)[32]>(ov));
                tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(ov + 32));
                tmem_wait_ld();
                float la, lb, lc, ld;
                f2_split(lsum0, la, lb);
                f2_split(lsum1, lc, ld);
                const float inv = 1.0f / ((la + lb) + (lc + ld));
                const int q = qt * BQ + r;
                if (q < a.N) {
                    const long orow = (long)(seq * a.N + q) * a.E + head * HD;
                    if (OUT_BF16) {
                        uint4 *dst = reinterpret_cast<uint4 *>(
                            reinterpret_cast<__nv_bfloat16 *>(a.out) + orow);
#pragma unroll
                        for (int d = 0; d < HD; d += 8) {
                            uint4 w;
                            w.x = pack_bf16x2(__uint_as_float(ov[d]) * inv, __uint_as_float(ov[d + 1]) * inv);
                            w.y = pack_bf16x2(__uint_as_float(ov[d + 2]) * inv, __uint_as_float(ov[d + 3]) * inv);
                            w.z = pack_bf16x2(__uint_as_float(ov[d + 4]) * inv, __uint_as_float(ov[d + 5]) * inv);
                            w.w = pack_bf16x2(__uint_as_float(ov[d + 6]) * inv, __uint_as_float(ov[d + 7]) * inv);
                            dst[d / 8] = w;
                        }
                    }
                    else {
                        float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(a.out) + orow);
#pragma unroll
                        for (int d = 0; d < HD; d += 4)
                            dst[d / 4] = make_float4(__uint_as_float(ov[d]) * inv, __uint_as_float(ov[d + 1]) * inv,
                                                     __uint_as_float(ov[d + 2]) * inv, __uint_as_float(ov[d + 3]) * inv);
                    }
                }
                tc_fence_before();
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TM_COLS);
    }
}

template <bool OUT_BF16>
int launch(const CUtensorMap &tq, const CUtensorMap &tkv, const AttnArgs &a, int grid, cudaStream_t s)
{
    auto kern = attn_tc_kernel<OUT_BF16>;
    cudaError_t e = smem_limit_once<attn_tc_kernel<OUT_BF16>>(SMEM_BYTES);
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
    if (nseq <= 0 || N <= 0 || heads <= 0 || E != heads * HD || (reinterpret_cast<uintptr_t>(out) & 15))
        return K_EARG;
    const uint64_t rows = (uint64_t)nseq * N;
    CUtensorMap tq, tkv;
    if (!make_tmap_bf16(&tq, qkv, rows, 3ull * E, 3ull * E, BQ) ||
        !make_tmap_bf16(&tkv, qkv, rows, 3ull * E, 3ull * E, BKV))
        return K_ETMAP;
    const int sms = device_sms();
    AttnArgs a;
    a.nseq = nseq;
    a.N = N;
    a.E = E;
    a.heads = heads;
    a.nqt = (N + BQ - 1) / BQ;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.err = err;
    const long nitems = (long)nseq * heads * a.nqt;
    if (nitems > 0x7fffffffL)
        return K_EARG;
    a.nitems = (int)nitems;
    const int grid = nitems < kCtasPerSm * sms ? (int)nitems : kCtasPerSm * sms;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    return out_bf16 ? launch<true>(tq, tkv, a, grid, st) : launch<false>(tq, tkv, a, grid, st);
}
