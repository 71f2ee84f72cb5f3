// SPDX-License-Identifier: Unlicense
// Fused self-attention of the PE backbone on tcgen05 tensor cores: one
// kernel replaces the reference's QK^T gemm -> softmax_rows -> P.V gemm
// sequence on a materialised fp32 score buffer (sam3_model.c:1000-1013,
// sam3_kernels.cl:637-656), for 24x24 windows (N = 576) and for global
// attention over the whole grid (N = 5184) alike.
//
// Input: bf16 qkv rows [nseq * N, 3E] (RoPE already applied to q and k by
// the QKV GEMM epilogue or by k_rope_cast_bf16), head h at column h*64.
// k_attn_tc_cross runs the same kernel on separate Q, K and V tensors with
// Nq query and Nk key rows per sequence (the mask decoder's token-to-image
// attention with keys shared by all prompts, the detector's queries over the
// image), optionally with an fp32 bias added to every scaled score (SAM 3's
// box relative position bias, softmax_ext in sam3_kernels.cl:890-921).
//
// Work items are (sequence, head, 128-query tile), query tile fastest so
// that CTAs running at the same time share a head's K/V in L2. Two CTAs run
// on each SM, each persistent (CTA c takes items c, c + grid, ...) with its
// own MMA thread and K/V stream: the two pipelines drift apart in phase, so
// one CTA's softmax runs while the other's tensor-core work or loads do, and
// a short launch balances at the granularity of one tile. A launch of few
// waves given a workspace (the standalone op, the detector, cross-
// attention) splits the items that do not fill the last wave over their KV
// range: each part writes its unnormalised rows with (offset, sum), and a
// merge kernel combines them (the encoder passes none: a tile's result
// must not depend on the batch it is encoded in). KV tiles hold 96
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

// nseq sequences of Nq query rows and Nk key / value rows (Q, K and V rows
// of sequence s start at s * Nq and s * Nk of their tensor maps; head h at
// column qcol / kcol / vcol + 64 h); out rows s * Nq + q, leading dimension
// ldo, head h at column 64 h. bias (BIAS instantiation): fp32 added to the
// scaled scores, [nseq, heads, Nq, Nk] in log2 units.
// Work units: the first nfull are whole items (sequence, head, query tile)
// over all nkv KV tiles; in a SPLIT launch each remaining item (the tail
// that does not fill a wave of CTAs) is split into tsplit parts of nkv_t
// KV tiles, each writing its unnormalised output and (offset, sum) per row
// to part ([part][128 rows][64 + 4] fp32: output, offset, sum, 2 unused,
// so that every row starts 16-byte aligned); combine_kernel merges them.
struct AttnArgs {
    int nseq, Nq, Nk, heads, nqt, nitems, nkv, nfull, tsplit, nkv_t;
    int qcol, kcol, vcol;
    long ldo;
    int ohd;  // output columns per head (16, 32 or 64): head h at column h * ohd
    int last_late;  // partial last query tiles ordered after all full ones
    int pdl;        // launched as a programmatic dependent (pdl.cuh)
    float scale_log2;
    void *out;
    const float *bias;
    float *part;
    int *err;
};
constexpr int kPartRow = HD + 4;
static_assert((kPartRow * 4) % 16 == 0, "partial rows 16-byte aligned");

// Item -> (sequence, head, query tile). Items run in order over the CTAs.
// Normally item = (seq * heads + head) * nqt + qt, keeping a head's query
// tiles together (its K/V read once from HBM). With last_late (short
// launches whose last query tile is partial) the full tiles come first and
// the partial ones last, so the final, incomplete wave holds the cheapest
// items.
__device__ __forceinline__ void item_coords(const AttnArgs &a, int item, int &seq, int &head,
                                            int &qt)
{
    int sh;
    if (a.last_late) {
        const int nmain = a.nseq * a.heads * (a.nqt - 1);
        if (item < nmain) {
            qt = item % (a.nqt - 1);
            sh = item / (a.nqt - 1);
        }
        else {
            qt = a.nqt - 1;
            sh = item - nmain;
        }
    }
    else {
        qt = item % a.nqt;
        sh = item / a.nqt;
    }
    head = sh % a.heads;
    seq = sh / a.heads;
}

// Scores of one KV tile as loaded from TMEM: keys at or beyond `valid`
// set to -inf; with BIAS, each score becomes s * scale_log2 + b (b: the
// row's bias for this tile, null for a row beyond the queries, which is only
// scaled).
template <bool BIAS>
__device__ __forceinline__ void prep_scores(uint32_t (&s)[BKV], int valid, const float *b,
                                            float scale_log2)
{
    if (valid < BKV) {
#pragma unroll
        for (int e = 0; e < BKV; e++)
            if (e >= valid)
                s[e] = __float_as_uint(-INFINITY);
    }
    if (!BIAS)
        return;
    if (!b) {
#pragma unroll
        for (int e = 0; e < BKV; e++)
            s[e] = __float_as_uint(__uint_as_float(s[e]) * scale_log2);
    }
    else if (valid >= BKV && !(reinterpret_cast<uintptr_t>(b) & 15)) {
        const float4 *b4 = reinterpret_cast<const float4 *>(b);
#pragma unroll
        for (int e = 0; e < BKV; e += 4) {
            const float4 v = __ldg(b4 + e / 4);
            s[e] = __float_as_uint(fmaf(__uint_as_float(s[e]), scale_log2, v.x));
            s[e + 1] = __float_as_uint(fmaf(__uint_as_float(s[e + 1]), scale_log2, v.y));
            s[e + 2] = __float_as_uint(fmaf(__uint_as_float(s[e + 2]), scale_log2, v.z));
            s[e + 3] = __float_as_uint(fmaf(__uint_as_float(s[e + 3]), scale_log2, v.w));
        }
    }
    else {
#pragma unroll
        for (int e = 0; e < BKV; e++)
            if (e < valid)
                s[e] = __float_as_uint(fmaf(__uint_as_float(s[e]), scale_log2, __ldg(b + e)));
    }
}

template <bool OUT_BF16, bool BIAS, bool SPLIT>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnArgs a)
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
    const int nmine = (int)blockIdx.x < a.nitems
                          ? (a.nitems - 1 - (int)blockIdx.x) / (int)gridDim.x + 1
                          : 0;
    // this CTA's units k < nwhole are whole items, the rest tail parts
    const int nwhole = !SPLIT ? nmine
                              : ((int)blockIdx.x < a.nfull
                                     ? min(nmine, (a.nfull - 1 - (int)blockIdx.x) / (int)gridDim.x + 1)
                                     : 0);
    const int total = nwhole * a.nkv + (nmine - nwhole) * a.nkv_t;
    auto tiles_of = [&](int k) { return k < nwhole ? a.nkv : a.nkv_t; };
    // item = (seq * heads + head) * nqt + qt; a tail part p of item i is
    // unit nfull + (i - nfull) * tsplit + p, its KV tiles start at j0
    auto coords = [&](int k, int &seq, int &head, int &qt, int &j0) {
        const int u = (int)blockIdx.x + k * (int)gridDim.x;
        int item = u;
        j0 = 0;
        if (SPLIT && u >= a.nfull) {
            const int v = u - a.nfull;
            item = a.nfull + v / a.tsplit;
            j0 = (v % a.tsplit) * a.nkv_t;
        }
        item_coords(a, item, seq, head, qt);
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
    // Launched as a programmatic dependent (pdl.cuh; the cross-attention
    // entry, whose callers chain short kernels): the setup above used only
    // this CTA's shared and tensor memory; global accesses wait below, and
    // the next kernel may be scheduled once every CTA has its tensor memory.
    // The encoder's launches keep plain stream order (measured: the 64-tile
    // step 2-3 % slower with its LayerNorm and attention as dependents).
    if (a.pdl)
        griddep_launch();
    griddep_wait();

    if (warp == kProducerWarp) {
        if (lane < 2) {
            const bool is_k = lane == 0;
            const CUtensorMap *tmX = is_k ? &tmK : &tmV;
            if (is_k)
                prefetch_tmap(&tmQ);
            prefetch_tmap(tmX);
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *empty = is_k ? k_empty : v_empty;
            uint8_t *ring = smem + (is_k ? OFF_K : OFF_V);
            int lastq = -1, lastg = -1, st = 0, use = 0;
            bool ok = true;
            for (int k = 0; k < nmine && ok; k++) {
                int seq, head, qt, j0;
                coords(k, seq, head, qt, j0);
                const int row0 = seq * a.Nk + j0 * BKV;
                if (is_k) {
                    if (!mbar_wait(&q_empty[k & 1], ((k >> 1) & 1) ^ 1, a.err, abort_flag))
                        break;
                    mbar_arrive_expect_tx(&q_full[k & 1], Q_BYTES);
                    tma_load_2d(smem + OFF_Q + (k & 1) * Q_BYTES, &tmQ, &q_full[k & 1],
                                a.qcol + head * HD, seq * a.Nq + qt * BQ);
                    lastq = k;
                }
                const int col = (is_k ? a.kcol : a.vcol) + head * HD;
                const int nkv = tiles_of(k);
                for (int j = 0; j < nkv; j++) {
                    if (!mbar_wait(&empty[st], (use & 1) ^ 1, a.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[st], KV_BYTES);
                    tma_load_2d(ring + st * KV_BYTES, tmX, &full[st], col, row0 + j * BKV);
                    lastg++;
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
                if (++c.j == tiles_of(c.k)) {
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
                if (c.j == tiles_of(c.k) - 1)
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
        // With a bias the scores are scaled and biased when loaded
        // (prep_scores), so the exponent step uses a unit scale.
        const float sl2 = BIAS ? 1.0f : a.scale_log2;
        const uint64_t sl2x2 = f2_make(sl2, sl2);
        bool ok = true;
        int g = 0;
        for (int k = 0; k < nmine && ok; k++) {
            int seq, head, qt, j0;
            coords(k, seq, head, qt, j0);
            const bool rows_live = qt * BQ + quarter * 32 < a.Nq;
            const int q = qt * BQ + r;
            const float *brow = BIAS && q < a.Nq
                                    ? a.bias + ((long)(seq * a.heads + head) * a.Nq + q) * a.Nk
                                    : nullptr;
            const bool is_part = SPLIT && k >= nwhole;
            const int nkv = tiles_of(k);
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
                    const int valid = a.Nk - (j0 + j) * BKV;
                    prep_scores<BIAS>(s, valid, brow ? brow + (j0 + j) * BKV : nullptr,
                                      a.scale_log2);
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
                        prep_scores<BIAS>(s, valid, brow ? brow + (j0 + j) * BKV : nullptr,
                                          a.scale_log2);
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
                const float lsum = (la + lb) + (lc + ld);
                if (is_part && q < a.Nq) {
                    const long v = (long)blockIdx.x + (long)k * gridDim.x - a.nfull;
                    float *pr = a.part + (v * BQ + r) * kPartRow;
                    float4 *dst = reinterpret_cast<float4 *>(pr);
#pragma unroll
                    for (int d = 0; d < HD; d += 4)
                        dst[d / 4] = make_float4(__uint_as_float(ov[d]), __uint_as_float(ov[d + 1]),
                                                 __uint_as_float(ov[d + 2]), __uint_as_float(ov[d + 3]));
                    pr[HD] = m_used;
                    pr[HD + 1] = lsum;
                }
                const float inv = 1.0f / lsum;
                if (!is_part && q < a.Nq) {
                    const long orow = (long)(seq * a.Nq + q) * a.ldo + head * a.ohd;
                    if (OUT_BF16) {
                        uint4 *dst = reinterpret_cast<uint4 *>(
                            reinterpret_cast<__nv_bfloat16 *>(a.out) + orow);
#pragma unroll
                        for (int d = 0; d < HD; d += 8) {
                            if (d >= a.ohd)
                                break;
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
                            if (d < a.ohd)
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

// Merges the tsplit partial results of each tail item's query rows:
// O = sum_p O_p 2^(m_p - M) / sum_p l_p 2^(m_p - M), M = max_p m_p. One
// warp per (tail item, row): the lanes first take the parts' offsets and
// sums (lane = part), then two output columns each, reading every part's
// row as one coalesced 256-byte load with the part's weight shuffled in.
template <bool OUT_BF16>
__global__ void __launch_bounds__(256) combine_kernel(const float *__restrict__ part, AttnArgs a,
                                                      int ntail)
{
    griddep_wait();  // a programmatic dependent with a.pdl (pdl.cuh)
    if (a.pdl)
        griddep_launch();
    static_assert(HD == 64, "two output columns per lane");
    const int lane = threadIdx.x & 31;
    const long nrows = (long)ntail * BQ, pstride = (long)BQ * kPartRow;
    for (long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < nrows;
         w += ((long)gridDim.x * blockDim.x) >> 5) {
        const int r = (int)(w % BQ);
        const long t = w / BQ;
        const long item = a.nfull + t;
        int seq, head, qt;
        item_coords(a, (int)item, seq, head, qt);
        const int q = qt * BQ + r;
        if (q >= a.Nq)
            continue;  // warp-uniform
        const float *p0 = part + ((t * a.tsplit) * BQ + r) * kPartRow;
        float M = -INFINITY;
        for (int sp = lane; sp < a.tsplit; sp += 32)
            M = fmaxf(M, p0[sp * pstride + HD]);
#pragma unroll
        for (int o = 16; o; o >>= 1)
            M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.0f, ox = 0.0f, oy = 0.0f;
        for (int s0 = 0; s0 < a.tsplit; s0 += 32) {
            const int sl = s0 + lane;
            const float2 ml = sl < a.tsplit ? *reinterpret_cast<const float2 *>(p0 + sl * pstride + HD)
                                            : make_float2(-INFINITY, 0.0f);
            const float fl = sl < a.tsplit ? exp2f(ml.x - M) : 0.0f;
            L = fmaf(ml.y, fl, L);
            const int n = min(32, a.tsplit - s0);
            const float *pc = p0 + s0 * pstride + 2 * lane;
#pragma unroll 4
            for (int j = 0; j < n; j++) {
                const float f = __shfl_sync(0xffffffffu, fl, j);
                const float2 v = *reinterpret_cast<const float2 *>(pc + j * pstride);
                ox = fmaf(v.x, f, ox);
                oy = fmaf(v.y, f, oy);
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1)
            L += __shfl_xor_sync(0xffffffffu, L, o);
        if (2 * lane >= a.ohd)
            continue;  // beyond the head's output columns
        const float inv = 1.0f / L;
        const long orow = (long)(seq * a.Nq + q) * a.ldo + head * a.ohd + 2 * lane;
        if (OUT_BF16)
            *reinterpret_cast<uint32_t *>(reinterpret_cast<__nv_bfloat16 *>(a.out) + orow) =
                pack_bf16x2(ox * inv, oy * inv);
        else
            *reinterpret_cast<float2 *>(reinterpret_cast<float *>(a.out) + orow) =
                make_float2(ox * inv, oy * inv);
    }
}

template <bool OUT_BF16, bool BIAS, bool SPLIT>
int launch(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv, const AttnArgs &a,
           int grid, cudaStream_t s)
{
    cudaError_t e = smem_limit_once<attn_tc_kernel<OUT_BF16, BIAS, SPLIT>>(SMEM_BYTES);
    if (e != cudaSuccess)
        return (int)e;
    int rc;
    if (a.pdl)
        rc = launch_pdl(attn_tc_kernel<OUT_BF16, BIAS, SPLIT>, dim3(grid), dim3(kThreads), SMEM_BYTES,
                        s, tq, tk, tv, a);
    else {
        attn_tc_kernel<OUT_BF16, BIAS, SPLIT><<<grid, kThreads, SMEM_BYTES, s>>>(tq, tk, tv, a);
        rc = (int)cudaGetLastError();
    }
    if (rc != 0 || !SPLIT)
        return rc;
    const int ntail = (a.nitems - a.nfull) / a.tsplit;
    const long n = (long)ntail * BQ * 32;  // a warp per row
    const long blocks = (n + 255) / 256;
    const dim3 cgrid((unsigned)(blocks < 148 * 32 ? blocks : 148 * 32));
    if (a.pdl)
        return launch_pdl(combine_kernel<OUT_BF16>, cgrid, dim3(256), 0, s, a.part, a, ntail);
    combine_kernel<OUT_BF16><<<cgrid, 256, 0, s>>>(a.part, a, ntail);
    return (int)cudaGetLastError();
}

// Work plan of a launch over `base` items of nkv KV tiles on 2 x sms CTA
// slots. Launches of many waves run whole items. Otherwise the items that
// do not fill the last wave (all of them when there are fewer items than
// slots, as for few query tiles over many keys) are split into parts: the divisor d of nkv that minimises the
// tail's time in KV-tile times, ceil(tail * d / slots) waves of nkv / d
// tiles plus kPartCost for a part's start and partial store, plus
// kMergeCost for the merge launch when d > 1 (measured: a 9-window launch
// whose 128 tail items split in 2 ran slower, the 16-head global one whose
// 64 tail items split in 9 faster). Returns the workspace bytes the split
// needs (0 for none).
size_t plan(AttnArgs &a, long base, int nkv, int sms)
{
    const long slots = 2L * sms;
    a.nkv = nkv;
    a.nfull = (int)base;
    a.tsplit = 1;
    a.nkv_t = nkv;
    a.nitems = (int)base;
    if (base >= 8 * slots)
        return 0;
    const long nfull = base / slots * slots;
    const long tail = base - nfull;
    if (tail == 0)
        return 0;
    constexpr long kPartCost = 3, kMergeCost = 4;
    int best = 1;
    long best_cost = (tail + slots - 1) / slots * (nkv + kPartCost);
    for (int d = 2; d <= nkv; d++) {
        if (nkv % d)
            continue;
        const long cost = (tail * d + slots - 1) / slots * (nkv / d + kPartCost) + kMergeCost;
        if (cost < best_cost) {
            best_cost = cost;
            best = d;
        }
    }
    if (best == 1)
        return 0;
    a.nfull = (int)nfull;
    a.tsplit = best;
    a.nkv_t = nkv / best;
    a.nitems = (int)(nfull + tail * best);
    return (size_t)tail * best * BQ * kPartRow * sizeof(float);
}

// Plans the launch (splitting only when ws holds the partial results) and
// runs it.
int run(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv, AttnArgs &a,
        bool out_bf16, void *ws, size_t ws_bytes, cudaStream_t st)
{
    a.nqt = (a.Nq + BQ - 1) / BQ;
    const long base = (long)a.nseq * a.heads * a.nqt;
    if (base > 0x3fffffffL || (long)a.nseq * a.Nq > 0x7fffffffL ||
        (long)a.nseq * a.Nk > 0x7fffffffL)
        return K_EARG;
    const int sms = device_sms();
    const int nkv = (a.Nk + BKV - 1) / BKV;
    size_t need = plan(a, base, nkv, sms);
    if (need && (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 15)))
        need = 0;  // no room for the partial results: whole items
    if (!need) {
        a.nfull = (int)base;
        a.tsplit = 1;
        a.nkv_t = nkv;
        a.nitems = (int)base;
    }
    a.part = need ? static_cast<float *>(ws) : nullptr;
    // Partial last query tiles go last in short launches (measured: the
    // detector's 201 queries 65-68 -> 62-63 us; the 9-window launch 398 ->
    // 420 TFLOP/s on one box, unchanged on two others; the fusion
    // encoder's 5184 tokens within 2 %), not in long ones, whose heads' K/V
    // late tiles would re-read from HBM.
    a.last_late = a.Nq % BQ != 0 && a.nqt > 1 && base < 8L * 2 * sms;
    if (a.nitems > 0x7fffffff)
        return K_EARG;
    const int grid = a.nitems < 2 * sms ? a.nitems : 2 * sms;
    const bool split = a.nitems != a.nfull;
    if (!a.bias && !split)
        return out_bf16 ? launch<true, false, false>(tq, tk, tv, a, grid, st)
                        : launch<false, false, false>(tq, tk, tv, a, grid, st);
    if (!a.bias)
        return out_bf16 ? launch<true, false, true>(tq, tk, tv, a, grid, st)
                        : launch<false, false, true>(tq, tk, tv, a, grid, st);
    if (out_bf16)
        return K_EARG;
    return split ? launch<false, true, true>(tq, tk, tv, a, grid, st)
                 : launch<false, true, false>(tq, tk, tv, a, grid, st);
}

// Workspace of a launch's plan.
size_t workspace(int nseq, int Nq, int Nk, int heads)
{
    if (nseq <= 0 || Nq <= 0 || Nk <= 0 || heads <= 0)
        return 0;
    AttnArgs a;
    const long base = (long)nseq * heads * ((Nq + BQ - 1) / BQ);
    return plan(a, base, (Nk + BKV - 1) / BKV, device_sms());
}

}  // namespace
}  // namespace sam3

extern "C" size_t k_attn_tc_workspace(int nseq, int N, int heads)
{
    return sam3::workspace(nseq, N, N, heads);
}

extern "C" int k_attn_tc(const void *qkv, int nseq, int N, int E, int heads, float scale,
                         void *out, int out_bf16, void *ws, size_t ws_bytes, int *err, k_stream s)
{
    using namespace sam3;
    if (nseq <= 0 || N <= 0 || heads <= 0 || E != heads * HD || (reinterpret_cast<uintptr_t>(out) & 15))
        return K_EARG;
    const uint64_t rows = (uint64_t)nseq * N;
    CUtensorMap tq, tkv;
    if (!make_tmap_bf16(&tq, qkv, rows, 3ull * E, 3ull * E, BQ) ||
        !make_tmap_bf16(&tkv, qkv, rows, 3ull * E, 3ull * E, BKV))
        return K_ETMAP;
    AttnArgs a;
    a.nseq = nseq;
    a.Nq = N;
    a.Nk = N;
    a.heads = heads;
    a.qcol = 0;
    a.kcol = E;
    a.vcol = 2 * E;
    a.ldo = E;
    a.ohd = HD;
    a.pdl = 0;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.bias = nullptr;
    a.err = err;
    return run(tq, tkv, tkv, a, out_bf16 != 0, ws, ws_bytes,
               reinterpret_cast<cudaStream_t>(s));
}

extern "C" size_t k_attn_tc_cross_workspace(int nseq, int Nq, int Nk, int heads)
{
    return sam3::workspace(nseq, Nq, Nk, heads);
}

extern "C" int k_attn_tc_cross(const void *Q, long ldq, const void *K, long ldk, const void *V,
                               long ldv, int nseq, int Nq, int Nk, int heads, float scale,
                               const float *bias, void *out, long ldo, int ohd, int out_bf16,
                               void *ws, size_t ws_bytes, int *err, k_stream s)
{
    using namespace sam3;
    const long W = (long)heads * HD;
    if (nseq <= 0 || Nq <= 0 || Nk <= 0 || heads <= 0 || ldq < W || ldk < W || ldv < W ||
        (ohd != 16 && ohd != 32 && ohd != HD) || ldo < (long)heads * ohd ||
        (ldo * (out_bf16 ? 2 : 4)) % 16 || (reinterpret_cast<uintptr_t>(out) & 15))
        return K_EARG;
    CUtensorMap tq, tk, tv;
    if (!make_tmap_bf16(&tq, Q, (uint64_t)nseq * Nq, (uint64_t)W, (uint64_t)ldq, BQ) ||
        !make_tmap_bf16(&tk, K, (uint64_t)nseq * Nk, (uint64_t)W, (uint64_t)ldk, BKV) ||
        !make_tmap_bf16(&tv, V, (uint64_t)nseq * Nk, (uint64_t)W, (uint64_t)ldv, BKV))
        return K_ETMAP;
    AttnArgs a;
    a.nseq = nseq;
    a.Nq = Nq;
    a.Nk = Nk;
    a.heads = heads;
    a.qcol = 0;
    a.kcol = 0;
    a.vcol = 0;
    a.ldo = ldo;
    a.ohd = ohd;
    a.pdl = 1;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.bias = bias;
    a.err = err;
    return run(tq, tk, tv, a, out_bf16 != 0, ws, ws_bytes, reinterpret_cast<cudaStream_t>(s));
}
