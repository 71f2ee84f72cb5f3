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
// Work items are pairs of 128-query tiles ("slots"). Per sequence and head
// the full tiles pair up (one K/V stream for both slots: 576 = 4.5 x 128 and
// 5184 = 40.5 x 128 give 2 and 20 such pairs); the leftover tile of each
// head (the 64-row tail here) pairs with the leftover of the next head, the
// two slots then streaming their own K and V. KV tiles hold 96 keys (576 =
// 6 x 96, 5184 = 54 x 96). Rows of a tail tile beyond N run through the
// tensor core but their softmax work is skipped and nothing is stored. The
// kernel is persistent: CTA c takes items c, c + grid, ... and streams their
// KV tiles back to back, so the pipeline is filled once per CTA and the next
// item's Q and first scores are loaded and computed while the current item
// finishes.
//
//   warps 0-3  softmax of query tile 0, warps 4-7 of tile 1 (one thread per
//              query row; warp w reads TMEM lanes 32*(w%4)...);
//   warp 8     TMA producers: lane 0 loads Q (two buffers) and the K ring,
//              lane 1 the V ring (three stages of one or two tiles each);
//   warp 9     TMEM owner and MMA issuer.
//
// Score tiles are numbered n = 2g + t (g: this CTA's KV tiles across items,
// t: query tile), and S(n) goes to TMEM score buffer n % 3 (96 fp32 columns
// each, at 0, 96, 192). The softmax writes P(n) into the first 48 columns
// of that buffer (pairs of 16-bit values, the TMEM A-operand layout), P.V(n)
// reads it from there, and S(n + 3) is issued into the same buffer right
// after P.V(n) (tensor-core operations of one thread run in issue order), so
// two score tiles are always computed ahead of the softmax. The output
// accumulator of tile t (80 columns at 288 + 80t) holds O in columns 0-63
// and, because every V tile is followed in shared memory by a tile of ones
// read as output columns 64-79, the row sum of P in column 64: the tensor
// core sums exactly the 16-bit P values it multiplies.
//
// Softmax per KV tile, one pass: the row's 96 scores in one TMEM round trip;
// row maximum with three-input max; x = s * scale * log2 e - m in packed
// fp32; 2^x on the MUFU unit, with 1/8 of the values on the FMA pipe
// (exp2_poly2); P packed to bf16 pairs. The running maximum is only
// raised (and O with its row sum rescaled in TMEM by 2^(m_old - m_new)) when
// the tile maximum exceeds it by more than 8 in log2 units, so P stays
// <= 2^8 and most tiles skip the rescale; the final division by the row sum
// makes the result independent of the offset used.
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>

namespace sam3 {
namespace {

constexpr int HD = 64;
constexpr int BQ = 128;
constexpr int BKV = 96;  // keys per KV tile (a multiple of 32)
constexpr int NO = HD + 16;               // O columns: 64 outputs + row-sum block
constexpr int NSB = 3;                    // TMEM score buffers
constexpr int KST = 3;                    // K and V ring stages
constexpr int kSoftmaxWarps = 8;          // 2 tiles x 4 lane quarters
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 32 * 10;
// Of every 8 pairs of scores, this many take the FMA-pipe exponential
// (exp2_poly2) instead of two MUFU instructions: the MUFU unit runs 16
// exponentials per clock per SM against 256 MMA flops per score.
constexpr int kPolyPairsPer16 = 1;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int Q_BYTES = BQ * HD * 2;     // 16 KB per query tile
constexpr int KV_BYTES = BKV * HD * 2;   // 12 KB per K or V tile
constexpr int K_STAGE = 2 * KV_BYTES;    // K of slot 0, K of slot 1
constexpr int V_STAGE = 2 * KV_BYTES;    // V of slot 0, V of slot 1
constexpr int OFF_Q = 0;                         // [buffer][slot]
constexpr int OFF_K = OFF_Q + 4 * Q_BYTES;       // K ring
constexpr int OFF_V = OFF_K + KST * K_STAGE;     // V ring
constexpr int OFF_ONES = OFF_V + KST * V_STAGE;  // one tile of ones behind every V
constexpr int OFF_BAR = OFF_ONES + KV_BYTES;
constexpr uint32_t TM_O = NSB * BKV;             // first O column
// q_full[2], q_empty[2], k_full[KST], k_empty[KST], v_full[KST],
// v_empty[KST], s_full[3], p_ready[3], pv_full[2 tiles][2], drain. A waiter never finds
// one of them two phases ahead of the phase it waits for: score buffer i is
// only refilled after P.V of its previous tile, which needs that tile's
// p_ready; pv_full is split by KV-tile parity so that the phase before the
// awaited one (P.V two KV tiles back) is always complete.
constexpr int NBAR = 4 + 4 * KST + 3 * NSB + 4 + 1;
constexpr int SMEM_BYTES = OFF_BAR + NBAR * 8 + 16 + 1024;
static_assert(SMEM_BYTES <= 232448, "attention smem");
static_assert(OFF_K % 1024 == 0 && OFF_V % 1024 == 0 && OFF_ONES % 1024 == 0 &&
                  KV_BYTES % 1024 == 0 && OFF_ONES - OFF_V < (1 << 18),
              "alignment, LBO range");
static_assert(TM_O + 2 * NO <= 512, "tensor memory");
static_assert(BKV % 32 == 0 && BKV <= 256, "KV tile");

struct AttnArgs {
    int nseq, N, E, heads;
    int nitems;
    // Work items per sequence: first the leftover tiles, with nleft == 2 per
    // head (an odd full tile and the partial tail) one item per head, with
    // nleft == 1 (only one of them) the leftover tiles of heads 2i and 2i+1,
    // one item per pair of heads (the second slot empty for an odd head
    // count); then heads * npf pairs of full 128-row tiles of one head.
    int npf, nleft, left_tile, per_seq;
    // Whether leftover tiles of different heads are paired (above), or each
    // head's tiles pair as (2i, 2i+1) with an odd last tile alone: the first
    // needs fewer, fuller items, which a long launch prefers; a launch of a
    // few waves is balanced better by the second's lighter last items.
    int pair_tails, nqt;
    float scale_log2;
    void *out;
    int *err;
};

// One query tile of an item: head, tile index within the sequence, and
// whether the slot is empty.
struct Slot {
    int head, qt;
    bool dead;
};

__device__ __forceinline__ void item_slots(const AttnArgs &a, int item, int &seq, Slot &s0,
                                           Slot &s1)
{
    seq = item / a.per_seq;
    int r = item - seq * a.per_seq;
    if (!a.pair_tails) {  // tiles (2i, 2i+1) of one head; an odd last tile alone
        const int npairs = a.per_seq / a.heads, h = r / npairs, pr = r - h * npairs;
        s0 = Slot{h, 2 * pr, false};
        s1 = Slot{h, 2 * pr + 1, 2 * pr + 1 >= a.nqt};
        return;
    }
    const int left_items = a.per_seq - a.heads * a.npf;
    if (r >= left_items) {  // leftover items first: a short launch ends on full pairs
        r -= left_items;
        const int h = r / a.npf, pr = r - h * a.npf;
        s0 = Slot{h, 2 * pr, false};
        s1 = Slot{h, 2 * pr + 1, false};
    }
    else if (a.nleft == 2) {
        s0 = Slot{r, a.left_tile, false};
        s1 = Slot{r, a.left_tile + 1, false};
    }
    else {
        const int h1 = 2 * r + 1;
        s0 = Slot{2 * r, a.left_tile, false};
        s1 = h1 < a.heads ? Slot{h1, a.left_tile, false} : Slot{2 * r, a.left_tile, true};
    }
}

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
    uint64_t *q_empty = q_full + 2;
    uint64_t *k_full = q_empty + 2;
    uint64_t *k_empty = k_full + KST;
    uint64_t *v_full = k_empty + KST;
    uint64_t *v_empty = v_full + KST;
    uint64_t *s_full = v_empty + KST;   // [score buffer]
    uint64_t *p_ready = s_full + NSB;   // [score buffer]
    uint64_t *pv_full = p_ready + NSB;  // [tile * 2 + KV-tile parity]
    uint64_t *drain = pv_full + 4;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int nkv = (a.N + BKV - 1) / BKV;
    // Items of this CTA and its total number of KV tiles.
    const int nmine = (int)blockIdx.x < a.nitems
                          ? (a.nitems - 1 - (int)blockIdx.x) / (int)gridDim.x + 1
                          : 0;
    const int total = nmine * nkv;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
        }
        for (int i = 0; i < KST; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < NSB; i++) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_ready[i], 4);
        }
        for (int i = 0; i < 4; i++)
            mbar_init(&pv_full[i], 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    // The ones tile read as P.V's output columns 64-79 (bf16 1.0 in both
    // halves of every word; the swizzle of a constant tile is immaterial).
    {
        const uint32_t one2 = 0x3F803F80u;
        for (int i = threadIdx.x; i < KV_BYTES / 16; i += kThreads)
            st_shared_v4(smem_addr(smem + OFF_ONES + i * 16), one2, one2, one2, one2);
        fence_proxy_async_smem();
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
            }
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *empty = is_k ? k_empty : v_empty;
            uint8_t *ring = smem + (is_k ? OFF_K : OFF_V);
            const int stride = is_k ? K_STAGE : V_STAGE;
            int lastq = -1, lastg = -1;
            bool ok = true;
            int st = 0, use = 0;  // ring stage and use count of KV tile g
            for (int k = 0; k < nmine && ok; k++) {
                int seq;
                Slot s0, s1;
                item_slots(a, (int)blockIdx.x + k * (int)gridDim.x, seq, s0, s1);
                const int row0 = seq * a.N;
                // The two slots share one K/V stream when they are the same
                // head (or the second is empty); else each has its own.
                const bool shared = s0.head == s1.head;
                if (is_k) {
                    // Q buffer k % 2 was last read by the S MMAs of item k-2.
                    if (!mbar_wait(&q_empty[k & 1], ((k >> 1) & 1) ^ 1, a.err, abort_flag))
                        break;
                    mbar_arrive_expect_tx(&q_full[k & 1], 2 * Q_BYTES);
                    tma_load_2d(smem + OFF_Q + ((k & 1) * 2) * Q_BYTES, &tmQ, &q_full[k & 1],
                                s0.head * HD, row0 + s0.qt * BQ);
                    tma_load_2d(smem + OFF_Q + ((k & 1) * 2 + 1) * Q_BYTES, &tmQ, &q_full[k & 1],
                                s1.head * HD, row0 + s1.qt * BQ);
                    lastq = k;
                }
                const int col0 = is_k ? a.E : 2 * a.E;
                for (int j = 0; j < nkv; j++) {
                    if (!mbar_wait(&empty[st], (use & 1) ^ 1, a.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[st], shared ? KV_BYTES : 2 * KV_BYTES);
                    tma_load_2d(ring + st * stride, &tmKV, &full[st], col0 + s0.head * HD,
                                row0 + j * BKV);
                    if (!shared)
                        tma_load_2d(ring + st * stride + KV_BYTES, &tmKV, &full[st],
                                    col0 + s1.head * HD, row0 + j * BKV);
                    lastg = k * nkv + j;
                    if (++st == KST) {
                        st = 0;
                        use++;
                    }
                }
            }
            // Let every issued copy land before the CTA can exit.
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
            constexpr uint32_t idPV = idesc_bf16_f32(BQ, NO, 0, 1);
            // Descriptors of the first 16-element K slice of the operand
            // regions. A tile or slice offset of d bytes adds d / 16 to the
            // start-address field (shared addresses stay below 2^18, so the
            // 14-bit field never carries): K-major slices are 32 bytes apart,
            // V slices (MN-major, 16 keys) 2048 bytes.
            // P.V's B operand is [V | ones]: the ones tile is the second
            // N-group, LBO bytes from the V tile. A V tile d bytes into the
            // ring moves the start-address field up and the LBO field down by
            // d / 16 (both 14-bit fields stay in range: no carry, no borrow).
            const uint64_t dQ = sw128_desc(smem_addr(smem + OFF_Q), 16, 1024);
            const uint64_t dK = sw128_desc(smem_addr(smem + OFF_K), 16, 1024);
            const uint64_t dV = sw128_desc(smem_addr(smem + OFF_V), OFF_ONES - OFF_V, 1024);
            auto v_desc = [&](int d) -> uint64_t {
                const uint64_t u = (uint64_t)(d >> 4);
                return dV + u - (u << 16);
            };
            const int nscore = 2 * total;
            // Per item: whether the slots share one K/V stream, and whether
            // the second slot is empty (no MMAs; its barriers are still
            // committed).
            auto item_kind = [&](int k, bool &shared, bool &dead1) {
                int seq;
                Slot s0, s1;
                item_slots(a, (int)blockIdx.x + k * (int)gridDim.x, seq, s0, s1);
                shared = s0.head == s1.head;
                dead1 = s1.dead;
            };
            // Cursor over score tiles n = 2g + t, kept by increments (this one
            // thread issues every MMA; its instruction count is on the
            // critical path).
            struct Cursor {
                int n, t;      // score tile, query tile
                int kst, kph;  // K/V ring stage of g and its use parity
                int gpar, j, k;
                int buf, bph;  // score buffer n % 3 and its use parity
                bool shared, dead1, dead;
            };
            auto advance = [&](Cursor &c) {
                c.n++;
                c.t ^= 1;
                if (++c.buf == NSB) {
                    c.buf = 0;
                    c.bph ^= 1;
                }
                if (c.t == 0) {
                    c.gpar ^= 1;
                    if (++c.kst == KST) {
                        c.kst = 0;
                        c.kph ^= 1;
                    }
                    if (++c.j == nkv) {
                        c.j = 0;
                        c.k++;
                        if (c.k < nmine)
                            item_kind(c.k, c.shared, c.dead1);
                    }
                }
                c.dead = c.t == 1 && c.dead1;
            };
            Cursor c0 = {0, 0, 0, 0, 0, 0, 0, 0, 0, true, false, false};
            item_kind(0, c0.shared, c0.dead1);
            Cursor ahead = c0, cur = c0;
            // S(n) = Q_t(item k) K(g)^T into score buffer n % 3. The first S of
            // an item waits for its Q; the last one releases the Q buffer.
            auto issue_s = [&](const Cursor &c) -> bool {
                if (c.t == 0) {
                    if (!mbar_wait(&k_full[c.kst], c.kph, a.err, abort_flag))
                        return false;
                    if (c.j == 0 && !mbar_wait(&q_full[c.k & 1], (c.k >> 1) & 1, a.err, abort_flag))
                        return false;
                    tc_fence_after();
                }
                if (!c.dead) {
                    const uint64_t qd = dQ + (uint64_t)((((c.k & 1) * 2 + c.t) * Q_BYTES) >> 4);
                    const uint64_t kd =
                        dK + (uint64_t)((c.kst * K_STAGE + (c.shared ? 0 : c.t) * KV_BYTES) >> 4);
                    const uint32_t dS = tmem_base + c.buf * BKV;
#pragma unroll
                    for (int kq = 0; kq < HD / 16; kq++)
                        tc_mma(dS, qd + 2 * kq, kd + 2 * kq, idS, kq != 0);
                }
                tc_commit(&s_full[c.buf]);
                if (c.t == 1) {
                    tc_commit(&k_empty[c.kst]);
                    if (c.j == nkv - 1)
                        tc_commit(&q_empty[c.k & 1]);
                }
                return true;
            };
            // O_t (+)= P(n) [V(g) | 1], P read from score buffer n % 3; the
            // first KV tile of an item resets O_t and its row sum.
            auto issue_pv = [&](const Cursor &c) -> bool {
                if (c.t == 0 && !mbar_wait(&v_full[c.kst], c.kph, a.err, abort_flag))
                    return false;
                if (!mbar_wait(&p_ready[c.buf], c.bph, a.err, abort_flag))
                    return false;
                tc_fence_after();
                if (!c.dead) {
                    const uint64_t vd = v_desc(c.kst * V_STAGE + (c.shared ? 0 : c.t) * KV_BYTES);
                    const uint32_t dO = tmem_base + TM_O + c.t * NO;
                    const uint32_t aP = tmem_base + c.buf * BKV;
#pragma unroll
                    for (int kk = 0; kk < BKV / 16; kk++)
                        tc_mma_ts(dO, aP + kk * 8, vd + 128 * kk, idPV, (c.j | kk) != 0);
                }
                tc_commit(&pv_full[c.t * 2 + c.gpar]);
                if (c.t == 1)
                    tc_commit(&v_empty[c.kst]);
                return true;
            };
            bool ok = true;
            for (int i = 0; ok && i < NSB && ahead.n < nscore; i++) {
                ok = issue_s(ahead);
                advance(ahead);
            }
            while (ok && cur.n < nscore) {
                ok = issue_pv(cur);
                if (ok && ahead.n < nscore) {
                    ok = issue_s(ahead);
                    advance(ahead);
                }
                advance(cur);
            }
            tc_commit(drain);
            volatile int no_abort = 0;
            mbar_wait(drain, 0, a.err, &no_abort);
        }
    }
    else if (warp < kSoftmaxWarps) {
        const int t = warp >> 2;            // query tile of the item
        const int quarter = warp & 3;       // TMEM lane quarter = rows 32q..32q+31
        const int r = quarter * 32 + lane;  // query row within the tile
        const uint32_t tL = tmem_base + ((uint32_t)(quarter * 32) << 16);
        const uint32_t tO = tL + TM_O + t * NO;
        const float sl2 = a.scale_log2;
        const uint64_t sl2x2 = f2_make(sl2, sl2);
        bool ok = true;
        // Score tile n = 2g + t: buffer n % 3 and its use parity, advanced
        // by increments (n grows by 2 per KV tile).
        int buf = t, bph = 0;
        for (int k = 0; k < nmine && ok; k++) {
            // Warps whose 32 query rows lie beyond N (the second half of a
            // partial tail tile) or in an empty slot keep the barrier protocol
            // but skip the softmax work; they store nothing.
            int seq;
            Slot s0, s1;
            item_slots(a, (int)blockIdx.x + k * (int)gridDim.x, seq, s0, s1);
            const Slot me = t ? s1 : s0;
            const bool rows_live = !me.dead && me.qt * BQ + quarter * 32 < a.N;
            float m_used = -INFINITY;
            for (int j = 0; j < nkv; j++) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s_full[buf], bph, a.err, abort_flag));
                if (!ok)
                    break;
                tc_fence_after();
                const uint32_t tS = tL + buf * BKV;
                bool resc = false;
                float factor = 1.0f;
                if (rows_live) {
                    // The whole score row in one TMEM round trip.
                    uint32_t s[BKV];
#pragma unroll
                    for (int c = 0; c < BKV / 32; c++)
                        tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
                    tmem_wait_ld();
                    const int valid = a.N - j * BKV;
                    if (valid < BKV) {  // only a sequence's last tile
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
                        m_used = m_tile;  // first tile of the item: O not yet written
                    }
                    else if (m_tile > m_used + kRescaleThreshold) {
                        resc = true;
                        factor = ex2_approx(m_used - m_tile);
                        m_used = m_tile;
                    }
                    // P = 2^(s * scale_log2 - m_used) as bf16 pairs, in place
                    // (s[i] holds keys 2i, 2i+1 for i < 48). Keys past N have
                    // s = -inf and get P = 0.
                    const uint64_t negm = f2_make(-m_used, -m_used);
#pragma unroll
                    for (int e = 0; e < BKV; e += 2) {
                        const uint64_t x2 = fma2(f2_make(__uint_as_float(s[e]),
                                                         __uint_as_float(s[e + 1])),
                                                 sl2x2, negm);
                        float x0, x1;
                        f2_split(x2, x0, x1);
                        uint32_t pp;
                        if (((e >> 1) & 7) >= 8 - kPolyPairsPer16) {
                            float p0, p1;
                            exp2_poly2(x0, x1, p0, p1);
                            pp = pack_bf16x2(p0, p1);
                        }
                        else {
                            pp = pack_bf16x2(ex2_approx(x0), ex2_approx(x1));
                        }
                        s[e >> 1] = pp;
                    }
#pragma unroll
                    for (int c = 0; c < BKV / 64; c++)
                        tmem_st32(tS + 32 * c, *reinterpret_cast<const uint32_t(*)[32]>(s + 32 * c));
                    if constexpr (BKV % 64 != 0)
                        tmem_st16(tS + BKV / 64 * 32,
                                  *reinterpret_cast<const uint32_t(*)[16]>(s + BKV / 64 * 32));
                }
                // A raised maximum rescales O and its row sum, which needs
                // P.V of the previous KV tile done; P.V(n) is only issued after
                // p_ready below.
                if (__any_sync(0xffffffffu, resc)) {
                    const int gp = k * nkv + j - 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&pv_full[t * 2 + (gp & 1)],
                                                           (gp >> 1) & 1, a.err, abort_flag));
                    if (!ok)
                        break;
                    tc_fence_after();
                    const uint64_t f2v = f2_make(factor, factor);
#pragma unroll
                    for (int c = 0; c < 3; c++) {
                        uint32_t o[32];
                        const int w = c < 2 ? 32 : 16;
                        if (c < 2)
                            tmem_ld32(tO + c * 32, o);
                        else
                            tmem_ld16(tO + 64, *reinterpret_cast<uint32_t(*)[16]>(o));
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            if (e < w) {
                                float o0, o1;
                                f2_split(mul2(f2_make(__uint_as_float(o[e]),
                                                      __uint_as_float(o[e + 1])),
                                              f2v),
                                         o0, o1);
                                o[e] = __float_as_uint(o0);
                                o[e + 1] = __float_as_uint(o1);
                            }
                        }
                        if (c < 2)
                            tmem_st32(tO + c * 32, o);
                        else
                            tmem_st16(tO + 64, *reinterpret_cast<const uint32_t(*)[16]>(o));
                    }
                }
                // P(n) (and a rescaled O) is in TMEM: ready for the MMA.
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&p_ready[buf]);
                if ((buf += 2) >= NSB) {
                    buf -= NSB;
                    bph ^= 1;
                }
            }
            if (!ok)
                break;
            // End of the item: O after P.V of its last KV tile, normalised by
            // the row sum in column 64.
            {
                const int gl = k * nkv + nkv - 1;
                ok = __all_sync(0xffffffffu, mbar_wait(&pv_full[t * 2 + (gl & 1)],
                                                       (gl >> 1) & 1, a.err, abort_flag));
                if (!ok)
                    break;
            }
            if (rows_live) {
                tc_fence_after();
                uint32_t ov[64];
                uint32_t lsum[16];
                tmem_ld32(tO, *reinterpret_cast<uint32_t(*)[32]>(ov));
                tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(ov + 32));
                tmem_ld16(tO + 64, lsum);
                tmem_wait_ld();
                const float inv = 1.0f / __uint_as_float(lsum[0]);
                const int q = me.qt * BQ + r;
                if (q < a.N) {
                    const long orow = (long)(seq * a.N + q) * a.E + me.head * HD;
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
                // O may now be reset by the next item's first P.V (issued
                // only after this warp's next p_ready arrival).
                tc_fence_before();
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
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    AttnArgs a;
    a.nseq = nseq;
    a.N = N;
    a.E = E;
    a.heads = heads;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.err = err;
    const int full = N / BQ, tail = N % BQ != 0;
    a.nqt = full + tail;
    a.npf = full / 2;
    a.nleft = (full & 1) + tail;
    a.left_tile = 2 * a.npf;  // the first leftover tile (odd full tile, or the tail)
    a.per_seq = heads * a.npf + (a.nleft == 2 ? heads : (a.nleft == 1 ? (heads + 1) / 2 : 0));
    a.pair_tails = (long)nseq * a.per_seq >= 8L * sms;
    if (!a.pair_tails)
        a.per_seq = heads * ((a.nqt + 1) / 2);
    const long nitems = (long)nseq * a.per_seq;
    if (nitems > 0x7fffffffL)
        return K_EARG;
    a.nitems = (int)nitems;
    const int grid = nitems < sms ? (int)nitems : sms;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    return out_bf16 ? launch<true>(tq, tkv, a, grid, st) : launch<false>(tq, tkv, a, grid, st);
}
