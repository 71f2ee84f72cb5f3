// SPDX-License-Identifier: Unlicense
// The mask decoder's fused attention (mha, sam3_model.c:419-451): 8 heads
// of c = dint / 8 channels, scale 1/sqrt(c), per-prompt strides sq / sk / sv
// (elements; 0 shares one K/V among all prompts), output [P * Nq, dint].
// It is bound by HBM, so both kernels are shaped around moving the bytes once
// with enough of them in flight:
//
//   few keys (Nk <= 64: image-to-token, token self-attention;
//   attn_fewkeys, sam3_kernels.cl:527-569): persistent CTAs, each taking a
//   contiguous range of 32-query units (so a prompt's K and V, a few KB, are
//   staged in shared memory once per CTA and prompt), one thread per
//   (query, head), the next unit's query loaded while the current one
//   computes; the 8 heads of a query sit in 8 adjacent threads (whole
//   512-byte rows per 8 threads); softmax over the keys from shared memory
//   (two passes for up to 8 keys, online beyond);
//
//   many keys (Nk > 64, c = 16: token-to-image; attn_manykeys,
//   sam3_kernels.cl:577-633): the prompts' 32-key chunks form one sequence
//   cut into equal ranges, one per CTA slot (two per SM), so that every SM
//   streams K/V (a prompt's K/V is 2.6 MB in fp32); a CTA (one range, for 8
//   queries) pulls the chunks of K and V with cp.async through a 3-stage
//   ring while its 256 threads (32 (query pair, head) items x 8 key lanes,
//   each K/V read serving two queries) run a blocked online softmax over the
//   oldest chunk with packed f32x2 arithmetic; at the end of each prompt in
//   its range it merges its key lanes and writes one (m, l, o) partial per
//   (query, head); a second kernel combines the partials of each prompt.
//
// The 8 different heads a warp reads at once fall on distinct shared-memory
// bank groups: rows padded to c + 4 floats per head (few keys) or 16-byte
// chunks rotated per head (many keys, rows stay 512 bytes for cp.async).
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

namespace sam3 {
namespace {

constexpr int kHeads = 8;

// Two floats rounded to nearest-even bf16, packed low / high.
__device__ __forceinline__ uint32_t bf16_pair(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem)
{
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_commit()
{
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------ few keys
constexpr int kFewSmall = 8;              // key counts up to this take two passes

template <int C>
__device__ __forceinline__ void load_q(const float *qp, float (&q)[C], float scale)
{
    const float4 *q4 = reinterpret_cast<const float4 *>(qp);
#pragma unroll
    for (int c = 0; c < C / 4; c++) {
        const float4 v = __ldg(q4 + c);
        q[4 * c] = v.x * scale;
        q[4 * c + 1] = v.y * scale;
        q[4 * c + 2] = v.z * scale;
        q[4 * c + 3] = v.w * scale;
    }
}

template <int C>
__global__ void __launch_bounds__(256, C == 16 ? 3 : 1) mha_few_kernel(const float *__restrict__ Q, long sq,
                                                      const float *__restrict__ K, long sk,
                                                      const float *__restrict__ V, long sv,
                                                      float *__restrict__ O, int P, int Nq,
                                                      int Nk, float scale)
{
    constexpr int D = C * kHeads, CP = C + 4, ROW = kHeads * CP;
    extern __shared__ float kv[];  // K rows then V rows, [Nk][8][CP] each
    float *ks = kv;
    float *vs = kv + Nk * ROW;
    const int h = threadIdx.x & 7, qt = threadIdx.x >> 3;
    // Units of 32 queries of one prompt; this CTA takes a contiguous range
    // (mostly one prompt, so its K/V are staged once), sized so that all
    // CTAs finish together.
    const int nqb = (Nq + 31) / 32;
    const long U = (long)P * nqb;
    const long u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
    float q[C];
    if (u0 < u1) {
        const long p = u0 / nqb;
        const int qi = (int)(u0 - p * nqb) * 32 + qt;
        if (qi < Nq)
            load_q<C>(Q + p * sq + (long)qi * D + h * C, q, scale);
    }
    long staged = -1;
#pragma unroll 1
    for (long u = u0; u < u1; u++) {
        const long p = u / nqb;
        const int qi = (int)(u - p * nqb) * 32 + qt;
        if (p != staged) {  // CTA-uniform: stage this prompt's K and V
            __syncthreads();
            const float *kb = K + p * sk, *vb = V + p * sv;
            for (int i = threadIdx.x; i < Nk * (D / 4); i += blockDim.x) {
                const int j = i / (D / 4), col = (i - j * (D / 4)) * 4;
                const int dst = j * ROW + (col / C) * CP + col % C;
                *reinterpret_cast<float4 *>(ks + dst) =
                    __ldg(reinterpret_cast<const float4 *>(kb + (long)j * D + col));
                *reinterpret_cast<float4 *>(vs + dst) =
                    __ldg(reinterpret_cast<const float4 *>(vb + (long)j * D + col));
            }
            __syncthreads();
            staged = p;
        }
        // The next unit's query in flight while this one computes.
        float qn[C];
        bool more = false;
        if (u + 1 < u1) {
            const long pn = (u + 1) / nqb;
            const int qin = (int)(u + 1 - pn * nqb) * 32 + qt;
            more = qin < Nq;
            if (more)
                load_q<C>(Q + pn * sq + (long)qin * D + h * C, qn, scale);
        }
        if (qi >= Nq) {
            if (more)
#pragma unroll
                for (int c = 0; c < C; c++)
                    q[c] = qn[c];
            continue;
        }
        float m = -INFINITY, l = 0.0f, o[C];
#pragma unroll
        for (int c = 0; c < C; c++)
            o[c] = 0.0f;
        if (Nk <= kFewSmall) {
            // Two passes over at most 8 keys: independent scores, one
            // maximum, then the exponentials and P.V without rescaling.
            float sc[kFewSmall];
#pragma unroll
            for (int j = 0; j < kFewSmall; j++) {
                sc[j] = -INFINITY;
                if (j < Nk) {
                    const float4 *kr = reinterpret_cast<const float4 *>(ks + j * ROW + h * CP);
                    float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;
#pragma unroll
                    for (int c = 0; c < C / 4; c++) {
                        const float4 k4 = kr[c];
                        d0 = fmaf(q[4 * c], k4.x, d0);
                        d1 = fmaf(q[4 * c + 1], k4.y, d1);
                        d2 = fmaf(q[4 * c + 2], k4.z, d2);
                        d3 = fmaf(q[4 * c + 3], k4.w, d3);
                    }
                    sc[j] = (d0 + d1) + (d2 + d3);
                    m = fmaxf(m, sc[j]);
                }
            }
#pragma unroll
            for (int j = 0; j < kFewSmall; j++) {
                if (j < Nk) {
                    const float e = __expf(sc[j] - m);
                    l += e;
                    const float4 *vr = reinterpret_cast<const float4 *>(vs + j * ROW + h * CP);
#pragma unroll
                    for (int c = 0; c < C / 4; c++) {
                        const float4 v4 = vr[c];
                        o[4 * c] = fmaf(e, v4.x, o[4 * c]);
                        o[4 * c + 1] = fmaf(e, v4.y, o[4 * c + 1]);
                        o[4 * c + 2] = fmaf(e, v4.z, o[4 * c + 2]);
                        o[4 * c + 3] = fmaf(e, v4.w, o[4 * c + 3]);
                    }
                }
            }
        }
        else
        for (int j = 0; j < Nk; j++) {
            const float4 *kr = reinterpret_cast<const float4 *>(ks + j * ROW + h * CP);
            float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;  // four short chains
#pragma unroll
            for (int c = 0; c < C / 4; c++) {
                const float4 k4 = kr[c];
                d0 = fmaf(q[4 * c], k4.x, d0);
                d1 = fmaf(q[4 * c + 1], k4.y, d1);
                d2 = fmaf(q[4 * c + 2], k4.z, d2);
                d3 = fmaf(q[4 * c + 3], k4.w, d3);
            }
            const float s = (d0 + d1) + (d2 + d3);
            const float mn = fmaxf(m, s), corr = __expf(m - mn), e = __expf(s - mn);
            l = l * corr + e;
            const float4 *vr = reinterpret_cast<const float4 *>(vs + j * ROW + h * CP);
#pragma unroll
            for (int c = 0; c < C / 4; c++) {
                const float4 v4 = vr[c];
                o[4 * c] = fmaf(e, v4.x, o[4 * c] * corr);
                o[4 * c + 1] = fmaf(e, v4.y, o[4 * c + 1] * corr);
                o[4 * c + 2] = fmaf(e, v4.z, o[4 * c + 2] * corr);
                o[4 * c + 3] = fmaf(e, v4.w, o[4 * c + 3] * corr);
            }
            m = mn;
        }
        const float inv = 1.0f / l;
        float4 *op = reinterpret_cast<float4 *>(O + (p * Nq + qi) * D + h * C);
#pragma unroll
        for (int c = 0; c < C / 4; c++)
            op[c] = make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv,
                                o[4 * c + 3] * inv);
        if (more) {
#pragma unroll
            for (int c = 0; c < C; c++)
                q[c] = qn[c];
        }
    }
}

// Image -> token attention (at most kFewSmall keys, 16 channels per head):
// the kernel above is bound by shared-memory bandwidth (every (query, head)
// thread reads its head's K and V rows for each key). Here a thread takes
// two queries of one head, so each K / V read from shared memory serves
// both: units of 64 queries, thread (head h, slot qt) computing queries
// qt and qt + 32 of the unit, the next unit's two queries in flight while
// this one computes. Same arithmetic per query as the small path above.
// Q_BF16: Q is read as bf16 (written so by its projection); OUT_BF16: O is
// written as bf16 (for a consumer that only feeds a GEMM).
template <bool Q_BF16, bool OUT_BF16>
__global__ void __launch_bounds__(256, 2) mha_few2_kernel(const void *__restrict__ Q, long sq,
                                                         const float *__restrict__ K, long sk,
                                                         const float *__restrict__ V, long sv,
                                                         void *__restrict__ O, int P, int Nq,
                                                         int Nk, float scale)
{
    constexpr int C = 16, D = C * kHeads, CP = C + 4, ROW = kHeads * CP;
    extern __shared__ float kv[];  // K rows then V rows, [Nk][8][CP] each
    float *ks = kv;
    float *vs = kv + Nk * ROW;
    const int h = threadIdx.x & 7, qt = threadIdx.x >> 3;
    const int nqb = (Nq + 63) / 64;
    const long U = (long)P * nqb;
    const long u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
    float q[2][C];
    auto load2 = [&](long u, float (&dst)[2][C]) {
        const long pu = u / nqb;
        const int qb = (int)(u - pu * nqb) * 64 + qt;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int qi = qb + 32 * i;
            if (qi >= Nq)
                continue;
            const long off = pu * sq + (long)qi * D + h * C;
            if (Q_BF16) {
                const uint4 *q4 =
                    reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(Q) + off);
#pragma unroll
                for (int c = 0; c < C / 8; c++) {
                    const uint4 w = __ldg(q4 + c);
                    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        dst[i][8 * c + 2 * k] = __uint_as_float(ws[k] << 16) * scale;
                        dst[i][8 * c + 2 * k + 1] = __uint_as_float(ws[k] & 0xffff0000u) * scale;
                    }
                }
            }
            else
                load_q<C>(reinterpret_cast<const float *>(Q) + off, dst[i], scale);
        }
    };
    if (u0 < u1)
        load2(u0, q);
    long staged = -1;
#pragma unroll 1
    for (long u = u0; u < u1; u++) {
        const long p = u / nqb;
        const int qb = (int)(u - p * nqb) * 64 + qt;
        if (p != staged) {  // CTA-uniform: stage this prompt's K and V
            __syncthreads();
            const float *kb = K + p * sk, *vb = V + p * sv;
            for (int i = threadIdx.x; i < Nk * (D / 4); i += blockDim.x) {
                const int j = i / (D / 4), col = (i - j * (D / 4)) * 4;
                const int dst = j * ROW + (col / C) * CP + col % C;
                *reinterpret_cast<float4 *>(ks + dst) =
                    __ldg(reinterpret_cast<const float4 *>(kb + (long)j * D + col));
                *reinterpret_cast<float4 *>(vs + dst) =
                    __ldg(reinterpret_cast<const float4 *>(vb + (long)j * D + col));
            }
            __syncthreads();
            staged = p;
        }
        float qn[2][C];
        const bool more = u + 1 < u1;
        if (more)
            load2(u + 1, qn);
        if (qb < Nq) {
            float sc[2][kFewSmall], m[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < kFewSmall; j++) {
                sc[0][j] = sc[1][j] = -INFINITY;
                if (j < Nk) {
                    const float4 *kr = reinterpret_cast<const float4 *>(ks + j * ROW + h * CP);
                    float d[2][4] = {};
#pragma unroll
                    for (int c = 0; c < C / 4; c++) {
                        const float4 k4 = kr[c];
#pragma unroll
                        for (int i = 0; i < 2; i++) {
                            d[i][0] = fmaf(q[i][4 * c], k4.x, d[i][0]);
                            d[i][1] = fmaf(q[i][4 * c + 1], k4.y, d[i][1]);
                            d[i][2] = fmaf(q[i][4 * c + 2], k4.z, d[i][2]);
                            d[i][3] = fmaf(q[i][4 * c + 3], k4.w, d[i][3]);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 2; i++) {
                        sc[i][j] = (d[i][0] + d[i][1]) + (d[i][2] + d[i][3]);
                        m[i] = fmaxf(m[i], sc[i][j]);
                    }
                }
            }
            float o[2][C], l[2] = {0.0f, 0.0f};
#pragma unroll
            for (int c = 0; c < C; c++)
                o[0][c] = o[1][c] = 0.0f;
#pragma unroll
            for (int j = 0; j < kFewSmall; j++) {
                if (j < Nk) {
                    float e[2];
#pragma unroll
                    for (int i = 0; i < 2; i++) {
                        e[i] = __expf(sc[i][j] - m[i]);
                        l[i] += e[i];
                    }
                    const float4 *vr = reinterpret_cast<const float4 *>(vs + j * ROW + h * CP);
#pragma unroll
                    for (int c = 0; c < C / 4; c++) {
                        const float4 v4 = vr[c];
#pragma unroll
                        for (int i = 0; i < 2; i++) {
                            o[i][4 * c] = fmaf(e[i], v4.x, o[i][4 * c]);
                            o[i][4 * c + 1] = fmaf(e[i], v4.y, o[i][4 * c + 1]);
                            o[i][4 * c + 2] = fmaf(e[i], v4.z, o[i][4 * c + 2]);
                            o[i][4 * c + 3] = fmaf(e[i], v4.w, o[i][4 * c + 3]);
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int qi = qb + 32 * i;
                if (qi < Nq) {
                    const float inv = 1.0f / l[i];
                    const long off = (p * Nq + qi) * D + h * C;
                    if (OUT_BF16) {
                        uint4 *op = reinterpret_cast<uint4 *>(
                            reinterpret_cast<__nv_bfloat16 *>(O) + off);
#pragma unroll
                        for (int c = 0; c < C / 8; c++)
                            op[c] = make_uint4(
                                bf16_pair(o[i][8 * c] * inv, o[i][8 * c + 1] * inv),
                                bf16_pair(o[i][8 * c + 2] * inv, o[i][8 * c + 3] * inv),
                                bf16_pair(o[i][8 * c + 4] * inv, o[i][8 * c + 5] * inv),
                                bf16_pair(o[i][8 * c + 6] * inv, o[i][8 * c + 7] * inv));
                    }
                    else {
                        float4 *op = reinterpret_cast<float4 *>(reinterpret_cast<float *>(O) + off);
#pragma unroll
                        for (int c = 0; c < C / 4; c++)
                            op[c] = make_float4(o[i][4 * c] * inv, o[i][4 * c + 1] * inv,
                                                o[i][4 * c + 2] * inv, o[i][4 * c + 3] * inv);
                    }
                }
            }
        }
        if (more) {
#pragma unroll
            for (int c = 0; c < C; c++) {
                q[0][c] = qn[0][c];
                q[1][c] = qn[1][c];
            }
        }
    }
}

// ------------------------------------------------------------ many keys
constexpr int kManyC = 16;                 // channels per head
constexpr int kManyD = kManyC * kHeads;    // 128
constexpr int kManyRow = kManyD;           // 128 floats per staged key
constexpr int kChunk = 32;                 // keys per staged chunk
constexpr int kStages = 3;                 // staged chunks in flight
constexpr int kLanes = 8;                  // key lanes per (query, head)
constexpr int kPart = 2 + kManyC;          // m, l, o[16]
constexpr float kManyLazy = 8.0f;          // rescale threshold (natural log units)
constexpr int kManySmem = kStages * 2 * kChunk * kManyRow * 4;  // K and V rings

// Position (in floats) of channels 4c..4c+3 of head h within a staged key
// row: the 16-byte chunks of a head are rotated by h / 2, so the 8 heads a
// warp reads at one c fall on 8 different 16-byte bank groups.
__device__ __forceinline__ int many_pos(int h, int c4)
{
    return h * kManyC + (((c4 + (h >> 1)) & 3) << 2);
}

// Byte offset of the 16-byte piece `half` (channels 8 half .. 8 half + 7)
// of head h within a staged bf16 key row (256 bytes): the halves of heads
// 4-7 are swapped, so the eight heads' reads of one half hit distinct banks.
__device__ __forceinline__ int many_pos_bf16(int h, int half)
{
    return h * 32 + ((half ^ (h >> 2)) & 1) * 16;
}

// Eight bf16 values (one 16-byte piece) widened to fp32 as four pairs
// (channels 2k, 2k + 1 in pair k) for the packed arithmetic.
__device__ __forceinline__ void widen8x2(const uint4 w, uint64_t (&f)[4])
{
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; k++)
        f[k] = f2_make(__uint_as_float(ws[k] << 16), __uint_as_float(ws[k] & 0xffff0000u));
}

// Work of the many-keys kernel: the P prompts' 32-key chunks taken as one
// sequence of T = P * nch chunks, CTA g of G doing chunks [g T / G,
// (g + 1) T / G) (whole prompts' shares differ by at most one chunk, and
// every SM slot gets one CTA). A CTA's range crosses at most `segs` prompts;
// it writes one partial per (prompt segment, query, head).
__host__ __device__ __forceinline__ long many_chunk0(long g, long T, long G)
{
    return g * T / G;
}

// KV_BF16: K and V are bf16 rows (as the decoder's projections write them);
// staged the same way in half the shared memory and widened on read. The
// dot products and P.V updates use the packed f32x2 instructions on channel
// pairs, with the same four partial sums per score and the same
// accumulation order as the scalar form.
template <bool KV_BF16>
__global__ void __launch_bounds__(256, 2) mha_many_split_kernel(
    const float *__restrict__ Q, long sq, const void *__restrict__ Kv, long sk,
    const void *__restrict__ Vv, long sv, float *__restrict__ part, int P, int Nq, int Nk,
    int segs, float scale)
{
    extern __shared__ __align__(16) float sm[];
    constexpr int ROWF = KV_BF16 ? kManyRow / 2 : kManyRow;  // staged row, in floats
    constexpr int BUF = 2 * kChunk * ROWF;                   // one stage: K rows, then V rows
    const int nch = (Nk + kChunk - 1) / kChunk;
    const long T = (long)P * nch, G = gridDim.x;
    const long c0 = many_chunk0(blockIdx.x, T, G), c1 = many_chunk0(blockIdx.x + 1, T, G);
    const int nloc = (int)(c1 - c0);
    const long p_first = c0 / nch;
    // Thread = (query pair, head, key lane): queries qg and qg + 4 of the
    // CTA's 8 share every K/V read from shared memory; a warp is one key lane.
    const int h = threadIdx.x & 7, qg = (threadIdx.x >> 3) & 3, lane = threadIdx.x >> 5;
    const int qa = blockIdx.z * 8 + qg, qb = qa + 4;

    // Chunk i of this CTA's range into stage b: 16-byte pieces into rotated rows.
    auto stage = [&](int i, int b) {
        const long idx = c0 + i, p = idx / nch;
        const int j0 = (int)(idx - p * nch) * kChunk, n = min(kChunk, Nk - j0);
        const char *kb = reinterpret_cast<const char *>(Kv) + p * sk * (KV_BF16 ? 2 : 4);
        const char *vb = reinterpret_cast<const char *>(Vv) + p * sv * (KV_BF16 ? 2 : 4);
        float *ks = sm + b * BUF, *vs = ks + kChunk * ROWF;
        constexpr int PIECES = kManyD * (KV_BF16 ? 2 : 4) / 16;  // per key row
        for (int t = threadIdx.x; t < n * PIECES; t += blockDim.x) {
            const int j = t / PIECES, pc = t - j * PIECES;
            int dst;  // in floats
            if (KV_BF16)
                dst = j * ROWF + many_pos_bf16(pc >> 1, pc & 1) / 4;
            else
                dst = j * ROWF + many_pos(pc / 4, pc % 4);
            const long src = ((long)(j0 + j) * PIECES + pc) * 16;  // bytes
            cp_async16(ks + dst, kb + src);
            cp_async16(vs + dst, vb + src);
        }
        cp_async_commit();
    };

    uint64_t q2[2][kManyC / 2], o2[2][kManyC / 2];
    float m[2], l[2];
    auto start_segment = [&](long p) {
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int qq = (u ? qb : qa) < Nq ? (u ? qb : qa) : 0;
            const float4 *qp =
                reinterpret_cast<const float4 *>(Q + p * sq + (long)qq * kManyD + h * kManyC);
#pragma unroll
            for (int c = 0; c < kManyC / 4; c++) {
                const float4 v = __ldg(qp + c);
                q2[u][2 * c] = f2_make(v.x * scale, v.y * scale);
                q2[u][2 * c + 1] = f2_make(v.z * scale, v.w * scale);
            }
            m[u] = -INFINITY;
            l[u] = 0.0f;
#pragma unroll
            for (int c = 0; c < kManyC / 2; c++)
                o2[u][c] = 0;
        }
    };
    // Merges the 8 key lanes of each (query, head) through stage b (free
    // when this runs: its chunk is consumed and the next one is not yet
    // requested) and writes segment k's partials; one query half per pass.
    auto flush = [&](int b, long k) {
        float *mer = sm + b * BUF;  // [7 lanes][32 (query, head)][kPart]
        static_assert(7 * 32 * kPart <= (KV_BF16 ? 2 * kChunk * kManyRow / 2 : 2 * kChunk * kManyRow),
                      "lane records fit in one stage");
#pragma unroll
        for (int u = 0; u < 2; u++) {  // unrolled: o2, m, l stay in registers
            const int slot = qg * kHeads + h;
            if (lane > 0) {
                float *mine = mer + ((lane - 1) * 32 + slot) * kPart;
                mine[0] = m[u];
                mine[1] = l[u];
#pragma unroll
                for (int c = 0; c < kManyC / 2; c++)
                    f2_split(o2[u][c], mine[2 + 2 * c], mine[3 + 2 * c]);
            }
            __syncthreads();
            const int qi = u ? qb : qa;
            if (lane == 0 && qi < Nq) {
                float M = m[u];
                for (int t = 0; t < kLanes - 1; t++)
                    M = fmaxf(M, mer[(t * 32 + slot) * kPart]);
                float acc[kManyC];
                const float f0 = m[u] == -INFINITY ? 0.0f : __expf(m[u] - M);
                float L = l[u] * f0;
#pragma unroll
                for (int c = 0; c < kManyC / 2; c++) {
                    float a0, a1;
                    f2_split(o2[u][c], a0, a1);
                    acc[2 * c] = a0 * f0;
                    acc[2 * c + 1] = a1 * f0;
                }
                for (int t = 0; t < kLanes - 1; t++) {
                    const float *pt = mer + (t * 32 + slot) * kPart;
                    const float f = pt[0] == -INFINITY ? 0.0f : __expf(pt[0] - M);
                    L += pt[1] * f;
#pragma unroll
                    for (int cc = 0; cc < kManyC; cc++)
                        acc[cc] = fmaf(pt[2 + cc], f, acc[cc]);
                }
                float *dst = part + (((blockIdx.x * (long)segs + k) * Nq + qi) * kHeads + h) * kPart;
                dst[0] = M;
                dst[1] = L;
#pragma unroll
                for (int cc = 0; cc < kManyC; cc++)
                    dst[2 + cc] = acc[cc];
            }
            __syncthreads();
        }
    };

    // Ring of kStages chunks: chunks i+1 and i+2 load while i computes (an
    // empty commit group keeps the wait count uniform at the tail).
    for (int i = 0; i < kStages - 1; i++) {
        if (i < nloc)
            stage(i, i);
        else
            cp_async_commit();
    }
    for (int i = 0; i < nloc; i++) {
        const int b = i % kStages;
        const long idx = c0 + i, p = idx / nch;
        const int ci = (int)(idx - p * nch);
        if (i == 0 || ci == 0)
            start_segment(p);
        if (i + kStages - 1 < nloc)  // its stage was released by the barrier below
            stage(i + kStages - 1, (i + kStages - 1) % kStages);
        else
            cp_async_commit();
        cp_async_wait<kStages - 1>();
        __syncthreads();
        const float *ks = sm + b * BUF, *vs = ks + kChunk * ROWF;
        const int n = min(kChunk, Nk - ci * kChunk);
        // This lane's keys of the chunk as one block per query: scores, block
        // maximum, one correction, then P.V.
        constexpr int KT = kChunk / kLanes;
        float s[2][KT];
        float bm[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int t = 0; t < KT; t++) {
            const int j = t * kLanes + lane;
            s[0][t] = s[1][t] = -INFINITY;
            if (j < n) {
                const float *kr = ks + j * ROWF;
                uint64_t dA[2] = {0, 0}, dB[2] = {0, 0};  // channel pairs (4c, 4c+1), (4c+2, 4c+3)
                if (KV_BF16) {
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        uint64_t kv[4];
                        widen8x2(*reinterpret_cast<const uint4 *>(
                                     reinterpret_cast<const char *>(kr) + many_pos_bf16(h, hf)),
                                 kv);
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            dA[u] = fma2(q2[u][4 * hf], kv[0], dA[u]);
                            dB[u] = fma2(q2[u][4 * hf + 1], kv[1], dB[u]);
                            dA[u] = fma2(q2[u][4 * hf + 2], kv[2], dA[u]);
                            dB[u] = fma2(q2[u][4 * hf + 3], kv[3], dB[u]);
                        }
                    }
                }
                else
#pragma unroll
                for (int cc = 0; cc < kManyC / 4; cc++) {
                    const ulonglong2 k2 = *reinterpret_cast<const ulonglong2 *>(kr + many_pos(h, cc));
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        dA[u] = fma2(q2[u][2 * cc], k2.x, dA[u]);
                        dB[u] = fma2(q2[u][2 * cc + 1], k2.y, dB[u]);
                    }
                }
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    float d0, d1, d2, d3;
                    f2_split(dA[u], d0, d1);
                    f2_split(dB[u], d2, d3);
                    s[u][t] = (d0 + d1) + (d2 + d3);
                    bm[u] = fmaxf(bm[u], s[u][t]);
                }
            }
        }
        if (bm[0] > -INFINITY) {  // the key count is the same for both queries
            uint64_t e2[2][KT];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                // The running maximum is raised (and o, l rescaled) only when
                // the block's maximum exceeds it by more than kManyLazy, so
                // e <= e^kManyLazy and most blocks skip the rescale; the
                // final normalisation makes the result independent of it.
                if (bm[u] > m[u] + kManyLazy) {
                    const float corr = __expf(m[u] - bm[u]);  // 0 on the first block
                    l[u] *= corr;
                    const uint64_t c2 = f2_make(corr, corr);
#pragma unroll
                    for (int cc = 0; cc < kManyC / 2; cc++)
                        o2[u][cc] = mul2(o2[u][cc], c2);
                    m[u] = bm[u];
                }
#pragma unroll
                for (int t = 0; t < KT; t++) {
                    const float e = __expf(s[u][t] - m[u]);  // 0 for keys past the chunk
                    l[u] += e;
                    e2[u][t] = f2_make(e, e);
                }
            }
#pragma unroll
            for (int t = 0; t < KT; t++) {
                const int j = t * kLanes + lane;
                if (j < n) {
                    const float *vr = vs + j * ROWF;
                    if (KV_BF16) {
#pragma unroll
                        for (int hf = 0; hf < 2; hf++) {
                            uint64_t vv[4];
                            widen8x2(*reinterpret_cast<const uint4 *>(
                                         reinterpret_cast<const char *>(vr) + many_pos_bf16(h, hf)),
                                     vv);
#pragma unroll
                            for (int ci2 = 0; ci2 < 4; ci2++)
#pragma unroll
                                for (int u = 0; u < 2; u++)
                                    o2[u][4 * hf + ci2] = fma2(e2[u][t], vv[ci2], o2[u][4 * hf + ci2]);
                        }
                    }
                    else
#pragma unroll
                    for (int cc = 0; cc < kManyC / 4; cc++) {
                        const ulonglong2 v2 = *reinterpret_cast<const ulonglong2 *>(vr + many_pos(h, cc));
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            o2[u][2 * cc] = fma2(e2[u][t], v2.x, o2[u][2 * cc]);
                            o2[u][2 * cc + 1] = fma2(e2[u][t], v2.y, o2[u][2 * cc + 1]);
                        }
                    }
                }
            }
        }
        __syncthreads();  // stage b may be refilled from the next iteration on
        if (ci == nch - 1 || i == nloc - 1)
            flush(b, p - p_first);
    }
}

// Combines the partials of each (prompt, query, head): those of the CTAs
// whose chunk ranges meet the prompt's chunks [p nch, (p + 1) nch), at
// segment p - (first prompt of the CTA).
__global__ void mha_many_combine_kernel(const float *__restrict__ part, float *__restrict__ O,
                                        int P, int Nq, int nch, int G, int segs)
{
    const long g = (long)blockIdx.x * blockDim.x + threadIdx.x;  // (p, qi, h)
    if (g >= (long)P * Nq * kHeads)
        return;
    const int h = (int)(g % kHeads);
    const int qi = (int)((g / kHeads) % Nq);
    const long p = g / ((long)kHeads * Nq);
    const long T = (long)P * nch;
    // CTA holding chunk c: the largest x with x T / G <= c, i.e.
    // ceil((c + 1) G / T) - 1.
    const long x0 = ((p * nch + 1) * G + T - 1) / T - 1;
    const long x1 = (((p + 1) * nch) * G + T - 1) / T - 1;
    auto rec = [&](long x) {
        const long k = p - many_chunk0(x, T, G) / nch;
        return part + (((x * segs + k) * Nq + qi) * kHeads + h) * kPart;
    };
    float M = -INFINITY;
    for (long x = x0; x <= x1; x++)
        M = fmaxf(M, rec(x)[0]);
    float L = 0.0f, acc[kManyC];
#pragma unroll
    for (int cc = 0; cc < kManyC; cc++)
        acc[cc] = 0.0f;
    for (long x = x0; x <= x1; x++) {
        const float *pt = rec(x);
        const float f = pt[0] == -INFINITY ? 0.0f : expf(pt[0] - M);
        L += pt[1] * f;
#pragma unroll
        for (int cc = 0; cc < kManyC; cc++)
            acc[cc] = fmaf(pt[2 + cc], f, acc[cc]);
    }
    const float inv = 1.0f / L;
    float4 *op = reinterpret_cast<float4 *>(O + (p * Nq + qi) * kManyD + h * kManyC);
#pragma unroll
    for (int cc = 0; cc < kManyC / 4; cc++)
        op[cc] = make_float4(acc[4 * cc] * inv, acc[4 * cc + 1] * inv, acc[4 * cc + 2] * inv,
                             acc[4 * cc + 3] * inv);
}

// Plan of the many-keys kernel: G CTAs per query group of 8 (two per SM
// over all groups, at most one per chunk) and the most prompt segments a
// CTA's chunk range can cross.
struct ManyPlan {
    int G, segs;
};

ManyPlan many_plan(int P, int Nq, int Nk, int num_sms)
{
    const long nch = (Nk + kChunk - 1) / kChunk, T = (long)P * nch;
    const long nz = (Nq + 7) / 8;
    long G = 2L * num_sms / nz;
    if (G < 1)
        G = 1;
    if (G > T)
        G = T;
    const long per = (T + G - 1) / G;  // chunks of the longest range
    return {(int)G, (int)((per - 1) / nch + 2)};
}

size_t many_workspace(int P, int Nq, int Nk, int num_sms)
{
    const ManyPlan pl = many_plan(P, Nq, Nk, num_sms);
    return (size_t)pl.G * pl.segs * Nq * kHeads * kPart * sizeof(float);
}

template <bool Q_BF16, bool OUT_BF16>
int launch_few2(int P, int Nq, int Nk, const void *qp, long sq, const float *kp, long sk,
                const float *vp, long sv, void *o, float scale, int num_sms, cudaStream_t st)
{
    const int smem = 2 * Nk * kHeads * (16 + 4) * 4;
    cudaError_t e = smem_limit_once<mha_few2_kernel<Q_BF16, OUT_BF16>>(smem);
    if (e != cudaSuccess)
        return (int)e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mha_few2_kernel<Q_BF16, OUT_BF16>,
                                                      256, smem);
    if (e != cudaSuccess)
        return (int)e;
    const long units = (long)P * ((Nq + 63) / 64);
    const long cap = (long)num_sms * (per_sm > 0 ? per_sm : 1);
    mha_few2_kernel<Q_BF16, OUT_BF16><<<(unsigned)(units < cap ? units : cap), 256, smem, st>>>(
        qp, sq, kp, sk, vp, sv, o, P, Nq, Nk, scale);
    return (int)cudaGetLastError();
}

template <int C>
int launch_few(int P, int Nq, int Nk, const float *qp, long sq, const float *kp, long sk,
               const float *vp, long sv, float *o, float scale, int num_sms, cudaStream_t st)
{
    if (C == 16 && Nk <= kFewSmall)
        return launch_few2<false, false>(P, Nq, Nk, qp, sq, kp, sk, vp, sv, o, scale, num_sms, st);
    const int smem = 2 * Nk * kHeads * (C + 4) * 4;
    auto kern = mha_few_kernel<C>;
    cudaError_t e = smem_limit_once<mha_few_kernel<C>>(smem);
    if (e != cudaSuccess)
        return (int)e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem);
    if (e != cudaSuccess)
        return (int)e;
    const long units = (long)P * ((Nq + 31) / 32);
    const long cap = (long)num_sms * (per_sm > 0 ? per_sm : 1);
    kern<<<(unsigned)(units < cap ? units : cap), 256, smem, st>>>(qp, sq, kp, sk, vp, sv, o, P,
                                                                    Nq, Nk, scale);
    return (int)cudaGetLastError();
}

template <bool KV_BF16>
int launch_many(int P, int Nq, int Nk, const float *qp, long sq, const void *kp, long sk,
                const void *vp, long sv, float *o, void *ws, size_t ws_bytes, float scale,
                int num_sms, cudaStream_t st)
{
    const ManyPlan pl = many_plan(P, Nq, Nk, num_sms);
    if (!ws || ws_bytes < many_workspace(P, Nq, Nk, num_sms))
        return K_EARG;
    const int smem = KV_BF16 ? kManySmem / 2 : kManySmem;
    cudaError_t e = smem_limit_once<mha_many_split_kernel<KV_BF16>>(smem);
    if (e != cudaSuccess)
        return (int)e;
    dim3 grid(pl.G, 1, (Nq + 7) / 8);
    mha_many_split_kernel<KV_BF16><<<grid, 256, smem, st>>>(
        qp, sq, kp, sk, vp, sv, static_cast<float *>(ws), P, Nq, Nk, pl.segs, scale);
    e = cudaGetLastError();
    if (e != cudaSuccess)
        return (int)e;
    const long total = (long)P * Nq * kHeads;
    mha_many_combine_kernel<<<(unsigned)((total + 127) / 128), 128, 0, st>>>(
        static_cast<const float *>(ws), o, P, Nq, (Nk + kChunk - 1) / kChunk, pl.G, pl.segs);
    return (int)cudaGetLastError();
}

}  // namespace
}  // namespace sam3

extern "C" size_t k_mha_workspace(int P, int Nq, int Nk, int dint, int num_sms)
{
    if (Nk <= 64 || dint != sam3::kManyD || P <= 0 || Nq <= 0)
        return 0;
    return sam3::many_workspace(P, Nq, Nk, num_sms);
}

extern "C" int k_mha(int P, int Nq, int Nk, int dint, const float *qp, long sq, const float *kp,
                     long sk, const float *vp, long sv, float *o, void *ws, size_t ws_bytes,
                     int num_sms, k_stream s)
{
    using namespace sam3;
    const int c = dint / kHeads;
    const float scale = 1.0f / sqrtf((float)c);
    if (P <= 0 || Nq <= 0 || Nk <= 0 || dint % kHeads || ((uintptr_t)qp & 15) ||
        ((uintptr_t)kp & 15) || ((uintptr_t)vp & 15) || ((uintptr_t)o & 15) || (sq & 3) ||
        (sk & 3) || (sv & 3) || P > 65535)
        return K_EARG;
    cudaStream_t st = STREAM(s);
    if (Nk > 64) {
        // The reference rejects the same shape (sam3_model.c:429-430).
        if (c != kManyC)
            return K_EARG;
        return launch_many<false>(P, Nq, Nk, qp, sq, kp, sk, vp, sv, o, ws, ws_bytes, scale,
                                  num_sms, st);
    }
    if (c == 16)
        return launch_few<16>(P, Nq, Nk, qp, sq, kp, sk, vp, sv, o, scale, num_sms, st);
    if (c == 32)
        return launch_few<32>(P, Nq, Nk, qp, sq, kp, sk, vp, sv, o, scale, num_sms, st);
    return K_EARG;
}

extern "C" int k_mha_i2t_bf16(int P, int Nq, int Nk, const void *qp, long sq, const float *kp,
                              long sk, const float *vp, long sv, void *o, int num_sms, k_stream s)
{
    using namespace sam3;
    if (P <= 0 || Nq <= 0 || Nk <= 0 || Nk > kFewSmall || ((uintptr_t)qp & 15) ||
        ((uintptr_t)kp & 15) || ((uintptr_t)vp & 15) || ((uintptr_t)o & 15) || (sq & 3) ||
        (sk & 3) || (sv & 3))
        return K_EARG;
    return launch_few2<true, true>(P, Nq, Nk, qp, sq, kp, sk, vp, sv, o, 1.0f / sqrtf(16.0f), num_sms,
                             reinterpret_cast<cudaStream_t>(s));
}

extern "C" int k_mha_t2i_bf16kv(int P, int Nq, int Nk, const float *qp, long sq, const void *kp,
                                long sk, const void *vp, long sv, float *o, void *ws,
                                size_t ws_bytes, int num_sms, k_stream s)
{
    using namespace sam3;
    if (P <= 0 || Nq <= 0 || Nk <= 64 || P > 65535 || ((uintptr_t)qp & 15) ||
        ((uintptr_t)kp & 15) || ((uintptr_t)vp & 15) || ((uintptr_t)o & 15) || (sq & 3) ||
        (sk & 7) || (sv & 7))
        return K_EARG;
    return launch_many<true>(P, Nq, Nk, qp, sq, kp, sk, vp, sv, o, ws, ws_bytes,
                             1.0f / sqrtf((float)kManyC), num_sms, STREAM(s));
}
