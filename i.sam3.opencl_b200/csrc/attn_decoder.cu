// SPDX-License-Identifier: Unlicense
// The mask decoder's fused attention (mha, sam3_model.c:419-451): 8 heads
// of c = dint / 8 channels, scale 1/sqrt(c), per-prompt strides sq / sk / sv
// (elements; 0 shares one K/V among all prompts), output [P * Nq, dint].
// It is bound by HBM, so both kernels are shaped around moving the bytes once
// with enough of them in flight:
//
//   few keys (Nk <= 64: image-to-token, token self-attention;
//   attn_fewkeys, sam3_kernels.cl:527-569): persistent CTAs, each taking a
//   contiguous range of query units (so a prompt's K and V, a few KB, are
//   loaded once per CTA and prompt). Up to 8 keys with c = 16 (the
//   decoder's image-to-token attention): warp = head, 16-query units on
//   mma.sync tensor tiles (bf16 hi / lo operand pairs), the softmax over a
//   query's 8 keys across the 4 lanes of a quad. Otherwise one thread per
//   (query, head) on the CUDA cores, the 8 heads of a query in 8 adjacent
//   threads (whole 512-byte rows per 8 threads), K and V staged in shared
//   memory, softmax in two passes for up to 8 keys, online beyond;
//
//   many keys (Nk > 64, c = 16: token-to-image; attn_manykeys,
//   sam3_kernels.cl:577-633): the prompts' 32-key chunks form one sequence
//   cut into equal ranges, one per CTA slot (two per SM), so that every SM
//   streams K/V (a prompt's K/V is 2.6 MB in fp32); in a CTA (one range,
//   for 8 queries) a producer warp loads the chunks of K and V by TMA into
//   a 3-stage ring (full / empty mbarriers), each head warp takes Q.K^T and
//   P.V of every chunk on the tensor cores (mma.sync, bf16 operand pairs
//   hi + lo for fp32 accuracy) with an online softmax on the accumulators;
//   at the end of each prompt in its range it writes one (m, l, o) partial
//   per (query, head); a second kernel combines the partials of each
//   prompt.
//
// Shared-memory layouts keep a warp's reads on distinct bank groups: rows
// padded to c + 4 floats per head (few keys: the 8 heads a warp reads), or
// per-head key tiles with XOR-swizzled 16-byte pieces (many keys: the 8
// key rows of a fragment).
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <type_traits>

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
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
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

// ------------------------------------------------------------ many keys
constexpr int kManyC = 16;                 // channels per head
constexpr int kManyD = kManyC * kHeads;    // 128
constexpr int kChunk = 32;                 // keys per staged chunk
constexpr int kStages = 3;                 // staged chunks in flight
constexpr int kPart = 4 + kManyC;          // m, l, 2 unused, o[16] (16-byte aligned)
constexpr float kManyLazy = 8.0f;          // rescale threshold (log2 units)
// One stage: K then V, each [8 heads][32 keys][16 channels].
constexpr int kManyStage = 2 * kHeads * kChunk * kManyC;  // elements
constexpr int kManySmem = kStages * kManyStage * 4;       // bytes, fp32 K/V ring

// The bf16 tensor-core step: D += A (16 x 16, row-major) . B (16 x 8).
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two fp32 values as bf16 pairs hi + lo (lo = the rounding residual of hi,
// itself rounded): hi + lo carries about 16 significant bits, so products
// of such pairs summed as hi.hi + hi.lo + lo.hi keep fp32-level accuracy
// for these 16-term dot products. Lower half = x0.
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t &hi, uint32_t &lo)
{
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(x1), "f"(x0));
    const float r0 = x0 - __uint_as_float(hi << 16);
    const float r1 = x1 - __uint_as_float(hi & 0xffff0000u);
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(r1), "f"(r0));
}

// Transpose of an 8 x 8 bf16 tile held one row pair per thread (the
// accumulator layout) into the column-pair layout of an MMA B operand.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x)
{
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *p, bool trans)
{
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    if (trans)
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
    else
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

// Staged key tile layout, per (K or V, head): 32 rows of the head's 16
// channels, written by one TMA box load with the hardware swizzle that
// matches the row size: fp32 rows are 64 bytes whose 16-byte pieces are
// XOR-ed with (row >> 1) & 3 (64-byte swizzle), bf16 rows 32 bytes whose
// two pieces are XOR-ed with (row >> 2) & 1 (32-byte swizzle); tiles start
// 1024-byte aligned. The fragment loads of one warp (8 rows x a few
// channels) then hit every bank group equally.
__device__ __forceinline__ int many_sw32(int row, int piece)  // fp32: float offset in row
{
    return (piece ^ ((row >> 1) & 3)) * 4;
}

__device__ __forceinline__ int many_sw16(int row, int piece)  // bf16: element offset in row
{
    return (piece ^ ((row >> 2) & 1)) * 8;
}

// The bf16 tensor-core step with K = 8: D += A (16 x 8) . B (8 x 8).
__device__ __forceinline__ void mma_bf16_k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0)
{
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// Image -> token attention (at most 8 keys, 16 channels per head) on the
// tensor cores: a CTA takes a contiguous range of 16-query units (mostly of
// one prompt, whose K and V fragments it loads once), warp w = head w. Per
// unit, S (16 queries x 8 keys) = Q . K^T by mma.sync m16n8k16 and O
// (16 queries x 16 channels) = P . V by two m16n8k8 in bf16 with fp32
// accumulation, fp32 operands split into bf16 pairs hi + lo and each
// product taken as hi.hi + lo.hi + hi.lo (a bf16 Q is exact: one term
// fewer); K carries scale * log2 e, so S is in log2 units. A query row's 8
// scores sit in the 4 lanes of a quad: its maximum and sum are two
// shuffles each, and P stays in the accumulator layout, which is the A
// layout of the P . V step. The next unit's Q fragment loads while this
// one computes. Q_BF16: Q is read as bf16 (written so by its projection);
// OUT_BF16: O is written as bf16 (for a consumer that only feeds a GEMM).
template <bool Q_BF16, bool OUT_BF16>
__global__ void __launch_bounds__(256) mha_few2_kernel(const void *__restrict__ Q, long sq,
                                                      long ldq, const float *__restrict__ K,
                                                      long sk,
                                                      const float *__restrict__ V, long sv,
                                                      void *__restrict__ O, int P, int Nq, int Nk,
                                                      float kscale)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    constexpr int D = kManyD;
    const int lane = threadIdx.x & 31, h = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int nqb = (Nq + 15) / 16;
    const long U = (long)P * nqb;
    const long u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
    if (u0 >= u1)
        return;
    // Q fragment of a unit: (row g | g + 8) x channels (2t, 2t+1 | 2t+8, 2t+9),
    // in the order a0 (g, lo), a1 (g+8, lo), a2 (g, hi), a3 (g+8, hi).
    using QRaw = typename std::conditional<Q_BF16, uint32_t, float2>::type;
    auto load_q = [&](long p, int q0, QRaw (&r)[4]) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int q = q0 + g + (k & 1) * 8;
            const long off = p * sq + (long)q * ldq + h * kManyC + 2 * t + (k >> 1) * 8;
            if (q < Nq) {
                if (Q_BF16)
                    reinterpret_cast<uint32_t &>(r[k]) =
                        __ldg(reinterpret_cast<const uint32_t *>(
                            reinterpret_cast<const __nv_bfloat16 *>(Q) + off));
                else
                    reinterpret_cast<float2 &>(r[k]) =
                        __ldg(reinterpret_cast<const float2 *>(reinterpret_cast<const float *>(Q) + off));
            }
            else {
                if (Q_BF16)
                    reinterpret_cast<uint32_t &>(r[k]) = 0u;
                else
                    reinterpret_cast<float2 &>(r[k]) = make_float2(0.0f, 0.0f);
            }
        }
    };
    // Unit cursors (prompt, first query), advanced without division.
    long pc = u0 / nqb, pn;
    int qc = (int)(u0 - pc * nqb) * 16, qn;
    pn = pc;
    qn = qc;
    auto advance = [&](long &p, int &q) {
        q += 16;
        if (q >= nqb * 16) {
            q = 0;
            p++;
        }
    };
    QRaw qr[4], qx[4];
    load_q(pc, qc, qr);
    advance(pn, qn);
    long staged = -1;
    uint32_t kh[2], kl[2], vh[2], vl[2];
#pragma unroll 1
    for (long u = u0; u < u1; u++) {
        if (pc != staged) {  // this prompt's K^T and V fragments
            float kv[4];
            const float *kb = K + pc * sk, *vb = V + pc * sv;
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const float *kr = kb + (long)g * D + h * kManyC + 2 * t + k * 8;
                kv[0] = g < Nk ? __ldg(kr) * kscale : 0.0f;
                kv[1] = g < Nk ? __ldg(kr + 1) * kscale : 0.0f;
                split_bf16x2(kv[0], kv[1], kh[k], kl[k]);
                const float *vr = vb + (long)(2 * t) * D + h * kManyC + k * 8 + g;
                kv[2] = 2 * t < Nk ? __ldg(vr) : 0.0f;
                kv[3] = 2 * t + 1 < Nk ? __ldg(vr + D) : 0.0f;
                split_bf16x2(kv[2], kv[3], vh[k], vl[k]);
            }
            staged = pc;
        }
        const bool more = u + 1 < u1;
        if (more)
            load_q(pn, qn, qx);
        uint32_t ah[4], al[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if (Q_BF16)
                ah[k] = reinterpret_cast<const uint32_t &>(qr[k]);
            else {
                const float2 x = reinterpret_cast<const float2 &>(qr[k]);
                split_bf16x2(x.x, x.y, ah[k], al[k]);
            }
        }
        float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // rows (g, g, g+8, g+8) x keys (2t, 2t+1)
        mma_bf16(sc, ah, kh[0], kh[1]);
        if (!Q_BF16)
            mma_bf16(sc, al, kh[0], kh[1]);
        mma_bf16(sc, ah, kl[0], kl[1]);
        if (2 * t >= Nk)
            sc[0] = sc[2] = -INFINITY;
        if (2 * t + 1 >= Nk)
            sc[1] = sc[3] = -INFINITY;
        float m0 = fmaxf(sc[0], sc[1]), m1 = fmaxf(sc[2], sc[3]);
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
        const float p0 = ex2_approx(sc[0] - m0), p1 = ex2_approx(sc[1] - m0);
        const float p2 = ex2_approx(sc[2] - m1), p3 = ex2_approx(sc[3] - m1);
        float l0 = p0 + p1, l1 = p2 + p3;
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        uint32_t ph0, pl0, ph1, pl1;
        split_bf16x2(p0, p1, ph0, pl0);
        split_bf16x2(p2, p3, ph1, pl1);
        const float i0 = 1.0f / l0, i1 = 1.0f / l1;
        const int qa = qc + g, qb = qa + 8;
#pragma unroll
        for (int nt = 0; nt < 2; nt++) {
            float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            mma_bf16_k8(o, ph0, ph1, vh[nt]);
            mma_bf16_k8(o, pl0, pl1, vh[nt]);
            mma_bf16_k8(o, ph0, ph1, vl[nt]);
            const long col = h * kManyC + nt * 8 + 2 * t;
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int q = r ? qb : qa;
                if (q >= Nq)
                    continue;
                const float inv = r ? i1 : i0;
                const long off = (pc * Nq + q) * D + col;
                if (OUT_BF16)
                    *reinterpret_cast<uint32_t *>(reinterpret_cast<__nv_bfloat16 *>(O) + off) =
                        bf16_pair(o[2 * r] * inv, o[2 * r + 1] * inv);
                else
                    *reinterpret_cast<float2 *>(reinterpret_cast<float *>(O) + off) =
                        make_float2(o[2 * r] * inv, o[2 * r + 1] * inv);
            }
        }
        if (more) {
#pragma unroll
            for (int k = 0; k < 4; k++)
                qr[k] = qx[k];
            pc = pn;
            qc = qn;
            advance(pn, qn);
        }
    }
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

// Token -> image attention on the tensor cores: warp w < 8 of the CTA is
// head w, for 8 queries of a prompt, over each staged chunk of 32 keys as
// two blocks of 16; warp 8 stages the chunks (TMA boxes of 32 keys x one
// head's 16 channels, K and V of every head, into a 3-stage ring guarded
// by full / empty mbarriers with bounded waits). KV_BF16: K and V given in
// bf16 (as the decoder's projections write them). Per block, S^T (16 keys x 8 queries) = K . Q^T and O^T (16
// channels x 8 queries) += V^T . P^T by mma.sync m16n8k16 in bf16 with
// fp32 accumulation, every fp32 operand split into a bf16 pair hi + lo
// and each product taken as hi.hi + lo.hi + hi.lo (K/V given in bf16 are
// exact: one term fewer). Q carries scale * log2 e, so S is in log2 units.
// Softmax per query over the chunk: maximum across the warp's 8 key
// groups by shuffles, the running maximum raised (O, l rescaled) only when
// the chunk's exceeds it by kManyLazy; P transposed into B fragments by
// movmatrix. At the end of each prompt in the CTA's range one (m, l, o)
// partial per (query, head). QG > 1 (keys and values shared by all
// prompts, whose queries the host flattens into one prompt): a warp takes
// QG groups of 8 queries, each chunk's K and V fragments loaded and split
// once for all of them.
constexpr int kManyThreads = 32 * (kHeads + 1);  // 8 head warps + the producer warp

template <bool KV_BF16, int QG = 1>
__global__ void __launch_bounds__(kManyThreads, 2) mha_many_split_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
    const float *__restrict__ Q, long sq, int k_per_prompt, int v_per_prompt,
    float *__restrict__ part, int P, int Nq, int Nk, int segs, float qscale, int *err)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    extern __shared__ __align__(16) float sm_raw[];
    constexpr int ESZ = KV_BF16 ? 2 : 4;
    constexpr int STAGE_B = kManyStage * ESZ;             // bytes per stage
    constexpr int TILE_B = kChunk * kManyC * ESZ;          // bytes per (K or V, head)
    char *smb = reinterpret_cast<char *>(
        (reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smb + kStages * STAGE_B);
    uint64_t *empty = full + kStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kStages);
    const int nch = (Nk + kChunk - 1) / kChunk;
    const long T = (long)P * nch, G = gridDim.x;
    const long c0 = many_chunk0(blockIdx.x, T, G), c1 = many_chunk0(blockIdx.x + 1, T, G);
    const int nloc = (int)(c1 - c0);
    const long p_first = c0 / nch;
    const int lane = threadIdx.x & 31, h = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int qz = blockIdx.z * 8 * QG;
    // Chunk cursors (prompt, chunk of the prompt), advanced without division.
    struct Cur {
        long p;
        int ci;
    };
    auto advance = [&](Cur &c) {
        if (++c.ci == nch) {
            c.ci = 0;
            c.p++;
        }
    };
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kHeads);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (h == kHeads) {  // producer warp: one thread issues the ring's TMA box loads
        if (lane == 0 && nloc > 0) {
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            Cur c = {p_first, (int)(c0 - p_first * nch)};
            int issued = 0;
            for (int i = 0; i < nloc; i++, advance(c)) {
                const int b = i % kStages;
                if (i >= kStages && !mbar_wait(&empty[b], ((i / kStages) - 1) & 1, err, abort_flag))
                    break;
                mbar_arrive_expect_tx(&full[b], 2 * kHeads * TILE_B);
                char *dst = smb + b * STAGE_B;
                const int j0 = c.ci * kChunk;
                const int zk = k_per_prompt ? (int)c.p : 0, zv = v_per_prompt ? (int)c.p : 0;
#pragma unroll
                for (int hh = 0; hh < kHeads; hh++) {
                    tma_load_3d(dst + hh * TILE_B, &tmK, &full[b], hh * kManyC, j0, zk);
                    tma_load_3d(dst + (kHeads + hh) * TILE_B, &tmV, &full[b], hh * kManyC, j0, zv);
                }
                issued = i + 1;
            }
            // copies in flight land before the CTA exits (bounded wait)
            volatile int no_abort = 0;
            for (int i = issued - kStages; i < issued; i++)
                if (i >= 0)
                    mbar_wait(&full[i % kStages], (i / kStages) & 1, err, &no_abort);
        }
        return;
    }

    uint32_t qh[QG][2], ql[QG][2];  // B fragments of Q^T (hi, lo) per query group
    float o[QG][2][4], m[QG][2], l[QG][2];  // O^T per key block (two MMA chains)
    auto start_segment = [&](long p) {
#pragma unroll
        for (int jq = 0; jq < QG; jq++) {
            const int qi = qz + 8 * jq + g;
            float2 x0 = make_float2(0.0f, 0.0f), x1 = x0;
            if (qi < Nq) {
                const float *qp = Q + p * sq + (long)qi * kManyD + h * kManyC + 2 * t;
                x0 = *reinterpret_cast<const float2 *>(qp);
                x1 = *reinterpret_cast<const float2 *>(qp + 8);
            }
            split_bf16x2(x0.x * qscale, x0.y * qscale, qh[jq][0], ql[jq][0]);
            split_bf16x2(x1.x * qscale, x1.y * qscale, qh[jq][1], ql[jq][1]);
#pragma unroll
            for (int k = 0; k < 4; k++)
                o[jq][0][k] = o[jq][1][k] = 0.0f;
            m[jq][0] = m[jq][1] = -INFINITY;
            l[jq][0] = l[jq][1] = 0.0f;
        }
    };
    // Segment k's partials: l summed over the 8 key groups; the lane of
    // key group g writes channels g and g + 8 of queries 2t, 2t + 1.
    auto flush = [&](long k) {
#pragma unroll
        for (int jq = 0; jq < QG; jq++) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                float L = l[jq][u];
                L += __shfl_xor_sync(0xffffffffu, L, 4);
                L += __shfl_xor_sync(0xffffffffu, L, 8);
                L += __shfl_xor_sync(0xffffffffu, L, 16);
                const int qi = qz + 8 * jq + 2 * t + u;
                if (qi < Nq) {
                    float *dst =
                        part + (((blockIdx.x * (long)segs + k) * Nq + qi) * kHeads + h) * kPart;
                    if (g == 0) {
                        dst[0] = m[jq][u];
                        dst[1] = L;
                    }
                    dst[4 + g] = o[jq][0][u] + o[jq][1][u];
                    dst[4 + g + 8] = o[jq][0][2 + u] + o[jq][1][2 + u];
                }
            }
        }
    };

    // Head warps: each waits for a stage, computes its head, releases the
    // stage (one arrival per warp); no CTA-wide barrier in the loop.
    Cur cur = {p_first, (int)(c0 - p_first * nch)};
    for (int i = 0; i < nloc; i++, advance(cur)) {
        const int b = i % kStages;
        const long p = cur.p;
        const int ci = cur.ci;
        if (i == 0 || ci == 0)
            start_segment(p);
        if (!__all_sync(0xffffffffu, mbar_wait(&full[b], (i / kStages) & 1, err, abort_flag)))
            break;
        const int n = min(kChunk, Nk - ci * kChunk);
        const char *tk = smb + b * STAGE_B + h * TILE_B;
        const char *tv = tk + kHeads * TILE_B;
        // K and V^T fragments of the two key blocks (bf16: ka / va; fp32:
        // hi in ka / va, lo in kb / vb), loaded by the first query group
        // and kept for the others.
        uint32_t ka[2][4], kb[2][4], va[2][4], vb[2][4];
#pragma unroll
        for (int jq = 0; jq < QG; jq++) {
            // S^T of the two key blocks: s[blk][0..3] = keys (g, g, g+8, g+8)
            // of the block x queries (2t, 2t+1, 2t, 2t+1) of group jq.
            float s[2][4];
#pragma unroll
            for (int blk = 0; blk < 2; blk++) {
                float (&d)[4] = s[blk];
                d[0] = d[1] = d[2] = d[3] = 0.0f;
                const int j = blk * 16 + g;
                if (KV_BF16) {
                    if (jq == 0) {
                        // rows of matrices 0..3: keys 0-7 / 8-15 x channels 0-7 / 8-15
                        const int mi = lane >> 3, rr = blk * 16 + (lane & 7) + (mi & 1) * 8;
                        ldmatrix_x4(ka[blk], tk + (rr * kManyC + many_sw16(rr, mi >> 1)) * 2,
                                    false);
                    }
                    mma_bf16(d, ka[blk], qh[jq][0], qh[jq][1]);
                    mma_bf16(d, ka[blk], ql[jq][0], ql[jq][1]);
                }
                else {
                    if (jq == 0) {
                        const float *kr = reinterpret_cast<const float *>(tk);
                        const float2 x0 = *reinterpret_cast<const float2 *>(
                            kr + j * kManyC + many_sw32(j, t >> 1) + 2 * (t & 1));
                        const float2 x1 = *reinterpret_cast<const float2 *>(
                            kr + (j + 8) * kManyC + many_sw32(j + 8, t >> 1) + 2 * (t & 1));
                        const float2 x2 = *reinterpret_cast<const float2 *>(
                            kr + j * kManyC + many_sw32(j, 2 + (t >> 1)) + 2 * (t & 1));
                        const float2 x3 = *reinterpret_cast<const float2 *>(
                            kr + (j + 8) * kManyC + many_sw32(j + 8, 2 + (t >> 1)) + 2 * (t & 1));
                        split_bf16x2(x0.x, x0.y, ka[blk][0], kb[blk][0]);
                        split_bf16x2(x1.x, x1.y, ka[blk][1], kb[blk][1]);
                        split_bf16x2(x2.x, x2.y, ka[blk][2], kb[blk][2]);
                        split_bf16x2(x3.x, x3.y, ka[blk][3], kb[blk][3]);
                    }
                    mma_bf16(d, ka[blk], qh[jq][0], qh[jq][1]);
                    mma_bf16(d, kb[blk], qh[jq][0], qh[jq][1]);
                    mma_bf16(d, ka[blk], ql[jq][0], ql[jq][1]);
                }
                if (j >= n)
                    d[0] = d[1] = -INFINITY;
                if (j + 8 >= n)
                    d[2] = d[3] = -INFINITY;
            }
            float bm[2];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                float x = fmaxf(fmaxf(s[0][u], s[0][2 + u]), fmaxf(s[1][u], s[1][2 + u]));
                x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 4));
                x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 8));
                x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 16));
                bm[u] = x;
                if (bm[u] > m[jq][u] + kManyLazy) {  // uniform over the lanes of query 2t + u
                    const float corr = exp2f(m[jq][u] - bm[u]);  // 0 on the first chunk
                    l[jq][u] *= corr;
                    o[jq][0][u] *= corr;
                    o[jq][0][2 + u] *= corr;
                    o[jq][1][u] *= corr;
                    o[jq][1][2 + u] *= corr;
                    m[jq][u] = bm[u];
                }
            }
#pragma unroll
            for (int blk = 0; blk < 2; blk++) {
                float pe[4];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    pe[k] = ex2_approx(s[blk][k] - m[jq][k & 1]);  // 0 for masked keys
                    l[jq][k & 1] += pe[k];
                }
                // P^T tiles (keys 0-7 / 8-15 x 8 queries) -> B fragments
                uint32_t ph0, pl0, ph1, pl1;
                split_bf16x2(pe[0], pe[1], ph0, pl0);
                split_bf16x2(pe[2], pe[3], ph1, pl1);
                ph0 = movmatrix_t(ph0);
                ph1 = movmatrix_t(ph1);
                pl0 = movmatrix_t(pl0);
                pl1 = movmatrix_t(pl1);
                if (KV_BF16) {
                    if (jq == 0) {
                        // V^T fragments: matrices (keys 0-7 / 8-15) x (channels 0-7 / 8-15),
                        // transposed
                        const int mi = lane >> 3;
                        const int rr = blk * 16 + (lane & 7) + (mi >> 1) * 8;
                        ldmatrix_x4(va[blk], tv + (rr * kManyC + many_sw16(rr, mi & 1)) * 2, true);
                    }
                    mma_bf16(o[jq][blk], va[blk], ph0, ph1);
                    mma_bf16(o[jq][blk], va[blk], pl0, pl1);
                }
                else {
                    if (jq == 0) {
                        const float *vr = reinterpret_cast<const float *>(tv);
                        const int k0 = blk * 16 + 2 * t;
                        auto ld = [&](int key, int ch) {
                            return vr[key * kManyC + many_sw32(key, ch >> 2) + (ch & 3)];
                        };
                        split_bf16x2(ld(k0, g), ld(k0 + 1, g), va[blk][0], vb[blk][0]);
                        split_bf16x2(ld(k0, g + 8), ld(k0 + 1, g + 8), va[blk][1], vb[blk][1]);
                        split_bf16x2(ld(k0 + 8, g), ld(k0 + 9, g), va[blk][2], vb[blk][2]);
                        split_bf16x2(ld(k0 + 8, g + 8), ld(k0 + 9, g + 8), va[blk][3],
                                     vb[blk][3]);
                    }
                    mma_bf16(o[jq][blk], va[blk], ph0, ph1);
                    mma_bf16(o[jq][blk], vb[blk], ph0, ph1);
                    mma_bf16(o[jq][blk], va[blk], pl0, pl1);
                }
            }
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[b]);  // this warp is done with stage b
        if (ci == nch - 1 || i == nloc - 1)
            flush(p - p_first);
    }
}

// Combines the partials of each (prompt, query, head): those of the CTAs
// whose chunk ranges meet the prompt's chunks [p nch, (p + 1) nch), at
// segment p - (first prompt of the CTA); offsets in log2 units. One warp
// per (prompt, query, head): the lanes take the records' offsets and sums
// (lane = record) for the maximum and the weights, then half-warps take
// alternate records, a lane one output channel, and the halves are added.
// OUT_BF16: O written as bf16 (the operand of the output projection).
template <bool OUT_BF16>
__global__ void __launch_bounds__(256) mha_many_combine_kernel(const float *__restrict__ part,
                                                               void *__restrict__ O, int P,
                                                               int Nq, int nch, int G, int segs)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    const long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;  // (p, qi, h)
    const int lane = threadIdx.x & 31;
    if (w >= (long)P * Nq * kHeads)
        return;  // warp-uniform
    const int h = (int)(w % kHeads);
    const int qi = (int)((w / kHeads) % Nq);
    const long p = w / ((long)kHeads * Nq);
    const long T = (long)P * nch;
    // CTA holding chunk c: the largest x with x T / G <= c, i.e.
    // ceil((c + 1) G / T) - 1.
    const long x0 = ((p * nch + 1) * G + T - 1) / T - 1;
    const long x1 = (((p + 1) * nch) * G + T - 1) / T - 1;
    const int nr = (int)(x1 - x0 + 1);
    // Only CTA x0 can start before the prompt (segment k0 > 0 of its
    // range); every later one starts inside it (segment 0).
    const long k0 = p - many_chunk0(x0, T, G) / nch;
    const float *base = part + ((x0 * segs * Nq + qi) * kHeads + h) * kPart;
    const long xstride = (long)segs * Nq * kHeads * kPart, kstride = (long)Nq * kHeads * kPart;
    auto rec = [&](int r) { return base + r * xstride + (r == 0 ? k0 * kstride : 0); };
    float M = -INFINITY;
    for (int r = lane; r < nr; r += 32)
        M = fmaxf(M, __ldg(rec(r)));
#pragma unroll
    for (int o = 16; o; o >>= 1)
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.0f, acc = 0.0f;
    const int half = lane >> 4, c = lane & 15;
    for (int r0 = 0; r0 < nr; r0 += 32) {
        float f = 0.0f;
        if (r0 + lane < nr) {
            const float2 ml = __ldg(reinterpret_cast<const float2 *>(rec(r0 + lane)));
            f = ml.x == -INFINITY ? 0.0f : exp2f(ml.x - M);
            L = fmaf(ml.y, f, L);
        }
        const int n = min(32, nr - r0);
#pragma unroll 4
        for (int jj = 0; jj < n; jj += 2) {  // same trip count in both halves
            const int j = jj + half;
            const float fj = __shfl_sync(0xffffffffu, f, j & 31);
            if (j < n)
                acc = fmaf(__ldg(rec(r0 + j) + 4 + c), fj, acc);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
        L += __shfl_xor_sync(0xffffffffu, L, o);
    acc += __shfl_xor_sync(0xffffffffu, acc, 16);
    if (half == 0) {
        const long i = (p * Nq + qi) * kManyD + h * kManyC + c;
        if constexpr (OUT_BF16)
            static_cast<__nv_bfloat16 *>(O)[i] = __float2bfloat16_rn(acc / L);
        else
            static_cast<float *>(O)[i] = acc / L;
    }
}

// Plan of the many-keys kernel: G CTAs per query group of 8 (two per SM
// over all groups, at most one per chunk) and the most prompt segments a
// CTA's chunk range can cross.
struct ManyPlan {
    int G, segs;
};

ManyPlan many_plan(int P, int Nq, int Nk, int num_sms, int qg = 1)
{
    const long nch = (Nk + kChunk - 1) / kChunk, T = (long)P * nch;
    const long nz = (Nq + 8 * qg - 1) / (8 * qg);
    long G = 2L * num_sms / nz;
    if (G < 1)
        G = 1;
    if (G > T)
        G = T;
    const long per = (T + G - 1) / G;  // chunks of the longest range
    return {(int)G, (int)((per - 1) / nch + 2)};
}

size_t many_workspace(int P, int Nq, int Nk, int num_sms, int qg = 1)
{
    const ManyPlan pl = many_plan(P, Nq, Nk, num_sms, qg);
    return (size_t)pl.G * pl.segs * Nq * kHeads * kPart * sizeof(float);
}

// Keys and values shared by all prompts, fp32, and the prompts' queries
// contiguous: the launch flattens them into one prompt of P * Nq queries in
// groups of 16 (two per warp), so each chunk's K / V fragments serve two
// groups. The flattened plan's workspace (k_mha_workspace reports the
// larger of the two).
constexpr int kManyFlatQG = 2;
bool many_flat(int P, int Nq, long sq, long sk, long sv, bool kv_bf16)
{
    return !kv_bf16 && sk == 0 && sv == 0 && (P == 1 || sq == (long)Nq * kManyD) &&
           (long)P * Nq >= 8 * kManyFlatQG && (long)P * Nq <= 0x7fffffffL;
}

template <bool Q_BF16, bool OUT_BF16>
int launch_few2(int P, int Nq, int Nk, const void *qp, long sq, long ldq, const float *kp,
                long sk, const float *vp, long sv, void *o, float scale, int num_sms,
                cudaStream_t st)
{
    int per_sm = 1;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per_sm, mha_few2_kernel<Q_BF16, OUT_BF16>, 256, 0);
    if (e != cudaSuccess)
        return (int)e;
    const long units = (long)P * ((Nq + 15) / 16);
    const long cap = (long)num_sms * (per_sm > 0 ? per_sm : 1);
    return launch_pdl(mha_few2_kernel<Q_BF16, OUT_BF16>, dim3((unsigned)(units < cap ? units : cap)),
                      dim3(256), 0, st, qp, sq, ldq, kp, sk, vp, sv, o, P, Nq, Nk,
                      scale * 1.4426950408889634f);
}

template <int C>
int launch_few(int P, int Nq, int Nk, const float *qp, long sq, const float *kp, long sk,
               const float *vp, long sv, float *o, float scale, int num_sms, cudaStream_t st)
{
    if (C == 16 && Nk <= kFewSmall)
        return launch_few2<false, false>(P, Nq, Nk, qp, sq, (long)kManyD, kp, sk, vp, sv, o, scale,
                                         num_sms, st);
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
    return launch_pdl(kern, dim3((unsigned)(units < cap ? units : cap)), dim3(256), smem, st, qp, sq,
                      kp, sk, vp, sv, o, P, Nq, Nk, scale);
}

template <bool KV_BF16>
int launch_many(int P, int Nq, int Nk, const float *qp, long sq, const void *kp, long sk,
                long kld, const void *vp, long sv, long vld, void *o, bool out_bf16, void *ws,
                size_t ws_bytes, float scale, int *err, int num_sms, cudaStream_t st)
{
    const bool flat = many_flat(P, Nq, sq, sk, sv, KV_BF16);
    if (flat) {
        Nq *= P;
        P = 1;
        sq = 0;
    }
    const int qg = flat ? kManyFlatQG : 1;
    const ManyPlan pl = many_plan(P, Nq, Nk, num_sms, qg);
    if (!ws || ws_bytes < many_workspace(P, Nq, Nk, num_sms, qg) ||
        (reinterpret_cast<uintptr_t>(ws) & 15) || !err)
        return K_EARG;
    // K and V as [P][Nk][128] boxes of 32 keys x one head's 16 channels
    // (prompt pitch sk / sv elements; 0: one block shared by all prompts)
    const CUtensorMapDataType dt =
        KV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const CUtensorMapSwizzle swz = KV_BF16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
    const uint32_t es = KV_BF16 ? 2 : 4;
    CUtensorMap tk, tv;
    if (!make_tmap_3d(&tk, dt, es, kp, (uint64_t)P, (uint64_t)Nk, kManyD, (uint64_t)kld,
                      (uint64_t)sk, kManyC, kChunk, swz) ||
        !make_tmap_3d(&tv, dt, es, vp, (uint64_t)P, (uint64_t)Nk, kManyD, (uint64_t)vld,
                      (uint64_t)sv, kManyC, kChunk, swz))
        return K_ETMAP;
    const int smem = (KV_BF16 ? kManySmem / 2 : kManySmem) + 1024 + 64;  // ring, alignment, barriers
    cudaError_t e = flat ? smem_limit_once<mha_many_split_kernel<KV_BF16, kManyFlatQG>>(smem)
                         : smem_limit_once<mha_many_split_kernel<KV_BF16>>(smem);
    if (e != cudaSuccess)
        return (int)e;
    dim3 grid(pl.G, 1, (Nq + 8 * qg - 1) / (8 * qg));
    int rc = flat ? launch_pdl(mha_many_split_kernel<KV_BF16, kManyFlatQG>, grid,
                               dim3(kManyThreads), smem, st, tk, tv, qp, sq, 0, 0,
                               static_cast<float *>(ws), P, Nq, Nk, pl.segs,
                               scale * 1.4426950408889634f, err)
                  : launch_pdl(mha_many_split_kernel<KV_BF16>, grid, dim3(kManyThreads), smem, st,
                               tk, tv, qp, sq, sk != 0, sv != 0, static_cast<float *>(ws), P, Nq,
                               Nk, pl.segs, scale * 1.4426950408889634f, err);
    if (rc != 0)
        return rc;
    const long total = (long)P * Nq * kHeads * 32;  // a warp per (prompt, query, head)
    const dim3 cgrid((unsigned)((total + 255) / 256));
    const float *part = static_cast<const float *>(ws);
    const int nch = (Nk + kChunk - 1) / kChunk;
    return out_bf16 ? launch_pdl(mha_many_combine_kernel<true>, cgrid, dim3(256), 0, st, part, o,
                                 P, Nq, nch, pl.G, pl.segs)
                    : launch_pdl(mha_many_combine_kernel<false>, cgrid, dim3(256), 0, st, part, o,
                                 P, Nq, nch, pl.G, pl.segs);
}

}  // namespace
}  // namespace sam3

extern "C" size_t k_mha_workspace(int P, int Nq, int Nk, int dint, int num_sms)
{
    if (Nk <= 64 || dint != sam3::kManyD || P <= 0 || Nq <= 0)
        return 0;
    const size_t a = sam3::many_workspace(P, Nq, Nk, num_sms);
    const size_t b = (long)P * Nq <= 0x7fffffffL
                         ? sam3::many_workspace(1, P * Nq, Nk, num_sms, sam3::kManyFlatQG)
                         : 0;
    return a > b ? a : b;
}

extern "C" int k_mha(int P, int Nq, int Nk, int dint, const float *qp, long sq, const float *kp,
                     long sk, const float *vp, long sv, float *o, void *ws, size_t ws_bytes,
                     int *err, int num_sms, k_stream s)
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
        return launch_many<false>(P, Nq, Nk, qp, sq, kp, sk, (long)kManyD, vp, sv, (long)kManyD, o,
                                  false, ws, ws_bytes, scale, err, num_sms, st);
    }
    if (c == 16)
        return launch_few<16>(P, Nq, Nk, qp, sq, kp, sk, vp, sv, o, scale, num_sms, st);
    if (c == 32)
        return launch_few<32>(P, Nq, Nk, qp, sq, kp, sk, vp, sv, o, scale, num_sms, st);
    return K_EARG;
}

extern "C" int k_mha_i2t_bf16(int P, int Nq, int Nk, const void *qp, long sq, long ldq,
                              const float *kp, long sk, const float *vp, long sv, void *o,
                              int num_sms, k_stream s)
{
    using namespace sam3;
    if (P <= 0 || Nq <= 0 || Nk <= 0 || Nk > kFewSmall || ((uintptr_t)qp & 15) ||
        ((uintptr_t)kp & 15) || ((uintptr_t)vp & 15) || ((uintptr_t)o & 15) || (sq & 3) ||
        ldq < kManyD || (ldq & 3) || (sk & 3) || (sv & 3))
        return K_EARG;
    return launch_few2<true, true>(P, Nq, Nk, qp, sq, ldq, kp, sk, vp, sv, o, 1.0f / sqrtf(16.0f),
                                   num_sms, reinterpret_cast<cudaStream_t>(s));
}

extern "C" int k_mha_t2i_bf16kv(int P, int Nq, int Nk, const float *qp, long sq, const void *kp,
                                long sk, long kld, const void *vp, long sv, long vld, void *o,
                                int out_bf16, void *ws, size_t ws_bytes, int *err, int num_sms,
                                k_stream s)
{
    using namespace sam3;
    if (P <= 0 || Nq <= 0 || Nk <= 64 || P > 65535 || ((uintptr_t)qp & 15) ||
        ((uintptr_t)kp & 15) || ((uintptr_t)vp & 15) || ((uintptr_t)o & 15) || (sq & 3) ||
        (sk & 7) || (sv & 7) || kld < kManyD || vld < kManyD || (kld & 7) || (vld & 7))
        return K_EARG;
    return launch_many<true>(P, Nq, Nk, qp, sq, kp, sk, kld, vp, sv, vld, o, out_bf16 != 0, ws,
                             ws_bytes, 1.0f / sqrtf((float)kManyC), err, num_sms, STREAM(s));
}
