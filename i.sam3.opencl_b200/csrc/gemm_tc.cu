// SPDX-License-Identifier: Unlicense
// Persistent tcgen05 GEMM for the backbone's linear layers (QKV, proj, fc1,
// fc2, patch embedding): C = epi(alpha * A . B^T) with bf16 operands, fp32
// accumulation in tensor memory and the reference GEMM's fused epilogue
// (bias, GELU/ReLU, residual; sam3_kernels.cl:57-69, 147-153), plus an
// optional RoPE rotation of the q/k columns (rope_apply,
// sam3_kernels.cl:679-698) so the QKV output feeds attention directly.
// The same kernel also runs the implicit-GEMM 3x3 convolution and the 2x2
// ConvTranspose (scatter in the epilogue) of the neck, and the mask
// decoder's two output-upscaling stages (LayerNorm2d + GELU, and GELU +
// mask logits, in the epilogue).
//
// One CTA per SM (or a CTA pair on the two SMs of a TPC), 10 warps:
//   warp 0    TMA producer: A/B k-blocks of 64 into a shared-memory ring;
//   warp 1    tensor-memory owner and MMA issuer (one elected thread; in a
//             pair, rank 0's): 128 x BN x 16 (pair: 256 x BN x 16,
//             cta_group::2) tcgen05.mma into one of two TMEM accumulators;
//   warps 2-9 epilogue, two warps per TMEM lane quarter (warp w reads lanes
//             32*(w%4)...), splitting the tile's 128-byte column chunks:
//             tcgen05.ld, epilogue math, the chunk written 128B-swizzled
//             into a per-warp staging tile and stored by TMA (coalesced,
//             asynchronous, rows/columns beyond C clipped by the tensor
//             map; an in-place fp32 residual is a TMA reduce-add). The
//             accumulator is released as soon as it is read, so the MMAs of
//             the next tile overlap the epilogue of this one.
// Tiles are visited m-major (all n-tiles of a row block back to back) so a
// row block of A is read from HBM once and re-read from L2.
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>

namespace sam3 {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 8;  // epilogue warps: two per TMEM lane quarter
constexpr int kStageTile = 32 * 128;  // one warp's 32 rows x 128 bytes

struct GemmEpi {
    int M, N, K;
    void *C;
    long ldc;
    const float *bias;
    const float *R;
    long ldr;
    int rmod;  // R row = m % rmod (0: R row = m)
    float alpha;
    int act;
    k_rope rope;
    int *err;
    int red;  // fp32 C updated in place: C += epilogue result by TMA reduce-add
};

// CONV3 geometry: 3x3 / pad-1 convolution of cimg maps cH x cW x (K / 9)
// channels (implicit GEMM); M tiles are 8 x 16 pixel blocks, cyb x cxb per map.
// Epilogue kinds beyond the generic one (bias, activation, residual, RoPE):
// the mask decoder's two output-upscaling stages and the scatter of a 2x2 /
// stride-2 ConvTranspose.
constexpr int kEpiGeneric = 0, kEpiLogits = 1, kEpiLn2d = 2, kEpiConvT = 3;

// Epilogue warps per CTA: four per TMEM lane quarter (one 32-column chunk
// each) for the mask logits, whose GELU chains are latency-bound with two;
// threads = a producer warp, an MMA warp and the epilogue warps.
__host__ __device__ constexpr int epi_warps(int epi) { return epi == kEpiLogits ? 16 : kEpiWarps; }
__host__ __device__ constexpr int gemm_threads(int epi) { return 64 + 32 * epi_warps(epi); }

// kEpiLogits / kEpiLn2d / kEpiConvT: cH x cW input maps; hyper = the
// prompts' hypernetwork vectors [P][3][32]; lnw / lnb = LayerNorm2d weight
// and bias; cout = ConvTranspose output channels.
struct ConvGeom {
    int cH, cW, cimg, cyb, cxb;
    const float *hyper, *lnw, *lnb;
    int cout;
};

// EPI_BUFS: staging tiles per epilogue warp. Single CTAs: one; the shared
// memory goes to a fourth A/B stage instead, which the main loop gains more
// from than the epilogue loses by waiting for its previous TMA store to be
// read. PAIR: each CTA of a pair holds half of the B tile (BN / 2 rows), so
// a stage is 32 KB. EW: epilogue warps with a staging tile (0 for the
// epilogues that store directly).
template <int BN, bool PAIR = false, int EW = kEpiWarps>
struct GemmSmem {
    static constexpr int STAGES = PAIR ? 6 : 4;
    static constexpr int EPI_BUFS = PAIR ? 1 : 1;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
    static constexpr int BAR_OFF = EPI_OFF + EW * EPI_BUFS * kStageTile;
    // full[S], empty[S], tfull[2], tempty[2], drain, then tmem base + abort
    static constexpr int BYTES = BAR_OFF + (2 * STAGES + 5) * 8 + 16 + 1024;
    static_assert(BYTES <= 232448, "GEMM shared memory");
};

// GELU(x) = 0.5 x (1 + erf(x / sqrt 2)) (sam3_kernels.cl:43-46) on a pair of
// values, with erf from Abramowitz & Stegun 7.1.26 (Hastings):
//   erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e^(-z^2),
//   t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7,
// so with h = erfc(|x| / sqrt 2) / 2 = t (...) 2^(-x^2 log2(e) / 2 - 1),
// GELU(x) = x (1 - h) for x >= 0 and x h for x < 0, i.e. max(x, 0) - |x| h
// for every x. Two MUFU operations per value (reciprocal, 2^x); the
// polynomial and products run in packed fp32. The result differs from the
// erf form by at most 4.2e-7 |x|-relative, far below the bf16 rounding of
// the output it feeds.
__device__ __forceinline__ void gelu_pair(float &x0, float &x1)
{
    const float kP = 0.3275911f * 0.70710678118654752f;
    const float kE = -0.72134752044448170f;  // -log2(e) / 2
    const float t0 = rcp_approx(fmaf(kP, fabsf(x0), 1.0f));
    const float t1 = rcp_approx(fmaf(kP, fabsf(x1), 1.0f));
    const uint64_t x = f2_make(x0, x1);
    const uint64_t t = f2_make(t0, t1);
    uint64_t q = fma2(f2_make(1.061405429f, 1.061405429f), t, f2_make(-1.453152027f, -1.453152027f));
    q = fma2(q, t, f2_make(1.421413741f, 1.421413741f));
    q = fma2(q, t, f2_make(-0.284496736f, -0.284496736f));
    q = fma2(q, t, f2_make(0.254829592f, 0.254829592f));
    float g0, g1;
    f2_split(fma2(mul2(x, f2_make(kE, kE)), x, f2_make(-1.0f, -1.0f)), g0, g1);
    q = mul2(mul2(q, t), f2_make(ex2_approx(g0), ex2_approx(g1)));
    float h0, h1;
    f2_split(q, h0, h1);
    x0 = fmaf(-fabsf(x0), h0, fmaxf(x0, 0.0f));
    x1 = fmaf(-fabsf(x1), h1, fmaxf(x1, 0.0f));
}

// Table row of the RoPE rotation for output row m.
__device__ __forceinline__ int rope_row(const k_rope &r, int m)
{
    if (r.mode == 1)
        return m % r.npos;
    const int T = r.grid * r.grid, w2 = r.ws * r.ws;
    const int t = m % T, w = t / w2, i = t % w2;
    const int y = (w / r.nwx) * r.ws + i / r.ws, x = (w % r.nwx) * r.ws + i % r.ws;
    return y * r.grid + x;
}

// Epilogue math on CW consecutive columns of row m starting at column n:
// alpha, bias, activation, residual, RoPE (the reference's order). rv / rot,
// when given, hold the chunk's residual values / (cos, sin) pairs already
// loaded into registers; otherwise they are read here. ACT false: the
// activation is known to be none (not compiled in).
template <int CW, bool ACT = true>
__device__ __forceinline__ void epilogue_math(const GemmEpi &p, int m, int n, float (&v)[CW],
                                              int rrow, const float4 *rv, const float2 *rot)
{
#pragma unroll
    for (int j = 0; j < CW; j++)
        v[j] *= p.alpha;
    const bool full = n + CW <= p.N;
    if (p.bias) {
        if (full) {
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
                const float4 b = __ldg(reinterpret_cast<const float4 *>(p.bias + n + j));
                v[j] += b.x;
                v[j + 1] += b.y;
                v[j + 2] += b.z;
                v[j + 3] += b.w;
            }
        }
        else {
#pragma unroll
            for (int j = 0; j < CW; j++)
                if (n + j < p.N)
                    v[j] += __ldg(p.bias + n + j);
        }
    }
    if (ACT && p.act == K_ACT_GELU) {
#pragma unroll
        for (int j = 0; j < CW; j += 2)
            gelu_pair(v[j], v[j + 1]);
    }
    else if (ACT && p.act == K_ACT_RELU) {
#pragma unroll
        for (int j = 0; j < CW; j++)
            v[j] = fmaxf(v[j], 0.0f);
    }
    if (p.R && m < p.M) {
        const float *rp = p.R + (long)(p.rmod ? m % p.rmod : m) * p.ldr + n;
        if (rv) {
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
                v[j] += rv[j / 4].x;
                v[j + 1] += rv[j / 4].y;
                v[j + 2] += rv[j / 4].z;
                v[j + 3] += rv[j / 4].w;
            }
        }
        else if (full && ((reinterpret_cast<uintptr_t>(rp) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
                const float4 q = *reinterpret_cast<const float4 *>(rp + j);
                v[j] += q.x;
                v[j + 1] += q.y;
                v[j + 2] += q.z;
                v[j + 3] += q.w;
            }
        }
        else {
#pragma unroll
            for (int j = 0; j < CW; j++)
                if (n + j < p.N)
                    v[j] += rp[j];
        }
    }
    if (p.rope.mode && n < 2 * p.rope.E) {
        // Chunks of 32 or 64 columns never straddle the q/k/v boundaries
        // (E % 64 == 0); each (2j, 2j+1) pair sits in one chunk.
        const float2 *cs = reinterpret_cast<const float2 *>(p.rope.cs) +
                           (long)rrow * (p.rope.hd / 2) + ((n % p.rope.hd) >> 1);
#pragma unroll
        for (int j = 0; j < CW; j += 2) {
            const float2 r = rot ? rot[j >> 1] : __ldg(cs + (j >> 1));
            const float a = v[j], b = v[j + 1];
            v[j] = a * r.x - b * r.y;
            v[j + 1] = a * r.y + b * r.x;
        }
    }
}

// Direct (non-TMA) store of one chunk of row m (its 128 bytes packed in
// pk: bf16 pairs or fp32 words); used when C's base or leading dimension is
// not 16-byte aligned.
template <int CW, bool OUT_BF16>
__device__ __forceinline__ void store_direct(const GemmEpi &p, int m, int n,
                                             const uint32_t (&pk)[32])
{
    if (m >= p.M)
        return;
    if (OUT_BF16) {
        uint16_t *cp = reinterpret_cast<uint16_t *>(p.C) + (long)m * p.ldc + n;
        for (int j = 0; j < CW; j++)
            if (n + j < p.N)
                cp[j] = (uint16_t)(pk[j >> 1] >> ((j & 1) * 16));
    }
    else {
        float *cp = reinterpret_cast<float *>(p.C) + (long)m * p.ldc + n;
        for (int j = 0; j < CW; j++)
            if (n + j < p.N)
                cp[j] = __uint_as_float(pk[j]);
    }
}

// Writes one row's 128 bytes into a 128B-swizzled staging tile: 16-byte
// chunk q of row r goes to chunk position q ^ (r & 7), the layout a
// SWIZZLE_128B tensor map expects; eight consecutive rows cover all 32 banks.
__device__ __forceinline__ void stage_row(uint32_t tile, int r, const uint32_t (&pk)[32])
{
    const uint32_t row = tile + r * 128;
#pragma unroll
    for (int q = 0; q < 8; q++)
        st_shared_v4(row + ((q ^ (r & 7)) << 4), pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                     pk[4 * q + 3]);
}

// LOGITS epilogue: the last output-upscaling stage of the mask decoder fused
// with the mask logits (sam3_model.c:1361-1366, 1387-1399). Row m of the
// GEMM is input pixel (prompt, y, x) of an H x W map, its 128 columns the
// ConvTranspose 2x2 (64 -> 32) outputs in sub-pixel-major order, so chunk c
// (32 columns) is sub-pixel d = c = 2 dy + dx of output pixel (2y + dy,
// 2x + dx). Per chunk: u = GELU(acc + bias + feat_s0[pixel]) over the 32
// channels (feat_s0 as k_dec_feat_subpix lays it out), dotted with the
// prompt's three hypernetwork vectors, written as the three logits of that
// pixel: the [P, 2H, 2W, 32] map is never stored.
// Output pixel of sub-pixel d of input row m.
__device__ __forceinline__ long logits_pixel(const ConvGeom &cg, int m, int d)
{
    const int x = m % cg.cW, y = (m / cg.cW) % cg.cH;
    return (2L * y + (d >> 1)) * (2L * cg.cW) + 2 * x + (d & 1);
}

// feat of sub-pixel d for row m (k_dec_feat_subpix layout [4][C][H*W]):
// channel c of the warp's 32 consecutive pixels is one 128-byte line. Read
// before the accumulator is waited for, so the L2 latency hides behind the
// tile's main loop.
template <int C>
__device__ __forceinline__ void feat_load(const GemmEpi &p, const ConvGeom &cg, int m, int d,
                                          float (&f)[C])
{
    if (m >= p.M)
        return;
    const int hw = cg.cW * cg.cH;
    const float *src = p.R + (long)d * C * hw + (m % hw);
#pragma unroll
    for (int c = 0; c < C; c++)
        f[c] = __ldg(src + c * hw);
}

// kEpiLn2d: the first output-upscaling stage of the mask decoder
// (sam3_model.c:1355-1360) as the epilogue of its ConvTranspose 2x2
// (256 -> 64) GEMM: row m is input pixel (prompt, y, x), its 256 columns in
// sub-pixel-major order, so a 64-column chunk is sub-pixel d of output pixel
// (2y + dy, 2x + dx). Per chunk: v = acc + bias + feat_s1[pixel] (as
// k_dec_feat_subpix lays it out), LayerNorm
// over the 64 channels (eps = p.alpha), GELU, written as the pixel's 64 bf16
// channels of the [P, 2H, 2W, 64] map.
__device__ __forceinline__ void ln2d_chunk(const GemmEpi &p, const ConvGeom &cg, int m, int d,
                                           float (&v)[64])
{
    if (m >= p.M)
        return;
    const int hw = cg.cW * cg.cH, pr = m / hw;
    const long opix = logits_pixel(cg, m, d) + (long)pr * 4 * hw;
    const float *f = p.R + (long)d * 64 * hw + (m - pr * hw);
    const float4 *bq = reinterpret_cast<const float4 *>(p.bias);
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const float4 bv = __ldg(bq + j);
        v[4 * j] = (v[4 * j] + bv.x) + __ldg(f + (4 * j) * hw);
        v[4 * j + 1] = (v[4 * j + 1] + bv.y) + __ldg(f + (4 * j + 1) * hw);
        v[4 * j + 2] = (v[4 * j + 2] + bv.z) + __ldg(f + (4 * j + 2) * hw);
        v[4 * j + 3] = (v[4 * j + 3] + bv.w) + __ldg(f + (4 * j + 3) * hw);
        sum += (v[4 * j] + v[4 * j + 1]) + (v[4 * j + 2] + v[4 * j + 3]);
    }
    const float mean = sum * (1.0f / 64.0f);
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < 64; j++) {
        const float e = v[j] - mean;
        sq = fmaf(e, e, sq);
    }
    const float inv = rsqrtf(sq * (1.0f / 64.0f) + p.alpha);
    const float4 *gq = reinterpret_cast<const float4 *>(cg.lnw);
    const float4 *tq = reinterpret_cast<const float4 *>(cg.lnb);
    uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.C) + opix * 64);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        float y[8];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const float4 g = __ldg(gq + 2 * j + h), t = __ldg(tq + 2 * j + h);
            y[4 * h] = fmaf((v[8 * j + 4 * h] - mean) * inv, g.x, t.x);
            y[4 * h + 1] = fmaf((v[8 * j + 4 * h + 1] - mean) * inv, g.y, t.y);
            y[4 * h + 2] = fmaf((v[8 * j + 4 * h + 2] - mean) * inv, g.z, t.z);
            y[4 * h + 3] = fmaf((v[8 * j + 4 * h + 3] - mean) * inv, g.w, t.w);
        }
        gelu_pair(y[0], y[1]);
        gelu_pair(y[2], y[3]);
        gelu_pair(y[4], y[5]);
        gelu_pair(y[6], y[7]);
        dst[j] = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                            pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
    }
}

// kEpiConvT: a 2x2 / stride-2 ConvTranspose as the epilogue of its GEMM:
// row m is input pixel (map, y, x), the columns sub-pixel-major (d * cout +
// co), so the 64-column chunk at column n is channels co0 .. co0 + 63 of
// sub-pixel d = n / cout of output pixel (2y + dy, 2x + dx). bias[co] and
// the activation are applied and the 64 bf16 values stored straight into
// the [maps, 2H, 2W, cout] map (one 128-byte run).
__device__ __forceinline__ void convt_chunk(const GemmEpi &p, const ConvGeom &cg, int m, int n,
                                            float (&v)[64])
{
    if (m >= p.M || n >= p.N)
        return;
    const int d = n / cg.cout, co0 = n % cg.cout;
    const int x = m % cg.cW, t = m / cg.cW, y = t % cg.cH, mp = t / cg.cH;
    const long opix = ((long)mp * 2 * cg.cH + 2 * y + (d >> 1)) * (2L * cg.cW) + 2 * x + (d & 1);
    const float4 *bq = reinterpret_cast<const float4 *>(p.bias + co0);
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const float4 bv = __ldg(bq + j);
        v[4 * j] += bv.x;
        v[4 * j + 1] += bv.y;
        v[4 * j + 2] += bv.z;
        v[4 * j + 3] += bv.w;
    }
    if (p.act == K_ACT_GELU) {
#pragma unroll
        for (int j = 0; j < 64; j += 2)
            gelu_pair(v[j], v[j + 1]);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.C) +
                                           opix * cg.cout + co0);
#pragma unroll
    for (int j = 0; j < 8; j++)
        dst[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                            pack_bf16x2(v[8 * j + 4], v[8 * j + 5]),
                            pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
}

__device__ __forceinline__ void logits_chunk(const GemmEpi &p, const ConvGeom &cg, int m, int d,
                                             const float (&v)[32], const float (&f)[32])
{
    if (m >= p.M)
        return;
    const int pr = m / (cg.cW * cg.cH);
    const long opix = logits_pixel(cg, m, d);
    const float4 *bq = reinterpret_cast<const float4 *>(p.bias);
    const float4 *h = reinterpret_cast<const float4 *>(cg.hyper + (long)pr * 96);
    // packed fp32 (the epilogue is issue-bound): the adds on channel pairs,
    // each logit as even / odd channel partial sums added at the end
    uint64_t a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float4 bv = __ldg(bq + j);
        float u0, u1, u2, u3;
        f2_split(add2(add2(f2_make(v[4 * j], v[4 * j + 1]), f2_make(bv.x, bv.y)),
                      f2_make(f[4 * j], f[4 * j + 1])),
                 u0, u1);
        f2_split(add2(add2(f2_make(v[4 * j + 2], v[4 * j + 3]), f2_make(bv.z, bv.w)),
                      f2_make(f[4 * j + 2], f[4 * j + 3])),
                 u2, u3);
        gelu_pair(u0, u1);
        gelu_pair(u2, u3);
        const uint64_t g01 = f2_make(u0, u1), g23 = f2_make(u2, u3);
        const float4 h0 = __ldg(h + j), h1 = __ldg(h + 8 + j), h2 = __ldg(h + 16 + j);
        a0 = fma2(g23, f2_make(h0.z, h0.w), fma2(g01, f2_make(h0.x, h0.y), a0));
        a1 = fma2(g23, f2_make(h1.z, h1.w), fma2(g01, f2_make(h1.x, h1.y), a1));
        a2 = fma2(g23, f2_make(h2.z, h2.w), fma2(g01, f2_make(h2.x, h2.y), a2));
    }
    float e0, o0, e1, o1, e2, o2;
    f2_split(a0, e0, o0);
    f2_split(a1, e1, o1);
    f2_split(a2, e2, o2);
    float *o = reinterpret_cast<float *>(p.C);
    const long onpix = 4L * cg.cH * cg.cW;
    o[((long)pr * 3 + 0) * onpix + opix] = e0 + o0;
    o[((long)pr * 3 + 1) * onpix + opix] = e1 + o1;
    o[((long)pr * 3 + 2) * onpix + opix] = e2 + o2;
}

// ROPE_PF: bf16 output whose tiles may need RoPE, with the row's (cos, sin)
// pairs held in registers and no activation (a separate instantiation: the
// register budget of the other epilogues does not carry them).
// CONV3: the A operand is a 3x3 / pad-1 convolution's implicit im2col: K =
// 9 taps x C channels in tap-major order (ky * 3 + kx, then c), each K block
// of 64 one 4-D TMA load of the input map (C, W, H, image) at the tap's
// shifted pixel block -- rows and columns outside the map read as zero, so
// the padding costs nothing and no im2col is ever written. An M tile is an
// 8 x 16 pixel block (row r = y * 16 + x; a CTA pair's tile is 16 x 16, rank
// r taking pixel rows 8r .. 8r + 7), and each epilogue warp's 32 rows (two
// pixel rows) leave as one 4-D TMA store into the NHWC output.
// PAIR: a cluster of two CTAs (the two SMs of a TPC) computes 256 x BN
// tiles with cta_group::2 MMAs: each CTA loads its 128 rows of A and half of
// the B tile into its own shared memory, both signalling rank 0's full
// barrier; rank 0 issues 256 x BN x 16 MMAs whose accumulator rows 0-127
// land in its tensor memory and 128-255 in rank 1's, and its commits arrive
// on both CTAs' barriers; each CTA's epilogue stores its own 128 rows and
// releases the accumulator on rank 0's barrier. Per SM this halves the B
// tile traffic from L2 into shared memory.
template <int BN, bool OUT_BF16, bool TMA_STORE, bool ROPE_PF, bool CONV3 = false,
          bool PAIR = false, int EPI = kEpiGeneric>
__global__ void __launch_bounds__(gemm_threads(EPI), 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const GemmEpi p,
                        const ConvGeom cg)
{
    // CONV3 pixel blocks: 8 x 16 per CTA; a pair's tile is 16 x 16, rank r
    // taking pixel rows 8r .. 8r + 7 of it.
    constexpr int CBH = PAIR ? 16 : 8;
    constexpr bool LOGITS = EPI == kEpiLogits;
    static_assert(!LOGITS || (BN == 128 && !OUT_BF16 && !TMA_STORE && !PAIR && !CONV3),
                  "the logits epilogue: one 128-column fp32 tile per row block");
    static_assert(EPI != kEpiLn2d || (BN == 256 && OUT_BF16 && !TMA_STORE && !ROPE_PF && !PAIR &&
                                      !CONV3),
                  "the LayerNorm2d epilogue: one 256-column tile per row block, bf16");
    static_assert(EPI != kEpiConvT || (BN == 256 && OUT_BF16 && !TMA_STORE && !ROPE_PF && !PAIR &&
                                       !CONV3),
                  "the ConvTranspose epilogue: bf16 out, direct stores");
    constexpr int EW = epi_warps(EPI);
    constexpr int CSTEP = EW / 4;  // chunk stride of an epilogue warp
    using L = GemmSmem<BN, PAIR, TMA_STORE ? EW : 0>;  // staging tiles for TMA stores only
    constexpr int STAGES = L::STAGES;
    constexpr int CW = OUT_BF16 ? 64 : 32;  // columns per 128-byte chunk
    constexpr int NCHUNK = BN / CW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], PAIR ? 2 * EW : EW);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, 2 * BN);
            tmem_relinquish_pair();
        }
        else {
            tmem_alloc(tmem_slot, 2 * BN);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR)
        cluster_sync_all();  // both CTAs' barriers exist before either signals the other
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched as a programmatic dependent of the previous kernel (pdl.cuh):
    // the setup above used only this CTA's shared and tensor memory (and the
    // tensor maps, kernel parameters); every global access below waits for
    // that kernel. The next kernel may be scheduled once every CTA has its
    // tensor memory.
    griddep_launch();
    griddep_wait();

    constexpr int TM = PAIR ? 2 * BM : BM;  // rows per tile
    const int first = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int num_m = CONV3 ? cg.cimg * cg.cyb * cg.cxb : (p.M + TM - 1) / TM;
    const int num_n = (p.N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int kblocks = (p.K + BK - 1) / BK;
    // Tile sequence of this CTA (or pair): every step-th tile; with RoPE a
    // contiguous range of the m-major order instead (same count +-1), so
    // that consecutive tiles share their rows and the epilogue keeps the
    // rows' (cos, sin) pairs in registers across them.
    int t_begin = first, t_end = num_tiles, t_step = step;
    if (ROPE_PF && p.rope.mode) {
        t_begin = (int)((long)first * num_tiles / step);
        t_end = (int)((long)(first + 1) * num_tiles / step);
        t_step = 1;
    }

    if (warp == 0) {
        if (elect_one()) {
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, last_parity = 0;
            bool ok = true;
            for (int t = t_begin; t < t_end && ok; t += t_step) {
                const int m0 = (t / num_n) * TM + (int)rank * BM, n0 = (t % num_n) * BN;
                int img = 0, py0 = 0, px0 = 0;
                if constexpr (CONV3) {
                    const int mt = t / num_n;
                    img = mt / (cg.cyb * cg.cxb);
                    py0 = ((mt / cg.cxb) % cg.cyb) * CBH + (int)rank * 8;
                    px0 = (mt % cg.cxb) * 16;
                }
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!(PAIR ? mbar_wait_cluster(&empty[stage], phase ^ 1, p.err, abort_flag)
                               : mbar_wait(&empty[stage], phase ^ 1, p.err, abort_flag))) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + stage * L::STAGE_BYTES;
                    if constexpr (PAIR) {
                        if (rank == 0)
                            mbar_arrive_expect_tx(&full[stage], 2 * L::STAGE_BYTES);
                        const uint32_t fb = mapa_shared(smem_addr(&full[stage]), 0);
                        if constexpr (CONV3) {
                            const int cblocks = p.K / (9 * BK), tap = kb / cblocks;
                            tma_load_4d_pair(sa, &tmA, fb, (kb % cblocks) * BK,
                                             px0 + tap % 3 - 1, py0 + tap / 3 - 1, img);
                        }
                        else
                            tma_load_2d_pair(sa, &tmA, fb, kb * BK, m0);
                        tma_load_2d_pair(sa + L::A_BYTES, &tmB, fb, kb * BK,
                                         n0 + (int)rank * (BN / 2));
                        issued_mask |= 1u << stage;
                        last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                        continue;
                    }
                    mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
                    if constexpr (CONV3) {
                        const int cblocks = p.K / (9 * BK), tap = kb / cblocks;
                        tma_load_4d(sa, &tmA, &full[stage], (kb % cblocks) * BK,
                                    px0 + tap % 3 - 1, py0 + tap / 3 - 1, img);
                    }
                    else
                        tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
                    tma_load_2d(sa + L::A_BYTES, &tmB, &full[stage], kb * BK, n0);
                    issued_mask |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Let every copy this thread issued land before the CTA exits
            // (in a pair, rank 0's barriers count both CTAs' copies; rank 1
            // is held by the closing cluster barrier).
            for (int s = 0; s < STAGES; s++)
                if (rank == 0 && (issued_mask & (1u << s))) {
                    volatile int no_abort = 0;
                    mbar_wait(&full[s], (last_parity >> s) & 1, p.err, &no_abort);
                }
        }
    }
    else if (warp == 1) {
        if (elect_one()) {
            if (rank == 0) {
                constexpr uint32_t idesc = idesc_bf16_f32(TM, BN, 0, 0);
                int stage = 0;
                uint32_t phase = 0;
                int acc = 0;
                uint32_t acc_phase = 0;
                bool ok = true;
                for (int t = t_begin; t < t_end && ok; t += t_step) {
                    if (!(PAIR ? mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, p.err, abort_flag)
                               : mbar_wait(&tempty[acc], acc_phase ^ 1, p.err, abort_flag)))
                        break;
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                    for (int kb = 0; kb < kblocks; kb++) {
                        if (!mbar_wait(&full[stage], phase, p.err, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = smem_addr(smem + stage * L::STAGE_BYTES);
                        const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
                        for (int k = 0; k < BK / 16; k++) {
                            if constexpr (PAIR)
                                tc_mma_pair(d, sw128_desc(sa + k * 32, 16, 1024),
                                            sw128_desc(sb + k * 32, 16, 1024), idesc,
                                            (kb | k) != 0);
                            else
                                tc_mma(d, sw128_desc(sa + k * 32, 16, 1024),
                                       sw128_desc(sb + k * 32, 16, 1024), idesc, (kb | k) != 0);
                        }
                        if constexpr (PAIR)
                            tc_commit_pair(&empty[stage], 3);
                        else
                            tc_commit(&empty[stage]);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok)
                        break;
                    if constexpr (PAIR)
                        tc_commit_pair(&tfull[acc], 3);
                    else
                        tc_commit(&tfull[acc]);
                    acc ^= 1;
                    if (acc == 0)
                        acc_phase ^= 1;
                }
                // Drain: one arrival (on both CTAs' barriers in a pair) once
                // every MMA issued above has completed.
                if constexpr (PAIR)
                    tc_commit_pair(drain, 3);
                else
                    tc_commit(drain);
            }
            // Tensor memory is idle before it is freed.
            volatile int no_abort = 0;
            if constexpr (PAIR)
                mbar_wait_cluster(drain, 0, p.err, &no_abort);
            else
                mbar_wait(drain, 0, p.err, &no_abort);
        }
    }
    else {
        const int ew = warp - 2;          // 0 .. EW - 1
        const int quarter = warp & 3;     // TMEM lane quarter this warp may read
        const int half = ew >> 2;         // which chunks of the tile (c % CSTEP)
        constexpr int kEpiBufs = L::EPI_BUFS;
        const uint32_t stage0 = smem_addr(smem + L::EPI_OFF + ew * kEpiBufs * kStageTile);
        int buf = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        if (TMA_STORE && lane == 0)
            prefetch_tmap(&tmC);
        float2 rc[ROPE_PF ? 32 : 1];  // this row's RoPE (cos, sin) pairs
        int rc_row = -1;               // the table row they are of
        for (int t = t_begin; t < t_end; t += t_step) {
            const int m0 = (t / num_n) * TM + (int)rank * BM, n0 = (t % num_n) * BN;
            int r0 = m0 + quarter * 32;
            int m = r0 + lane;
            int cimg = 0, cy = 0, cx0 = 0;
            if constexpr (CONV3) {
                // this warp's rows: pixel rows cy, cy + 1 of the block, x
                // cx0 .. cx0 + 15; m = the pixel's index in the NHWC output
                // (p.M when outside the map)
                const int mt = t / num_n;
                cimg = mt / (cg.cyb * cg.cxb);
                cy = ((mt / cg.cxb) % cg.cyb) * CBH + (int)rank * 8 + 2 * quarter;
                cx0 = (mt % cg.cxb) * 16;
                const int py = cy + lane / 16, px = cx0 + lane % 16;
                m = (py < cg.cH && px < cg.cW) ? (cimg * cg.cH + py) * cg.cW + px : p.M;
                r0 = cy < cg.cH ? 0 : p.M;  // the chunk's store is issued when r0 < p.M
            }
            const int rrow = p.rope.mode ? rope_row(p.rope, m < p.M ? m : 0) : 0;
            // Global reads issued before the accumulator wait, so that their
            // latency hides behind the tile's main loop: with bf16 output the
            // row's 32 RoPE (cos, sin) pairs when the row changed (every
            // 64-column chunk is one head and uses all of them); with fp32
            // output the residual of this warp's first chunk (later chunks
            // are fetched one ahead).
            const bool rope_tile = ROPE_PF && p.rope.mode && p.rope.hd == 64 && n0 < 2 * p.rope.E;
            if (ROPE_PF && rope_tile && rrow != rc_row) {
                rc_row = rrow;
                const float4 *cs = reinterpret_cast<const float4 *>(p.rope.cs) + (long)rrow * 16;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float4 q = __ldg(cs + j);
                    rc[2 * j] = make_float2(q.x, q.y);
                    rc[2 * j + 1] = make_float2(q.z, q.w);
                }
            }
            const bool rfast = !OUT_BF16 && !LOGITS && p.R && m < p.M && n0 + BN <= p.N &&
                               (p.ldr & 3) == 0 &&
                               (reinterpret_cast<uintptr_t>(p.R) & 15) == 0;
            const float *rrowp =
                rfast ? p.R + (long)(p.rmod ? m % p.rmod : m) * p.ldr + n0 : nullptr;
            float4 rnext[OUT_BF16 ? 1 : CW / 4];
            if (!OUT_BF16 && rfast) {
#pragma unroll
                for (int j = 0; j < CW / 4; j++)
                    rnext[j] = *reinterpret_cast<const float4 *>(rrowp + half * CW + 4 * j);
            }
            // mask logits: the feat values of the warp's chunks, read ahead
            // as well
            constexpr int LCH = LOGITS ? NCHUNK / CSTEP : 1;
            float fpre[LCH][LOGITS ? 32 : 1];
            if constexpr (LOGITS) {
#pragma unroll
                for (int cc = 0; cc < LCH; cc++)
                    feat_load<32>(p, cg, m, half + CSTEP * cc, fpre[cc]);
            }
            const bool ok = PAIR ? mbar_wait_cluster(&tfull[acc], acc_phase, p.err, abort_flag)
                                 : mbar_wait(&tfull[acc], acc_phase, p.err, abort_flag);
            if (!__all_sync(0xffffffffu, ok))
                break;
            tc_fence_after();
            const uint32_t tbase =
                tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
            if constexpr (LOGITS) {
                // the warp's chunks' accumulators first, then the tile is
                // released
                float va[LCH][32];
#pragma unroll
                for (int cc = 0; cc < LCH; cc++) {
                    uint32_t r[32];
                    tmem_ld32(tbase + (half + CSTEP * cc) * CW, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        va[cc][j] = __uint_as_float(r[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&tempty[acc]);
#pragma unroll
                for (int cc = 0; cc < LCH; cc++)
                    logits_chunk(p, cg, m, half + CSTEP * cc, va[cc], fpre[cc]);
                acc ^= 1;
                if (acc == 0)
                    acc_phase ^= 1;
            }
            else if constexpr (EPI == kEpiLn2d) {
                // chunks half and half + CSTEP (sub-pixels); the tile is
                // released once the second chunk's accumulator is loaded
                static_assert(NCHUNK == 2 * CSTEP, "two chunks per epilogue warp");
                float v[64];
#pragma unroll 1
                for (int cc = 0; cc < 2; cc++) {
                    {
                        uint32_t r[32], r2[32];
                        tmem_ld32(tbase + (half + CSTEP * cc) * CW, r);
                        tmem_ld32(tbase + (half + CSTEP * cc) * CW + 32, r2);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            v[j] = __uint_as_float(r[j]);
                            v[32 + j] = __uint_as_float(r2[j]);
                        }
                    }
                    if (cc == 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0)
                            mbar_arrive(&tempty[acc]);
                    }
                    ln2d_chunk(p, cg, m, half + CSTEP * cc, v);
                }
                acc ^= 1;
                if (acc == 0)
                    acc_phase ^= 1;
            }
            else {
#pragma unroll 1
                for (int c = half; c < NCHUNK; c += CSTEP) {
                    const int n = n0 + c * CW;
                    if (n >= p.N)
                        continue;  // warp-uniform: a chunk entirely beyond C
                    uint32_t pk[32];  // the chunk's 128-byte output row
                    float v32[OUT_BF16 ? 1 : 32];
                    if constexpr (OUT_BF16 && !ROPE_PF) {
                        // 64 columns in one TMEM round trip.
                        float v[64];
                        {
                            uint32_t r[32], r2[32];
                            tmem_ld32(tbase + c * CW, r);
                            tmem_ld32(tbase + c * CW + 32, r2);
                            tmem_wait_ld();
#pragma unroll
                            for (int j = 0; j < 32; j++) {
                                v[j] = __uint_as_float(r[j]);
                                v[32 + j] = __uint_as_float(r2[j]);
                            }
                        }
                        if constexpr (EPI == kEpiConvT) {
                            convt_chunk(p, cg, m, n, v);
                            continue;
                        }
                        epilogue_math<64>(p, m, n, v, rrow, nullptr, nullptr);
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            pk[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
                    }
                    else if constexpr (OUT_BF16) {
                        // With the row's RoPE pairs held in registers: 64 columns
                        // in two halves of 32 (fewer live registers).
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            float v[32];
                            {
                                uint32_t r[32];
                                tmem_ld32(tbase + c * CW + h * 32, r);
                                tmem_wait_ld();
#pragma unroll
                                for (int j = 0; j < 32; j++)
                                    v[j] = __uint_as_float(r[j]);
                            }
                            epilogue_math<32, false>(p, m, n + h * 32, v, rrow, nullptr,
                                              rope_tile && n < 2 * p.rope.E ? rc + h * 16 : nullptr);
#pragma unroll
                            for (int j = 0; j < 16; j++)
                                pk[h * 16 + j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
                        }
                    }
                    else {
                        float4 rcur[CW / 4];
#pragma unroll
                        for (int j = 0; j < CW / 4; j++)
                            rcur[j] = rnext[j];
                        if (rfast && c + CSTEP < NCHUNK) {
#pragma unroll
                            for (int j = 0; j < CW / 4; j++)
                                rnext[j] = *reinterpret_cast<const float4 *>(rrowp + (c + CSTEP) * CW +
                                                                             4 * j);
                        }
                        {
                            uint32_t r[32];
                            tmem_ld32(tbase + c * CW, r);
                            tmem_wait_ld();
#pragma unroll
                            for (int j = 0; j < 32; j++)
                                v32[j] = __uint_as_float(r[j]);
                        }
                        epilogue_math<32>(p, m, n, v32, rrow, rfast ? rcur : nullptr, nullptr);
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            pk[j] = __float_as_uint(v32[j]);
                    }
                    if (TMA_STORE) {
                        // The store issued kEpiBufs chunks ago used this buffer.
                        if (lane == 0)
                            bulk_wait_read<kEpiBufs - 1>();
                        __syncwarp();
                        const uint32_t tile = stage0 + buf * kStageTile;
                        stage_row(tile, lane, pk);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0 && r0 < p.M) {
                            const void *src = smem + L::EPI_OFF + ew * kEpiBufs * kStageTile +
                                              buf * kStageTile;
                            if constexpr (CONV3)
                                tma_store_4d(&tmC, src, n, cx0, cy, cimg);
                            else if (!OUT_BF16 && p.red)
                                tma_reduce_add_2d(&tmC, src, n, r0);
                            else
                                tma_store_2d(&tmC, src, n, r0);
                            bulk_commit();
                        }
                        buf = (buf + 1) % kEpiBufs;
                    }
                    else
                        store_direct<CW, OUT_BF16>(p, m, n, pk);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (PAIR)
                        mbar_arrive_cluster(mapa_shared(smem_addr(&tempty[acc]), 0));
                    else
                        mbar_arrive(&tempty[acc]);
                }
                acc ^= 1;
                if (acc == 0)
                    acc_phase ^= 1;
            }
        }
        if (TMA_STORE && lane == 0)
            bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    // In a pair, neither CTA leaves (nor frees tensor memory) while the
    // other's MMAs, copies or arrivals may still touch its shared memory.
    if constexpr (PAIR)
        cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR)
            tmem_dealloc_pair(tmem_base, 2 * BN);
        else
            tmem_dealloc(tmem_base, 2 * BN);
    }
}

template <int BN, bool OUT_BF16, bool TMA_STORE, bool ROPE_PF = false, bool CONV3 = false,
          int EPI = kEpiGeneric>
int launch(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tc,
           const GemmEpi &p, int num_sms, cudaStream_t s,
           const ConvGeom &cg = ConvGeom{0, 0, 0, 0, 0})
{
    using L = GemmSmem<BN, false, TMA_STORE ? epi_warps(EPI) : 0>;
    auto kern = gemm_bf16_tc_kernel<BN, OUT_BF16, TMA_STORE, ROPE_PF, CONV3, false, EPI>;
    cudaError_t e =
        smem_limit_once<gemm_bf16_tc_kernel<BN, OUT_BF16, TMA_STORE, ROPE_PF, CONV3, false, EPI>>(
            L::BYTES);
    if (e != cudaSuccess)
        return (int)e;
    const int tiles = (CONV3 ? cg.cimg * cg.cyb * cg.cxb : (p.M + BM - 1) / BM) *
                      ((p.N + BN - 1) / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    return launch_pdl(kern, dim3(grid), dim3(gemm_threads(EPI)), L::BYTES, s, ta, tb, tc, p, cg);
}

// Co-resident clusters of two CTAs of the pair kernel, per device (0: not
// known yet; -1: none).
static int g_pair_clusters[64];

// The pair kernel over 256 x 256 tiles: a persistent grid of as many CTA
// pairs as can be resident at once (each cluster on the two SMs of a TPC).
// Returns 1 when pairs cannot be launched here (the caller uses single CTAs).
template <bool OUT_BF16, bool ROPE_PF, bool CONV3 = false>
int launch_pair(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tc,
                const GemmEpi &p, int num_sms, cudaStream_t s,
                const ConvGeom &cg = ConvGeom{0, 0, 0, 0, 0})
{
    constexpr int BN = 256;
    using L = GemmSmem<BN, true>;
    auto kern = gemm_bf16_tc_kernel<BN, OUT_BF16, true, ROPE_PF, CONV3, true>;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return 1;
    cudaError_t e =
        smem_limit_once<gemm_bf16_tc_kernel<BN, OUT_BF16, true, ROPE_PF, CONV3, true>>(L::BYTES);
    if (e != cudaSuccess)
        return (int)e;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms / 2 > 0 ? num_sms / 2 : 1));
    cfg.blockDim = dim3(gemm_threads(kEpiGeneric));
    cfg.dynamicSmemBytes = L::BYTES;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (g_pair_clusters[dev] == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = -1;
        }
        g_pair_clusters[dev] = n;
    }
    if (g_pair_clusters[dev] < 0)
        return 1;
    const int tiles = (CONV3 ? cg.cimg * cg.cyb * cg.cxb : (p.M + 2 * BM - 1) / (2 * BM)) *
                      ((p.N + BN - 1) / BN);
    const int pairs = tiles < g_pair_clusters[dev] ? tiles : g_pair_clusters[dev];
    cfg.gridDim = dim3(2 * pairs);
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, p, cg);
    return e == cudaSuccess ? (int)cudaGetLastError() : (int)e;
}

template <int BN>
int launch_bn(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tc, bool tma,
              bool bf16, const GemmEpi &p, int num_sms, cudaStream_t s)
{
    if (bf16)
        return tma ? (p.rope.mode && p.rope.hd == 64 && p.act == K_ACT_NONE
                          ? launch<BN, true, true, true>(ta, tb, tc, p, num_sms, s)
                          : launch<BN, true, true>(ta, tb, tc, p, num_sms, s))
                   : launch<BN, true, false>(ta, tb, tc, p, num_sms, s);
    return tma ? launch<BN, false, true>(ta, tb, tc, p, num_sms, s)
               : launch<BN, false, false>(ta, tb, tc, p, num_sms, s);
}

}  // namespace
}  // namespace sam3

extern "C" int k_gemm_bf16_tc(int M, int N, int K, const void *A, int lda, const void *B,
                              int ldb, void *C, int ldc, int c_bf16, const float *bias,
                              const float *R, int ldr, int rmod, float alpha, int act,
                              const struct k_rope *rope, int *err, int num_sms, k_stream s)
{
    using namespace sam3;
    if (M <= 0 || N <= 0 || K <= 0 || (lda & 7) || (ldb & 7) || lda < K || ldb < K)
        return K_EARG;
    if (rope && rope->mode && (rope->hd != 64 || (rope->E & 63) || 2 * rope->E > N))
        return K_EARG;
    if (bias && (reinterpret_cast<uintptr_t>(bias) & 15))
        return K_EARG;
    // 128-wide tiles for N <= 128, and where 256-wide ones would leave more
    // than half of the SMs without a tile (the decoder's token stream: 512
    // rows, 4 tiles at N = 256): twice the CTAs, half the serial MMA work
    // per CTA.
    const long tiles256 = (long)((M + BM - 1) / BM) * ((N + 255) / 256);
    const int BN = N <= 128 || tiles256 < num_sms / 2 ? 128 : 256;
    CUtensorMap ta, tb, tc, tb_half;
    if (!make_tmap_bf16(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM) ||
        !make_tmap_bf16(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, (uint32_t)BN))
        return K_ETMAP;
    // TMA stores need a 16-byte aligned base and row pitch; else direct stores.
    const bool tma = c_bf16 ? make_tmap_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C,
                                           (uint64_t)M, (uint64_t)N, (uint64_t)ldc, 64, 32)
                            : make_tmap_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, C,
                                           (uint64_t)M, (uint64_t)N, (uint64_t)ldc, 32, 32);
    if (!tma)
        tc = ta;  // unused by the direct-store kernels
    GemmEpi p;
    p.M = M;
    p.N = N;
    p.K = K;
    p.C = C;
    p.ldc = ldc;
    p.bias = bias;
    p.R = R;
    p.ldr = ldr;
    p.rmod = rmod;
    p.alpha = alpha;
    p.act = act;
    if (rope)
        p.rope = *rope;
    else
        p.rope = k_rope{nullptr, 0, 0, 0, 0, 0, 0, 0};
    p.err = err;
    // In-place residual (C = R, the residual stream x += f(x)): the epilogue
    // leaves the residual read to L2 and reduce-adds its result into C, so
    // no epilogue warp waits on residual loads. Same arithmetic: the fp32
    // sum of the epilogue value and C's element, one rounding.
    p.red = 0;
    if (!c_bf16 && tma && R && reinterpret_cast<const void *>(R) == C && ldr == ldc &&
        rmod == 0) {
        p.R = nullptr;
        p.red = 1;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    if (BN == 128)
        return launch_bn<128>(ta, tb, tc, tma, c_bf16 != 0, p, num_sms, st);
    // CTA pairs (256 x 256 tiles) when there are enough tiles to give every
    // pair of SMs at least one, with TMA stores, and the main loop or the
    // in-place reduce-add carries the tile: bf16 output, K above 1024, or an
    // fp32 residual updated in place (the attention projection, K = 1024:
    // 830 -> 935 TFLOP/s in pairs once its epilogue stopped reading the
    // residual; other fp32-output GEMMs with short K stay on single CTAs).
    const long pair_tiles = (long)((M + 2 * BM - 1) / (2 * BM)) * ((N + 255) / 256);
    if (tma && pair_tiles >= num_sms / 2 && (c_bf16 || K > 1024 || p.red) &&
        make_tmap_bf16(&tb_half, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 128)) {
        const bool rope64 = p.rope.mode && p.rope.hd == 64 && p.act == K_ACT_NONE;
        const int rc = c_bf16 ? (rope64 ? launch_pair<true, true>(ta, tb_half, tc, p, num_sms, st)
                                        : launch_pair<true, false>(ta, tb_half, tc, p, num_sms, st))
                              : launch_pair<false, false>(ta, tb_half, tc, p, num_sms, st);
        if (rc != 1)
            return rc;
    }
    return launch_bn<256>(ta, tb, tc, tma, c_bf16 != 0, p, num_sms, st);
}

extern "C" int k_conv3x3_bf16_tc(const void *X, int nimg, int H, int W, int C, const void *Wt,
                                 int N, const float *bias, const float *R, void *out,
                                 int out_bf16, int *err, int num_sms, k_stream s)
{
    using namespace sam3;
    if (nimg <= 0 || H <= 0 || W <= 0 || C <= 0 || C % BK || N <= 0 || N % 64 ||
        (bias && (reinterpret_cast<uintptr_t>(bias) & 15)) ||
        (R && (reinterpret_cast<uintptr_t>(R) & 15)))
        return K_EARG;
    const int BN = N <= 128 ? 128 : 256;
    const int K = 9 * C;
    CUtensorMap ta, tb, tc;
    if (!make_tmap_nhwc(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, X, (uint64_t)nimg,
                        (uint64_t)H, (uint64_t)W, (uint64_t)C, BK, 16, 8) ||
        !make_tmap_bf16(&tb, Wt, (uint64_t)N, (uint64_t)K, (uint64_t)K, (uint32_t)BN) ||
        !(out_bf16 ? make_tmap_nhwc(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, (uint64_t)nimg,
                                    (uint64_t)H, (uint64_t)W, (uint64_t)N, 64, 16, 2)
                   : make_tmap_nhwc(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, out, (uint64_t)nimg,
                                    (uint64_t)H, (uint64_t)W, (uint64_t)N, 32, 16, 2)))
        return K_ETMAP;
    GemmEpi p;
    p.M = nimg * H * W;
    p.N = N;
    p.K = K;
    p.C = out;
    p.ldc = N;
    p.bias = bias;
    p.R = R;
    p.ldr = N;
    p.rmod = 1;  // R: one row added to every pixel
    p.alpha = 1.0f;
    p.act = K_ACT_NONE;
    p.rope = k_rope{nullptr, 0, 0, 0, 0, 0, 0, 0};
    p.err = err;
    p.red = 0;
    ConvGeom cg{};
    cg.cH = H;
    cg.cW = W;
    cg.cimg = nimg;
    cg.cyb = (H + 7) / 8;
    cg.cxb = (W + 15) / 16;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    if (BN == 128)
        return out_bf16 ? launch<128, true, true, false, true>(ta, tb, tc, p, num_sms, st, cg)
                        : launch<128, false, true, false, true>(ta, tb, tc, p, num_sms, st, cg);
    // CTA pairs over 16 x 16 pixel blocks (K = 9C is long, so the halved B
    // traffic pays, as for fc2) when one map alone gives every pair of SMs a
    // tile: decided per map size, not per batch, so a map's result does not
    // depend on how many maps are convolved with it.
    ConvGeom cgp = cg;
    cgp.cyb = (H + 15) / 16;
    CUtensorMap tb_half;
    if (N == 256 && (long)cgp.cyb * cgp.cxb >= num_sms / 2 &&
        make_tmap_bf16(&tb_half, Wt, (uint64_t)N, (uint64_t)K, (uint64_t)K, 128)) {
        const int rc = out_bf16 ? launch_pair<true, false, true>(ta, tb_half, tc, p, num_sms, st, cgp)
                                : launch_pair<false, false, true>(ta, tb_half, tc, p, num_sms, st, cgp);
        if (rc != 1)
            return rc;
    }
    return out_bf16 ? launch<256, true, true, false, true>(ta, tb, tc, p, num_sms, st, cg)
                    : launch<256, false, true, false, true>(ta, tb, tc, p, num_sms, st, cg);
}

extern "C" int k_dec_convt_logits(const void *X, int P, int H, int W, const void *Wt,
                                  const float *bias, const float *feat, const float *hyper,
                                  float *out, int *err, int num_sms, k_stream s)
{
    using namespace sam3;
    if (P <= 0 || H <= 0 || W <= 0 || (long)P * H * W > 0x7fffffffL ||
        (reinterpret_cast<uintptr_t>(bias) & 15) || (reinterpret_cast<uintptr_t>(feat) & 15) ||
        (reinterpret_cast<uintptr_t>(hyper) & 15))
        return K_EARG;
    const int M = P * H * W;
    CUtensorMap ta, tb;
    if (!make_tmap_bf16(&ta, X, (uint64_t)M, 64, 64, BM) ||
        !make_tmap_bf16(&tb, Wt, 128, 64, 64, 128))
        return K_ETMAP;
    GemmEpi p;
    p.M = M;
    p.N = 128;
    p.K = 64;
    p.C = out;
    p.ldc = 0;
    p.bias = bias;
    p.R = feat;
    p.ldr = 32;
    p.rmod = 0;
    p.alpha = 1.0f;
    p.act = K_ACT_NONE;
    p.rope = k_rope{nullptr, 0, 0, 0, 0, 0, 0, 0};
    p.err = err;
    p.red = 0;
    ConvGeom cg{H, W, P, 0, 0, hyper, nullptr, nullptr};
    return launch<128, false, false, false, false, kEpiLogits>(
        ta, tb, ta, p, num_sms, reinterpret_cast<cudaStream_t>(s), cg);
}

extern "C" int k_dec_convt_ln2d(const void *X, int P, int H, int W, const void *Wt,
                                const float *bias, const float *feat, const float *lnw,
                                const float *lnb, float eps, void *out, int *err, int num_sms,
                                k_stream s)
{
    using namespace sam3;
    if (P <= 0 || H <= 0 || W <= 0 || (long)P * H * W > 0x7fffffffL ||
        (reinterpret_cast<uintptr_t>(bias) & 15) || (reinterpret_cast<uintptr_t>(feat) & 15) ||
        (reinterpret_cast<uintptr_t>(lnw) & 15) || (reinterpret_cast<uintptr_t>(lnb) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15))
        return K_EARG;
    const int M = P * H * W;
    CUtensorMap ta, tb;
    if (!make_tmap_bf16(&ta, X, (uint64_t)M, 256, 256, BM) ||
        !make_tmap_bf16(&tb, Wt, 256, 256, 256, 256))
        return K_ETMAP;
    GemmEpi p;
    p.M = M;
    p.N = 256;
    p.K = 256;
    p.C = out;
    p.ldc = 0;
    p.bias = bias;
    p.R = feat;
    p.ldr = 64;
    p.rmod = 0;
    p.alpha = eps;
    p.act = K_ACT_NONE;
    p.rope = k_rope{nullptr, 0, 0, 0, 0, 0, 0, 0};
    p.err = err;
    p.red = 0;
    ConvGeom cg{H, W, P, 0, 0, nullptr, lnw, lnb};
    return launch<256, true, false, false, false, kEpiLn2d>(
        ta, tb, ta, p, num_sms, reinterpret_cast<cudaStream_t>(s), cg);
}

extern "C" int k_convt2x2_bf16_tc(const void *X, int nimg, int H, int W, int cin, const void *Wt,
                                  int cout, const float *bias, int act, void *out, int *err,
                                  int num_sms, k_stream s)
{
    using namespace sam3;
    if (nimg <= 0 || H <= 0 || W <= 0 || cin <= 0 || cin % 8 || cout <= 0 || cout % 64 ||
        (long)nimg * H * W > 0x7fffffffL || (reinterpret_cast<uintptr_t>(bias) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15))
        return K_EARG;
    const int M = nimg * H * W, N = 4 * cout;
    CUtensorMap ta, tb;
    if (!make_tmap_bf16(&ta, X, (uint64_t)M, (uint64_t)cin, (uint64_t)cin, BM) ||
        !make_tmap_bf16(&tb, Wt, (uint64_t)N, (uint64_t)cin, (uint64_t)cin, 256))
        return K_ETMAP;
    GemmEpi p;
    p.M = M;
    p.N = N;
    p.K = cin;
    p.C = out;
    p.ldc = 0;
    p.bias = bias;
    p.R = nullptr;
    p.ldr = 0;
    p.rmod = 0;
    p.alpha = 1.0f;
    p.act = act;
    p.rope = k_rope{nullptr, 0, 0, 0, 0, 0, 0, 0};
    p.err = err;
    p.red = 0;
    ConvGeom cg{H, W, nimg, 0, 0, nullptr, nullptr, nullptr, cout};
    return launch<256, true, false, false, false, kEpiConvT>(
        ta, tb, ta, p, num_sms, reinterpret_cast<cudaStream_t>(s), cg);
}
