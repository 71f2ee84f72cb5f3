// SPDX-License-Identifier: Unlicense
// fp32 CUDA-core kernels: the backbone attention in reference precision
// (the "fp32-reference mode" of the global-attention config) and the
// reference-contract batched GEMM used for operands the tensor-core path
// does not take (sam3_kernels.cl:57-156). The mask decoder's attention is in
// attn_decoder.cu.
#include "kernels.h"
#include "tc_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace sam3 {
namespace {

// ------------------------------------------------------ fp32 attention
// One thread per query row (128 per CTA), K/V tiles of 32 keys staged in
// shared memory, online softmax per tile with expf. hd = 64. Q, O and the
// dot products are held as fp32 pairs for the packed f32x2 instructions
// (each lane an IEEE fp32 fma; a score is four interleaved partial sums).
constexpr int F_HD = 64;
constexpr int F_BQ = 128;
constexpr int F_BK = 32;

__global__ void __launch_bounds__(F_BQ) attn_f32_kernel(const float *__restrict__ qkv, int nseq,
                                                       int N, int E, int heads, float scale,
                                                       float *__restrict__ out)
{
    __shared__ __align__(16) float ks[F_BK][F_HD];
    __shared__ __align__(16) float vs[F_BK][F_HD];
    const int nqt = (N + F_BQ - 1) / F_BQ;
    const int qt = blockIdx.x % nqt;
    const int h = (blockIdx.x / nqt) % heads;
    const int seq = blockIdx.x / (nqt * heads);
    const long ld = 3L * E;
    const long base = (long)seq * N * ld;
    const int qi = qt * F_BQ + threadIdx.x;
    const bool valid = qi < N;
    uint64_t q2[F_HD / 2], o2[F_HD / 2];
    const float *qp = qkv + base + (long)(valid ? qi : 0) * ld + h * F_HD;
#pragma unroll
    for (int d = 0; d < F_HD; d += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(qp + d);
        q2[d / 2] = f2_make(v.x * scale, v.y * scale);
        q2[d / 2 + 1] = f2_make(v.z * scale, v.w * scale);
        o2[d / 2] = o2[d / 2 + 1] = 0;
    }
    float m = -INFINITY, l = 0.0f;
    for (int k0 = 0; k0 < N; k0 += F_BK) {
        __syncthreads();
        for (int i = threadIdx.x; i < F_BK * F_HD / 4; i += F_BQ) {
            const int kr = i / (F_HD / 4), c = (i % (F_HD / 4)) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (k0 + kr < N) {
                const float *row = qkv + base + (long)(k0 + kr) * ld + h * F_HD + c;
                kv = *reinterpret_cast<const float4 *>(row + E);
                vv = *reinterpret_cast<const float4 *>(row + 2 * E);
            }
            *reinterpret_cast<float4 *>(&ks[kr][c]) = kv;
            *reinterpret_cast<float4 *>(&vs[kr][c]) = vv;
        }
        __syncthreads();
        const int nk = min(F_BK, N - k0);
        float s[F_BK];
        float mx = m;
#pragma unroll
        for (int j = 0; j < F_BK; j++) {
            uint64_t a0 = 0, a1 = 0;
#pragma unroll
            for (int d = 0; d < F_HD; d += 4) {
                const ulonglong2 k2 = *reinterpret_cast<const ulonglong2 *>(&ks[j][d]);
                a0 = fma2(q2[d / 2], k2.x, a0);
                a1 = fma2(q2[d / 2 + 1], k2.y, a1);
            }
            float x0, x1, x2, x3;
            f2_split(a0, x0, x1);
            f2_split(a1, x2, x3);
            const float acc = (x0 + x1) + (x2 + x3);
            s[j] = j < nk ? acc : -INFINITY;
            mx = fmaxf(mx, s[j]);
        }
        const float corr = expf(m - mx);
        l *= corr;
        const uint64_t c2 = f2_make(corr, corr);
#pragma unroll
        for (int d = 0; d < F_HD / 2; d++)
            o2[d] = mul2(o2[d], c2);
#pragma unroll
        for (int j = 0; j < F_BK; j++) {
            const float p = expf(s[j] - mx);
            l += p;
            const uint64_t p2 = f2_make(p, p);
#pragma unroll
            for (int d = 0; d < F_HD; d += 4) {
                const ulonglong2 v2 = *reinterpret_cast<const ulonglong2 *>(&vs[j][d]);
                o2[d / 2] = fma2(p2, v2.x, o2[d / 2]);
                o2[d / 2 + 1] = fma2(p2, v2.y, o2[d / 2 + 1]);
            }
        }
        m = mx;
    }
    if (valid) {
        const float inv = 1.0f / l;
        float *op = out + ((long)seq * N + qi) * E + h * F_HD;
#pragma unroll
        for (int d = 0; d < F_HD; d += 4) {
            float a, b, c, e;
            f2_split(o2[d / 2], a, b);
            f2_split(o2[d / 2 + 1], c, e);
            *reinterpret_cast<float4 *>(op + d) = make_float4(a * inv, b * inv, c * inv, e * inv);
        }
    }
}

// ------------------------------------------------------ SIMT GEMM
// The reference GEMM contract (sam3_kernels.cl:57-69) on CUDA cores, any
// strides, operands fp32 / bf16 / fp16: 64 x 64 tile per 256 threads, 4 x 4
// outputs per thread, K steps of 16 through shared memory.
__device__ __forceinline__ float ld_any(const void *p, int dt, long i)
{
    if (dt == 1)
        return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    if (dt == 2)
        return __half2float(reinterpret_cast<const __half *>(p)[i]);
    return reinterpret_cast<const float *>(p)[i];
}

__device__ __forceinline__ float act_fn(float v, int act)
{
    if (act == K_ACT_GELU)
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    if (act == K_ACT_RELU)
        return fmaxf(v, 0.0f);
    return v;
}

__global__ void __launch_bounds__(256) gemm_simt_kernel(
    int M, int N, int K, const void *A, int adt, long aoff, int lda, long sa0, long sa1,
    const void *B, int bdt, long boff, int ldb, long sb0, long sb1, int transb, float *C,
    long coff, int ldc, long sc0, long sc1, int nb1, const float *bias, const float *R, long roff,
    float alpha, int act)
{
    __shared__ float As[16][65];
    __shared__ float Bs[16][65];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int n0 = blockIdx.x * 64, m0 = blockIdx.y * 64;
    const long b = blockIdx.z, b0 = b / nb1, b1 = b % nb1;
    const long ao = aoff + b0 * sa0 + b1 * sa1;
    const long bo = boff + b0 * sb0 + b1 * sb1;
    const long co = coff + b0 * sc0 + b1 * sc1;
    const long ro = roff + b0 * sc0 + b1 * sc1;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int l = threadIdx.x; l < 1024; l += 256) {
            const int r = l >> 4, c = l & 15;
            const int gm = m0 + r, gk = k0 + c;
            As[c][r] = (gm < M && gk < K) ? ld_any(A, adt, ao + (long)gm * lda + gk) : 0.0f;
            if (transb) {
                const int gn = n0 + r;
                Bs[c][r] = (gn < N && gk < K) ? ld_any(B, bdt, bo + (long)gn * ldb + gk) : 0.0f;
            }
            else {
                const int kk = l >> 6, nn = l & 63;
                const int gk2 = k0 + kk, gn = n0 + nn;
                Bs[kk][nn] = (gn < N && gk2 < K) ? ld_any(B, bdt, bo + (long)gk2 * ldb + gn) : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) {
            float a[4], bb[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                a[i] = As[k][ty + 16 * i];
                bb[i] = Bs[k][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + ty + 16 * i;
        if (m >= M)
            continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tx + 16 * j;
            if (n >= N)
                continue;
            float v = alpha * acc[i][j];
            if (bias)
                v += bias[n];
            v = act_fn(v, act);
            if (R)
                v += R[ro + (long)m * ldc + n];
            C[co + (long)m * ldc + n] = v;
        }
    }
}

}  // namespace
}  // namespace sam3

using namespace sam3;
#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

extern "C" int k_attn_f32(const float *qkv, int nseq, int N, int E, int heads, int hd,
                          float scale, float *out, k_stream s)
{
    if (hd != F_HD || E != heads * hd || nseq <= 0 || N <= 0 || ((uintptr_t)qkv & 15) ||
        ((uintptr_t)out & 15))
        return K_EARG;
    const long grid = (long)nseq * heads * ((N + F_BQ - 1) / F_BQ);
    attn_f32_kernel<<<(int)grid, F_BQ, 0, STREAM(s)>>>(qkv, nseq, N, E, heads, scale, out);
    return (int)cudaGetLastError();
}

extern "C" int k_gemm_simt(int M, int N, int K, const void *A, int adt, long aoff, int lda,
                           long sa0, long sa1, const void *B, int bdt, long boff, int ldb,
                           long sb0, long sb1, int transb, float *C, long coff, int ldc, long sc0,
                           long sc1, int nb, int nb1, const float *bias, const float *R, long roff,
                           float alpha, int act, k_stream s)
{
    if (M <= 0 || N <= 0 || K <= 0 || nb <= 0 || nb1 <= 0 || nb > 65535)
        return K_EARG;
    dim3 grid((N + 63) / 64, (M + 63) / 64, nb);
    gemm_simt_kernel<<<grid, 256, 0, STREAM(s)>>>(M, N, K, A, adt, aoff, lda, sa0, sa1, B, bdt,
                                                  boff, ldb, sb0, sb1, transb, C, coff, ldc, sc0,
                                                  sc1, nb1, bias, R, roff, alpha, act);
    return (int)cudaGetLastError();
}
