// SPDX-License-Identifier: Unlicense
// The detector's attention (sam3_text.c attend :305-343: Q.K^T / sqrt(hd),
// softmax_ext with an optional causal mask or box relative position bias
// (sam3_kernels.cl:889-921), P.V), in two forms:
//   - large self-attention without mask or bias (the fusion encoder's 6
//     layers over the 5184 image tokens, 8 heads of 32): the q/k/v rows are
//     packed to bf16 with each head zero-padded to 64 columns and run through
//     the tcgen05 flash kernel (attn_tc.cu), then the 32 real columns of each
//     head are written back in fp32. The padding doubles the tensor-core
//     work of a kernel whose softmax, not its tensor core, is the bound;
//   - cross-attention over the image (at least 1024 keys, no causal mask:
//     the decoder's 201 queries with or without the box bias): q, k and v
//     padded the same way and run through the cross form of the tcgen05
//     kernel, the box bias expanded by rpb_bias_kernel into a dense fp32
//     term that the kernel adds to the scaled scores, keys split over CTAs
//     when the queries alone do not fill the GPU;
//   - everything else (the prompt cross-attention, the causal text
//     encoder, the fp32 mode): an fp32 flash kernel on the CUDA cores with
//     the keys split over CTAs (online softmax per split, merged by a
//     combine kernel).
#include "kernels.h"
#include "pdl.cuh"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace sam3 {
namespace {

inline int grid_for(long n, int block)
{
    long g = (n + block - 1) / block;
    return (int)(g < 1 ? 1 : (g > 0x7fffffffL ? 0x7fffffffL : g));
}

// q, k, v fp32 [N, ld*] (head h at column h * hd) -> bf16 [N, 3 * heads * 64]
// (q | k | v blocks, head h at column h * 64), columns hd..63 of each head
// zero. A CTA per kPackRows rows, a thread per 4 output columns.
constexpr int kPackRows = 4;
__global__ void __launch_bounds__(128) pack_qkv_kernel(const float *__restrict__ q, int ldq,
                                                       const float *__restrict__ k, int ldk,
                                                       const float *__restrict__ v, int ldv,
                                                       long N, int heads, int hd,
                                                       uint2 *__restrict__ out)
{
    const int e4 = heads * 16;  // 4-column groups per block of q, k or v
    for (int r = 0; r < kPackRows; r++) {
        const long n = (long)blockIdx.x * kPackRows + r;
        if (n >= N)
            return;
#pragma unroll
        for (int blk = 0; blk < 3; blk++) {
            const float *src = blk == 0 ? q + n * ldq : (blk == 1 ? k + n * ldk : v + n * ldv);
            uint2 *dst = out + (n * 3 + blk) * e4;
            for (int c4 = threadIdx.x; c4 < e4; c4 += blockDim.x) {
                const int h = c4 >> 4, d = (c4 & 15) * 4;
                float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (d < hd)
                    x = __ldg(reinterpret_cast<const float4 *>(src + h * hd + d));
                __nv_bfloat162 lo = __floats2bfloat162_rn(x.x, x.y), hi = __floats2bfloat162_rn(x.z, x.w);
                dst[c4] = make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
            }
        }
    }
}

// fp32 [N, heads * 64] -> O [N, ldo]: the first hd columns of each head.
__global__ void __launch_bounds__(256) unpack_heads_kernel(const float *__restrict__ in, long N,
                                                           int heads, int hd,
                                                           float *__restrict__ O, int ldo)
{
    const int per = heads * hd / 4;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < N * per;
         i += (long)gridDim.x * blockDim.x) {
        const long n = i / per;
        const int c = (int)(i % per) * 4, h = c / hd, d = c % hd;
        *reinterpret_cast<float4 *>(O + n * ldo + c) =
            *reinterpret_cast<const float4 *>(in + (n * heads + h) * 64 + d);
    }
}

// One operand of a cross-attention, fp32 or bf16 [rows, ld] (head h at
// column h * hd) -> bf16 [rows, heads * 64] with columns hd..63 of each
// head zero (the tcgen05 attention's layout). A CTA per kPackRows rows, a
// thread per 4 output columns.
template <bool SRC_BF16>
__global__ void __launch_bounds__(128) pad_heads_kernel(const void *__restrict__ src, long ld,
                                                        long rows, int heads, int hd,
                                                        uint2 *__restrict__ out)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    const int e4 = heads * 16;
    for (int r = 0; r < kPackRows; r++) {
        const long n = (long)blockIdx.x * kPackRows + r;
        if (n >= rows)
            return;
        for (int c4 = threadIdx.x; c4 < e4; c4 += blockDim.x) {
            const int h = c4 >> 4, d = (c4 & 15) * 4;
            uint2 w = make_uint2(0u, 0u);
            if (d < hd) {
                if (SRC_BF16)
                    w = __ldg(reinterpret_cast<const uint2 *>(
                        reinterpret_cast<const __nv_bfloat16 *>(src) + n * ld + h * hd + d));
                else {
                    const float4 x = __ldg(reinterpret_cast<const float4 *>(
                        reinterpret_cast<const float *>(src) + n * ld + h * hd + d));
                    __nv_bfloat162 lo = __floats2bfloat162_rn(x.x, x.y),
                                   hi = __floats2bfloat162_rn(x.z, x.w);
                    w = make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
                }
            }
            out[n * e4 + c4] = w;
        }
    }
}

// SAM 3's box relative position bias of softmax_ext (sam3_kernels.cl:
// 890-921) as a dense [heads, Nq, Nk] term for the tensor-core attention, in
// log2 units: bias[(h Nq + i) Nk + j] = (dy[(i H + y) nh + h] + dx[(i W +
// x) nh + h]) log2 e for key j = y W + x. One CTA per (head, query) row:
// the row's H + W terms (strided by nh in dy / dx) are gathered into
// shared memory once, then the Nk outputs are written 4 at a time (W a
// multiple of 4 keeps the 4 keys of a store in one y) - a write-bound pass.
__global__ void __launch_bounds__(256) rpb_bias_kernel(const float *__restrict__ dy,
                                                       const float *__restrict__ dx, int Nq,
                                                       int Nk, int W, int heads,
                                                       float *__restrict__ bias)
{
    extern __shared__ float rpb_s[];  // [H] dy terms, then [W] dx terms
    const int H = Nk / W;
    const int h = blockIdx.x / Nq, i = blockIdx.x - h * Nq;
    float *dys = rpb_s, *dxs = rpb_s + H;
    for (int t = threadIdx.x; t < H + W; t += blockDim.x)
        rpb_s[t] = t < H ? __ldg(dy + ((long)i * H + t) * heads + h) * 1.4426950408889634f
                         : __ldg(dx + ((long)i * W + (t - H)) * heads + h) * 1.4426950408889634f;
    __syncthreads();
    float *row = bias + (long)blockIdx.x * Nk;
    if (!(W & 3) && !(reinterpret_cast<uintptr_t>(row) & 15)) {
        float4 *row4 = reinterpret_cast<float4 *>(row);
        for (int j4 = threadIdx.x; j4 < Nk / 4; j4 += blockDim.x) {
            const int y = (4 * j4) / W, x = 4 * j4 - y * W;
            const float b = dys[y];
            row4[j4] = make_float4(b + dxs[x], b + dxs[x + 1], b + dxs[x + 2], b + dxs[x + 3]);
        }
    }
    else {
        for (int j = threadIdx.x; j < Nk; j += blockDim.x) {
            const int y = j / W;
            row[j] = dys[y] + dxs[j - y * W];
        }
    }
}

constexpr int kQB = 32;    // queries per CTA
constexpr int kLanes = 8;  // key lanes per query
constexpr int kKC = 32;    // keys per shared-memory chunk

// fp32 flash attention of one head over one key range [k0, k1): CTA =
// (query block, head, split), 256 threads = 32 queries x 8 key lanes (the 8
// lanes of a query are adjacent threads of one warp); each 32-key chunk of
// K and V is staged in shared memory and a lane takes every 8th key.
// Scores: (q . k) / sqrt(hd), then -inf past the query (causal) or
// + dy[(i * H + y) * nh + h] + dx[(i * W + x) * nh + h] for key j = y * W +
// x (box relative position bias). Online softmax per lane, the 8 lanes
// merged with warp shuffles, the split's (max, sum, unnormalised output)
// written for the combine kernel.
template <int HD>
__global__ void __launch_bounds__(256) attend_split_kernel(
    const float *__restrict__ Q, int ldq, const float *__restrict__ K, int ldk,
    const float *__restrict__ V, int ldv, int Nq, int Nk, int heads, int causal,
    const float *__restrict__ dy, const float *__restrict__ dx, int W, int nsplit, float scale,
    float *__restrict__ part)
{
    __shared__ float ks[kKC][HD + 1], vs[kKC][HD + 1];
    const int qb = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
    const int ql = threadIdx.x / kLanes, lane = threadIdx.x % kLanes;
    const int i = qb * kQB + ql;
    const bool live = i < Nq;
    const int per = (Nk + nsplit - 1) / nsplit;
    const int k0 = split * per, k1 = min(Nk, k0 + per);
    const int H = W > 0 ? Nk / W : 0;
    float q[HD], acc[HD];
#pragma unroll
    for (int d = 0; d < HD; d++) {
        q[d] = live ? Q[(long)i * ldq + h * HD + d] : 0.0f;
        acc[d] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    for (int c0 = k0; c0 < k1; c0 += kKC) {
        __syncthreads();
        for (int e = threadIdx.x; e < kKC * HD; e += blockDim.x) {
            const int r = e / HD, d = e % HD, j = c0 + r;
            ks[r][d] = j < k1 ? K[(long)j * ldk + h * HD + d] : 0.0f;
            vs[r][d] = j < k1 ? V[(long)j * ldv + h * HD + d] : 0.0f;
        }
        __syncthreads();
        if (!live)
            continue;
        for (int r = lane; r < kKC; r += kLanes) {
            const int j = c0 + r;
            if (j >= k1)
                break;
            float s = 0.0f;
#pragma unroll
            for (int d = 0; d < HD; d++)
                s = fmaf(q[d], ks[r][d], s);
            s *= scale;
            if (causal && j > i)
                continue;
            if (dy)
                s += __ldg(dy + ((long)i * H + j / W) * heads + h) +
                     __ldg(dx + ((long)i * W + j % W) * heads + h);
            const float mn = fmaxf(m, s);
            const float corr = expf(m - mn), p = expf(s - mn);
            l = l * corr + p;
#pragma unroll
            for (int d = 0; d < HD; d++)
                acc[d] = fmaf(p, vs[r][d], acc[d] * corr);
            m = mn;
        }
    }
    // merge the 8 lanes of each query (adjacent threads of one warp)
#pragma unroll
    for (int off = 1; off < kLanes; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
        const float mm = fmaxf(m, m2);
        const float w1 = m == -INFINITY ? 0.0f : expf(m - mm);
        const float w2 = m2 == -INFINITY ? 0.0f : expf(m2 - mm);
        l = l * w1 + l2 * w2;
#pragma unroll
        for (int d = 0; d < HD; d++)
            acc[d] = acc[d] * w1 + __shfl_xor_sync(0xffffffffu, acc[d], off) * w2;
        m = mm;
    }
    if (lane == 0 && live) {
        float *pp = part + (((long)split * Nq + i) * heads + h) * (HD + 2);
        pp[0] = m;
        pp[1] = l;
#pragma unroll
        for (int d = 0; d < HD; d++)
            pp[2 + d] = acc[d];
    }
}

// Combine the splits of each (query, head): O = sum_s o_s e^(m_s - m) /
// sum_s l_s e^(m_s - m).
__global__ void __launch_bounds__(256) attend_combine_kernel(const float *__restrict__ part,
                                                             int Nq, int heads, int hd,
                                                             int nsplit, float *__restrict__ O,
                                                             int ldo)
{
    for (long t = (long)blockIdx.x * blockDim.x + threadIdx.x; t < (long)Nq * heads * hd;
         t += (long)gridDim.x * blockDim.x) {
        const int d = (int)(t % hd);
        const long qh = t / hd;  // i * heads + h
        float mm = -INFINITY;
        for (int s = 0; s < nsplit; s++)
            mm = fmaxf(mm, part[((long)s * Nq * heads + qh) * (hd + 2)]);
        float ll = 0.0f, o = 0.0f;
        for (int s = 0; s < nsplit; s++) {
            const float *pp = part + ((long)s * Nq * heads + qh) * (hd + 2);
            const float w = pp[0] == -INFINITY ? 0.0f : expf(pp[0] - mm);
            ll += pp[1] * w;
            o += pp[2 + d] * w;
        }
        const long i = qh / heads;
        const int h = (int)(qh % heads);
        O[i * ldo + h * hd + d] = o / ll;
    }
}

}  // namespace
}  // namespace sam3

using namespace sam3;

#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

extern "C" int k_pack_qkv_pad64(const float *q, int ldq, const float *k, int ldk, const float *v,
                                int ldv, long N, int heads, int hd, void *out, k_stream s)
{
    if (N <= 0 || heads <= 0 || hd <= 0 || hd > 64 || (hd & 3) || (ldq & 3) || (ldk & 3) ||
        (ldv & 3) || (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(k) & 15) ||
        (reinterpret_cast<uintptr_t>(v) & 15) || (reinterpret_cast<uintptr_t>(out) & 7))
        return K_EARG;
    pack_qkv_kernel<<<grid_for(N, kPackRows), 128, 0, STREAM(s)>>>(
        q, ldq, k, ldk, v, ldv, N, heads, hd, reinterpret_cast<uint2 *>(out));
    return (int)cudaGetLastError();
}

extern "C" int k_unpack_heads64(const float *in, long N, int heads, int hd, float *O, int ldo,
                                k_stream s)
{
    if (N <= 0 || heads <= 0 || hd <= 0 || hd > 64 || (hd & 3) || (ldo & 3) ||
        (reinterpret_cast<uintptr_t>(O) & 15) || (reinterpret_cast<uintptr_t>(in) & 15))
        return K_EARG;
    const int grid = grid_for(N * heads * hd / 4, 256);
    unpack_heads_kernel<<<grid < 148 * 16 ? grid : 148 * 16, 256, 0, STREAM(s)>>>(in, N, heads, hd,
                                                                                  O, ldo);
    return (int)cudaGetLastError();
}

extern "C" int k_pad_heads64(const void *src, int src_bf16, long ld, long rows, int heads, int hd,
                             void *out, k_stream s)
{
    if (rows <= 0 || heads <= 0 || hd <= 0 || hd > 64 || (hd & 3) || (ld & 3) ||
        (reinterpret_cast<uintptr_t>(src) & (src_bf16 ? 7 : 15)) ||
        (reinterpret_cast<uintptr_t>(out) & 7))
        return K_EARG;
    const int g = grid_for(rows, kPackRows);
    if (src_bf16)
        return launch_pdl(pad_heads_kernel<true>, dim3(g), dim3(128), 0, STREAM(s), src, ld, rows,
                          heads, hd, reinterpret_cast<uint2 *>(out));
    return launch_pdl(pad_heads_kernel<false>, dim3(g), dim3(128), 0, STREAM(s), src, ld, rows,
                      heads, hd, reinterpret_cast<uint2 *>(out));
}

extern "C" int k_rpb_bias(const float *dy, const float *dx, int Nq, int Nk, int W, int heads,
                          float *bias, k_stream s)
{
    if (Nq <= 0 || Nk <= 0 || W <= 0 || Nk % W || heads <= 0)
        return K_EARG;
    const long rows = (long)heads * Nq;
    const size_t smem = (size_t)(Nk / W + W) * sizeof(float);
    if (rows > 0x7fffffffL || smem > 48 * 1024)
        return K_EARG;
    rpb_bias_kernel<<<(int)rows, 256, smem, STREAM(s)>>>(dy, dx, Nq, Nk, W, heads, bias);
    return (int)cudaGetLastError();
}

extern "C" int k_attend_splits(int Nq, int Nk, int heads, int num_sms)
{
    const long blocks = (long)((Nq + kQB - 1) / kQB) * heads;
    long ns = (2L * num_sms + blocks - 1) / blocks;
    const long max_ns = (Nk + 255) / 256;  // at least 256 keys per split
    if (ns > max_ns)
        ns = max_ns;
    return (int)(ns < 1 ? 1 : ns);
}

extern "C" size_t k_attend_workspace(int Nq, int Nk, int heads, int hd, int num_sms)
{
    return (size_t)k_attend_splits(Nq, Nk, heads, num_sms) * Nq * heads * (hd + 2) * sizeof(float);
}

extern "C" int k_attend_simt(int Nq, int Nk, int heads, int hd, const float *Q, int ldq,
                             const float *K, int ldk, const float *V, int ldv, float *O, int ldo,
                             int causal, const float *dy, const float *dx, int W, void *ws,
                             size_t ws_bytes, int num_sms, k_stream s)
{
    if (Nq <= 0 || Nk <= 0 || heads <= 0 || heads > 65535 || (hd != 32 && hd != 64) ||
        ((dy != nullptr) != (dx != nullptr)) || (dy && (W <= 0 || Nk % W)) ||
        ws_bytes < k_attend_workspace(Nq, Nk, heads, hd, num_sms))
        return K_EARG;
    const int ns = k_attend_splits(Nq, Nk, heads, num_sms);
    const dim3 grid((Nq + kQB - 1) / kQB, heads, ns);
    const float scale = 1.0f / sqrtf((float)hd);
    float *part = reinterpret_cast<float *>(ws);
    if (hd == 32)
        attend_split_kernel<32><<<grid, 256, 0, STREAM(s)>>>(Q, ldq, K, ldk, V, ldv, Nq, Nk, heads,
                                                            causal, dy, dx, W, ns, scale, part);
    else
        attend_split_kernel<64><<<grid, 256, 0, STREAM(s)>>>(Q, ldq, K, ldk, V, ldv, Nq, Nk, heads,
                                                            causal, dy, dx, W, ns, scale, part);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return (int)e;
    const int g = grid_for((long)Nq * heads * hd, 256);
    attend_combine_kernel<<<g < 148 * 16 ? g : 148 * 16, 256, 0, STREAM(s)>>>(part, Nq, heads, hd,
                                                                             ns, O, ldo);
    return (int)cudaGetLastError();
}
