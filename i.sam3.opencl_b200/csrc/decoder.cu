// SPDX-License-Identifier: Unlicense
// Kernels of the point-prompt mask decoder around its attention
// (sam3_model.c sam_decode :1239-1399): the ConvTranspose scatter of the
// output upscaling, the mask logits, the hypernetwork / IoU heads that the
// reference runs on the host, the positional-encoding add fused with the
// cast of a GEMM operand, and the weight layout change of the ConvTranspose
// GEMM operands.
#include "kernels.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace sam3 {
namespace {

inline int grid_for(long n, int block)
{
    long g = (n + block - 1) / block;
    return (int)(g < 1 ? 1 : (g > 0x7fffffffL ? 0x7fffffffL : g));
}

__device__ __forceinline__ float act_fn(float v, int act)
{
    if (act == K_ACT_GELU)
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    if (act == K_ACT_RELU)
        return fmaxf(v, 0.0f);
    return v;
}

// convt_scatter (sam3_kernels.cl:762-781). One thread per GEMM element
// group (p, y, x, co): the four sub-pixel values G[row, co*4 .. co*4+3] in
// one 16-byte load, each written to its output pixel (2y+dy, 2x+dx). co is
// the fastest index, so loads and each of the four stores are coalesced.
// Per value: (G + bias) + add, then the activation, as the reference.
__global__ void __launch_bounds__(256) convt_scatter_kernel(const float4 *__restrict__ G,
                                                            float *__restrict__ out,
                                                            const float *__restrict__ bias,
                                                            const float *__restrict__ add, int H,
                                                            int W, int Co, long total, int act)
{
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x) {
        const int co = (int)(i % Co);
        const long pix = i / Co;  // (p * H + y) * W + x
        const int x = (int)(pix % W);
        const long py = pix / W;
        const int y = (int)(py % H);
        const long p = py / H;
        const float4 g = G[i];
        const float bc = __ldg(bias + co);
        const float gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
        for (int d = 0; d < 4; d++) {
            const int oy = 2 * y + (d >> 1), ox = 2 * x + (d & 1);
            const long o_img = ((long)oy * 2 * W + ox) * Co + co;  // index within one prompt
            float v = gv[d] + bc;
            if (add)
                v += __ldg(add + o_img);
            out[p * 4L * H * W * Co + o_img] = act_fn(v, act);
        }
    }
}

// mask_logits (sam3_kernels.cl:787-807): one thread per (prompt, pixel),
// the pixel's 32 channels as eight 16-byte loads (consecutive threads read
// consecutive 128-byte rows), three dot products with the prompt's
// hypernetwork outputs, three coalesced stores.
__global__ void __launch_bounds__(256) mask_logits_kernel(const float4 *__restrict__ U,
                                                          const float *__restrict__ hyper,
                                                          float *__restrict__ out, int npix,
                                                          long total)
{
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x) {
        const long p = i / npix;
        const int pix = (int)(i % npix);
        const float4 *h = reinterpret_cast<const float4 *>(hyper + p * 96);
        float acc[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 u = U[i * 8 + j];
#pragma unroll
            for (int m = 0; m < 3; m++) {
                const float4 w = __ldg(h + m * 8 + j);
                acc[m] += (u.x * w.x + u.y * w.y) + (u.z * w.z + u.w * w.w);
            }
        }
#pragma unroll
        for (int m = 0; m < 3; m++)
            out[(p * 3 + m) * (long)npix + pix] = acc[m];
    }
}

// Hypernetwork MLPs 1-3 and the IoU head (host_mlp3 / host_linear,
// sam3_model.c:1188-1210, 1370-1385): block (p, m) runs MLP m on its token
// (mask token m for m < 3 -> rows 3..5, the IoU token row 1 for m = 3):
// 256 -> 256 (ReLU) -> 256 (ReLU) -> nout. A warp per output row, lanes
// over the inputs, double accumulation as host_linear. Outputs: hyper
// [P, 96] (m * 32 + o), iou [P, 3] = sigmoid(out[1..3]) of the IoU head.
__global__ void __launch_bounds__(256) dec_heads_kernel(const float *__restrict__ tok,
                                                        const k_dec_heads_w a,
                                                        float *__restrict__ hyper,
                                                        float *__restrict__ iou)
{
    __shared__ float xs[256], hs[256];
    const int p = blockIdx.x, m = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = m < 3 ? 3 + m : 1;
    const float *t = tok + ((long)p * 8 + row) * 256;
    xs[threadIdx.x] = t[threadIdx.x];
    __syncthreads();
    const int nout = m < 3 ? 32 : 4;
    for (int l = 0; l < 3; l++) {
        const float *W = a.w[m][l], *B = a.b[m][l];
        const int no = l < 2 ? 256 : nout;
        const float *in = (l & 1) ? hs : xs;
        float *o = (l & 1) ? xs : hs;
        for (int r = warp; r < no; r += 8) {
            const float *wr = W + (long)r * 256;
            double acc = 0.0;
#pragma unroll
            for (int k = 0; k < 8; k++)
                acc += (double)__ldg(wr + lane + 32 * k) * (double)in[lane + 32 * k];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
                acc += __shfl_xor_sync(0xffffffffu, acc, off);
            if (lane == 0) {
                acc += (double)__ldg(B + r);
                o[r] = (l < 2 && acc < 0.0) ? 0.0f : (float)acc;
            }
        }
        __syncthreads();
    }
    // layers write hs, xs, hs: the output is in hs
    if (m < 3) {
        if (threadIdx.x < 32)
            hyper[(long)p * 96 + m * 32 + threadIdx.x] = hs[threadIdx.x];
    }
    else if (threadIdx.x < 3)
        iou[p * 3 + threadIdx.x] = 1.0f / (1.0f + expf(-hs[1 + threadIdx.x]));
}

// out = bf16(x[i] + a[i % amod]): the positional-encoding add of a decoder
// Linear's input fused with its cast to the GEMM operand type; four values
// per thread (n and amod multiples of 4, 16-byte aligned inputs).
__global__ void __launch_bounds__(256) add_cast_kernel(const float4 *__restrict__ x,
                                                       const float4 *__restrict__ a, long n4,
                                                       long amod4, uint2 *__restrict__ out)
{
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (long)gridDim.x * blockDim.x) {
        const float4 v = x[i], w = __ldg(a + i % amod4);
        __nv_bfloat162 lo = __floats2bfloat162_rn(v.x + w.x, v.y + w.y);
        __nv_bfloat162 hi = __floats2bfloat162_rn(v.z + w.z, v.w + w.w);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t *>(&lo);
        o.y = *reinterpret_cast<uint32_t *>(&hi);
        out[i] = o;
    }
}

// src [rows, cols] fp32 -> dst [cols, rows] bf16 (round to nearest even),
// through 32 x 32 shared-memory tiles.
__global__ void transpose_cast_kernel(const float *__restrict__ src, int rows, int cols,
                                      __nv_bfloat16 *__restrict__ dst)
{
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int r = r0 + j, c = c0 + threadIdx.x;
        if (r < rows && c < cols)
            tile[j][threadIdx.x] = src[(long)r * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int c = c0 + j, r = r0 + threadIdx.x;
        if (r < rows && c < cols)
            dst[(long)c * rows + r] = __float2bfloat16_rn(tile[threadIdx.x][j]);
    }
}

}  // namespace
}  // namespace sam3

using namespace sam3;

#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

extern "C" int k_convt_scatter(const float *G, float *out, const float *bias, const float *add,
                               int P, int H, int W, int Co, int act, k_stream s)
{
    if (P <= 0 || H <= 0 || W <= 0 || Co <= 0 || (reinterpret_cast<uintptr_t>(G) & 15))
        return K_EARG;
    const long total = (long)P * H * W * Co;
    const int grid = grid_for(total, 256);
    convt_scatter_kernel<<<grid < 148 * 16 ? grid : 148 * 16, 256, 0, STREAM(s)>>>(
        reinterpret_cast<const float4 *>(G), out, bias, add, H, W, Co, total, act);
    return (int)cudaGetLastError();
}

extern "C" int k_mask_logits(const float *U, const float *hyper, float *out, int P, int npix,
                             k_stream s)
{
    if (P <= 0 || npix <= 0 || (reinterpret_cast<uintptr_t>(U) & 15) ||
        (reinterpret_cast<uintptr_t>(hyper) & 15))
        return K_EARG;
    const long total = (long)P * npix;
    const int grid = grid_for(total, 256);
    mask_logits_kernel<<<grid < 148 * 16 ? grid : 148 * 16, 256, 0, STREAM(s)>>>(
        reinterpret_cast<const float4 *>(U), hyper, out, npix, total);
    return (int)cudaGetLastError();
}

extern "C" int k_dec_heads(const float *tok, int P, const k_dec_heads_w *hw, float *hyper,
                           float *iou, k_stream s)
{
    if (P <= 0 || P > 65535 || !hw)
        return K_EARG;
    dec_heads_kernel<<<dim3(P, 4), 256, 0, STREAM(s)>>>(tok, *hw, hyper, iou);
    return (int)cudaGetLastError();
}

extern "C" int k_add_cast_bf16(const float *x, const float *a, long n, long amod, void *out,
                               k_stream s)
{
    if (n < 0 || amod <= 0 || (n & 3) || (amod & 3) || (reinterpret_cast<uintptr_t>(x) & 15) ||
        (reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(out) & 7))
        return K_EARG;
    if (n == 0)
        return 0;
    const int grid = grid_for(n / 4, 256);
    add_cast_kernel<<<grid < 148 * 16 ? grid : 148 * 16, 256, 0, STREAM(s)>>>(
        reinterpret_cast<const float4 *>(x), reinterpret_cast<const float4 *>(a), n / 4, amod / 4,
        reinterpret_cast<uint2 *>(out));
    return (int)cudaGetLastError();
}

extern "C" int k_transpose_cast_bf16(const float *src, int rows, int cols, void *dst, k_stream s)
{
    if (rows <= 0 || cols <= 0)
        return K_EARG;
    transpose_cast_kernel<<<dim3((cols + 31) / 32, (rows + 31) / 32), dim3(32, 8), 0, STREAM(s)>>>(
        src, rows, cols, reinterpret_cast<__nv_bfloat16 *>(dst));
    return (int)cudaGetLastError();
}
