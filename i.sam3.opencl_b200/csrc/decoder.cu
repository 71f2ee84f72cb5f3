// SPDX-License-Identifier: Unlicense
// Kernels of the point-prompt mask decoder around its attention
// (sam3_model.c sam_decode :1239-1399): the ConvTranspose scatter of the
// output upscaling, the mask logits, the hypernetwork / IoU heads that the
// reference runs on the host, the fused LayerNorm / upscaling passes of the
// decoder's image stream, and the weight layout change of the ConvTranspose
// GEMM operands.
#include "kernels.h"
#include "tc_ptx.cuh"

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
// over the inputs, double accumulation as host_linear; 32 warps, four rows
// each per pass, so a 256-row layer is two passes (each pass waits for its
// weight rows from L2: few passes, short latency chain). Outputs: hyper
// [P, 96] (m * 32 + o), iou [P, 3] = sigmoid(out[1..3]) of the IoU head.
constexpr int kHeadWarps = 32;

__global__ void __launch_bounds__(32 * kHeadWarps) dec_heads_kernel(const float *__restrict__ tok,
                                                        const k_dec_heads_w a,
                                                        float *__restrict__ hyper,
                                                        float *__restrict__ iou)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    __shared__ float xs[256], hs[256];
    const int p = blockIdx.x, m = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = m < 3 ? 3 + m : 1;
    const float *t = tok + ((long)p * 8 + row) * 256;
    if (threadIdx.x < 256)
        xs[threadIdx.x] = t[threadIdx.x];
    __syncthreads();
    const int nout = m < 3 ? 32 : 4;
    for (int l = 0; l < 3; l++) {
        const float *W = a.w[m][l], *B = a.b[m][l];
        const int no = l < 2 ? 256 : nout;
        const float *in = (l & 1) ? hs : xs;
        float *o = (l & 1) ? xs : hs;
        // Four rows per pass (r0 + W i, W = kHeadWarps): four independent
        // accumulation and reduction chains per warp; each row's sum is
        // formed in the same order as with one row at a time.
        for (int r0 = warp; r0 < no; r0 += 4 * kHeadWarps) {
            double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const double xv = (double)in[lane + 32 * k];
#pragma unroll
                for (int i = 0; i < 4; i++)
                    if (r0 + kHeadWarps * i < no)
                        acc[i] += (double)__ldg(W + (long)(r0 + kHeadWarps * i) * 256 + lane +
                                                32 * k) *
                                  xv;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int i = 0; i < 4; i++)
                    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], off);
            if (lane == 0) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int r = r0 + kHeadWarps * i;
                    if (r < no) {
                        const double v = acc[i] + (double)__ldg(B + r);
                        o[r] = (l < 2 && v < 0.0) ? 0.0f : (float)v;
                    }
                }
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

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// LayerNorm of the decoder's image stream (256 channels, norm4 of the
// image -> token attention, sam3_model.c:1309/1348) with the outputs its
// consumers need written in the same pass. R (optional) is the residual
// shared by every prompt, row % T, added to X before the statistics (layer
// 0's input: the image embedding), so the output projection before this
// kernel stores plainly. Y (fp32, may alias X), Yb = bf16(Y) (operand of
// the value projection and of the first upscaling GEMM) and Yk = bf16(Y +
// pe[row % T]) (keys + dense positional encoding, operand of the key /
// query projections); each NULL = not written. The token stream's norms
// use it too (T = rows, pe = the tokens' positional encoding). One warp
// per row, 8 values per lane; two-pass mean / variance as the reference.
__global__ void __launch_bounds__(256) ln_keys_kernel(const float *X,
                                                      const float *__restrict__ R, float *Y,
                                                      const float *__restrict__ g,
                                                      const float *__restrict__ b, long rows,
                                                      float eps, const float *__restrict__ pe,
                                                      int T, uint2 *__restrict__ Yb,
                                                      uint2 *__restrict__ Yk)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    const float4 *x = reinterpret_cast<const float4 *>(X + row * 256);
    float4 v[2] = {x[lane], x[32 + lane]};
    if (R) {  // the residual shared by all prompts, added as the GEMM epilogue would
        const float4 *rr = reinterpret_cast<const float4 *>(R + (row % T) * 256);
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const float4 a = __ldg(rr + i * 32 + lane);
            v[i].x += a.x;
            v[i].y += a.y;
            v[i].z += a.z;
            v[i].w += a.w;
        }
    }
    const float mean =
        warp_sum((v[0].x + v[0].y) + (v[0].z + v[0].w) + (v[1].x + v[1].y) + (v[1].z + v[1].w)) /
        256.0f;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float a = v[i].x - mean, c = v[i].y - mean, d = v[i].z - mean, e = v[i].w - mean;
        q += (a * a + c * c) + (d * d + e * e);
    }
    const float inv = rsqrtf(warp_sum(q) / 256.0f + eps);
    const float4 *pr = reinterpret_cast<const float4 *>(pe + (row % T) * 256);
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int c4 = i * 32 + lane;
        const float4 gg = __ldg(reinterpret_cast<const float4 *>(g) + c4);
        const float4 bt = __ldg(reinterpret_cast<const float4 *>(b) + c4);
        float4 y;
        y.x = (v[i].x - mean) * inv * gg.x + bt.x;
        y.y = (v[i].y - mean) * inv * gg.y + bt.y;
        y.z = (v[i].z - mean) * inv * gg.z + bt.z;
        y.w = (v[i].w - mean) * inv * gg.w + bt.w;
        if (Y)
            reinterpret_cast<float4 *>(Y + row * 256)[c4] = y;
        if (Yb)
            Yb[row * 64 + c4] = make_uint2(pack2(y.x, y.y), pack2(y.z, y.w));
        if (Yk) {
            const float4 p4 = __ldg(pr + c4);
            Yk[row * 64 + c4] =
                make_uint2(pack2(y.x + p4.x, y.y + p4.y), pack2(y.z + p4.z, y.w + p4.w));
        }
    }
}

// src [rows, cols] fp32 -> dst [cols, rows] bf16 (round to nearest even),
// through 32 x 32 shared-memory tiles. With dmajor, source column
// c = co * 4 + d becomes destination row d * (cols / 4) + co.
__global__ void transpose_cast_kernel(const float *__restrict__ src, int rows, int cols,
                                      int dmajor, __nv_bfloat16 *__restrict__ dst)
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
        const int oc = dmajor ? (c & 3) * (cols >> 2) + (c >> 2) : c;
        if (r < rows && c < cols)
            dst[(long)oc * rows + r] = __float2bfloat16_rn(tile[threadIdx.x][j]);
    }
}

// The upscaling epilogues' per-pixel residual in the layout they read:
// feat [(2H) * (2W), C] (NHWC of one image) -> out [4][C][H * W] with
// out[(d * C + c) * H * W + y * W + x] = feat[(2y + d / 2, 2x + d % 2)][c],
// i.e. for ConvTranspose input pixel (y, x), sub-pixel d, channel c. An
// epilogue thread owns one input pixel (GEMM row), so the 32 threads of a
// warp read one channel of 32 consecutive pixels as one 128-byte line
// instead of 32 lines. Through 32 x 32 shared-memory tiles, both sides
// coalesced.
__global__ void feat_subpix_kernel(const float *__restrict__ feat, int H, int W, int C,
                                   float *__restrict__ out)
{
    __shared__ float tile[32][33];
    const int HW = H * W, d = blockIdx.z;
    const int i0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int i = i0 + j;
        if (i < HW) {
            const int y = i / W, x = i - y * W;
            const long pix = (long)(2 * y + (d >> 1)) * (2 * W) + 2 * x + (d & 1);
            tile[j][threadIdx.x] = feat[pix * C + c0 + threadIdx.x];
        }
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int i = i0 + threadIdx.x;
        if (i < HW)
            out[(long)(d * C + c0 + j) * HW + i] = tile[threadIdx.x][j];
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
    return launch_pdl(dec_heads_kernel, dim3(P, 4), dim3(32 * kHeadWarps), 0, STREAM(s), tok, *hw,
                      hyper, iou);
}

extern "C" int k_transpose_cast_bf16(const float *src, int rows, int cols, int dmajor, void *dst,
                                     k_stream s)
{
    if (rows <= 0 || cols <= 0 || (dmajor && (cols & 3)))
        return K_EARG;
    transpose_cast_kernel<<<dim3((cols + 31) / 32, (rows + 31) / 32), dim3(32, 8), 0, STREAM(s)>>>(
        src, rows, cols, dmajor, reinterpret_cast<__nv_bfloat16 *>(dst));
    return (int)cudaGetLastError();
}

extern "C" int k_dec_feat_subpix(const float *feat, int H, int W, int C, float *out, k_stream s)
{
    if (!feat || !out || H <= 0 || W <= 0 || C <= 0 || C % 32 || (long)H * W > 0x7fffffffL / C)
        return K_EARG;
    feat_subpix_kernel<<<dim3((H * W + 31) / 32, C / 32, 4), dim3(32, 8), 0, STREAM(s)>>>(
        feat, H, W, C, out);
    return (int)cudaGetLastError();
}

extern "C" int k_dec_ln_keys(const float *X, const float *R, float *Y, const float *g,
                             const float *b, long rows, float eps, const float *pe, int T, void *Yb,
                             void *Yk, k_stream s)
{
    if (rows <= 0 || T <= 0 || (!Y && !Yb && !Yk) || (Yk && !pe) ||
        (reinterpret_cast<uintptr_t>(X) & 15) ||
        (reinterpret_cast<uintptr_t>(R) & 15) ||
        (reinterpret_cast<uintptr_t>(Y) & 15) || (reinterpret_cast<uintptr_t>(pe) & 15) ||
        (reinterpret_cast<uintptr_t>(Yb) & 7) || (reinterpret_cast<uintptr_t>(Yk) & 7))
        return K_EARG;
    return launch_pdl(ln_keys_kernel, dim3(grid_for(rows, 8)), dim3(256), 0, STREAM(s), X, R, Y, g,
                      b, rows, eps, pe, T, reinterpret_cast<uint2 *>(Yb),
                      reinterpret_cast<uint2 *>(Yk));
}

