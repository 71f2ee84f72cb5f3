// SPDX-License-Identifier: Unlicense
// Data-movement kernels of the SimpleFPN neck (sam3_model.c neck_level
// :1071-1095, conv3x3 :1032-1054, convt2x2 :1058-1065): the 2x2 / stride-2
// ConvTranspose scatter from its GEMM form and the 3x3 weight permutation.
// The matrix work itself, the 3x3 convolutions included, runs on the tcgen05
// GEMM (gemm_tc.cu). The scatter moves 16-byte chunks of channels: every
// load and store is coalesced.
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

__device__ __forceinline__ uint32_t pack2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// ConvTranspose scatter (convt_scatter, sam3_kernels.cl:762-781) from a
// GEMM output whose columns are sub-pixel-major (d * C + co, d = 2 dy + dx;
// the weight rows are stored in that order), so output pixel (2y+dy, 2x+dx)
// is one contiguous run of C values. One thread per 8 channels:
// act(G + bias) in fp32, stored bf16 (the operand of the next GEMM).
// G fp32 [n * H * W, 4C], out bf16 [n, 2H, 2W, C].
__global__ void __launch_bounds__(256) convt_scatter_bf16_kernel(const float4 *__restrict__ G,
                                                                 const float *__restrict__ bias,
                                                                 int H, int W, int C, int act,
                                                                 long total,
                                                                 uint4 *__restrict__ out)
{
    const int c8 = C >> 3;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x) {
        const int j = (int)(i % c8);
        const long q = i / c8;  // (input pixel, d)
        const int d = (int)(q & 3);
        const long ip = q >> 2;
        const int x = (int)(ip % W);
        const long py = ip / W;
        const int y = (int)(py % H);
        const long p = py / H;
        const float4 a = G[(ip * 4 + d) * (C >> 2) + 2 * j];
        const float4 b = G[(ip * 4 + d) * (C >> 2) + 2 * j + 1];
        const float4 ba = __ldg(reinterpret_cast<const float4 *>(bias) + 2 * j);
        const float4 bb = __ldg(reinterpret_cast<const float4 *>(bias) + 2 * j + 1);
        const long opix = (p * 2 * H + 2 * y + (d >> 1)) * 2L * W + 2 * x + (d & 1);
        out[opix * c8 + j] = make_uint4(
            pack2(act_fn(a.x + ba.x, act), act_fn(a.y + ba.y, act)),
            pack2(act_fn(a.z + ba.z, act), act_fn(a.w + ba.w, act)),
            pack2(act_fn(b.x + bb.x, act), act_fn(b.y + bb.y, act)),
            pack2(act_fn(b.z + bb.z, act), act_fn(b.w + bb.w, act)));
    }
}

}  // namespace
}  // namespace sam3

using namespace sam3;

#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

extern "C" int k_convt_scatter_bf16(const float *G, const float *bias, int n, int H, int W, int C,
                                    int act, void *out, k_stream s)
{
    if (n <= 0 || H <= 0 || W <= 0 || C <= 0 || (C & 7) || (reinterpret_cast<uintptr_t>(G) & 15) ||
        (reinterpret_cast<uintptr_t>(bias) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
        return K_EARG;
    const long total = (long)n * H * W * 4 * (C >> 3);
    const int grid = grid_for(total, 256);
    convt_scatter_bf16_kernel<<<grid < 148 * 16 ? grid : 148 * 16, 256, 0, STREAM(s)>>>(
        reinterpret_cast<const float4 *>(G), bias, H, W, C, act, total,
        reinterpret_cast<uint4 *>(out));
    return (int)cudaGetLastError();
}

// Conv2d weight [cout, cin, 3, 3] (fp32) -> bf16 [cout, 9 * cin] with
// columns tap-major ((ky * 3 + kx) * cin + c), the K order of the
// implicit-GEMM 3x3 convolution (k_conv3x3_bf16_tc).
__global__ void permute_conv3x3_kernel(const float *__restrict__ src, int cout, int cin,
                                       __nv_bfloat16 *__restrict__ dst)
{
    const long n = (long)cout * cin * 9;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const long o = i / (9L * cin);
        const int rem = (int)(i % (9L * cin));
        const int tap = rem / cin, c = rem % cin;
        dst[i] = __float2bfloat16_rn(src[o * 9L * cin + (long)c * 9 + tap]);
    }
}

extern "C" int k_permute_conv3x3_bf16(const float *src, int cout, int cin, void *dst, k_stream s)
{
    if (cout <= 0 || cin <= 0)
        return K_EARG;
    const int grid = grid_for((long)cout * cin * 9, 256);
    permute_conv3x3_kernel<<<grid < 148 * 8 ? grid : 148 * 8, 256, 0, STREAM(s)>>>(
        src, cout, cin, reinterpret_cast<__nv_bfloat16 *>(dst));
    return (int)cudaGetLastError();
}
