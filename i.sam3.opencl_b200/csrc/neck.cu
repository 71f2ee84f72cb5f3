// SPDX-License-Identifier: Unlicense
// Weight layout of the SimpleFPN neck's 3x3 convolutions (sam3_model.c
// conv3x3 :1032-1054): the permutation to the K order of the implicit-GEMM
// convolution. All of the neck's arithmetic runs on the tcgen05 GEMM
// (gemm_tc.cu: ConvTranspose with its scatter in the epilogue, 1x1, and the
// implicit 3x3).
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

}  // namespace
}  // namespace sam3

using namespace sam3;

#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

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
