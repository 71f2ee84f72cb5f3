// SPDX-License-Identifier: Unlicense
// The encoder's input path on the device (image.c image_encoder_input
// :346-371): a crop of an interleaved 8-bit RGB image resized to the
// encoder's side with torchvision's uint8 antialiased bilinear (aa_resize,
// image.c:209-339: per output pixel a fixed-point triangle filter over a
// window of input pixels, the horizontal pass first, each pass rounded and
// clipped to 8 bits), and the reference's float normalisation. Integer
// arithmetic throughout the resize, so the result equals the reference's bit
// for bit. Windows and weights come from the host (one small table per
// axis); one thread per output pixel, the three channels together.
#include "kernels.h"

#include <cuda_runtime.h>

namespace sam3 {
namespace {

inline int grid_for(long n, int block)
{
    long g = (n + block - 1) / block;
    return (int)(g < 1 ? 1 : (g > 0x7fffffffL ? 0x7fffffffL : g));
}

__device__ __forceinline__ uint8_t clip8(long long v, int prec)
{
    v >>= prec;
    return v < 0 ? 0 : v > 255 ? 255 : (uint8_t)v;
}

// One axis of the resize: output position o < nout of each of `lines`
// lines; byte strides between lines and between pixels along the axis,
// separately for source and destination (the horizontal pass reads the
// crop with the image's row pitch; the vertical pass walks columns). With
// line_fastest, consecutive threads take consecutive lines (the vertical
// pass: consecutive x, so loads and stores stay contiguous).
__global__ void __launch_bounds__(256) resize_pass_kernel(
    const uint8_t *__restrict__ src, long s_line, long s_step, uint8_t *__restrict__ dst,
    long d_line, long d_step, int lines, int nout, int line_fastest,
    const int *__restrict__ bounds, const int *__restrict__ kk, int ksize, int prec)
{
    const long n = (long)lines * nout;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int o = line_fastest ? (int)(i / lines) : (int)(i % nout);
        const long line = line_fastest ? i % lines : i / nout;
        const int lo = __ldg(bounds + 2 * o), cnt = __ldg(bounds + 2 * o + 1);
        const int *k = kk + (long)o * ksize;
        long long a0 = 1LL << (prec - 1), a1 = a0, a2 = a0;
        const uint8_t *s = src + line * s_line + (long)lo * s_step;
        for (int t = 0; t < cnt; t++) {
            const long long w = __ldg(k + t);
            a0 += (long long)s[0] * w;
            a1 += (long long)s[1] * w;
            a2 += (long long)s[2] * w;
            s += s_step;
        }
        uint8_t *d = dst + line * d_line + (long)o * d_step;
        d[0] = clip8(a0, prec);
        d[1] = clip8(a1, prec);
        d[2] = clip8(a2, prec);
    }
}

// Crop copy without resampling (the reference skips the resize when the
// crop already has the encoder's size).
__global__ void crop_copy_kernel(const uint8_t *__restrict__ src, long pitch, int w, int h,
                                 uint8_t *__restrict__ dst)
{
    const long n = (long)w * h * 3;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const long y = i / ((long)w * 3), r = i % ((long)w * 3);
        dst[i] = src[y * pitch + r];
    }
}

// out[c][y][x] = (u / 255 - 0.5) / 0.5 (image.c:360-366), CHW fp32.
__global__ void normalize_chw_kernel(const uint8_t *__restrict__ tile, int side,
                                     float *__restrict__ out)
{
    const long n = (long)side * side;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
#pragma unroll
        for (int c = 0; c < 3; c++)
            out[c * n + i] = (tile[i * 3 + c] / 255.0f - 0.5f) / 0.5f;
    }
}

}  // namespace
}  // namespace sam3

using namespace sam3;

#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

extern "C" int k_resize_pass_u8(const uint8_t *src, long s_line, long s_step, uint8_t *dst,
                                long d_line, long d_step, int lines, int nout, int line_fastest,
                                const int *bounds, const int *kk, int ksize, int prec, k_stream s)
{
    if (lines <= 0 || nout <= 0 || ksize <= 0 || prec < 1 || prec > 22)
        return K_EARG;
    const int grid = grid_for((long)lines * nout, 256);
    resize_pass_kernel<<<grid < 148 * 16 ? grid : 148 * 16, 256, 0, STREAM(s)>>>(
        src, s_line, s_step, dst, d_line, d_step, lines, nout, line_fastest, bounds, kk, ksize,
        prec);
    return (int)cudaGetLastError();
}

extern "C" int k_crop_copy_u8(const uint8_t *src, long pitch, int w, int h, uint8_t *dst,
                              k_stream s)
{
    if (w <= 0 || h <= 0)
        return K_EARG;
    const int grid = grid_for((long)w * h * 3, 256);
    crop_copy_kernel<<<grid < 148 * 16 ? grid : 148 * 16, 256, 0, STREAM(s)>>>(src, pitch, w, h,
                                                                               dst);
    return (int)cudaGetLastError();
}

extern "C" int k_normalize_chw(const uint8_t *tile, int side, float *out, k_stream s)
{
    if (side <= 0)
        return K_EARG;
    const int grid = grid_for((long)side * side, 256);
    normalize_chw_kernel<<<grid < 148 * 16 ? grid : 148 * 16, 256, 0, STREAM(s)>>>(tile, side, out);
    return (int)cudaGetLastError();
}
