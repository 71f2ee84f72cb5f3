// SPDX-License-Identifier: Unlicense
// Memory-bound kernels of the PE backbone path and the reference-contract
// helpers: LayerNorm (one warp per row, 128-bit loads, row kept in
// registers), RoPE, window (un)partition, add_bcast, patch extraction with
// the uint8 -> [-1, 1] input normalisation, casts, row permutations and the
// seeded generator. Each kernel cites the reference kernel it replaces.
#include "kernels.h"
#include "sam3_synth.h"
#include "tc_ptx.cuh"

#include <cuda_bf16.h>

namespace sam3 {
namespace {

inline int grid_for(long n, int block)
{
    long g = (n + block - 1) / block;
    return (int)(g < 1 ? 1 : (g > 0x7fffffffL ? 0x7fffffffL : g));
}

__device__ __forceinline__ float gelu_erf(float x)
{
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ float act_fn(float v, int act)
{
    if (act == K_ACT_GELU)
        return gelu_erf(v);
    if (act == K_ACT_RELU)
        return fmaxf(v, 0.0f);
    return v;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------- LayerNorm
// layernorm (sam3_kernels.cl:489-514): two-pass mean / variance, eps inside
// the square root, optional activation. One warp per row; the row stays in
// registers (NV float4 per lane), so X is read once and Y written once.
template <int NV, bool OUT_BF16>
__global__ void __launch_bounds__(256) ln_reg_kernel(const float *__restrict__ X, void *Y,
                                                     const float *__restrict__ g,
                                                     const float *__restrict__ b, long rows, int C,
                                                     float eps, int act)
{
    const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    const float4 *x = reinterpret_cast<const float4 *>(X + row * C);
    float4 v[NV];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        v[i] = x[i * 32 + lane];
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
    const float mean = warp_sum(s) / C;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
        q += (a * a + bb * bb) + (c * c + d * d);
    }
    const float inv = rsqrtf(warp_sum(q) / C + eps);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    const float4 *b4 = reinterpret_cast<const float4 *>(b);
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const int c4 = i * 32 + lane;
        const float4 gg = __ldg(g4 + c4), bt = __ldg(b4 + c4);
        float4 y;
        y.x = act_fn((v[i].x - mean) * inv * gg.x + bt.x, act);
        y.y = act_fn((v[i].y - mean) * inv * gg.y + bt.y, act);
        y.z = act_fn((v[i].z - mean) * inv * gg.z + bt.z, act);
        y.w = act_fn((v[i].w - mean) * inv * gg.w + bt.w, act);
        if (OUT_BF16) {
            uint2 p;
            p.x = pack_bf16x2(y.x, y.y);
            p.y = pack_bf16x2(y.z, y.w);
            reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(Y) + row * C)[c4] = p;
        }
        else
            reinterpret_cast<float4 *>(reinterpret_cast<float *>(Y) + row * C)[c4] = y;
    }
}

// Any C: one warp per row, three passes over global memory.
template <bool OUT_BF16>
__global__ void __launch_bounds__(256) ln_any_kernel(const float *__restrict__ X, void *Y,
                                                     const float *__restrict__ g,
                                                     const float *__restrict__ b, long rows, int C,
                                                     float eps, int act)
{
    const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    const float *x = X + row * C;
    float s = 0.0f;
    for (int c = lane; c < C; c += 32)
        s += x[c];
    const float mean = warp_sum(s) / C;
    float q = 0.0f;
    for (int c = lane; c < C; c += 32) {
        const float d = x[c] - mean;
        q += d * d;
    }
    const float inv = rsqrtf(warp_sum(q) / C + eps);
    // Read every input before the first write: Y may alias X.
    __syncwarp();
    for (int c = lane; c < C; c += 32) {
        const float y = act_fn((x[c] - mean) * inv * g[c] + b[c], act);
        if (OUT_BF16)
            reinterpret_cast<__nv_bfloat16 *>(Y)[row * C + c] = __float2bfloat16_rn(y);
        else
            reinterpret_cast<float *>(Y)[row * C + c] = y;
    }
}

// ---------------------------------------------------------------- softmax
// softmax_rows (sam3_kernels.cl:637-656): in place, one warp per row.
__global__ void __launch_bounds__(256) softmax_rows_kernel(float *S, long rows, int L)
{
    const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    float *s = S + row * L;
    float m = -INFINITY;
    for (int j = lane; j < L; j += 32)
        m = fmaxf(m, s[j]);
    m = warp_max(m);
    float sum = 0.0f;
    for (int j = lane; j < L; j += 32) {
        const float v = expf(s[j] - m);
        s[j] = v;
        sum += v;
    }
    const float inv = 1.0f / warp_sum(sum);
    for (int j = lane; j < L; j += 32)
        s[j] *= inv;
}

// ---------------------------------------------------------------- RoPE
// rope_apply (sam3_kernels.cl:679-698): pair (2j, 2j+1) of q and k of row r
// rotated by cs[(r % npos) * hd/2 + j]. One thread per pair.
__global__ void rope_apply_kernel(float *qkv, long rows, int E, int hd, int npos,
                                  const float2 *__restrict__ cs)
{
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int half = E / 2;
    if (gid >= rows * 2 * half)
        return;
    const int pr = (int)(gid % half);
    const long rest = gid / half;
    const int qk = (int)(rest % 2);
    const long r = rest / 2;
    const int nf = hd / 2, h = pr / nf, j = pr % nf;
    float2 *x = reinterpret_cast<float2 *>(qkv + r * 3 * E + qk * E + h * hd + 2 * j);
    const float2 rot = __ldg(cs + (r % npos) * nf + j);
    const float2 v = *x;
    *x = make_float2(v.x * rot.x - v.y * rot.y, v.x * rot.y + v.y * rot.x);
}

// fp32 qkv -> bf16 qkv, RoPE on q and k, plain cast of v. A CTA per
// kRopeRows rows, a thread per 4 columns (two pairs) of a row, 32-bit index
// math (the table row r % npos once per row).
constexpr int kRopeRows = 2;
__global__ void __launch_bounds__(256) rope_cast_kernel(const float *__restrict__ qkv, long rows,
                                                        int E, int hd, int npos,
                                                        const float2 *__restrict__ cs,
                                                        __nv_bfloat16 *__restrict__ out)
{
    const int per_row = 3 * E / 4, nf = hd / 2;
#pragma unroll
    for (int rr = 0; rr < kRopeRows; rr++) {
        const long r = (long)blockIdx.x * kRopeRows + rr;
        if (r >= rows)
            return;
        const float4 *src = reinterpret_cast<const float4 *>(qkv + r * 3 * E);
        uint2 *dst = reinterpret_cast<uint2 *>(out + r * 3 * E);
        const float2 *trow = cs + (long)(int)(r % npos) * nf;
        for (int k = threadIdx.x; k < per_row; k += blockDim.x) {
            const int c = 4 * k;
            float4 v = __ldg(src + k);
            if (c < 2 * E) {
                const int j = (c % hd) / 2;
                const float2 r0 = __ldg(trow + j), r1 = __ldg(trow + j + 1);
                v = make_float4(v.x * r0.x - v.y * r0.y, v.x * r0.y + v.y * r0.x,
                                v.z * r1.x - v.w * r1.y, v.z * r1.y + v.w * r1.x);
            }
            dst[k] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
        }
    }
}

// ---------------------------------------------------------------- misc
// add_bcast (sam3_kernels.cl:701-708).
__global__ void add_bcast_kernel(float *out, const float *a, const float *b, long n, long bmod)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        out[i] = a[i] + b[i % bmod];
}

// out = bf16(a + b): the sum rounded once to bf16 (the same value as the
// fp32 sum followed by a cast), for a sum whose only reader is a GEMM.
__global__ void add_bf16_kernel(const float *__restrict__ a, const float *__restrict__ b,
                                __nv_bfloat16 *__restrict__ out, long n)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        out[i] = __float2bfloat16_rn(a[i] + b[i]);
}

// window_partition (sam3_kernels.cl:712-724): window-major row r = (window
// w, in-window position i) <- token (y, x), zero past the image. A CTA per
// row; V4: 16-byte copies (C % 4 == 0, 16-byte aligned buffers).
template <bool V4>
__global__ void __launch_bounds__(256) window_partition_kernel(const float *__restrict__ X,
                                                               float *__restrict__ out, int H,
                                                               int C, int ws, int nwx)
{
    const int r = blockIdx.x;
    const int w = r / (ws * ws), i = r - w * (ws * ws);
    const int y = (w / nwx) * ws + i / ws, x = (w % nwx) * ws + i % ws;
    const bool in = y < H && x < H;
    const float *src = X + ((long)y * H + x) * C;
    float *dst = out + (long)r * C;
    if (V4) {
        for (int c = threadIdx.x; c < C / 4; c += blockDim.x)
            reinterpret_cast<float4 *>(dst)[c] =
                in ? __ldg(reinterpret_cast<const float4 *>(src) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    else {
        for (int c = threadIdx.x; c < C; c += blockDim.x)
            dst[c] = in ? src[c] : 0.0f;
    }
}

// window_unpartition_add (sam3_kernels.cl:728-741): token (y, x) += its
// window-major row. A CTA per token.
template <bool V4>
__global__ void __launch_bounds__(256) window_unpartition_add_kernel(float *__restrict__ X,
                                                                     const float *__restrict__ Wd,
                                                                     int H, int C, int ws, int nwx)
{
    const int t = blockIdx.x;
    const int y = t / H, x = t - y * H;
    const int w = (y / ws) * nwx + x / ws, i = (y % ws) * ws + x % ws;
    float *dst = X + (long)t * C;
    const float *src = Wd + ((long)w * ws * ws + i) * C;
    if (V4) {
        for (int c = threadIdx.x; c < C / 4; c += blockDim.x) {
            float4 a = reinterpret_cast<float4 *>(dst)[c];
            const float4 b = __ldg(reinterpret_cast<const float4 *>(src) + c);
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
            reinterpret_cast<float4 *>(dst)[c] = a;
        }
    }
    else {
        for (int c = threadIdx.x; c < C; c += blockDim.x)
            dst[c] += src[c];
    }
}

// patch_im2col (sam3_kernels.cl:661-672).
__global__ void patch_im2col_kernel(const float *img, float *out, int side, int grid, int ps)
{
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int k = 3 * ps * ps;
    const long t = gid / k;
    if (t >= (long)grid * grid)
        return;
    const int col = (int)(gid % k);
    const int c = col / (ps * ps), ky = (col % (ps * ps)) / ps, kx = col % ps;
    const int ty = (int)(t / grid), tx = (int)(t % grid);
    out[gid] = img[((long)c * side + ty * ps + ky) * side + tx * ps + kx];
}

// Patch rows straight from uint8 HWC tiles, normalised as
// image_encoder_input does (image.c:360-366), in window-major token order,
// bf16, K padded with zeros to kpad. One CTA per window row of one tile: the
// ws patches of the row come from ps image rows of ws * ps * 3 contiguous
// bytes, staged in shared memory with 16-byte loads (byte loads when the
// rows are not 16-byte aligned); a table maps each patch column (channel,
// ky, kx) to its byte in the staged rows, and each thread then writes 8
// output columns of one token with one 16-byte store.
__global__ void __launch_bounds__(256) patch_embed_in_kernel(const uint8_t *__restrict__ rgb,
                                                             int side, int grid, int ps, int ws,
                                                             int kpad, __nv_bfloat16 *out)
{
    extern __shared__ uint8_t patch_smem[];
    const int rowbytes = ws * ps * 3;
    const int K = 3 * ps * ps;
    int *coloff = reinterpret_cast<int *>(patch_smem);
    uint8_t *st = patch_smem + (((size_t)K * 4 + 15) & ~(size_t)15);
    const int nwx = grid / ws, nwin = nwx * nwx;
    int bid = (int)blockIdx.x;
    const int iy = bid % ws;
    bid /= ws;
    const int w = bid % nwin, tile = bid / nwin;
    const int ty = (w / nwx) * ws + iy, tx0 = (w % nwx) * ws;
    const uint8_t *src = rgb + ((long)tile * side * side + (long)ty * ps * side + (long)tx0 * ps) * 3;
    const long pitch = (long)side * 3;
    for (int col = threadIdx.x; col < K; col += blockDim.x) {
        const int c = col / (ps * ps), rem = col - c * ps * ps;
        const int ky = rem / ps, kx = rem - ky * ps;
        coloff[col] = ky * rowbytes + kx * 3 + c;
    }
    if (!(((uintptr_t)src | (uintptr_t)pitch | (uintptr_t)rowbytes) & 15)) {
        const int n16 = rowbytes / 16;
        for (int i = threadIdx.x; i < ps * n16; i += blockDim.x) {
            const int r = i / n16, c16 = i - r * n16;
            reinterpret_cast<uint4 *>(st)[i] =
                *reinterpret_cast<const uint4 *>(src + (long)r * pitch + 16 * c16);
        }
    }
    else {
        for (int i = threadIdx.x; i < ps * rowbytes; i += blockDim.x) {
            const int r = i / rowbytes;
            st[i] = src[(long)r * pitch + (i - r * rowbytes)];
        }
    }
    __syncthreads();
    const int groups = kpad / 8;
    const long row0 = (long)tile * grid * grid + (long)w * ws * ws + (long)iy * ws;
    for (int i = threadIdx.x; i < ws * groups; i += blockDim.x) {
        const int j = i / groups, g0 = (i - j * groups) * 8;
        const uint8_t *pj = st + j * ps * 3;
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int col = g0 + e;
            v[e] = col < K ? ((float)pj[coloff[col]] / 255.0f - 0.5f) / 0.5f : 0.0f;
        }
        uint4 p;
        p.x = pack_bf16x2(v[0], v[1]);
        p.y = pack_bf16x2(v[2], v[3]);
        p.z = pack_bf16x2(v[4], v[5]);
        p.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4 *>(out + (row0 + j) * kpad + g0) = p;
    }
}

// Eight values per thread: two 16-byte loads, one 16-byte store.
__global__ void cast_f32_bf16_v8_kernel(const float4 *__restrict__ x, uint4 *__restrict__ y,
                                        long n8)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (long)gridDim.x * blockDim.x) {
        const float4 a = x[2 * i], b = x[2 * i + 1];
        y[i] = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                          pack_bf16x2(b.z, b.w));
    }
}

__global__ void cast_f32_bf16_kernel(const float *x, __nv_bfloat16 *y, long n)
{
    griddep_wait();  // launched as a programmatic dependent (pdl.cuh)
    griddep_launch();
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        y[i] = __float2bfloat16_rn(x[i]);
}

__global__ void cast_bf16_f32_kernel(const __nv_bfloat16 *x, float *y, long n)
{
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        y[i] = __bfloat162float(x[i]);
}

// Row r of the window-major layout <-> raster row of the same token.
__device__ __forceinline__ long raster_of(long r, int grid, int ws)
{
    const long T = (long)grid * grid;
    const long tile = r / T;
    const int t = (int)(r % T), w2 = ws * ws, nwx = grid / ws;
    const int w = t / w2, i = t % w2;
    const int y = (w / nwx) * ws + i / ws, x = (w % nwx) * ws + i % ws;
    return tile * T + (long)y * grid + x;
}

// dir 0: y[raster] = x[window-major]; dir 1: y[window-major] = x[raster].
__global__ void permute_rows_kernel(const float *__restrict__ x, float *__restrict__ y, long rows,
                                    int grid, int ws, int C, int dir)
{
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int c4 = C / 4;
    if (gid >= rows * c4)
        return;
    const long r = gid / c4;
    const int c = (int)(gid % c4);
    const long p = raster_of(r, grid, ws);
    const float4 *src = reinterpret_cast<const float4 *>(x + (dir == 0 ? r : p) * C);
    float4 *dst = reinterpret_cast<float4 *>(y + (dir == 0 ? p : r) * C);
    dst[c] = src[c];
}

// Device copy of sam3_synth_normal: same hash, same Irwin-Hall sum, one
// correctly rounded multiply and add.
__global__ void synth_normal_kernel(uint64_t base, long n, float mean, float std, float *out32,
                                    __nv_bfloat16 *out16)
{
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    const float z = sam3_normal_at(base, (uint64_t)i);
    const float v = __fadd_rn(mean, __fmul_rn(std, z));
    if (out16)
        out16[i] = __float2bfloat16_rn(v);
    else
        out32[i] = v;
}

}  // namespace
}  // namespace sam3

using namespace sam3;

#define STREAM(s) reinterpret_cast<cudaStream_t>(s)
#define LAUNCH_RET() return (int)cudaGetLastError()

extern "C" int k_layernorm(const float *X, void *Y, int y_bf16, const float *g, const float *b,
                           long rows, int C, float eps, int act, k_stream s)
{
    if (rows <= 0 || C <= 0)
        return rows == 0 ? 0 : K_EARG;
    const int grid = grid_for(rows, 8);
    const bool vec = (C % 128 == 0) && !((uintptr_t)X & 15) && !((uintptr_t)Y & 15) &&
                     !((uintptr_t)g & 15) && !((uintptr_t)b & 15);
#define LN_REG(NV)                                                                          \
    if (vec && C == NV * 128) {                                                             \
        if (y_bf16)                                                                         \
            ln_reg_kernel<NV, true><<<grid, 256, 0, STREAM(s)>>>(X, Y, g, b, rows, C, eps, act); \
        else                                                                                \
            ln_reg_kernel<NV, false><<<grid, 256, 0, STREAM(s)>>>(X, Y, g, b, rows, C, eps, act); \
        LAUNCH_RET();                                                                       \
    }
    LN_REG(2)
    LN_REG(4)
    LN_REG(8)
    LN_REG(16)
#undef LN_REG
    if (y_bf16)
        ln_any_kernel<true><<<grid, 256, 0, STREAM(s)>>>(X, Y, g, b, rows, C, eps, act);
    else
        ln_any_kernel<false><<<grid, 256, 0, STREAM(s)>>>(X, Y, g, b, rows, C, eps, act);
    LAUNCH_RET();
}

extern "C" int k_softmax_rows(float *S, long rows, int L, k_stream s)
{
    if (rows <= 0)
        return 0;
    softmax_rows_kernel<<<grid_for(rows, 8), 256, 0, STREAM(s)>>>(S, rows, L);
    LAUNCH_RET();
}

extern "C" int k_rope_apply(float *qkv, long rows, int E, int hd, int npos, const float *cs,
                            k_stream s)
{
    if (hd % 2 || E % hd || npos <= 0)
        return K_EARG;
    const long n = rows * E;
    rope_apply_kernel<<<grid_for(n, 256), 256, 0, STREAM(s)>>>(
        qkv, rows, E, hd, npos, reinterpret_cast<const float2 *>(cs));
    LAUNCH_RET();
}

extern "C" int k_rope_cast_bf16(const float *qkv, long rows, int E, int hd, int npos,
                                const float *cs, void *out, k_stream s)
{
    if (hd % 4 || E % hd || npos <= 0 || ((uintptr_t)qkv & 15) || ((uintptr_t)out & 7))
        return K_EARG;
    rope_cast_kernel<<<grid_for(rows, kRopeRows), 256, 0, STREAM(s)>>>(
        qkv, rows, E, hd, npos, reinterpret_cast<const float2 *>(cs),
        reinterpret_cast<__nv_bfloat16 *>(out));
    LAUNCH_RET();
}

extern "C" int k_add_bcast(float *out, const float *a, const float *b, long n, long bmod,
                           k_stream s)
{
    if (n <= 0)
        return 0;
    if (bmod <= 0)
        return K_EARG;
    return launch_pdl(add_bcast_kernel, dim3(grid_for(n, 256)), dim3(256), 0, STREAM(s), out, a, b,
                      n, bmod);
}

extern "C" int k_add_bf16(const float *a, const float *b, void *out, long n, k_stream s)
{
    if (n <= 0)
        return K_EARG;
    return launch_pdl(add_bf16_kernel, dim3(grid_for(n, 256)), dim3(256), 0, STREAM(s), a, b,
                      reinterpret_cast<__nv_bfloat16 *>(out), n);
}

extern "C" int k_window_partition(const float *X, float *out, int H, int C, int ws, int nwx,
                                  k_stream s)
{
    const long rows = (long)nwx * nwx * ws * ws;
    if (rows <= 0 || C <= 0)
        return rows == 0 ? 0 : K_EARG;
    if (rows > 0x7fffffffL)
        return K_EARG;
    const bool v4 = !(C & 3) && !((uintptr_t)X & 15) && !((uintptr_t)out & 15);
    if (v4)
        window_partition_kernel<true><<<(unsigned)rows, 256, 0, STREAM(s)>>>(X, out, H, C, ws, nwx);
    else
        window_partition_kernel<false><<<(unsigned)rows, 256, 0, STREAM(s)>>>(X, out, H, C, ws, nwx);
    LAUNCH_RET();
}

extern "C" int k_window_unpartition_add(float *X, const float *Wd, int H, int C, int ws, int nwx,
                                        k_stream s)
{
    const long rows = (long)H * H;
    if (rows <= 0 || C <= 0)
        return rows == 0 ? 0 : K_EARG;
    if (rows > 0x7fffffffL)
        return K_EARG;
    const bool v4 = !(C & 3) && !((uintptr_t)X & 15) && !((uintptr_t)Wd & 15);
    if (v4)
        window_unpartition_add_kernel<true><<<(unsigned)rows, 256, 0, STREAM(s)>>>(X, Wd, H, C, ws,
                                                                                   nwx);
    else
        window_unpartition_add_kernel<false><<<(unsigned)rows, 256, 0, STREAM(s)>>>(X, Wd, H, C, ws,
                                                                                    nwx);
    LAUNCH_RET();
}

extern "C" int k_patch_im2col(const float *img, float *out, int side, int grid, int ps,
                              k_stream s)
{
    const long n = (long)grid * grid * 3 * ps * ps;
    patch_im2col_kernel<<<grid_for(n, 256), 256, 0, STREAM(s)>>>(img, out, side, grid, ps);
    LAUNCH_RET();
}

extern "C" int k_patch_embed_in(const uint8_t *rgb, int ntile, int side, int grid, int ps, int ws,
                                int kpad, void *out, k_stream s)
{
    if (kpad % 8 || kpad < 3 * ps * ps || grid % ws || ((uintptr_t)out & 15) || ntile <= 0 ||
        side < grid * ps)
        return K_EARG;
    const size_t smem = (((size_t)3 * ps * ps * 4 + 15) & ~(size_t)15) + (size_t)ps * ws * ps * 3;
    if (smem > 227 * 1024)
        return K_EARG;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(
            patch_embed_in_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess)
            return (int)e;
    }
    const long blocks = (long)ntile * (grid / ws) * (grid / ws) * ws;
    if (blocks > 0x7fffffffL)
        return K_EARG;
    patch_embed_in_kernel<<<(unsigned)blocks, 256, smem, STREAM(s)>>>(
        rgb, side, grid, ps, ws, kpad, reinterpret_cast<__nv_bfloat16 *>(out));
    LAUNCH_RET();
}

extern "C" int k_cast_f32_bf16(const float *x, void *y, long n, k_stream s)
{
    if (n <= 0)
        return 0;
    if (n % 8 == 0 && !((uintptr_t)x & 15) && !((uintptr_t)y & 15)) {
        const int g = grid_for(n / 8, 256);
        return launch_pdl(cast_f32_bf16_v8_kernel, dim3(g < 148 * 16 ? g : 148 * 16), dim3(256), 0,
                          STREAM(s), reinterpret_cast<const float4 *>(x),
                          reinterpret_cast<uint4 *>(y), n / 8);
    }
    return launch_pdl(cast_f32_bf16_kernel, dim3(grid_for(n, 256)), dim3(256), 0, STREAM(s), x,
                      reinterpret_cast<__nv_bfloat16 *>(y), n);
}

extern "C" int k_cast_bf16_f32(const void *x, float *y, long n, k_stream s)
{
    if (n <= 0)
        return 0;
    cast_bf16_f32_kernel<<<grid_for(n, 256), 256, 0, STREAM(s)>>>(
        reinterpret_cast<const __nv_bfloat16 *>(x), y, n);
    LAUNCH_RET();
}

extern "C" int k_unpermute_rows(const float *x, float *y, int ntile, int grid, int ws, int C,
                                k_stream s)
{
    if (C % 4 || grid % ws)
        return K_EARG;
    const long rows = (long)ntile * grid * grid;
    permute_rows_kernel<<<grid_for(rows * (C / 4), 256), 256, 0, STREAM(s)>>>(x, y, rows, grid, ws,
                                                                               C, 0);
    LAUNCH_RET();
}

extern "C" int k_permute_rows(const float *x, float *y, int ntile, int grid, int ws, int C,
                              k_stream s)
{
    if (C % 4 || grid % ws)
        return K_EARG;
    const long rows = (long)ntile * grid * grid;
    permute_rows_kernel<<<grid_for(rows * (C / 4), 256), 256, 0, STREAM(s)>>>(x, y, rows, grid, ws,
                                                                               C, 1);
    LAUNCH_RET();
}

extern "C" int k_synth_normal(uint64_t seed, uint64_t stream, long n, float mean, float std,
                              void *out, int out_bf16, k_stream s)
{
    if (n <= 0)
        return 0;
    const uint64_t base = sam3_stream_base(seed, stream);
    synth_normal_kernel<<<grid_for(n, 256), 256, 0, STREAM(s)>>>(
        base, n, mean, std, out_bf16 ? nullptr : reinterpret_cast<float *>(out),
        out_bf16 ? reinterpret_cast<__nv_bfloat16 *>(out) : nullptr);
    LAUNCH_RET();
}

// ---------------------------------------------------------------- diagnostics
namespace sam3 {
namespace {
__global__ void diag_exp2_kernel(const float *x, float *y_poly, float *y_mufu, int n)
{
    const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i + 1 < n) {
        exp2_poly2(x[i], x[i + 1], y_poly[i], y_poly[i + 1]);
        y_mufu[i] = ex2_approx(x[i]);
        y_mufu[i + 1] = ex2_approx(x[i + 1]);
    }
}
// One thread waits on an mbarrier that nothing arrives on, with the given
// limit: the bounded wait must give up, record kErrWaitTimeout in *err and
// leave the context usable. status[0] = the wait's result (0: timed out),
// status[1] = the abort flag it raised.
__global__ void diag_wait_timeout_kernel(int *err, int *status, uint64_t limit_ns)
{
    __shared__ uint64_t bar;
    __shared__ volatile int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
        const bool ok = mbar_wait(&bar, 0, err, &abort_flag, limit_ns);
        status[0] = ok ? 1 : 0;
        status[1] = abort_flag;
    }
}
}  // namespace
}  // namespace sam3

extern "C" int cb_diag_wait_timeout(int *err, int *status, int limit_us, void *stream)
{
    if (!err || !status || limit_us <= 0 || limit_us > 1000000)
        return 3;  // CB_EARG
    sam3::diag_wait_timeout_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        err, status, (uint64_t)limit_us * 1000);
    return cudaGetLastError() == cudaSuccess ? 0 : 4;  // CB_OK / CB_ECUDA
}

extern "C" int cb_diag_exp2(const float *x, float *y_poly, float *y_mufu, int n, void *stream)
{
    if (!x || !y_poly || !y_mufu || n <= 0 || (n & 1))
        return 3;  // CB_EARG
    diag_exp2_kernel<<<grid_for(n / 2, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        x, y_poly, y_mufu, n);
    return cudaGetLastError() == cudaSuccess ? 0 : 4;  // CB_OK / CB_ECUDA
}
