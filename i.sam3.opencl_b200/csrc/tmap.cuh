// SPDX-License-Identifier: Unlicense
// Host helper: 2D TMA descriptors for bf16 row-major matrices with 128-byte
// swizzle, via the driver entry point cuTensorMapEncodeTiled (fetched once
// through the runtime, so the library needs no -lcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sam3 {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// rows x cols bf16 matrix, leading dimension ld elements; box box_rows x 64
// (one 128-byte swizzle span). Out-of-range elements read as zero.
// Returns false on failure (base not 16-byte aligned, ld*2 not a multiple of
// 16, or the encode call failing).
inline bool make_tmap_bf16(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                           uint64_t ld, uint32_t box_rows)
{
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15) || box_rows > 256 ||
        rows == 0 || cols == 0)
        return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// General 2D tile map: rows x cols elements of `esize` bytes (dtype), leading
// dimension ld elements, box box_rows x box_cols, 128-byte swizzle (box_cols
// * esize must be 128 or less).
inline bool make_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t esize,
                         const void *base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_cols, uint32_t box_rows)
{
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || ((ld * esize) & 15) ||
        box_rows > 256 || box_cols * esize > 128 || rows == 0 || cols == 0)
        return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * esize};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// 3-D map over n blocks of rows x cols elements (row pitch ld, block pitch
// bld elements; bld 0: one block), box box_cols x box_rows x 1 with the
// given swizzle (box_cols * esize must not exceed the swizzle span).
// Out-of-range elements read as zero.
inline bool make_tmap_3d(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t esize,
                         const void *base, uint64_t n, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint64_t bld, uint32_t box_cols, uint32_t box_rows,
                         CUtensorMapSwizzle swz)
{
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || ((ld * esize) & 15) ||
        ((bld * esize) & 15) || box_rows > 256 || rows == 0 || cols == 0 || n == 0)
        return false;
    if (bld == 0)
        n = 1;
    cuuint64_t dims[3] = {cols, rows, n};
    cuuint64_t strides[2] = {ld * esize, (bld ? bld : rows * ld) * esize};
    cuuint32_t box[3] = {box_cols, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D map over n images of h x w pixels of c channels (channels innermost,
// packed), box box_c x box_w x box_h x 1 with 128-byte swizzle (box_c *
// esize = 128 or less). Out-of-range elements read as zero; stores clip.
inline bool make_tmap_nhwc(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t esize,
                           const void *base, uint64_t n, uint64_t h, uint64_t w, uint64_t c,
                           uint32_t box_c, uint32_t box_w, uint32_t box_h)
{
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || ((c * esize) & 15) ||
        box_c * esize > 128 || box_w > 256 || box_h > 256 || !n || !h || !w || !c)
        return false;
    cuuint64_t dims[4] = {c, w, h, n};
    cuuint64_t strides[3] = {c * esize, w * c * esize, h * w * c * esize};
    cuuint32_t box[4] = {box_c, box_w, box_h, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(map, dtype, 4, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// Raises kernel Kern's dynamic shared-memory limit to `bytes` once per
// device (the attribute persists; setting it before every launch costs host
// time in front of short kernels).
template <auto Kern>
inline cudaError_t smem_limit_once(int bytes)
{
    static int set[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (set[dev] >= bytes)
        return cudaSuccess;
    const cudaError_t e =
        cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess)
        set[dev] = bytes;
    return e;
}

// Multiprocessor count of the current device, queried once per device.
inline int device_sms()
{
    static int sms[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return 148;
    if (!sms[dev] &&
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 148;
    return sms[dev];
}

}  // namespace sam3
