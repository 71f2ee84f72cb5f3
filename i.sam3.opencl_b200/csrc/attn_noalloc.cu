// SPDX-License-Identifier: Unlicense
// cb_attention_noalloc: the tensor-core attention of cb_attention for fp32
// Q/K/V, for callers that cannot allocate device memory. cb_attention
// converts fp32 qkv into bf16 (RoPE applied) in the backend's scratch
// buffer, which the backend grows with cudaMalloc on demand; this entry
// point instead stages that bf16 copy in a fixed array compiled into the
// library, so it never calls cudaMalloc, cudaFree or any allocating routine.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds its SAM3_NOALLOC_SCRATCH_BYTES (32 MiB) from module load
// until the process exits. In host code the array's name is only a
// host-side stand-in, so the device address is looked up with
// cudaGetSymbolAddress once per device, with that device current, on the
// first call made on it.
#include "kernels.h"
#include "sam3_cuda.h"

#include <cuda_runtime.h>
#include <stdint.h>

#define SAM3_NOALLOC_SCRATCH_BYTES (32u << 20)
#define SAM3_NOALLOC_MAX_DEVICES 64

namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[SAM3_NOALLOC_SCRATCH_BYTES];
static __device__ __align__(256) int g_noalloc_err;

// Device addresses of the two variables, per device ordinal (null = not set
// up). Read and written with atomic loads / stores, so two host threads
// making their first call on one device at the same time both look the
// addresses up (the same values) without a data race. Never invalidated: a
// cudaDeviceReset leaves them stale (documented in sam3_cuda.h).
static void *g_scratch_addr[SAM3_NOALLOC_MAX_DEVICES];
static void *g_err_addr[SAM3_NOALLOC_MAX_DEVICES];

void *load_addr(void *const *slot)
{
    return __atomic_load_n(slot, __ATOMIC_ACQUIRE);
}

int status_of(cudaError_t e)
{
    return e == cudaSuccess ? CB_OK : CB_ECUDA;
}

int status_of_launch(int rc)
{
    if (rc == 0)
        return CB_OK;
    return (rc == K_EARG || rc == K_ETMAP) ? CB_EARG : CB_ECUDA;
}

// Looks up the device addresses of the static array and error word for the
// current device (first call on each device only).
int setup_current_device(int dev)
{
    if (load_addr(&g_scratch_addr[dev]) && load_addr(&g_err_addr[dev]))
        return CB_OK;
    void *s = nullptr, *e = nullptr;
    cudaError_t rc = cudaGetSymbolAddress(&s, g_noalloc_scratch);
    if (rc != cudaSuccess)
        return CB_ECUDA;
    rc = cudaGetSymbolAddress(&e, g_noalloc_err);
    if (rc != cudaSuccess)
        return CB_ECUDA;
    __atomic_store_n(&g_err_addr[dev], e, __ATOMIC_RELEASE);
    __atomic_store_n(&g_scratch_addr[dev], s, __ATOMIC_RELEASE);
    return CB_OK;
}

}  // namespace

extern "C" int cb_attention_noalloc(const float *qkv, int nseq, int N, int E, int heads,
                                    const float *cs, int npos, float scale, float *out,
                                    int *err, void *stream)
{
    const int hd = 64;
    if (!qkv || !out || nseq <= 0 || N <= 0 || heads <= 0 || E != heads * hd ||
        (cs && npos <= 0))
        return CB_EARG;
    const uint64_t rows = (uint64_t)nseq * (uint64_t)N;
    if (rows * 3ull * (uint64_t)E * 2ull > SAM3_NOALLOC_SCRATCH_BYTES)
        return CB_EARG;  // larger than the static scratch array
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= SAM3_NOALLOC_MAX_DEVICES)
        return CB_ENODEV;
    const int st = setup_current_device(dev);
    if (st != CB_OK)
        return st;
    k_stream s = reinterpret_cast<k_stream>(stream);
    int *errp = err;
    if (!errp) {
        // The library's own error word keeps the previous call's value:
        // clear it first.
        errp = static_cast<int *>(load_addr(&g_err_addr[dev]));
        int rc = status_of(cudaMemsetAsync(errp, 0, sizeof(int),
                                           reinterpret_cast<cudaStream_t>(stream)));
        if (rc != CB_OK)
            return rc;
    }
    void *scratch = load_addr(&g_scratch_addr[dev]);
    int rc = cs ? k_rope_cast_bf16(qkv, (long)rows, E, hd, npos, cs, scratch, s)
                : k_cast_f32_bf16(qkv, scratch, (long)rows * 3 * E, s);
    if (rc != 0)
        return status_of_launch(rc);
    return status_of_launch(k_attn_tc(scratch, nseq, N, E, heads, scale, out, 0, NULL, 0, errp,
                                      s));
}
