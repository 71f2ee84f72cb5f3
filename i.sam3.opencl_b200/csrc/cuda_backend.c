/* SPDX-License-Identifier: Unlicense */
/* Device, stream and buffer management of the C-ABI (include/sam3_cuda.h):
 * the B200 counterpart of the reference's ocl_backend.c. Every entry point
 * returns a status code instead of exiting (the reference calls
 * G_fatal_error through ocl_check, ocl_backend.c:72-77). */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "backend_internal.h"

size_t cbi_dtype_size(int dtype)
{
    switch (dtype) {
    case CB_F32:
        return 4;
    case CB_BF16:
    case CB_F16:
        return 2;
    case CB_U8:
        return 1;
    default:
        return 0;
    }
}

const char *cb_errstr(int status)
{
    switch (status) {
    case CB_OK:
        return "success";
    case CB_ENODEV:
        return "no usable CUDA device (compute capability 10.x required)";
    case CB_EALLOC:
        return "allocation failed";
    case CB_EARG:
        return "invalid argument, shape, stride or alignment";
    case CB_ECUDA:
        return "CUDA runtime error";
    case CB_ETIMEOUT:
        return "a device-side wait timed out";
    case CB_EDTYPE:
        return "operand dtype not supported by this operation";
    default:
        return "unknown status";
    }
}

int cbi_fail(cb_backend *b, int status, const char *what)
{
    if (b)
        snprintf(b->last_error, sizeof(b->last_error), "%s: %s", what,
                 cb_errstr(status));
    return status;
}

int cbi_kstatus(cb_backend *b, int rc, const char *what)
{
    if (rc == 0)
        return CB_OK;
    if (rc == K_EARG)
        return cbi_fail(b, CB_EARG, what);
    if (rc == K_ETMAP) {
        if (b)
            snprintf(b->last_error, sizeof(b->last_error),
                     "%s: TMA descriptor rejected (alignment or extent)", what);
        return CB_EARG;
    }
    if (b)
        snprintf(b->last_error, sizeof(b->last_error), "%s: %s", what,
                 cudaGetErrorString((cudaError_t)rc));
    return CB_ECUDA;
}

int cbi_enter(cb_backend *b)
{
    int cur = -1;

    if (!b)
        return CB_EARG;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != b->device) {
        cudaError_t e = cudaSetDevice(b->device);

        if (e != cudaSuccess)
            return cbi_kstatus(b, (int)e, "cudaSetDevice");
    }
    return CB_OK;
}

int cb_init(cb_backend **out, int device)
{
    cb_backend *b;
    struct cudaDeviceProp prop;
    int n = 0;
    cudaError_t e;

    if (!out)
        return CB_EARG;
    *out = NULL;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n)
        return CB_ENODEV;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10)
        return CB_ENODEV;
    b = calloc(1, sizeof(*b));
    if (!b)
        return CB_EALLOC;
    b->device = device;
    b->num_sms = prop.multiProcessorCount;
    e = cudaSetDevice(device);
    if (e == cudaSuccess)
        e = cudaStreamCreateWithFlags(&b->own_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess)
        e = cudaMalloc((void **)&b->d_err, sizeof(int));
    if (e == cudaSuccess)
        e = cudaMemset(b->d_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        cb_free(b);
        return CB_ECUDA;
    }
    b->stream = b->own_stream;
    *out = b;
    return CB_OK;
}

void cb_free(cb_backend *b)
{
    if (!b)
        return;
    cudaSetDevice(b->device);
    if (b->own_stream)
        cudaStreamSynchronize(b->own_stream);
    cudaFree(b->scratch);
    cudaFree(b->d_err);
    if (b->pend) {
        int i;

        for (i = 0; i < CBI_PROF_PENDING; i++) {
            if (b->pend[i].ev[0])
                cudaEventDestroy(b->pend[i].ev[0]);
            if (b->pend[i].ev[1])
                cudaEventDestroy(b->pend[i].ev[1]);
        }
        free(b->pend);
    }
    if (b->own_stream)
        cudaStreamDestroy(b->own_stream);
    free(b);
}

const char *cb_last_error(const cb_backend *b)
{
    return b ? b->last_error : "no backend";
}

int cb_device(const cb_backend *b)
{
    return b ? b->device : -1;
}

int cb_num_sms(const cb_backend *b)
{
    return b ? b->num_sms : 0;
}

int cbi_scratch(cb_backend *b, size_t bytes, void **out)
{
    if (bytes > b->scratch_bytes) {
        void *p = NULL;
        cudaError_t e;

        /* The old buffer may still be read by queued work. */
        cudaStreamSynchronize(b->stream);
        cudaFree(b->scratch);
        b->scratch = NULL;
        b->scratch_bytes = 0;
        e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess)
            return cbi_fail(b, CB_EALLOC, "scratch");
        b->scratch = p;
        b->scratch_bytes = bytes;
    }
    *out = b->scratch;
    return CB_OK;
}

static int new_mem(void *ptr, size_t bytes, int dtype, int owned, cb_mem *out)
{
    cb_mem m = malloc(sizeof(*m));

    if (!m)
        return CB_EALLOC;
    m->ptr = ptr;
    m->bytes = bytes;
    m->dtype = dtype;
    m->owned = owned;
    *out = m;
    return CB_OK;
}

int cb_alloc(cb_backend *b, size_t bytes, int dtype, cb_mem *out)
{
    void *p = NULL;
    int rc;

    if (!out || !cbi_dtype_size(dtype))
        return cbi_fail(b, CB_EARG, "cb_alloc");
    *out = NULL;
    CB_TRY(cbi_enter(b));
    if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess)
        return cbi_fail(b, CB_EALLOC, "cb_alloc");
    rc = new_mem(p, bytes, dtype, 1, out);
    if (rc != CB_OK)
        cudaFree(p);
    return rc;
}

int cb_wrap(cb_backend *b, void *dptr, size_t bytes, int dtype, cb_mem *out)
{
    if (!out || !cbi_dtype_size(dtype))
        return cbi_fail(b, CB_EARG, "cb_wrap");
    return new_mem(dptr, bytes, dtype, 0, out);
}

int cb_write(cb_backend *b, cb_mem dst, size_t off, const void *src, size_t n)
{
    cudaError_t e;

    if (!dst || off + n > dst->bytes)
        return cbi_fail(b, CB_EARG, "cb_write");
    CB_TRY(cbi_enter(b));
    e = cudaMemcpyAsync((char *)dst->ptr + off, src, n, cudaMemcpyHostToDevice,
                        b->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(b->stream);
    return cbi_kstatus(b, (int)e, "cb_write");
}

int cb_read(cb_backend *b, cb_mem src, size_t off, void *dst, size_t n)
{
    cudaError_t e;

    if (!src || off + n > src->bytes)
        return cbi_fail(b, CB_EARG, "cb_read");
    CB_TRY(cbi_enter(b));
    e = cudaMemcpyAsync(dst, (const char *)src->ptr + off, n,
                        cudaMemcpyDeviceToHost, b->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(b->stream);
    return cbi_kstatus(b, (int)e, "cb_read");
}

int cb_upload(cb_backend *b, const void *src, size_t bytes, int dtype,
              cb_mem *out)
{
    int rc = cb_alloc(b, bytes, dtype, out);

    if (rc == CB_OK && bytes) {
        rc = cb_write(b, *out, 0, src, bytes);
        if (rc != CB_OK)
            cb_release(out);
    }
    return rc;
}

/* IEEE binary16, round to nearest even (the rounding the reference's
 * f32_to_f16 uses for precision=fp16 weights, ocl_backend.c:521-558). */
static uint16_t f32_to_f16_rne(float f)
{
    uint32_t x, sign, mag;
    int e;

    memcpy(&x, &f, 4);
    sign = (x >> 16) & 0x8000u;
    mag = x & 0x7fffffffu;
    if (mag >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (mag > 0x7f800000u ? 0x200u : 0));
    e = (int)(mag >> 23) - 127;
    if (e > 15)
        return (uint16_t)(sign | 0x7c00u);
    if (e < -25)
        return (uint16_t)sign;
    {
        /* Value = m * 2^(e-23) with the hidden bit; target ulp 2^-24 for
         * subnormals, 2^(e-10) otherwise. */
        uint32_t m = (mag & 0x7fffffu) | 0x800000u;
        int shift = e < -14 ? (-14 - e) + 13 : 13;
        uint32_t r = m >> shift, rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        uint32_t h;

        if (rem > half || (rem == half && (r & 1)))
            r++;
        if (e < -14)
            h = r; /* subnormal (a carry into 0x400 gives the smallest normal) */
        else
            h = ((uint32_t)(e + 15) << 10) + (r - 0x400u); /* carry may bump exp */
        return (uint16_t)(sign | h);
    }
}

int cb_upload_weight(cb_backend *b, const float *src, size_t count, int dtype,
                     cb_mem *out)
{
    int rc;

    if (dtype == CB_F32)
        return cb_upload(b, src, count * 4, CB_F32, out);
    if (dtype == CB_BF16) {
        void *tmp = NULL;

        CB_TRY(cb_alloc(b, count * 2, CB_BF16, out));
        rc = cbi_scratch(b, count * 4, &tmp);
        if (rc == CB_OK)
            rc = cbi_kstatus(b,
                            (int)cudaMemcpyAsync(tmp, src, count * 4,
                                                 cudaMemcpyHostToDevice, b->stream),
                            "cb_upload_weight");
        if (rc == CB_OK)
            rc = cbi_kstatus(b, k_cast_f32_bf16(tmp, (*out)->ptr, (long)count,
                                               (k_stream)b->stream),
                            "cb_upload_weight");
        if (rc == CB_OK)
            rc = cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream),
                            "cb_upload_weight");
        if (rc != CB_OK)
            cb_release(out);
        return rc;
    }
    if (dtype == CB_F16) {
        uint16_t *h = malloc(count * 2);
        size_t i;

        if (!h)
            return CB_EALLOC;
        for (i = 0; i < count; i++)
            h[i] = f32_to_f16_rne(src[i]);
        rc = cb_upload(b, h, count * 2, CB_F16, out);
        free(h);
        return rc;
    }
    return cbi_fail(b, CB_EDTYPE, "cb_upload_weight");
}

int cb_release(cb_mem *m)
{
    if (!m || !*m)
        return CB_OK;
    if ((*m)->owned)
        cudaFree((*m)->ptr);
    free(*m);
    *m = NULL;
    return CB_OK;
}

void *cb_ptr(cb_mem m)
{
    return m ? m->ptr : NULL;
}

size_t cb_bytes(cb_mem m)
{
    return m ? m->bytes : 0;
}

int cb_dtype(cb_mem m)
{
    return m ? m->dtype : -1;
}

int cb_device_error(cb_backend *b)
{
    int v = 0;

    if (cbi_enter(b) != CB_OK)
        return -1;
    if (cudaMemcpy(&v, b->d_err, sizeof(int), cudaMemcpyDeviceToHost) !=
        cudaSuccess)
        return -1;
    return v;
}

int cb_clear_error(cb_backend *b)
{
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b, (int)cudaMemset(b->d_err, 0, sizeof(int)),
                      "cb_clear_error");
}

int cb_sync(cb_backend *b)
{
    int v;

    CB_TRY(cbi_enter(b));
    CB_TRY(cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "cb_sync"));
    v = cb_device_error(b);
    if (v > 0)
        return cbi_fail(b, CB_ETIMEOUT, "cb_sync");
    return v < 0 ? cbi_fail(b, CB_ECUDA, "cb_sync") : CB_OK;
}

/* ---------------------------------------------------------------- profile */

static void prof_fold(cb_backend *b)
{
    int i;

    for (i = 0; i < b->prof_npend; i++) {
        struct cbi_prof_pending *p = &b->pend[i];
        float ms = 0.0f;

        if (cudaEventElapsedTime(&ms, p->ev[0], p->ev[1]) == cudaSuccess)
            b->prof[p->entry].ms += ms;
    }
    b->prof_npend = 0;
}

int cb_profile(cb_backend *b, int on)
{
    int i;

    if (!b)
        return CB_EARG;
    CB_TRY(cbi_enter(b));
    if (on && !b->pend) {
        b->pend = calloc(CBI_PROF_PENDING, sizeof(*b->pend));
        if (!b->pend)
            return CB_EALLOC;
        for (i = 0; i < CBI_PROF_PENDING; i++)
            if (cudaEventCreate(&b->pend[i].ev[0]) != cudaSuccess ||
                cudaEventCreate(&b->pend[i].ev[1]) != cudaSuccess)
                return cbi_fail(b, CB_ECUDA, "cb_profile");
    }
    if (on) {
        cudaStreamSynchronize(b->stream);
        b->prof_n = 0;
        b->prof_npend = 0;
        memset(b->prof, 0, sizeof(b->prof));
    }
    b->prof_on = on;
    b->prof_cur = -1;
    return CB_OK;
}

void cbi_prof_begin(cb_backend *b, const char *name, double flops, double bytes)
{
    int i;

    b->prof_cur = -1;
    if (!b->prof_on)
        return;
    if (b->prof_npend == CBI_PROF_PENDING) {
        /* out of event pairs: fold what has completed so far */
        cudaStreamSynchronize(b->stream);
        prof_fold(b);
    }
    for (i = 0; i < b->prof_n && strcmp(b->prof[i].name, name) != 0; i++)
        ;
    if (i == b->prof_n) {
        if (b->prof_n == CBI_PROF_ENTRIES)
            return;
        b->prof[b->prof_n++].name = name;
    }
    b->prof[i].calls++;
    b->prof[i].flops += flops;
    b->prof[i].bytes += bytes;
    b->pend[b->prof_npend].entry = i;
    cudaEventRecord(b->pend[b->prof_npend].ev[0], b->stream);
    b->prof_cur = i;
}

void cbi_prof_end(cb_backend *b)
{
    if (!b->prof_on || b->prof_cur < 0)
        return;
    cudaEventRecord(b->pend[b->prof_npend].ev[1], b->stream);
    b->prof_npend++;
    b->prof_cur = -1;
}

int cb_profile_entry(cb_backend *b, int i, const char **name, long *calls,
                     double *ms, double *flops, double *bytes)
{
    if (!b)
        return CB_EARG;
    CB_TRY(cbi_enter(b));
    if (b->prof_npend) {
        CB_TRY(cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "cb_profile_entry"));
        prof_fold(b);
    }
    if (i < 0 || i >= b->prof_n)
        return CB_EARG;
    if (name)
        *name = b->prof[i].name;
    if (calls)
        *calls = b->prof[i].calls;
    if (ms)
        *ms = b->prof[i].ms;
    if (flops)
        *flops = b->prof[i].flops;
    if (bytes)
        *bytes = b->prof[i].bytes;
    return CB_OK;
}

int cb_set_stream(cb_backend *b, void *stream)
{
    cudaStream_t next;

    if (!b)
        return CB_EARG;
    next = stream ? (cudaStream_t)stream : b->own_stream;
    if (next != b->stream) {
        /* the backend's scratch buffer is reused by every launch: work on
         * the new stream starts after the old stream's */
        cudaEvent_t ev;

        CB_TRY(cbi_enter(b));
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess)
            return cbi_fail(b, CB_ECUDA, "set_stream: event");
        if (cudaEventRecord(ev, b->stream) != cudaSuccess ||
            cudaStreamWaitEvent(next, ev, 0) != cudaSuccess) {
            cudaEventDestroy(ev);
            return cbi_fail(b, CB_ECUDA, "set_stream: order");
        }
        cudaEventDestroy(ev);
    }
    b->stream = next;
    return CB_OK;
}

void *cb_stream(const cb_backend *b)
{
    return b ? (void *)b->stream : NULL;
}

int cb_synth_normal(cb_backend *b, uint64_t seed, uint64_t stream, float mean,
                    float std, cb_mem out, size_t count)
{
    if (!out || (out->dtype != CB_F32 && out->dtype != CB_BF16) ||
        count * cbi_dtype_size(out->dtype) > out->bytes)
        return cbi_fail(b, CB_EARG, "cb_synth_normal");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_synth_normal(seed, stream, (long)count, mean, std,
                                     out->ptr, out->dtype == CB_BF16,
                                     (k_stream)b->stream),
                      "cb_synth_normal");
}
