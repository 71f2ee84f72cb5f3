/* SPDX-License-Identifier: Unlicense */
/* Private definitions shared by the C host files of the backend. */
#ifndef SAM3_BACKEND_INTERNAL_H
#define SAM3_BACKEND_INTERNAL_H

#include <cuda_runtime_api.h>

#include "kernels.h"
#include "sam3_cuda.h"

#define CBI_PROF_ENTRIES 64
#define CBI_PROF_PENDING 4096

struct cbi_prof_entry {
    const char *name;
    long calls;
    double ms, flops, bytes;
};

struct cbi_prof_pending {
    int entry;
    cudaEvent_t ev[2];
};

struct cb_backend {
    int device;
    int num_sms;
    cudaStream_t own_stream;
    cudaStream_t stream;
    int *d_err;          /* device error word written by kernels */
    void *scratch;       /* grown on demand (cbi_scratch) */
    size_t scratch_bytes;
    char last_error[256];
    /* profiler */
    int prof_on;
    int prof_n;
    struct cbi_prof_entry prof[CBI_PROF_ENTRIES];
    int prof_npend;
    struct cbi_prof_pending *pend; /* CBI_PROF_PENDING event pairs */
    int prof_cur;                  /* entry of the open bracket, -1 none */
};

struct cb_mem_s {
    void *ptr;
    size_t bytes;
    int dtype;
    int owned;
};

/* Record a failure on the backend and return its status code. */
int cbi_fail(cb_backend *b, int status, const char *what);
/* Map a launcher result (cudaError_t or K_E*) to a status code. */
int cbi_kstatus(cb_backend *b, int rc, const char *what);
/* Make the current device the backend's (every entry point calls this). */
int cbi_enter(cb_backend *b);
/* Scratch buffer of at least `bytes` on the backend's device. */
int cbi_scratch(cb_backend *b, size_t bytes, void **out);
size_t cbi_dtype_size(int dtype);
/* Profiler brackets around one kernel launch (no-ops when profiling is
 * off): name must be a string literal. */
void cbi_prof_begin(cb_backend *b, const char *name, double flops,
                    double bytes);
void cbi_prof_end(cb_backend *b);

#define CB_TRY(x)                                                              \
    do {                                                                       \
        int rc_ = (x);                                                         \
        if (rc_ != CB_OK)                                                      \
            return rc_;                                                        \
    } while (0)

#endif
