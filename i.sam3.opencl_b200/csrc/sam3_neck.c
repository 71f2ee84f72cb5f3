/* SPDX-License-Identifier: Unlicense */
/* The SimpleFPN neck of the point-prompt head and the decoder's
 * high-resolution projections (sam3_model.c: load_neck :585-622,
 * load_point_neck :642-654, conv3x3 :1032-1054, convt2x2 :1058-1065,
 * neck_level :1071-1095, point_neck :1098-1110), batched over tiles.
 *
 * Every convolution is a tcgen05 GEMM with bf16 operands and fp32
 * accumulation:
 *   - ConvTranspose 2x2 / stride 2: the GEMM of the map with the weight
 *     stored as [cout * 4, cin] in sub-pixel-major row order (d * cout + co),
 *     so each 64-column chunk of a row is 64 channels of one output pixel;
 *     the epilogue adds the bias, applies the activation and writes them
 *     into the upsampled bf16 map (the next GEMM's operand);
 *   - 1x1: a GEMM with the bias in its epilogue, bf16 out;
 *   - 3x3 / pad 1: an implicit GEMM (k_conv3x3_bf16_tc) against the weight
 *     permuted to tap-major columns ((ky * 3 + kx) * 256 + c): each K block
 *     is a TMA load of the input map at the tap's shifted 8 x 16 pixel
 *     block, zero outside the map, so no im2col is written (the reference
 *     materialises one in 128 MB bands); the image embedding's no_mem_embed
 *     add (sam3_model.c:1109) is the GEMM's broadcast residual.
 * The conv_s0 / conv_s1 projections read the level outputs in bf16 and
 * write the decoder's fp32 feat_s0 / feat_s1. */
#include <stdlib.h>
#include <string.h>

#include "backend_internal.h"
#include "sam3_synth.h"

#define NECK_DIM 256

struct cb_neck {
    cb_backend *b;
    int grid, E, max_tiles, T;
    void *w[SAM3_NT_COUNT]; /* bf16 GEMM weights (layouts above), fp32 vectors */
    void *xb;               /* bf16 [R, E], R = max_tiles * T */
    void *a0;               /* bf16 [4R, E / 2] */
    void *a1;               /* bf16 [16R, E / 4] */
    void *c1;               /* bf16 [16R, 256] */
    void *c3;               /* bf16 [16R, 256] */
};

static int neck_is_matrix(int i, int E)
{
    int r, c, k;

    sam3_neck_tensor(i, E, &r, &c, &k);
    return r > 0 && k == SAM3_INIT_W;
}

static int nalloc(cb_neck *n, void **p, size_t bytes)
{
    if (cudaMalloc(p, bytes ? bytes : 16) != cudaSuccess) {
        *p = NULL;
        return cbi_fail(n->b, CB_EALLOC, "neck buffers");
    }
    return CB_OK;
}

void cb_neck_free(cb_neck *n)
{
    int i;

    if (!n)
        return;
    cbi_enter(n->b);
    cudaStreamSynchronize(n->b->stream);
    for (i = 0; i < SAM3_NT_COUNT; i++)
        cudaFree(n->w[i]);
    cudaFree(n->xb);
    cudaFree(n->a0);
    cudaFree(n->a1);
    cudaFree(n->c1);
    cudaFree(n->c3);
    free(n);
}

int cb_neck_create(cb_backend *b, int grid, int embed, int max_tiles, cb_neck **out)
{
    cb_neck *n;
    size_t R, T;
    int i, rc = CB_OK;

    if (!b || !out)
        return CB_EARG;
    *out = NULL;
    if (grid <= 0 || grid > 512 || embed <= 0 || embed % 64 || max_tiles <= 0)
        return cbi_fail(b, CB_EARG, "neck config");
    CB_TRY(cbi_enter(b));
    n = calloc(1, sizeof(*n));
    if (!n)
        return CB_EALLOC;
    n->b = b;
    n->grid = grid;
    n->E = embed;
    n->max_tiles = max_tiles;
    n->T = grid * grid;
    T = (size_t)n->T;
    R = (size_t)max_tiles * T;
#define A(p, bytes) \
    if (rc == CB_OK) rc = nalloc(n, (void **)&(p), (bytes))
    for (i = 0; i < SAM3_NT_COUNT; i++) {
        int r, c, k;

        sam3_neck_tensor(i, embed, &r, &c, &k);
        A(n->w[i], (size_t)r * c * (neck_is_matrix(i, embed) ? 2 : 4));
    }
    A(n->xb, R * embed * 2);
    A(n->a0, 4 * R * (embed / 2) * 2);
    A(n->a1, 16 * R * (embed / 4) * 2);
    A(n->c1, 16 * R * NECK_DIM * 2);
    A(n->c3, 16 * R * NECK_DIM * 2);
#undef A
    if (rc != CB_OK) {
        cb_neck_free(n);
        return rc;
    }
    *out = n;
    return CB_OK;
}

/* Device copy of tensor i from fp32 values on the device (checkpoint
 * layout): ConvTranspose weights -> bf16 [cout * 4, cin] sub-pixel-major,
 * 3x3 weights -> bf16 [cout, 9 * cin] tap-major, other matrices -> bf16 as
 * they are, vectors fp32. */
static int neck_store(cb_neck *n, int i, const float *f32)
{
    cb_backend *b = n->b;
    const k_stream st = (k_stream)b->stream;
    int r, c, k, t;

    sam3_neck_tensor(i, n->E, &r, &c, &k);
    if (!r)
        return CB_OK;
    t = i < SAM3_NT_S0_W ? i % 8 : -1;
    if (t == 0 || t == 2)
        return cbi_kstatus(b, k_transpose_cast_bf16(f32, r, c, 1, n->w[i], st), "neck weights");
    if (t == 6)
        return cbi_kstatus(b, k_permute_conv3x3_bf16(f32, r, c / 9, n->w[i], st), "neck weights");
    if (neck_is_matrix(i, n->E))
        return cbi_kstatus(b, k_cast_f32_bf16(f32, n->w[i], (long)r * c, st), "neck weights");
    return cbi_kstatus(b,
                       (int)cudaMemcpyAsync(n->w[i], f32, (size_t)r * c * 4,
                                            cudaMemcpyDeviceToDevice, b->stream),
                       "neck weights");
}

int cb_neck_init_random(cb_neck *n, uint64_t seed, float std)
{
    cb_backend *b;
    void *s = NULL;
    int i;

    if (!n)
        return CB_EARG;
    b = n->b;
    CB_TRY(cbi_enter(b));
    CB_TRY(cbi_scratch(b, (size_t)n->E * n->E * 2 * 4, &s));
    for (i = 0; i < SAM3_NT_COUNT; i++) {
        int r, c, k;

        sam3_neck_tensor(i, n->E, &r, &c, &k);
        if (!r)
            continue;
        CB_TRY(cbi_kstatus(b,
                           k_synth_normal(seed, SAM3_STREAM_NECKW + (uint64_t)i, (long)r * c,
                                          0.0f, std, s, 0, (k_stream)b->stream),
                           "neck init"));
        CB_TRY(neck_store(n, i, (const float *)s));
        /* the scratch buffer is reused by the next tensor */
        CB_TRY(cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "neck init"));
    }
    return CB_OK;
}

int cb_neck_set_weight(cb_neck *n, int which, const float *src, size_t count)
{
    cb_backend *b;
    void *s = NULL;
    int r, c, k;

    if (!n || !src)
        return CB_EARG;
    b = n->b;
    if (which < 0 || which >= SAM3_NT_COUNT)
        return cbi_fail(b, CB_EARG, "neck set_weight: tensor");
    sam3_neck_tensor(which, n->E, &r, &c, &k);
    if (!r || count != (size_t)r * c)
        return cbi_fail(b, CB_EARG, "neck set_weight: shape");
    CB_TRY(cbi_enter(b));
    CB_TRY(cbi_scratch(b, count * 4, &s));
    CB_TRY(cbi_kstatus(b,
                       (int)cudaMemcpyAsync(s, src, count * 4, cudaMemcpyHostToDevice, b->stream),
                       "neck set_weight"));
    CB_TRY(neck_store(n, which, (const float *)s));
    return cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "neck set_weight");
}

/* One launch bracketed by the profiler, its result mapped to a status. */
#define LAUNCH(name, flops, bytes, call)                                       \
    do {                                                                       \
        int lrc_;                                                              \
        cbi_prof_begin(b, name, (double)(flops), (double)(bytes));             \
        lrc_ = (call);                                                         \
        cbi_prof_end(b);                                                       \
        CB_TRY(cbi_kstatus(b, lrc_, name));                                    \
    } while (0)

/* C[rows, N] = A[rows, K] W^T (+ bias) (+ R[m % rmod]); A bf16, C bf16 or
 * fp32. */
static int ngemm(cb_neck *n, const char *name, const void *A, long rows, int K, int N, int wi,
                 int bi, void *C, int c_bf16, const float *R, int rmod)
{
    cb_backend *b = n->b;
    const double dr = (double)rows;

    LAUNCH(name, 2.0 * dr * K * N, dr * K * 2 + (double)K * N * 2 + dr * N * (c_bf16 ? 2 : 4),
           k_gemm_bf16_tc((int)rows, N, K, A, K, n->w[wi], K, C, N, c_bf16,
                          bi >= 0 ? (const float *)n->w[bi] : NULL, R, N, rmod, 1.0f,
                          K_ACT_NONE, NULL, b->d_err, b->num_sms, (k_stream)b->stream));
    return CB_OK;
}

/* convt2x2 (sam3_model.c:1058-1065) of nt maps H x W x cin (bf16 A): one
 * GEMM whose epilogue adds the bias, applies the activation and writes the
 * upsampled map out bf16 [nt, 2H, 2W, cout]. */
static int convt(cb_neck *n, const void *A, int nt, int H, int W, int cin, int cout, int wi,
                 int bi, int act, void *out)
{
    cb_backend *b = n->b;
    const double rows = (double)nt * H * W;

    LAUNCH("neck_gemm_convt", 2.0 * rows * cin * 4 * cout,
           rows * cin * 2 + 4.0 * cout * cin * 2 + rows * 4 * cout * 2,
           k_convt2x2_bf16_tc(A, nt, H, W, cin, n->w[wi], cout, (const float *)n->w[bi], act, out,
                              b->d_err, b->num_sms, (k_stream)b->stream));
    return CB_OK;
}

/* conv3x3 (sam3_model.c:1032-1054) of nt maps side x side x 256 (bf16 X)
 * as one implicit tcgen05 GEMM (no im2col), + bias (+ R broadcast row). */
static int conv3(cb_neck *n, const void *X, int nt, int side, int wi, int bi, void *out,
                 int out_bf16, const float *R)
{
    cb_backend *b = n->b;
    const double rows = (double)nt * side * side;

    LAUNCH("neck_conv3x3", 2.0 * rows * 9 * NECK_DIM * NECK_DIM,
           rows * NECK_DIM * 2 + 9.0 * NECK_DIM * NECK_DIM * 2 + rows * NECK_DIM * (out_bf16 ? 2 : 4),
           k_conv3x3_bf16_tc(X, nt, side, side, NECK_DIM, n->w[wi], NECK_DIM,
                             (const float *)n->w[bi], R, out, out_bf16, b->d_err, b->num_sms,
                             (k_stream)b->stream));
    return CB_OK;
}

#define LV(l, t) (SAM3_NT_LEVEL + 8 * (l) + (t))

int cb_neck_run(cb_neck *n, cb_mem x, int ntile, cb_mem emb, cb_mem feat_s0, cb_mem feat_s1)
{
    cb_backend *b;
    int G, E;
    long R;

    if (!n || !x || !emb || !feat_s0 || !feat_s1)
        return CB_EARG;
    b = n->b;
    G = n->grid;
    E = n->E;
    R = (long)ntile * n->T;
    if (ntile <= 0 || ntile > n->max_tiles || x->dtype != CB_F32 || emb->dtype != CB_F32 ||
        feat_s0->dtype != CB_F32 || feat_s1->dtype != CB_F32 ||
        x->bytes < (size_t)R * E * 4 || emb->bytes < (size_t)R * NECK_DIM * 4 ||
        feat_s0->bytes < (size_t)16 * R * 32 * 4 || feat_s1->bytes < (size_t)4 * R * 64 * 4)
        return cbi_fail(b, CB_EARG, "neck_run: shapes");
    CB_TRY(cbi_enter(b));
    LAUNCH("neck_cast", 0, (double)R * E * 6,
           k_cast_f32_bf16((const float *)x->ptr, n->xb, R * E, (k_stream)b->stream));

    /* level 0, scale 4: ConvT E -> E/2 (GELU), ConvT E/2 -> E/4, 1x1, 3x3;
     * then conv_s0 (sam3_model.c:1076-1083, 1102-1103) */
    CB_TRY(convt(n, n->xb, ntile, G, G, E, E / 2, LV(0, 0), LV(0, 1), K_ACT_GELU, n->a0));
    CB_TRY(convt(n, n->a0, ntile, 2 * G, 2 * G, E / 2, E / 4, LV(0, 2), LV(0, 3), K_ACT_NONE,
                 n->a1));
    CB_TRY(ngemm(n, "neck_gemm_1x1", n->a1, 16 * R, E / 4, NECK_DIM, LV(0, 4), LV(0, 5), n->c1, 1,
                 NULL, 0));
    CB_TRY(conv3(n, n->c1, ntile, 4 * G, LV(0, 6), LV(0, 7), n->c3, 1, NULL));
    CB_TRY(ngemm(n, "neck_gemm_s", n->c3, 16 * R, NECK_DIM, 32, SAM3_NT_S0_W, SAM3_NT_S0_B,
                 feat_s0->ptr, 0, NULL, 0));

    /* level 1, scale 2: ConvT E -> E/2, 1x1, 3x3; then conv_s1 */
    CB_TRY(convt(n, n->xb, ntile, G, G, E, E / 2, LV(1, 0), LV(1, 1), K_ACT_NONE, n->a0));
    CB_TRY(ngemm(n, "neck_gemm_1x1", n->a0, 4 * R, E / 2, NECK_DIM, LV(1, 4), LV(1, 5), n->c1, 1,
                 NULL, 0));
    CB_TRY(conv3(n, n->c1, ntile, 2 * G, LV(1, 6), LV(1, 7), n->c3, 1, NULL));
    CB_TRY(ngemm(n, "neck_gemm_s", n->c3, 4 * R, NECK_DIM, 64, SAM3_NT_S1_W, SAM3_NT_S1_B,
                 feat_s1->ptr, 0, NULL, 0));

    /* level 2, scale 1: 1x1, 3x3, + no_mem_embed -> the image embedding */
    CB_TRY(ngemm(n, "neck_gemm_1x1", n->xb, R, E, NECK_DIM, LV(2, 4), LV(2, 5), n->c1, 1, NULL,
                 0));
    CB_TRY(conv3(n, n->c1, ntile, G, LV(2, 6), LV(2, 7), emb->ptr, 0,
                 (const float *)n->w[SAM3_NT_NO_MEM]));
    return CB_OK;
}
