/* SPDX-License-Identifier: Unlicense */
/* The point-prompt mask decoder (sam3_model.c: load_decoder :656-755,
 * decoder caches :877-902 and :1153-1170, pe_encode :760-773, sam_decode
 * :1239-1399) on the B200 kernels of this library.
 *
 * Data flow and precision. The token stream (P * 8 rows of 256) and the
 * per-prompt image stream ("keys", P * 5184 rows of 256) stay fp32, as in
 * the reference; every Linear runs on the tcgen05 GEMM with bf16 operands
 * and fp32 accumulation, its fp32 input rounded to bf16 once. The decoder
 * attention (k_mha) reads fp32 Q/K/V. Fusions against the reference's op
 * sequence:
 *   - keys = Linear(bo) + src: the add_bcast of src (shared by all
 *     prompts) is the GEMM epilogue's residual with row m % 5184;
 *   - the LayerNorm of keys (norm4) also writes bf16(keys) and
 *     bf16(keys + dense PE), the operands of the next token -> image
 *     attention's projections, of layer 1's image queries and of the first
 *     upscaling GEMM: no separate add_bcast or cast passes over keys;
 *   - the ConvTranspose weights are stored as [cout * 4, cin] bf16, so both
 *     upscaling convolutions are plain tcgen05 GEMMs; the first one's
 *     scatter + feat_s1 + LayerNorm2d + GELU is one pass writing bf16, the
 *     second one's scatter + feat_s0 + GELU is dotted with the
 *     hypernetwork outputs in the same pass, so the [P, 288, 288, 32] map
 *     is never stored;
 *   - the hypernetwork and IoU MLPs run on the device (dec_heads), so the
 *     decode does not stop for a host round trip before the logits.
 * Everything runs on the backend stream; cb_decode blocks only to return
 * the IoU predictions. */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "backend_internal.h"
#include "sam3_synth.h"

#define DEC_GRID 72
#define DEC_T (DEC_GRID * DEC_GRID)
#define DEC_DIM 256
#define DEC_NTOK 8
#define DEC_IMG 1008
#define DEC_LOWRES 288
#define DEC_EPS 1e-5f
#define LN2D_EPS 1e-6f

/* Tensors that are GEMM weights (stored bf16 on the device). */
static int is_gemm_weight(int i)
{
    int r, c, k;

    if (i == SAM3_DT_UP0_W || i == SAM3_DT_UP3_W)
        return 1;
    if (i >= SAM3_DT_NF_W)
        return 0;
    sam3_dec_tensor(i, &r, &c, &k);
    return k == SAM3_INIT_W;
}

/* Tensors the host needs (prompt encoding, token setup). */
static int is_host_tensor(int i)
{
    return i >= SAM3_DT_GAUSS;
}

struct cb_decoder {
    cb_backend *b;
    int batch;
    void *w[SAM3_DT_COUNT];     /* device: bf16 [out, in] GEMM weights, else fp32 */
    float *hw[SAM3_DT_COUNT];   /* host copies of the prompt-side tensors */
    int have_image;
    /* image-side state (sam_encode's decoder caches) */
    float *src, *srcpe, *pe_img, *kp0, *vp0, *qp0, *feat_s0, *feat_s1;
    /* token stream [batch * 8, 256] and its scratch */
    float *qpe, *qry, *sq, *sk, *sv, *so, *sh;
    void *tok_bf16;             /* bf16 [batch * 8, 2048] GEMM operand */
    /* layer 1's token -> image key projection and image -> token query
     * projection stacked ([256, 256] bf16 weight, [256] bias): both read
     * kin, so one GEMM writes [keys | queries] rows of 256 */
    void *w_kq1;
    float *b_kq1;
    void *qv_bf16;              /* bf16(qry) [batch * 8, 256] from a layer's
                                 * last token norm: input of its image ->
                                 * token values and of the next layer's
                                 * self-attention values */
    /* per-prompt image stream */
    float *keys;                /* [batch * T, 256] */
    void *keys_bf16, *kin_bf16; /* bf16 [batch * T, 256] */
    float *bk, *bv;             /* [batch * T, 128] fp32-sized: bf16 keys /
                                 * values of the token -> image attention
                                 * (layer 1: bk holds [keys | queries] rows
                                 * of 256 bf16) */
    void *bo_bf16;              /* bf16 [batch * T, 128] */
    void *u1_bf16;              /* bf16 [batch * 4T, 64] */
    float *hyper, *iou;         /* [batch, 96], [batch, 3] */
    void *mha_ws;
    size_t mha_ws_bytes;
    /* layer 0's token -> image attention on the tensor cores: the shared
     * keys / values with heads padded to 64 columns (bf16 [T, 512], set
     * with the image), the queries in that layout, and the key-split
     * workspace (the kernel writes the 16 real columns of each head) */
    void *k0_pad, *v0_pad, *q_pad;
    void *xws;
    size_t xws_bytes;
    float *h_tok;               /* host [batch * 8, 256] */
};

static int dalloc(cb_decoder *d, void **p, size_t bytes)
{
    if (cudaMalloc(p, bytes ? bytes : 16) != cudaSuccess) {
        *p = NULL;
        return cbi_fail(d->b, CB_EALLOC, "decoder buffers");
    }
    return CB_OK;
}

void cb_decoder_free(cb_decoder *d)
{
    int i;

    if (!d)
        return;
    cbi_enter(d->b);
    cudaStreamSynchronize(d->b->stream);
    for (i = 0; i < SAM3_DT_COUNT; i++) {
        cudaFree(d->w[i]);
        free(d->hw[i]);
    }
    {
        void *dev[] = {d->src, d->srcpe, d->pe_img, d->kp0, d->vp0, d->qp0, d->feat_s0,
                       d->feat_s1, d->qpe, d->qry, d->sq, d->sk, d->sv, d->so,
                       d->sh, d->tok_bf16, d->qv_bf16, d->w_kq1, d->b_kq1, d->keys,
                       d->keys_bf16, d->kin_bf16,
                       d->bk, d->bv, d->bo_bf16, d->u1_bf16,
                       d->hyper, d->iou, d->mha_ws, d->k0_pad, d->v0_pad, d->q_pad,
                       d->xws};

        for (i = 0; i < (int)(sizeof(dev) / sizeof(dev[0])); i++)
            cudaFree(dev[i]);
    }
    free(d->h_tok);
    free(d);
}

int cb_decoder_create(cb_backend *b, int batch, cb_decoder **out)
{
    cb_decoder *d;
    const size_t T = DEC_T, B = (size_t)batch, nt = B * DEC_NTOK;
    size_t ws_t2i, ws_i2t;
    int i, rc = CB_OK;

    if (!b || !out)
        return CB_EARG;
    *out = NULL;
    if (batch <= 0 || batch > 1024)
        return cbi_fail(b, CB_EARG, "decoder batch");
    CB_TRY(cbi_enter(b));
    d = calloc(1, sizeof(*d));
    if (!d)
        return CB_EALLOC;
    d->b = b;
    d->batch = batch;
#define A(p, n) \
    if (rc == CB_OK) rc = dalloc(d, (void **)&(p), (n))
    for (i = 0; i < SAM3_DT_COUNT; i++) {
        int r, c, k;

        sam3_dec_tensor(i, &r, &c, &k);
        A(d->w[i], (size_t)r * c * (is_gemm_weight(i) ? 2 : 4));
        if (rc == CB_OK && is_host_tensor(i)) {
            d->hw[i] = calloc((size_t)r * c, sizeof(float));
            if (!d->hw[i])
                rc = CB_EALLOC;
        }
    }
    A(d->src, T * DEC_DIM * 4);
    A(d->srcpe, T * DEC_DIM * 4);
    A(d->pe_img, T * DEC_DIM * 4);
    A(d->kp0, T * 128 * 4);
    A(d->vp0, T * 128 * 4);
    A(d->qp0, T * 128 * 4);
    A(d->feat_s0, 16 * T * 32 * 4);
    A(d->feat_s1, 4 * T * 64 * 4);
    A(d->qpe, nt * DEC_DIM * 4);
    A(d->qry, nt * DEC_DIM * 4);
    A(d->sq, nt * DEC_DIM * 4);
    A(d->sk, nt * DEC_DIM * 4);
    A(d->sv, nt * DEC_DIM * 4);
    A(d->so, nt * DEC_DIM * 4);
    A(d->sh, nt * 2048 * 4);
    A(d->tok_bf16, nt * 2048 * 2);
    A(d->qv_bf16, nt * DEC_DIM * 2);
    A(d->w_kq1, (size_t)256 * DEC_DIM * 2);
    A(d->b_kq1, (size_t)256 * 4);
    A(d->keys, B * T * DEC_DIM * 4);
    A(d->keys_bf16, B * T * DEC_DIM * 2);
    A(d->kin_bf16, B * T * DEC_DIM * 2);
    A(d->bk, B * T * 128 * 4);
    A(d->bv, B * T * 128 * 4);
    A(d->bo_bf16, B * T * 128 * 2);
    A(d->u1_bf16, B * 4 * T * 64 * 2);
    A(d->hyper, B * 96 * 4);
    A(d->iou, B * 3 * 4);
    ws_t2i = k_mha_workspace(batch, DEC_NTOK, DEC_T, 128, b->num_sms);
    ws_i2t = k_mha_workspace(batch, DEC_T, DEC_NTOK, 128, b->num_sms);
    d->mha_ws_bytes = ws_t2i > ws_i2t ? ws_t2i : ws_i2t;
    A(d->mha_ws, d->mha_ws_bytes);
    A(d->k0_pad, T * 512 * 2);
    A(d->v0_pad, T * 512 * 2);
    A(d->q_pad, nt * 512 * 2);
    for (i = 1; i <= batch; i++) {  /* fewer prompts split the keys more */
        const size_t w = k_attn_tc_cross_workspace(1, i * DEC_NTOK, DEC_T, 8);

        if (w > d->xws_bytes)
            d->xws_bytes = w;
    }
    A(d->xws, d->xws_bytes);
#undef A
    if (rc == CB_OK) {
        d->h_tok = malloc(nt * DEC_DIM * sizeof(float));
        if (!d->h_tok)
            rc = CB_EALLOC;
    }
    if (rc != CB_OK) {
        cb_decoder_free(d);
        return rc;
    }
    *out = d;
    return CB_OK;
}

/* ---------------------------------------------------------------- weights */

/* One launch bracketed by the profiler, its result mapped to a status. */
#define LAUNCH(name, flops, bytes, call)                                       \
    do {                                                                       \
        int lrc_;                                                              \
        cbi_prof_begin(b, name, (double)(flops), (double)(bytes));             \
        lrc_ = (call);                                                         \
        cbi_prof_end(b);                                                       \
        CB_TRY(cbi_kstatus(b, lrc_, name));                                    \
    } while (0)

/* PositionEmbeddingRandom of normalised (x, y) (pe_encode,
 * sam3_model.c:760-773): 128 sines then 128 cosines of
 * 2 pi (x' g[i] + y' g[128 + i]), x' = 2x - 1, y' = 2y - 1. */
static void pe_encode(const float *gauss, float x, float y, float *out)
{
    int i;

    x = 2.0f * x - 1.0f;
    y = 2.0f * y - 1.0f;
    for (i = 0; i < DEC_DIM / 2; i++) {
        float v = x * gauss[i] + y * gauss[DEC_DIM / 2 + i];

        v *= 2.0f * (float)M_PI;
        out[i] = sinf(v);
        out[DEC_DIM / 2 + i] = cosf(v);
    }
}

/* Dense positional encoding of the 72 x 72 grid (sam3_model.c:886-892). */
static int compute_pe_img(cb_decoder *d)
{
    cb_backend *b = d->b;
    float *pe = malloc((size_t)DEC_T * DEC_DIM * sizeof(float));
    int x, y, rc;

    if (!pe)
        return CB_EALLOC;
    for (y = 0; y < DEC_GRID; y++)
        for (x = 0; x < DEC_GRID; x++)
            pe_encode(d->hw[SAM3_DT_GAUSS], (x + 0.5f) / DEC_GRID, (y + 0.5f) / DEC_GRID,
                      pe + ((size_t)y * DEC_GRID + x) * DEC_DIM);
    rc = cbi_kstatus(b,
                     (int)cudaMemcpyAsync(d->pe_img, pe, (size_t)DEC_T * DEC_DIM * 4,
                                          cudaMemcpyHostToDevice, b->stream),
                     "decoder pe");
    if (rc == CB_OK)
        rc = cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "decoder pe");
    free(pe);
    return rc;
}

/* Decoder tensor indices: attention block blk's tensor t, layer l's
 * tensor t. */
#define ATT(blk, t) (SAM3_DT_ATTN + 8 * (blk) + (t))
#define LAY(l, t) (SAM3_DT_LAYER + 12 * (l) + (t))
enum { QW = 0, QB, KW, KB, VW, VB, OW, OB };
enum { N1W = 0, N1B, N2W, N2B, N3W, N3B, N4W, N4B, M1W, M1B, M2W, M2B };

/* Device copy of tensor i from fp32 values already on the device (rows x
 * cols in the checkpoint layout): bf16 for GEMM weights (the ConvTranspose
 * ones transposed to [cout * 4, cin]), fp32 otherwise. */
static int store_tensor(cb_decoder *d, int i, const float *f32)
{
    cb_backend *b = d->b;
    const k_stream st = (k_stream)b->stream;
    int r, c, k;

    sam3_dec_tensor(i, &r, &c, &k);
    /* ConvTranspose weights [cin, cout * 4] -> GEMM operands [cout * 4, cin]
     * with rows in sub-pixel-major order d * cout + co: a sub-pixel's
     * channels are one column chunk of the GEMM's fused epilogue. */
    if (i == SAM3_DT_UP0_W || i == SAM3_DT_UP3_W)
        return cbi_kstatus(b, k_transpose_cast_bf16(f32, r, c, 1, d->w[i], st),
                           "decoder weights");
    if (is_gemm_weight(i))
        CB_TRY(cbi_kstatus(b, k_cast_f32_bf16(f32, d->w[i], (long)r * c, st),
                           "decoder weights"));
    else
        CB_TRY(cbi_kstatus(b,
                           (int)cudaMemcpyAsync(d->w[i], f32, (size_t)r * c * 4,
                                                cudaMemcpyDeviceToDevice, b->stream),
                           "decoder weights"));
    /* the stacked copy of layer 1's key (rows 0-127) and query (128-255)
     * projections */
    {
        const int kq = i == ATT(SAM3_DA_L1_T2I, KW) || i == ATT(SAM3_DA_L1_T2I, KB) ? 0
                       : i == ATT(SAM3_DA_L1_I2T, QW) || i == ATT(SAM3_DA_L1_I2T, QB) ? 1
                                                                                       : -1;
        if (kq >= 0) {
            const int w = i == ATT(SAM3_DA_L1_T2I, KW) || i == ATT(SAM3_DA_L1_I2T, QW);
            const size_t bytes = w ? (size_t)128 * DEC_DIM * 2 : (size_t)128 * 4;
            char *dst = w ? (char *)d->w_kq1 : (char *)d->b_kq1;
            return cbi_kstatus(b,
                               (int)cudaMemcpyAsync(dst + kq * bytes, d->w[i], bytes,
                                                    cudaMemcpyDeviceToDevice, b->stream),
                               "decoder weights");
        }
    }
    return CB_OK;
}

static void init_params(int kind, float std, float *mean, float *sd)
{
    *mean = kind == SAM3_INIT_LNW ? 1.0f : 0.0f;
    *sd = kind == SAM3_INIT_EMB ? 1.0f
          : (kind == SAM3_INIT_LNW || kind == SAM3_INIT_LNB) ? 0.1f : std;
}

int cb_decoder_init_random(cb_decoder *d, uint64_t seed, float std)
{
    cb_backend *b;
    void *s = NULL;
    int i;

    if (!d)
        return CB_EARG;
    b = d->b;
    CB_TRY(cbi_enter(b));
    CB_TRY(cbi_scratch(b, (size_t)2048 * 256 * 4, &s));
    for (i = 0; i < SAM3_DT_COUNT; i++) {
        int r, c, k;
        float mean, sd;

        sam3_dec_tensor(i, &r, &c, &k);
        init_params(k, std, &mean, &sd);
        CB_TRY(cbi_kstatus(b,
                           k_synth_normal(seed, SAM3_STREAM_DECW + (uint64_t)i, (long)r * c,
                                          mean, sd, s, 0, (k_stream)b->stream),
                           "decoder init"));
        CB_TRY(store_tensor(d, i, (const float *)s));
        if (d->hw[i])
            sam3_synth_normal(seed, SAM3_STREAM_DECW + (uint64_t)i, (size_t)r * c, mean, sd,
                              d->hw[i]);
        /* the scratch buffer is reused by the next tensor */
        CB_TRY(cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "decoder init"));
    }
    d->have_image = 0;
    return compute_pe_img(d);
}

int cb_decoder_set_weight(cb_decoder *d, int which, const float *src, size_t count)
{
    cb_backend *b;
    void *s = NULL;
    int r, c, k;

    if (!d || !src)
        return CB_EARG;
    b = d->b;
    if (which < 0 || which >= SAM3_DT_COUNT)
        return cbi_fail(b, CB_EARG, "decoder set_weight: tensor");
    sam3_dec_tensor(which, &r, &c, &k);
    if (count != (size_t)r * c)
        return cbi_fail(b, CB_EARG, "decoder set_weight: shape");
    CB_TRY(cbi_enter(b));
    CB_TRY(cbi_scratch(b, count * 4, &s));
    CB_TRY(cbi_kstatus(b,
                       (int)cudaMemcpyAsync(s, src, count * 4, cudaMemcpyHostToDevice,
                                            b->stream),
                       "decoder set_weight"));
    CB_TRY(store_tensor(d, which, (const float *)s));
    CB_TRY(cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "decoder set_weight"));
    if (d->hw[which])
        memcpy(d->hw[which], src, count * 4);
    d->have_image = 0;
    if (which == SAM3_DT_GAUSS)
        return compute_pe_img(d);
    return CB_OK;
}

/* ---------------------------------------------------------------- layers */

/* Y[rows, out] = act(Xb W^T + bias) (+ R[m % rmod] when R): Xb bf16
 * [rows, in], W bf16 [out, in], Y fp32. */
static int lin16(cb_decoder *d, const char *name, const void *Xb, long rows, int in, int out,
                 int wi, int bi, float *Y, const float *R, int rmod, int act)
{
    cb_backend *b = d->b;
    const double dr = (double)rows;

    LAUNCH(name, 2.0 * dr * in * out,
           dr * in * 2 + (double)in * out * 2 + dr * out * 4 * (R ? 2 : 1),
           k_gemm_bf16_tc((int)rows, out, in, Xb, in, d->w[wi], in, Y, out, 0,
                          bi >= 0 ? (const float *)d->w[bi] : NULL, R, out, rmod, 1.0f, act,
                          NULL, b->d_err, b->num_sms, (k_stream)b->stream));
    return CB_OK;
}

/* Y bf16 [rows, out] = X W^T + bias, for outputs read only by an attention
 * kernel that takes bf16. */
static int lin16h(cb_decoder *d, const char *name, const void *Xb, long rows, int in, int out,
                  int wi, int bi, void *Y)
{
    cb_backend *b = d->b;
    const double dr = (double)rows;

    LAUNCH(name, 2.0 * dr * in * out, dr * in * 2 + (double)in * out * 2 + dr * out * 2,
           k_gemm_bf16_tc((int)rows, out, in, Xb, in, d->w[wi], in, Y, out, 1,
                          (const float *)d->w[bi], NULL, out, 0, 1.0f, K_ACT_NONE, NULL,
                          b->d_err, b->num_sms, (k_stream)b->stream));
    return CB_OK;
}

/* The same on an fp32 X of the image stream, rounded to bf16 into xs
 * first. */
static int lin32(cb_decoder *d, const char *name, const float *X, void *xs, long rows, int in,
                 int out, int wi, int bi, float *Y, const float *R, int rmod, int act)
{
    cb_backend *b = d->b;

    LAUNCH("dec_cast", 0, (double)rows * in * 6,
           k_cast_f32_bf16(X, xs, rows * in, (k_stream)b->stream));
    return lin16(d, name, xs, rows, in, out, wi, bi, Y, R, rmod, act);
}

/* A Linear of the token stream (8 rows per prompt): Y = act(X W^T + bias)
 * (+ Y when residual), X rounded to bf16 into the token operand buffer. */
static int lintok(cb_decoder *d, const float *X, long rows, int in, int out, int wi, int bi,
                  float *Y, int residual, int act)
{
    return lin32(d, "dec_gemm_tok", X, d->tok_bf16, rows, in, out, wi, bi, Y,
                 residual ? Y : NULL, 0, act);
}

/* The same on the X that the previous lintok rounded into the token
 * operand buffer (no second rounding pass). */
static int lintok_again(cb_decoder *d, long rows, int in, int out, int wi, int bi, float *Y,
                        int residual, int act)
{
    return lin16(d, "dec_gemm_tok", d->tok_bf16, rows, in, out, wi, bi, Y, residual ? Y : NULL, 0,
                 act);
}

static int ln(cb_decoder *d, float *X, void *Y, int y_bf16, long rows, int C, int wi, int bi,
              float eps, int act)
{
    cb_backend *b = d->b;

    LAUNCH("dec_layernorm", 8.0 * rows * C, (double)rows * C * (y_bf16 ? 6 : 8),
           k_layernorm(X, Y, y_bf16, (const float *)d->w[wi], (const float *)d->w[bi], rows, C,
                       eps, act, (k_stream)b->stream));
    return CB_OK;
}

static int add(cb_decoder *d, float *out, const float *a, const float *bb, long n, long bmod)
{
    cb_backend *b = d->b;

    LAUNCH("dec_add", (double)n, (double)n * 12,
           k_add_bcast(out, a, bb, n, bmod, (k_stream)b->stream));
    return CB_OK;
}

/* A norm of the token stream (LayerNorm of qry in place, weights wi / bi)
 * that also writes the bf16 operands of the Linears after it in the same
 * pass: yb = bf16(qry) (NULL: none) and, with pe, tok_bf16 = bf16(qry +
 * qpe), the queries / keys input of the next attention. Each attention
 * step reads tok_bf16 as the last norm left it (lintok_again): qry does not
 * change between a norm and the attention projections that follow it (the
 * image -> token attention updates the image stream only). */
static int lntok(cb_decoder *d, long nt, int wi, int bi, void *yb, int pe)
{
    cb_backend *b = d->b;

    LAUNCH("dec_layernorm", 8.0 * nt * DEC_DIM,
           (double)nt * DEC_DIM * (8 + (yb ? 2 : 0) + (pe ? 6 : 0)),
           k_dec_ln_keys(d->qry, NULL, d->qry, (const float *)d->w[wi], (const float *)d->w[bi],
                         nt, DEC_EPS, d->qpe, (int)nt, yb, pe ? d->tok_bf16 : NULL,
                         (k_stream)b->stream));
    return CB_OK;
}

static int mha(cb_decoder *d, int P, int Nq, int Nk, int dint, const float *q, long sq,
               const float *k, long sk, const float *v, long sv, float *o)
{
    cb_backend *b = d->b;

    LAUNCH(Nk > 64 ? "dec_mha_t2i" : (Nq > 64 ? "dec_mha_i2t" : "dec_mha_self"),
           4.0 * P * Nq * (double)Nk * dint,
           4.0 * ((double)P * Nq * dint * 2 + (sk ? (double)P : 1.0) * Nk * dint * 2),
           k_mha(P, Nq, Nk, dint, q, sq, k, sk, v, sv, o, d->mha_ws, d->mha_ws_bytes,
                 b->d_err, b->num_sms, (k_stream)b->stream));
    return CB_OK;
}

/* Token -> image attention of the P prompts' queries sq on bf16 keys and
 * values (prompt strides sk / sv in elements, 0: shared by all prompts; key
 * row stride kld, value rows of 128) into so's storage as bf16 [P * 8, 128],
 * the operand of the output projection (no rounding pass). */
static int mha_t2i(cb_decoder *d, int P, const void *k, long sk, long kld, const void *v,
                   long sv)
{
    cb_backend *b = d->b;
    const long nt = (long)P * DEC_NTOK;

    if (!sk && !sv) {
        /* keys shared by all prompts (layer 0): one cross-attention of the
         * P * 8 queries over the image on the tensor cores, heads of 16
         * padded to 64 (the keys once per image, in set_image) */
        LAUNCH("dec_pad", 0, (double)nt * 128 * 4 + (double)nt * 512 * 2,
               k_pad_heads64(d->sq, 0, 128, nt, 8, 16, d->q_pad,
                             (k_stream)b->stream));
        LAUNCH("dec_mha_t2i", 4.0 * nt * (double)DEC_T * 128,
               (double)nt * 512 * 2 + 2.0 * DEC_T * 512 * 2 + (double)nt * 128 * 4,
               k_attn_tc_cross(d->q_pad, 512, d->k0_pad, 512, d->v0_pad, 512, 1, (int)nt, DEC_T,
                               8, 0.25f, NULL, d->so, 128, 16, 1, d->xws, d->xws_bytes, b->d_err,
                               (k_stream)b->stream));
        return CB_OK;
    }
    LAUNCH("dec_mha_t2i", 4.0 * P * DEC_NTOK * (double)DEC_T * 128,
           4.0 * (double)P * DEC_NTOK * 128 * 2 + 2.0 * (sk ? (double)P : 1.0) * DEC_T * 128 * 2,
           k_mha_t2i_bf16kv(P, DEC_NTOK, DEC_T, d->sq, DEC_NTOK * 128, k, sk, kld, v, sv, 128,
                            d->so, 1, d->mha_ws, d->mha_ws_bytes, b->d_err, b->num_sms,
                            (k_stream)b->stream));
    return CB_OK;
}

int cb_decoder_set_image(cb_decoder *d, cb_mem emb, cb_mem feat_s0, cb_mem feat_s1)
{
    cb_backend *b;
    const size_t T = DEC_T;

    if (!d || !emb || !feat_s0 || !feat_s1)
        return CB_EARG;
    b = d->b;
    if (emb->dtype != CB_F32 || feat_s0->dtype != CB_F32 || feat_s1->dtype != CB_F32 ||
        emb->bytes < T * DEC_DIM * 4 || feat_s0->bytes < 16 * T * 32 * 4 ||
        feat_s1->bytes < 4 * T * 64 * 4)
        return cbi_fail(b, CB_EARG, "decoder set_image");
    CB_TRY(cbi_enter(b));
    /* the upscaling residuals, sub-pixel-major and channel-major, the
     * layout the two upscaling epilogues read */
    LAUNCH("dec_feat", 0, 2.0 * 16 * T * 32 * 4,
           k_dec_feat_subpix((const float *)feat_s0->ptr, 2 * DEC_GRID, 2 * DEC_GRID, 32,
                             d->feat_s0, (k_stream)b->stream));
    LAUNCH("dec_feat", 0, 2.0 * 4 * T * 64 * 4,
           k_dec_feat_subpix((const float *)feat_s1->ptr, DEC_GRID, DEC_GRID, 64, d->feat_s1,
                             (k_stream)b->stream));
    /* src = emb + no_mask_embed, srcpe = src + dense PE; the layer-0
     * projections every prompt shares (sam3_model.c:1160-1168) */
    CB_TRY(add(d, d->src, (const float *)emb->ptr, (const float *)d->w[SAM3_DT_NO_MASK],
               (long)T * DEC_DIM, DEC_DIM));
    CB_TRY(add(d, d->srcpe, d->src, d->pe_img, (long)T * DEC_DIM, (long)T * DEC_DIM));
    /* kp0 / vp0 are read only by the token -> image attention, as bf16 */
    LAUNCH("dec_cast", 0, (double)T * DEC_DIM * 6,
           k_cast_f32_bf16(d->srcpe, d->kin_bf16, (long)T * DEC_DIM, (k_stream)b->stream));
    CB_TRY(lin16h(d, "dec_gemm_img", d->kin_bf16, (long)T, DEC_DIM, 128,
                  ATT(SAM3_DA_L0_T2I, KW), ATT(SAM3_DA_L0_T2I, KB), d->kp0));
    LAUNCH("dec_cast", 0, (double)T * DEC_DIM * 6,
           k_cast_f32_bf16(d->src, d->kin_bf16, (long)T * DEC_DIM, (k_stream)b->stream));
    CB_TRY(lin16h(d, "dec_gemm_img", d->kin_bf16, (long)T, DEC_DIM, 128,
                  ATT(SAM3_DA_L0_T2I, VW), ATT(SAM3_DA_L0_T2I, VB), d->vp0));
    LAUNCH("dec_pad", 0, (double)T * 128 * 2 * 2 + (double)T * 512 * 2 * 2,
           k_pad_heads64(d->kp0, 1, 128, (long)T, 8, 16, d->k0_pad, (k_stream)b->stream));
    LAUNCH("dec_pad", 0, 0,
           k_pad_heads64(d->vp0, 1, 128, (long)T, 8, 16, d->v0_pad, (k_stream)b->stream));
    /* qp0 is read only by the image -> token attention, as bf16 */
    LAUNCH("dec_cast", 0, (double)T * DEC_DIM * 6,
           k_cast_f32_bf16(d->srcpe, d->kin_bf16, (long)T * DEC_DIM, (k_stream)b->stream));
    LAUNCH("dec_gemm_img", 2.0 * T * DEC_DIM * 128,
           (double)T * DEC_DIM * 2 + DEC_DIM * 128.0 * 2 + (double)T * 128 * 2,
           k_gemm_bf16_tc(T, 128, DEC_DIM, d->kin_bf16, DEC_DIM, d->w[ATT(SAM3_DA_L0_I2T, QW)],
                          DEC_DIM, d->qp0, 128, 1, (const float *)d->w[ATT(SAM3_DA_L0_I2T, QB)],
                          NULL, 128, 0, 1.0f, K_ACT_NONE, NULL, b->d_err, b->num_sms,
                          (k_stream)b->stream));
    d->have_image = 1;
    return CB_OK;
}

/* ---------------------------------------------------------------- decode */

/* Token -> image attention on per-prompt keys, residual into the queries
 * (t2i_attention, sam3_model.c:1212-1229). Its image-side operands, keys and
 * kin = keys + dense PE in bf16, were written by the LayerNorm that ended
 * the previous image -> token attention (ln_keys); kin serves layer 1's
 * image -> token queries as well. */
static int t2i_attention(cb_decoder *d, int P, int blk)
{
    const long nt = (long)P * DEC_NTOK, rows = (long)P * DEC_T;

    CB_TRY(lintok_again(d, nt, DEC_DIM, 128, ATT(blk, QW), ATT(blk, QB), d->sq, 0,
                  K_ACT_NONE));
    if (blk == SAM3_DA_L1_T2I) {
        cb_backend *b = d->b;

        /* keys and layer 1's image -> token queries from kin in one GEMM:
         * [keys | queries] rows of 256 bf16 in bk's storage */
        LAUNCH("dec_gemm_img", 2.0 * rows * DEC_DIM * 256,
               (double)rows * DEC_DIM * 2 + DEC_DIM * 256.0 * 2 + (double)rows * 256 * 2,
               k_gemm_bf16_tc((int)rows, 256, DEC_DIM, d->kin_bf16, DEC_DIM, d->w_kq1, DEC_DIM,
                              d->bk, 256, 1, d->b_kq1, NULL, 256, 0, 1.0f, K_ACT_NONE, NULL,
                              b->d_err, b->num_sms, (k_stream)b->stream));
    }
    else
        CB_TRY(lin16h(d, "dec_gemm_img", d->kin_bf16, rows, DEC_DIM, 128, ATT(blk, KW),
                      ATT(blk, KB), d->bk));
    CB_TRY(lin16h(d, "dec_gemm_img", d->keys_bf16, rows, DEC_DIM, 128, ATT(blk, VW),
                  ATT(blk, VB), d->bv));
    {
        const long kld = blk == SAM3_DA_L1_T2I ? 256 : 128;

        CB_TRY(mha_t2i(d, P, d->bk, (long)DEC_T * kld, kld, d->bv, (long)DEC_T * 128));
    }
    return lin16(d, "dec_gemm_tok", d->so, nt, 128, DEC_DIM, ATT(blk, OW), ATT(blk, OB), d->qry,
                 d->qry, 0, K_ACT_NONE);
}

/* token_mlp (sam3_model.c:1231-1237): 256 -> 2048 (ReLU) -> 256, residual.
 * The hidden layer is written once, in bf16 (into sh's storage), as the
 * second GEMM's operand. */
static int token_mlp(cb_decoder *d, int P, int l)
{
    cb_backend *b = d->b;
    const long nt = (long)P * DEC_NTOK;
    const double dr = (double)nt;

    /* tok_bf16 = bf16(qry), written by the norm before (lntok) */
    LAUNCH("dec_gemm_tok", 2.0 * dr * DEC_DIM * 2048,
           dr * DEC_DIM * 2 + (double)DEC_DIM * 2048 * 2 + dr * 2048 * 2,
           k_gemm_bf16_tc((int)nt, 2048, DEC_DIM, d->tok_bf16, DEC_DIM, d->w[LAY(l, M1W)], DEC_DIM,
                          d->sh, 2048, 1, (const float *)d->w[LAY(l, M1B)], NULL, 2048, 0, 1.0f,
                          K_ACT_RELU, NULL, b->d_err, b->num_sms, (k_stream)b->stream));
    return lin16(d, "dec_gemm_tok", d->sh, nt, 2048, DEC_DIM, LAY(l, M2W), LAY(l, M2B), d->qry,
                 d->qry, 0, K_ACT_NONE);
}

/* Self attention of the tokens; layer 0 without positional encoding and
 * without residual (skip_first_layer_pe), layer 1 with both
 * (sam3_model.c:1269-1282, 1311-1324). */
static int self_attention(cb_decoder *d, int P, int l)
{
    const long nt = (long)P * DEC_NTOK;
    const int blk = l ? SAM3_DA_L1_SELF : SAM3_DA_L0_SELF;

    if (l)  /* tok_bf16 = bf16(qry + qpe) from layer 0's last token norm */
        CB_TRY(lintok_again(d, nt, DEC_DIM, DEC_DIM, ATT(blk, QW), ATT(blk, QB), d->sq, 0,
                            K_ACT_NONE));
    else
        CB_TRY(lintok(d, d->qry, nt, DEC_DIM, DEC_DIM, ATT(blk, QW), ATT(blk, QB), d->sq, 0,
                      K_ACT_NONE));
    CB_TRY(lintok_again(d, nt, DEC_DIM, DEC_DIM, ATT(blk, KW), ATT(blk, KB), d->sk, 0, K_ACT_NONE));
    /* The values' input bf16(qry) is already rounded: in layer 0 by the
     * queries' projection above, in layer 1 by layer 0's last token norm
     * (qry is unchanged since). */
    if (l)
        CB_TRY(lin16(d, "dec_gemm_tok", d->qv_bf16, nt, DEC_DIM, DEC_DIM, ATT(blk, VW),
                     ATT(blk, VB), d->sv, NULL, 0, K_ACT_NONE));
    else
        CB_TRY(lintok_again(d, nt, DEC_DIM, DEC_DIM, ATT(blk, VW), ATT(blk, VB), d->sv, 0,
                            K_ACT_NONE));
    CB_TRY(mha(d, P, DEC_NTOK, DEC_NTOK, DEC_DIM, d->sq, DEC_NTOK * DEC_DIM, d->sk,
               DEC_NTOK * DEC_DIM, d->sv, DEC_NTOK * DEC_DIM, d->so));
    return lintok(d, d->so, nt, DEC_DIM, DEC_DIM, ATT(blk, OW), ATT(blk, OB), d->qry, l,
                  K_ACT_NONE);
}

/* Image -> token attention of layer l (sam3_model.c:1297-1309, 1334-1348):
 * queries from the image stream (the shared layer-0 projection, or kin of
 * layer 1), keys and values from the tokens; the output projection lands
 * in keys, + keys as the GEMM residual (layer 1) or + src (layer 0: the
 * add_bcast of sam3_model.c:1307, row m % T, added by norm4 before its
 * statistics), then norm4, which also writes the bf16 operands keys and
 * keys + PE of the next token -> image attention (and of the upscaling).
 * After layer 1 nothing reads the fp32 keys again, so that LayerNorm writes
 * only the bf16 copies. */
static int i2t_attention(cb_decoder *d, int P, int l)
{
    const long nt = (long)P * DEC_NTOK, rows = (long)P * DEC_T;
    const int blk = l ? SAM3_DA_L1_I2T : SAM3_DA_L0_I2T;

    /* layer 1's queries: columns 128-255 of the [keys | queries] rows that
     * layer 1's token -> image attention projected from kin (unchanged
     * since: the token steps in between leave the image stream alone) */
    CB_TRY(lintok_again(d, nt, DEC_DIM, 128, ATT(blk, KW), ATT(blk, KB), d->sk, 0,
                  K_ACT_NONE));
    /* keys from tok_bf16, values from qv_bf16: both written by the norm
     * before (lntok) */
    CB_TRY(lin16(d, "dec_gemm_tok", d->qv_bf16, nt, DEC_DIM, 128, ATT(blk, VW), ATT(blk, VB),
                 d->sv, NULL, 0, K_ACT_NONE));
    {
        cb_backend *b = d->b;

        /* the attention output is read only by the output projection: bf16 */
        LAUNCH("dec_mha_i2t", 4.0 * P * DEC_T * (double)DEC_NTOK * 128,
               (double)P * DEC_T * 128 * (4 + 2),
               k_mha_i2t_bf16(P, DEC_T, DEC_NTOK,
                              l ? (const void *)((const uint16_t *)d->bk + 128) : d->qp0,
                              l ? (long)DEC_T * 256 : 0, l ? 256 : 128, d->sk, DEC_NTOK * 128,
                              d->sv, DEC_NTOK * 128, d->bo_bf16, b->num_sms,
                              (k_stream)b->stream));
    }
    CB_TRY(lin16(d, "dec_gemm_img", d->bo_bf16, rows, 128, DEC_DIM, ATT(blk, OW), ATT(blk, OB),
                 d->keys, l ? d->keys : NULL, 0, K_ACT_NONE));
    {
        cb_backend *b = d->b;

        LAUNCH("dec_ln_keys", 8.0 * rows * DEC_DIM, (double)rows * DEC_DIM * (l ? 8 : 12),
               k_dec_ln_keys(d->keys, l ? NULL : d->src, l ? NULL : d->keys,
                             (const float *)d->w[LAY(l, N4W)],
                             (const float *)d->w[LAY(l, N4B)], rows, DEC_EPS, d->pe_img, DEC_T,
                             d->keys_bf16, d->kin_bf16, (k_stream)b->stream));
    }
    return CB_OK;
}

/* Prompt tokens (sam3_model.c:1249-1263): object score token, IoU token,
 * 4 mask tokens, the point's encoding + point_embeddings[1], and
 * not_a_point (the padding point SAM appends without a box). */
static void prompt_tokens(const cb_decoder *d, int P, const float *points, float *tok)
{
    int p, i;

    for (p = 0; p < P; p++) {
        float *t = tok + (size_t)p * DEC_NTOK * DEC_DIM;

        memcpy(t, d->hw[SAM3_DT_OBJ_TOKEN], DEC_DIM * sizeof(float));
        memcpy(t + DEC_DIM, d->hw[SAM3_DT_IOU_TOKEN], DEC_DIM * sizeof(float));
        memcpy(t + 2 * DEC_DIM, d->hw[SAM3_DT_MASK_TOKENS], 4 * DEC_DIM * sizeof(float));
        pe_encode(d->hw[SAM3_DT_GAUSS], (points[2 * p] + 0.5f) / DEC_IMG,
                  (points[2 * p + 1] + 0.5f) / DEC_IMG, t + 6 * DEC_DIM);
        for (i = 0; i < DEC_DIM; i++) {
            t[6 * DEC_DIM + i] += d->hw[SAM3_DT_POINT_EMB + 1][i];
            t[7 * DEC_DIM + i] = d->hw[SAM3_DT_NOT_A_POINT][i];
        }
    }
}

int cb_decode(cb_decoder *d, int P, const float *points, float *iou, cb_mem lowres)
{
    cb_backend *b;
    struct k_dec_heads_w heads;
    long nt, rows;
    int l, m;

    if (!d || !points || !iou || !lowres)
        return CB_EARG;
    b = d->b;
    if (P <= 0 || P > d->batch || lowres->dtype != CB_F32 ||
        lowres->bytes < (size_t)P * 3 * DEC_LOWRES * DEC_LOWRES * 4)
        return cbi_fail(b, CB_EARG, "decode: batch or lowres buffer");
    if (!d->have_image)
        return cbi_fail(b, CB_EARG, "decode: no image (cb_decoder_set_image)");
    CB_TRY(cbi_enter(b));
    nt = (long)P * DEC_NTOK;
    rows = (long)P * DEC_T;

    prompt_tokens(d, P, points, d->h_tok);
    CB_TRY(cbi_kstatus(b,
                       (int)cudaMemcpyAsync(d->qpe, d->h_tok, (size_t)nt * DEC_DIM * 4,
                                            cudaMemcpyHostToDevice, b->stream),
                       "decode: tokens"));
    CB_TRY(cbi_kstatus(b,
                       (int)cudaMemcpyAsync(d->qry, d->qpe, (size_t)nt * DEC_DIM * 4,
                                            cudaMemcpyDeviceToDevice, b->stream),
                       "decode: tokens"));

    /* Layer 0: self attention (no PE, no residual), token -> image on the
     * shared layer-0 projections, MLP, image -> token. */
    CB_TRY(self_attention(d, P, 0));
    CB_TRY(lntok(d, nt, LAY(0, N1W), LAY(0, N1B), NULL, 1));
    CB_TRY(lintok_again(d, nt, DEC_DIM, 128, ATT(SAM3_DA_L0_T2I, QW),
                  ATT(SAM3_DA_L0_T2I, QB), d->sq, 0, K_ACT_NONE));
    CB_TRY(mha_t2i(d, P, d->kp0, 0, 128, d->vp0, 0));
    CB_TRY(lin16(d, "dec_gemm_tok", d->so, nt, 128, DEC_DIM, ATT(SAM3_DA_L0_T2I, OW),
                 ATT(SAM3_DA_L0_T2I, OB), d->qry, d->qry, 0, K_ACT_NONE));
    CB_TRY(lntok(d, nt, LAY(0, N2W), LAY(0, N2B), d->tok_bf16, 0));
    CB_TRY(token_mlp(d, P, 0));
    CB_TRY(lntok(d, nt, LAY(0, N3W), LAY(0, N3B), d->qv_bf16, 1));
    CB_TRY(i2t_attention(d, P, 0));

    /* Layer 1. */
    CB_TRY(self_attention(d, P, 1));
    CB_TRY(lntok(d, nt, LAY(1, N1W), LAY(1, N1B), NULL, 1));
    CB_TRY(t2i_attention(d, P, SAM3_DA_L1_T2I));
    CB_TRY(lntok(d, nt, LAY(1, N2W), LAY(1, N2B), d->tok_bf16, 0));
    CB_TRY(token_mlp(d, P, 1));
    CB_TRY(lntok(d, nt, LAY(1, N3W), LAY(1, N3B), d->qv_bf16, 1));
    CB_TRY(i2t_attention(d, P, 1));

    /* Final token -> image attention (its queries' input tok_bf16 from
     * layer 1's last token norm). */
    CB_TRY(t2i_attention(d, P, SAM3_DA_FINAL_T2I));
    CB_TRY(ln(d, d->qry, d->qry, 0, nt, DEC_DIM, SAM3_DT_NF_W, SAM3_DT_NF_B, DEC_EPS,
              K_ACT_NONE));

    /* Hypernetwork MLPs 1..3 and the IoU head on the final tokens
     * (sam3_model.c:1368-1386), first: the last upscaling stage takes their
     * outputs. */
    for (m = 0; m < 4; m++)
        for (l = 0; l < 3; l++) {
            const int base = m < 3 ? SAM3_DT_HYPER + 6 * (m + 1) : SAM3_DT_IOU;

            heads.w[m][l] = (const float *)d->w[base + 2 * l];
            heads.b[m][l] = (const float *)d->w[base + 2 * l + 1];
        }
    LAUNCH("dec_heads", 2.0 * P * 4 * (2 * 65536.0 + 32 * 256), (double)P * 4 * 2 * 65536 * 4,
           k_dec_heads(d->qry, P, &heads, d->hyper, d->iou, (k_stream)b->stream));

    /* Output upscaling (sam3_model.c:1353-1366) and mask_logits
     * (:1387-1399) as two tcgen05 GEMMs with fused epilogues: ConvT
     * 256 -> 64 on the bf16 keys + bias + feat_s1 + LayerNorm2d + GELU,
     * written as the bf16 operand of ConvT 64 -> 32, whose epilogue adds
     * feat_s0, applies GELU and dots with the hypernetwork outputs,
     * straight to the logits. */
    LAUNCH("dec_up1", 2.0 * rows * DEC_DIM * 256,
           (double)rows * DEC_DIM * 2 + (double)rows * 4 * 64 * 2,
           k_dec_convt_ln2d(d->keys_bf16, P, DEC_GRID, DEC_GRID, d->w[SAM3_DT_UP0_W],
                            (const float *)d->w[SAM3_DT_UP0_B], d->feat_s1,
                            (const float *)d->w[SAM3_DT_UP1_W],
                            (const float *)d->w[SAM3_DT_UP1_B], LN2D_EPS, d->u1_bf16, b->d_err,
                            b->num_sms, (k_stream)b->stream));
    LAUNCH("dec_up2_logits", 2.0 * 4 * rows * 64 * 128 + 2.0 * P * 3 * 32 * DEC_LOWRES * DEC_LOWRES,
           (double)4 * rows * 64 * 2 + (double)P * 3 * DEC_LOWRES * DEC_LOWRES * 4,
           k_dec_convt_logits(d->u1_bf16, P, 2 * DEC_GRID, 2 * DEC_GRID, d->w[SAM3_DT_UP3_W],
                              (const float *)d->w[SAM3_DT_UP3_B], d->feat_s0, d->hyper,
                              (float *)lowres->ptr, b->d_err, b->num_sms, (k_stream)b->stream));
    CB_TRY(cbi_kstatus(b,
                       (int)cudaMemcpyAsync(iou, d->iou, (size_t)P * 3 * 4,
                                            cudaMemcpyDeviceToHost, b->stream),
                       "decode: iou"));
    return cb_sync(b);
}
