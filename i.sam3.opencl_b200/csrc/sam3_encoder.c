/* SPDX-License-Identifier: Unlicense */
/* The PE ViT trunk (sam3_model.c: load_encoder :473-581, alloc_buffers
 * :815-916, vit_block :981-1028, sam_encode_trunk :1112-1144) on the
 * tensor-core path, batched over image tiles.
 *
 * Layout: tokens are kept in window-major order (token r of a tile belongs
 * to window r / ws^2, in-window index r % ws^2) for the whole trunk. The
 * windowed blocks then need no partition/unpartition copies
 * (sam3_kernels.cl:712-741 are folded away); the global blocks attend over
 * all tokens of the tile, which is order-independent for keys, and take
 * their RoPE rotation from each token's raster position in the QKV
 * epilogue. The patch embedding writes rows in that order and the output
 * is permuted back to raster order once at the end.
 *
 * Per block, on the backend stream:
 *   LN1 (fp32 x -> bf16)  QKV GEMM (+bias, RoPE, bf16 out)  attention
 *   (tcgen05, bf16 out)  proj GEMM (+bias, +x residual, fp32 in place)
 *   LN2 (-> bf16)  fc1 GEMM (+bias, GELU, bf16)  fc2 GEMM (+bias, +x).
 * Matrices are bf16 (operands of tcgen05.mma), vectors and the residual
 * stream fp32. */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "backend_internal.h"
#include "sam3_synth.h"

struct enc_block {
    void *qkvw, *projw, *fc1w, *fc2w; /* bf16 [out, in] */
    float *n1w, *n1b, *n2w, *n2b, *qkvb, *projb, *fc1b, *fc2b;
};

struct cb_encoder {
    cb_backend *b;
    struct cb_encoder_config cfg;
    int T, hd, kpad, ws2, nwin;
    void *pe_w;      /* bf16 [E, kpad] */
    float *pos;      /* fp32 [T, E], window-major rows */
    float *lnpw, *lnpb;
    float *rope_win; /* [ws^2, hd/2, 2] */
    float *rope_glob; /* [T, hd/2, 2], raster positions */
    struct enc_block *blk;
    /* work buffers, max_tiles tiles */
    float *x;        /* fp32 [rows, E] */
    void *xn;        /* bf16 [rows, E] */
    void *qkv;       /* bf16 [rows, 3E] */
    void *attn;      /* bf16 [rows, E] */
    void *h;         /* bf16 [rows, max(mlp, kpad)] */
    /* cb_encode_tiles_host pipeline: two staging buffers per direction,
     * chunk tiles each, a stream per copy direction and their events */
    int chunk;
    uint8_t *tiles[2];
    float *out_dev[2];
    cudaStream_t h2d, d2h;
    cudaEvent_t ev_in[2], ev_done[2], ev_out[2];
};

void cb_encoder_default_config(struct cb_encoder_config *c)
{
    c->embed = 1024;
    c->depth = 32;
    c->heads = 16;
    c->mlp = 4096;
    c->grid = 72;
    c->patch = 14;
    c->window = 24;
    c->max_tiles = 1;
    c->global_mask = (1ull << 7) | (1ull << 15) | (1ull << 23) | (1ull << 31);
}

static int dev_alloc(cb_encoder *e, void **p, size_t bytes)
{
    if (cudaMalloc(p, bytes ? bytes : 16) != cudaSuccess) {
        *p = NULL;
        return cbi_fail(e->b, CB_EALLOC, "encoder buffers");
    }
    return CB_OK;
}

void cb_encoder_free(cb_encoder *e)
{
    int i;

    if (!e)
        return;
    cbi_enter(e->b);
    cudaStreamSynchronize(e->b->stream);
    if (e->h2d)
        cudaStreamSynchronize(e->h2d);
    if (e->d2h)
        cudaStreamSynchronize(e->d2h);
    if (e->blk)
        for (i = 0; i < e->cfg.depth; i++) {
            struct enc_block *k = &e->blk[i];

            cudaFree(k->qkvw);
            cudaFree(k->projw);
            cudaFree(k->fc1w);
            cudaFree(k->fc2w);
            cudaFree(k->n1w);
            cudaFree(k->n1b);
            cudaFree(k->n2w);
            cudaFree(k->n2b);
            cudaFree(k->qkvb);
            cudaFree(k->projb);
            cudaFree(k->fc1b);
            cudaFree(k->fc2b);
        }
    free(e->blk);
    cudaFree(e->pe_w);
    cudaFree(e->pos);
    cudaFree(e->lnpw);
    cudaFree(e->lnpb);
    cudaFree(e->rope_win);
    cudaFree(e->rope_glob);
    cudaFree(e->x);
    cudaFree(e->xn);
    cudaFree(e->qkv);
    cudaFree(e->attn);
    cudaFree(e->h);
    for (i = 0; i < 2; i++) {
        cudaFree(e->tiles[i]);
        cudaFree(e->out_dev[i]);
        if (e->ev_in[i])
            cudaEventDestroy(e->ev_in[i]);
        if (e->ev_done[i])
            cudaEventDestroy(e->ev_done[i]);
        if (e->ev_out[i])
            cudaEventDestroy(e->ev_out[i]);
    }
    if (e->h2d)
        cudaStreamDestroy(e->h2d);
    if (e->d2h)
        cudaStreamDestroy(e->d2h);
    free(e);
}

int cb_encoder_create(cb_backend *b, const struct cb_encoder_config *cfg,
                      cb_encoder **out)
{
    cb_encoder *e;
    const struct cb_encoder_config *c = cfg;
    size_t E, rows, hcols;
    int i, rc = CB_OK;

    if (!b || !cfg || !out)
        return CB_EARG;
    *out = NULL;
    if (c->embed <= 0 || c->heads <= 0 || c->embed != c->heads * 64 ||
        c->depth <= 0 || c->depth > 64 || c->mlp <= 0 || c->mlp % 64 ||
        c->grid <= 0 || c->patch <= 0 || c->window <= 0 ||
        c->grid % c->window || c->max_tiles <= 0)
        return cbi_fail(b, CB_EARG, "encoder config");
    CB_TRY(cbi_enter(b));
    e = calloc(1, sizeof(*e));
    if (!e)
        return CB_EALLOC;
    e->b = b;
    e->cfg = *c;
    e->T = c->grid * c->grid;
    e->hd = 64;
    e->kpad = (3 * c->patch * c->patch + 63) / 64 * 64;
    e->ws2 = c->window * c->window;
    e->nwin = (c->grid / c->window) * (c->grid / c->window);
    E = (size_t)c->embed;
    rows = (size_t)c->max_tiles * e->T;
    hcols = (size_t)(c->mlp > e->kpad ? c->mlp : e->kpad);
    e->blk = calloc((size_t)c->depth, sizeof(struct enc_block));
    if (!e->blk) {
        free(e);
        return CB_EALLOC;
    }
#define A(p, n) \
    if (rc == CB_OK) rc = dev_alloc(e, (void **)&(p), (n))
    A(e->pe_w, E * e->kpad * 2);
    A(e->pos, (size_t)e->T * E * 4);
    A(e->lnpw, E * 4);
    A(e->lnpb, E * 4);
    A(e->rope_win, (size_t)e->ws2 * e->hd * 4);
    A(e->rope_glob, (size_t)e->T * e->hd * 4);
    for (i = 0; i < c->depth; i++) {
        struct enc_block *k = &e->blk[i];

        A(k->qkvw, 3 * E * E * 2);
        A(k->projw, E * E * 2);
        A(k->fc1w, (size_t)c->mlp * E * 2);
        A(k->fc2w, (size_t)c->mlp * E * 2);
        A(k->n1w, E * 4);
        A(k->n1b, E * 4);
        A(k->n2w, E * 4);
        A(k->n2b, E * 4);
        A(k->qkvb, 3 * E * 4);
        A(k->projb, E * 4);
        A(k->fc1b, (size_t)c->mlp * 4);
        A(k->fc2b, E * 4);
    }
    A(e->x, rows * E * 4);
    A(e->xn, rows * E * 2);
    A(e->qkv, rows * 3 * E * 2);
    A(e->attn, rows * E * 2);
    A(e->h, rows * hcols * 2);
#undef A
    if (rc == CB_OK && cudaMemset(e->pe_w, 0, E * e->kpad * 2) != cudaSuccess)
        rc = CB_ECUDA;
    if (rc != CB_OK) {
        cb_encoder_free(e);
        return rc;
    }
    *out = e;
    return CB_OK;
}

/* ---------------------------------------------------------------- weights */

static int upload_f32(cb_encoder *e, float *dst, const float *src, size_t n)
{
    return cbi_kstatus(e->b,
                      (int)cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyHostToDevice,
                                           e->b->stream),
                      "encoder weights");
}

/* fp32 [rows, cols] host -> bf16 [rows, ld] device (ld >= cols; padding
 * columns untouched). */
static int upload_bf16(cb_encoder *e, void *dst, const float *src, size_t rows,
                       size_t cols, size_t ld)
{
    void *s = NULL;
    cb_backend *b = e->b;

    CB_TRY(cbi_scratch(b, rows * cols * 6, &s));
    CB_TRY(cbi_kstatus(b,
                      (int)cudaMemcpyAsync(s, src, rows * cols * 4,
                                           cudaMemcpyHostToDevice, b->stream),
                      "encoder weights"));
    CB_TRY(cbi_kstatus(b,
                      k_cast_f32_bf16((const float *)s, (char *)s + rows * cols * 4,
                                      (long)(rows * cols), (k_stream)b->stream),
                      "encoder weights"));
    CB_TRY(cbi_kstatus(b,
                      (int)cudaMemcpy2DAsync(dst, ld * 2, (char *)s + rows * cols * 4,
                                             cols * 2, cols * 2, rows,
                                             cudaMemcpyDeviceToDevice, b->stream),
                      "encoder weights"));
    /* the scratch buffer is reused by the next call */
    return cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "encoder weights");
}

static int fill_f32(cb_encoder *e, float *dst, float v, size_t n)
{
    float *h = malloc(n * 4);
    size_t i;
    int rc;

    if (!h)
        return CB_EALLOC;
    for (i = 0; i < n; i++)
        h[i] = v;
    rc = upload_f32(e, dst, h, n);
    if (rc == CB_OK)
        rc = cbi_kstatus(e->b, (int)cudaStreamSynchronize(e->b->stream),
                        "encoder weights");
    free(h);
    return rc;
}

int cb_encoder_set_weight(cb_encoder *e, int which, int block, const float *src,
                          size_t count)
{
    const size_t E = (size_t)e->cfg.embed, mlp = (size_t)e->cfg.mlp;
    const size_t kin = 3 * (size_t)e->cfg.patch * e->cfg.patch;
    struct enc_block *k;
    cb_backend *b = e->b;
    int rc;

    CB_TRY(cbi_enter(b));
    switch (which) {
    case CB_W_PATCH_W:
        if (count != E * kin)
            return cbi_fail(b, CB_EARG, "set_weight: patch_embed shape");
        return upload_bf16(e, e->pe_w, src, E, kin, (size_t)e->kpad);
    case CB_W_POS: {
        void *s = NULL;

        if (count != (size_t)e->T * E)
            return cbi_fail(b, CB_EARG, "set_weight: pos_embed shape");
        CB_TRY(cbi_scratch(b, count * 4, &s));
        CB_TRY(upload_f32(e, (float *)s, src, count));
        rc = cbi_kstatus(b,
                        k_permute_rows((const float *)s, e->pos, 1, e->cfg.grid,
                                       e->cfg.window, (int)E, (k_stream)b->stream),
                        "set_weight: pos");
        if (rc == CB_OK)
            rc = cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "set_weight");
        return rc;
    }
    case CB_W_LN_PRE_W:
    case CB_W_LN_PRE_B:
        if (count != E)
            return cbi_fail(b, CB_EARG, "set_weight: ln_pre shape");
        rc = upload_f32(e, which == CB_W_LN_PRE_W ? e->lnpw : e->lnpb, src, E);
        break;
    case CB_W_ROPE_WIN:
        if (count != (size_t)e->ws2 * e->hd)
            return cbi_fail(b, CB_EARG, "set_weight: window rope shape");
        rc = upload_f32(e, e->rope_win, src, count);
        break;
    case CB_W_ROPE_GLOB:
        if (count != (size_t)e->T * e->hd)
            return cbi_fail(b, CB_EARG, "set_weight: global rope shape");
        rc = upload_f32(e, e->rope_glob, src, count);
        break;
    default:
        if (block < 0 || block >= e->cfg.depth)
            return cbi_fail(b, CB_EARG, "set_weight: block");
        k = &e->blk[block];
        switch (which) {
        case CB_W_QKV_W:
            if (count != 3 * E * E)
                return cbi_fail(b, CB_EARG, "set_weight: qkv shape");
            return upload_bf16(e, k->qkvw, src, 3 * E, E, E);
        case CB_W_PROJ_W:
            if (count != E * E)
                return cbi_fail(b, CB_EARG, "set_weight: proj shape");
            return upload_bf16(e, k->projw, src, E, E, E);
        case CB_W_FC1_W:
            if (count != mlp * E)
                return cbi_fail(b, CB_EARG, "set_weight: fc1 shape");
            return upload_bf16(e, k->fc1w, src, mlp, E, E);
        case CB_W_FC2_W:
            if (count != mlp * E)
                return cbi_fail(b, CB_EARG, "set_weight: fc2 shape");
            return upload_bf16(e, k->fc2w, src, E, mlp, mlp);
        case CB_W_N1_W:
        case CB_W_N1_B:
        case CB_W_N2_W:
        case CB_W_N2_B:
        case CB_W_PROJ_B:
        case CB_W_FC2_B:
            if (count != E)
                return cbi_fail(b, CB_EARG, "set_weight: vector shape");
            rc = upload_f32(e,
                            which == CB_W_N1_W   ? k->n1w
                            : which == CB_W_N1_B ? k->n1b
                            : which == CB_W_N2_W ? k->n2w
                            : which == CB_W_N2_B ? k->n2b
                            : which == CB_W_PROJ_B ? k->projb
                                                   : k->fc2b,
                            src, E);
            break;
        case CB_W_QKV_B:
            if (count != 3 * E)
                return cbi_fail(b, CB_EARG, "set_weight: qkv bias shape");
            rc = upload_f32(e, k->qkvb, src, count);
            break;
        case CB_W_FC1_B:
            if (count != mlp)
                return cbi_fail(b, CB_EARG, "set_weight: fc1 bias shape");
            rc = upload_f32(e, k->fc1b, src, count);
            break;
        default:
            return cbi_fail(b, CB_EARG, "set_weight: unknown tensor");
        }
    }
    if (rc == CB_OK)
        rc = cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "set_weight");
    return rc;
}

int cb_encoder_init_random(cb_encoder *e, uint64_t seed, float std, double theta)
{
    const size_t E = (size_t)e->cfg.embed, mlp = (size_t)e->cfg.mlp;
    const size_t kin = 3 * (size_t)e->cfg.patch * e->cfg.patch;
    cb_backend *b = e->b;
    k_stream st;
    void *s = NULL;
    float *tab;
    int i, rc = CB_OK;

    CB_TRY(cbi_enter(b));
    st = (k_stream)b->stream;
    /* patch_embed [E, 3p^2] -> bf16 [E, kpad] (padding stays zero) */
    CB_TRY(cbi_scratch(b, E * kin * 2 + (size_t)e->T * E * 4, &s));
    CB_TRY(cbi_kstatus(b, k_synth_normal(seed, SAM3_STREAM_PATCH_W, (long)(E * kin),
                                        0.0f, std, s, 1, st),
                      "init_random"));
    CB_TRY(cbi_kstatus(b,
                      (int)cudaMemcpy2DAsync(e->pe_w, (size_t)e->kpad * 2, s, kin * 2,
                                             kin * 2, E, cudaMemcpyDeviceToDevice,
                                             b->stream),
                      "init_random"));
    /* pos_embed on the raster grid -> window-major rows */
    CB_TRY(cbi_kstatus(b, k_synth_normal(seed, SAM3_STREAM_POS, (long)(e->T * E), 0.0f,
                                        std, (char *)s + E * kin * 2, 0, st),
                      "init_random"));
    CB_TRY(cbi_kstatus(b,
                      k_permute_rows((const float *)((char *)s + E * kin * 2), e->pos,
                                     1, e->cfg.grid, e->cfg.window, (int)E, st),
                      "init_random"));
    CB_TRY(cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "init_random"));
    CB_TRY(fill_f32(e, e->lnpw, 1.0f, E));
    CB_TRY(fill_f32(e, e->lnpb, 0.0f, E));
    for (i = 0; i < e->cfg.depth && rc == CB_OK; i++) {
        struct enc_block *k = &e->blk[i];
        const uint64_t s0 = SAM3_STREAM_BLOCK0 + 16 * (uint64_t)i;

        rc = cbi_kstatus(b, k_synth_normal(seed, s0 + SAM3_BT_QKV_W, (long)(3 * E * E),
                                          0.0f, std, k->qkvw, 1, st), "init_random");
        if (rc == CB_OK)
            rc = cbi_kstatus(b, k_synth_normal(seed, s0 + SAM3_BT_PROJ_W, (long)(E * E),
                                              0.0f, std, k->projw, 1, st), "init_random");
        if (rc == CB_OK)
            rc = cbi_kstatus(b, k_synth_normal(seed, s0 + SAM3_BT_FC1_W, (long)(mlp * E),
                                              0.0f, std, k->fc1w, 1, st), "init_random");
        if (rc == CB_OK)
            rc = cbi_kstatus(b, k_synth_normal(seed, s0 + SAM3_BT_FC2_W, (long)(mlp * E),
                                              0.0f, std, k->fc2w, 1, st), "init_random");
        if (rc == CB_OK)
            rc = fill_f32(e, k->n1w, 1.0f, E);
        if (rc == CB_OK)
            rc = fill_f32(e, k->n2w, 1.0f, E);
        if (rc == CB_OK) {
            cudaMemsetAsync(k->n1b, 0, E * 4, b->stream);
            cudaMemsetAsync(k->n2b, 0, E * 4, b->stream);
            cudaMemsetAsync(k->qkvb, 0, 3 * E * 4, b->stream);
            cudaMemsetAsync(k->projb, 0, E * 4, b->stream);
            cudaMemsetAsync(k->fc1b, 0, mlp * 4, b->stream);
            cudaMemsetAsync(k->fc2b, 0, E * 4, b->stream);
        }
    }
    CB_TRY(rc);
    /* 2D axial RoPE tables (host-generated, as the checkpoint's freqs_cis
     * would be) */
    tab = malloc((size_t)e->T * e->hd * 4);
    if (!tab)
        return CB_EALLOC;
    sam3_synth_rope_axial(e->cfg.window, e->hd, theta, tab);
    rc = upload_f32(e, e->rope_win, tab, (size_t)e->ws2 * e->hd);
    if (rc == CB_OK)
        rc = cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "init_random");
    sam3_synth_rope_axial(e->cfg.grid, e->hd, theta, tab);
    if (rc == CB_OK)
        rc = upload_f32(e, e->rope_glob, tab, (size_t)e->T * e->hd);
    if (rc == CB_OK)
        rc = cbi_kstatus(b, (int)cudaStreamSynchronize(b->stream), "init_random");
    free(tab);
    return rc;
}

/* ---------------------------------------------------------------- forward */

/* One launch bracketed by the profiler, its result mapped to a status. */
#define LAUNCH(name, flops, bytes, call)                                       \
    do {                                                                       \
        int lrc_;                                                              \
        cbi_prof_begin(b, name, (double)(flops), (double)(bytes));             \
        lrc_ = (call);                                                         \
        cbi_prof_end(b);                                                       \
        CB_TRY(cbi_kstatus(b, lrc_, name));                                    \
    } while (0)

static int run_blocks(cb_encoder *e, int ntile, int first, int last)
{
    cb_backend *b = e->b;
    const k_stream st = (k_stream)b->stream;
    const int E = e->cfg.embed, mlp = e->cfg.mlp, heads = e->cfg.heads;
    const int rows = ntile * e->T;
    const double R = rows, dE = E, dM = mlp;
    const float scale = 1.0f / sqrtf((float)e->hd);
    int i;

    for (i = first; i < last; i++) {
        const struct enc_block *k = &e->blk[i];
        const int global = (int)((e->cfg.global_mask >> i) & 1);
        const int nseq = global ? ntile : ntile * e->nwin;
        const int N = global ? e->T : e->ws2;
        struct k_rope rope;

        rope.cs = global ? e->rope_glob : e->rope_win;
        rope.mode = global ? 2 : 1;
        rope.E = E;
        rope.hd = e->hd;
        rope.npos = global ? e->T : e->ws2;
        rope.ws = e->cfg.window;
        rope.nwx = e->cfg.grid / e->cfg.window;
        rope.grid = e->cfg.grid;

        LAUNCH("layernorm", 8 * R * dE, R * dE * 6,
               k_layernorm(e->x, e->xn, 1, k->n1w, k->n1b, rows, E, 1e-5f,
                           K_ACT_NONE, st));
        LAUNCH("gemm_qkv", 2 * R * 3 * dE * dE, R * dE * 2 + 3 * dE * dE * 2 + R * 3 * dE * 2,
               k_gemm_bf16_tc(rows, 3 * E, E, e->xn, E, k->qkvw, E, e->qkv, 3 * E, 1,
                              k->qkvb, NULL, 0, 0, 1.0f, K_ACT_NONE, &rope, b->d_err,
                              b->num_sms, st));
        LAUNCH(global ? "attn_global" : "attn_window",
               4.0 * nseq * heads * (double)N * N * e->hd, R * 4 * dE * 2,
               k_attn_tc(e->qkv, nseq, N, E, heads, scale, e->attn, 1, NULL, 0, b->d_err,
                         st));  /* whole items: a tile's result never depends on its batch */
        LAUNCH("gemm_proj", 2 * R * dE * dE, R * dE * 2 + dE * dE * 2 + R * dE * 8,
               k_gemm_bf16_tc(rows, E, E, e->attn, E, k->projw, E, e->x, E, 0, k->projb,
                              e->x, E, 0, 1.0f, K_ACT_NONE, NULL, b->d_err, b->num_sms,
                              st));
        LAUNCH("layernorm", 8 * R * dE, R * dE * 6,
               k_layernorm(e->x, e->xn, 1, k->n2w, k->n2b, rows, E, 1e-5f,
                           K_ACT_NONE, st));
        LAUNCH("gemm_fc1", 2 * R * dM * dE, R * dE * 2 + dM * dE * 2 + R * dM * 2,
               k_gemm_bf16_tc(rows, mlp, E, e->xn, E, k->fc1w, E, e->h, mlp, 1, k->fc1b,
                              NULL, 0, 0, 1.0f, K_ACT_GELU, NULL, b->d_err, b->num_sms,
                              st));
        LAUNCH("gemm_fc2", 2 * R * dM * dE, R * dM * 2 + dM * dE * 2 + R * dE * 8,
               k_gemm_bf16_tc(rows, E, mlp, e->h, mlp, k->fc2w, mlp, e->x, E, 0, k->fc2b,
                              e->x, E, 0, 1.0f, K_ACT_NONE, NULL, b->d_err, b->num_sms,
                              st));
    }
    return CB_OK;
}

static int encode_dev(cb_encoder *e, const uint8_t *tiles, int ntile, float *out)
{
    cb_backend *b = e->b;
    const k_stream st = (k_stream)b->stream;
    const int E = e->cfg.embed;
    const int rows = ntile * e->T;
    const int side = e->cfg.grid * e->cfg.patch;
    const double R = rows, dE = E, kp = e->kpad;

    /* patch embedding: uint8 -> normalised bf16 patch rows (window-major),
     * GEMM with the conv weight (no bias) + pos_embed residual, ln_pre */
    LAUNCH("patch_in", 0, (double)ntile * side * side * 3 + R * kp * 2,
           k_patch_embed_in(tiles, ntile, side, e->cfg.grid, e->cfg.patch,
                            e->cfg.window, e->kpad, e->h, st));
    LAUNCH("gemm_patch", 2 * R * dE * 3 * e->cfg.patch * e->cfg.patch,
           R * kp * 2 + dE * kp * 2 + R * dE * 4 + e->T * dE * 4,
           k_gemm_bf16_tc(rows, E, e->kpad, e->h, e->kpad, e->pe_w, e->kpad, e->x, E, 0,
                          NULL, e->pos, E, e->T, 1.0f, K_ACT_NONE, NULL, b->d_err,
                          b->num_sms, st));
    LAUNCH("layernorm", 8 * R * dE, R * dE * 8,
           k_layernorm(e->x, e->x, 0, e->lnpw, e->lnpb, rows, E, 1e-5f, K_ACT_NONE, st));
    CB_TRY(run_blocks(e, ntile, 0, e->cfg.depth));
    LAUNCH("unpermute", 0, R * dE * 8,
           k_unpermute_rows(e->x, out, ntile, e->cfg.grid, e->cfg.window, E, st));
    return CB_OK;
}

int cb_encode_tiles(cb_encoder *e, cb_mem tiles, int ntile, cb_mem out)
{
    const size_t side = (size_t)e->cfg.grid * e->cfg.patch;

    if (!e || !tiles || !out || ntile <= 0 || ntile > e->cfg.max_tiles ||
        tiles->dtype != CB_U8 || out->dtype != CB_F32 ||
        tiles->bytes < (size_t)ntile * side * side * 3 ||
        out->bytes < (size_t)ntile * e->T * e->cfg.embed * 4)
        return cbi_fail(e ? e->b : NULL, CB_EARG, "encode_tiles");
    CB_TRY(cbi_enter(e->b));
    return encode_dev(e, (const uint8_t *)tiles->ptr, ntile, (float *)out->ptr);
}

int cb_encode_blocks(cb_encoder *e, cb_mem x, int ntile, int first, int last)
{
    cb_backend *b;
    const k_stream st = e ? (k_stream)e->b->stream : NULL;

    if (!e || !x || ntile <= 0 || ntile > e->cfg.max_tiles || first < 0 ||
        last > e->cfg.depth || first > last || x->dtype != CB_F32 ||
        x->bytes < (size_t)ntile * e->T * e->cfg.embed * 4)
        return cbi_fail(e ? e->b : NULL, CB_EARG, "encode_blocks");
    b = e->b;
    CB_TRY(cbi_enter(b));
    CB_TRY(cbi_kstatus(b, k_permute_rows((const float *)x->ptr, e->x, ntile,
                                        e->cfg.grid, e->cfg.window, e->cfg.embed,
                                        st), "encode_blocks"));
    CB_TRY(run_blocks(e, ntile, first, last));
    return cbi_kstatus(b, k_unpermute_rows(e->x, (float *)x->ptr, ntile, e->cfg.grid,
                                          e->cfg.window, e->cfg.embed, st),
                      "encode_blocks");
}

/* Chunk of the host-buffer pipeline: about a quarter of the batch, so that
 * the copies in and out of neighbouring chunks hide behind the compute and
 * only the first chunk's upload and the last chunk's download stay exposed,
 * but at least 4 tiles: smaller chunks leave the GEMMs and the attention
 * with wave tails that cost more than the exposed copies save (with 8 tiles
 * per GPU, two chunks of 4), at most max_tiles. */
static int host_chunk(const cb_encoder *e, int ntile)
{
    int c = (ntile + 3) / 4;

    if (c < 4)
        c = ntile < 4 ? ntile : 4;
    return c > e->cfg.max_tiles ? e->cfg.max_tiles : c;
}

static int host_pipeline_setup(cb_encoder *e, int chunk)
{
    const size_t side = (size_t)e->cfg.grid * e->cfg.patch;
    const size_t tile_in = side * side * 3;
    const size_t tile_out = (size_t)e->T * e->cfg.embed * 4;
    int i;

    if (e->chunk >= chunk)
        return CB_OK;
    for (i = 0; i < 2; i++) {
        cudaFree(e->tiles[i]);
        cudaFree(e->out_dev[i]);
        e->tiles[i] = NULL;
        e->out_dev[i] = NULL;
    }
    e->chunk = 0;
    for (i = 0; i < 2; i++) {
        CB_TRY(dev_alloc(e, (void **)&e->tiles[i], tile_in * chunk));
        CB_TRY(dev_alloc(e, (void **)&e->out_dev[i], tile_out * chunk));
        if (!e->ev_in[i] &&
            (cudaEventCreateWithFlags(&e->ev_in[i], cudaEventDisableTiming) != cudaSuccess ||
             cudaEventCreateWithFlags(&e->ev_done[i], cudaEventDisableTiming) != cudaSuccess ||
             cudaEventCreateWithFlags(&e->ev_out[i], cudaEventDisableTiming) != cudaSuccess))
            return cbi_fail(e->b, CB_ECUDA, "encode_tiles_host: events");
    }
    if (!e->h2d && (cudaStreamCreateWithFlags(&e->h2d, cudaStreamNonBlocking) != cudaSuccess ||
                    cudaStreamCreateWithFlags(&e->d2h, cudaStreamNonBlocking) != cudaSuccess))
        return cbi_fail(e->b, CB_ECUDA, "encode_tiles_host: streams");
    e->chunk = chunk;
    return CB_OK;
}

/* Host-to-host encode as a three-stage pipeline over chunks: chunk c's
 * host-to-device copy (h2d stream) and chunk c-1's device-to-host copy (d2h
 * stream) run while chunk c-1 / c computes on the backend stream. Buffer
 * c % 2 is reused by chunk c + 2 only after its copy out (outputs) and its
 * encode (inputs) are done, which the events order. */
int cb_encode_tiles_host(cb_encoder *e, const uint8_t *tiles, int ntile,
                         float *out)
{
    size_t side, tile_in, tile_out;
    cb_backend *b;
    int chunk, t0, c, n, tail, lim, nfull;

    if (!e || !tiles || !out || ntile <= 0)
        return cbi_fail(e ? e->b : NULL, CB_EARG, "encode_tiles_host");
    b = e->b;
    side = (size_t)e->cfg.grid * e->cfg.patch;
    tile_in = side * side * 3;
    tile_out = (size_t)e->T * e->cfg.embed * 4;
    CB_TRY(cbi_enter(b));
    chunk = host_chunk(e, ntile);
    CB_TRY(host_pipeline_setup(e, chunk));
    /* The last chunk's read-back is the copy nothing overlaps: when the
     * batch spans more than two chunks plus a small one, it ends with a
     * chunk of 4 tiles and the rest is cut into near-equal chunks of at
     * most `chunk` (64 tiles: 15 + 15 + 15 + 15 + 4). */
    tail = ntile >= 2 * chunk + 4 && chunk > 4 ? 4 : 0;
    lim = ntile - tail;
    nfull = (lim + chunk - 1) / chunk;
    for (t0 = 0, c = 0; t0 < ntile; t0 += n, c++) {
        const int i = c & 1;

        n = c < nfull ? lim / nfull + (c < lim % nfull) : tail;

        if (c >= 2)  /* chunk c - 2's encode has read tiles[i] */
            CB_TRY(cbi_kstatus(b, (int)cudaStreamWaitEvent(e->h2d, e->ev_done[i], 0),
                              "encode_tiles_host"));
        CB_TRY(cbi_kstatus(b, (int)cudaMemcpyAsync(e->tiles[i], tiles + t0 * tile_in,
                                                  n * tile_in, cudaMemcpyHostToDevice,
                                                  e->h2d), "encode_tiles_host"));
        CB_TRY(cbi_kstatus(b, (int)cudaEventRecord(e->ev_in[i], e->h2d), "encode_tiles_host"));
        CB_TRY(cbi_kstatus(b, (int)cudaStreamWaitEvent(b->stream, e->ev_in[i], 0),
                          "encode_tiles_host"));
        if (c >= 2)  /* chunk c - 2's outputs have left out_dev[i] */
            CB_TRY(cbi_kstatus(b, (int)cudaStreamWaitEvent(b->stream, e->ev_out[i], 0),
                              "encode_tiles_host"));
        CB_TRY(encode_dev(e, e->tiles[i], n, e->out_dev[i]));
        CB_TRY(cbi_kstatus(b, (int)cudaEventRecord(e->ev_done[i], b->stream),
                          "encode_tiles_host"));
        CB_TRY(cbi_kstatus(b, (int)cudaStreamWaitEvent(e->d2h, e->ev_done[i], 0),
                          "encode_tiles_host"));
        CB_TRY(cbi_kstatus(b, (int)cudaMemcpyAsync((char *)out + t0 * tile_out,
                                                  e->out_dev[i], n * tile_out,
                                                  cudaMemcpyDeviceToHost, e->d2h),
                          "encode_tiles_host"));
        CB_TRY(cbi_kstatus(b, (int)cudaEventRecord(e->ev_out[i], e->d2h), "encode_tiles_host"));
    }
    CB_TRY(cbi_kstatus(b, (int)cudaStreamSynchronize(e->d2h), "encode_tiles_host"));
    return cb_sync(b);
}
