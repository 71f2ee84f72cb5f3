/* SPDX-License-Identifier: Unlicense
 *
 * A C consumer of the drop-in boundary: the reference's vit_block
 * (sam3_model.c:981-1028) written the way the reference writes it, against
 * include/sam3_cuda.h, with the operator macros of INTEGRATION.md section 3
 * pasted unchanged and the one call-site change of section 4 (the fused
 * cb_attention in place of rope_apply + the per-head-chunk gemm / softmax_rows
 * / gemm loop). Compiled by tests/test_c_abi.py with gcc -std=gnu11 and
 * linked against libsam3cuda.so; the test compares what it writes with the
 * oracle's vit_block on the same seeded weights.
 *
 *   vit_block_abi <out.f32> <seed> <block kind: 0 windowed, 1 global>
 *
 * Weights come from the library's seeded generator (sam3_synth_normal) with
 * the streams of cb_encoder_init_random / the oracle's TrunkWeights (block i
 * = the test's block index 0 or 1 of a 2-block trunk): matrices N(0, 0.02)
 * uploaded as bf16 (the tensor-core operands), LayerNorm gamma 1 / beta 0,
 * biases 0. x = N(0, 1) from stream 99. Activations stay fp32, as in the
 * reference. Exit status 0 on success; any failed call prints its status
 * and exits 1 (the G_fatal_error path of the reference). */
#include "sam3_cuda.h"
#include "sam3_synth.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>

/* ---- what the port of sam3_model.c would carry ------------------------ */
#define SAM_GRID 72
#define ENC_EPS 1e-5f
#define ACT_NONE 0
#define ACT_GELU 1

struct sam_model {
    cb_backend *cb;
    int embed, heads, hd, mlp;
    cb_mem x, xn, xw, qkv, attn, tmp, mlpbuf;
    cb_mem rope_win, rope_glob;
};

struct vit_block {
    cb_mem n1w, n1b, qkvw, qkvb, projw, projb, n2w, n2b, l1w, l1b, l2w, l2b;
    int window;
};

struct geom {
    int s, nwx, nwin, N;
};

static void G_fatal_error(const char *fmt, const char *a, const char *b)
{
    fprintf(stderr, fmt, a, b);
    fputc('\n', stderr);
    exit(1);
}

static void cb_fatal(cb_backend *cb, int rc)
{
    if (rc != CB_OK)
        G_fatal_error("CUDA backend: %s (%s)", cb_errstr(rc), cb_last_error(cb));
}

/* ---- INTEGRATION.md section 3, verbatim ------------------------------- */
typedef struct cb_opnd opnd_t;           /* struct opnd (sam3_ops.h:19-24) */
#define opnd cb_opnd
#define mat(buf, off, ld) cb_mat(buf, off, ld)
#define bmat(buf, off, ld, s0, s1) cb_bmat(buf, off, ld, s0, s1)
#define gemm(m, M, N, K, A, B, tb, C, nb, nb1, bias, R, roff, alpha, act) \
    cb_fatal((m)->cb, cb_gemm((m)->cb, M, N, K, A, B, tb, C, nb, nb1, bias, R, roff, alpha, act))
#define linear(m, rows, in, out, X, xoff, W, b, Y, yoff, act, res) \
    cb_fatal((m)->cb, cb_linear((m)->cb, rows, in, out, X, xoff, W, b, Y, yoff, act, res))
#define layernorm(m, rows, C, X, Y, g, b, eps, act) \
    cb_fatal((m)->cb, cb_layernorm((m)->cb, rows, C, X, Y, g, b, eps, act))
#define add_bcast(m, out, a, b, n, bmod) \
    cb_fatal((m)->cb, cb_add_bcast((m)->cb, out, a, b, n, bmod))
/* ---------------------------------------------------------------------- */

/* sam3_model.c's static helpers, ported to the operators they launch. */
static struct geom block_geom(const struct vit_block *b)
{
    struct geom g;

    g.s = b->window ? b->window : SAM_GRID;
    g.nwx = SAM_GRID / g.s;
    g.nwin = g.nwx * g.nwx;
    g.N = g.s * g.s;
    return g;
}

static void window_partition(struct sam_model *m, cb_mem X, cb_mem out, int H, int C, int ws,
                             int nwx)
{
    cb_fatal(m->cb, cb_window_partition(m->cb, X, out, H, C, ws, nwx));
}

static void window_unpartition_add(struct sam_model *m, cb_mem X, cb_mem Wd, int H, int C,
                                   int ws, int nwx)
{
    cb_fatal(m->cb, cb_window_unpartition_add(m->cb, X, Wd, H, C, ws, nwx));
}

/* One ViT block, x updated in place: the reference's sequence with the
 * section 4 call-site change. */
static void vit_block(struct sam_model *m, const struct vit_block *b)
{
    const struct geom g = block_geom(b);
    const int T = SAM_GRID * SAM_GRID, E = m->embed, hd = m->hd;
    const long rows = (long)g.nwin * g.N;
    const float scale = 1.0f / sqrtf((float)hd);
    cb_mem A = m->xn;

    layernorm(m, T, E, m->x, m->xn, b->n1w, b->n1b, ENC_EPS, ACT_NONE);
    if (b->window) {
        window_partition(m, m->xn, m->xw, SAM_GRID, E, g.s, g.nwx);
        A = m->xw;
    }
    linear(m, (int)rows, E, 3 * E, A, 0, b->qkvw, b->qkvb, m->qkv, 0, ACT_NONE, 0);
    cb_fatal(m->cb, cb_attention(m->cb, m->qkv, g.nwin, g.N, E, m->heads, hd,
                                 b->window ? m->rope_win : m->rope_glob, g.N,
                                 scale, CB_ATTN_TC, m->attn));
    if (b->window) {
        linear(m, (int)rows, E, E, m->attn, 0, b->projw, b->projb, m->tmp, 0, ACT_NONE, 0);
        window_unpartition_add(m, m->x, m->tmp, SAM_GRID, E, g.s, g.nwx);
    }
    else
        linear(m, T, E, E, m->attn, 0, b->projw, b->projb, m->x, 0, ACT_NONE, 1);

    layernorm(m, T, E, m->x, m->xn, b->n2w, b->n2b, ENC_EPS, ACT_NONE);
    linear(m, T, E, m->mlp, m->xn, 0, b->l1w, b->l1b, m->mlpbuf, 0, ACT_GELU, 0);
    linear(m, T, m->mlp, E, m->mlpbuf, 0, b->l2w, b->l2b, m->x, 0, ACT_NONE, 1);
}

/* ---- the test driver: load_encoder's uploads for one block ------------ */
static float *host_normal(uint64_t seed, uint64_t stream, size_t n, float std)
{
    float *p = malloc(n * sizeof(float));

    if (!p)
        G_fatal_error("%s%s", "out of host memory", "");
    sam3_synth_normal(seed, stream, n, 0.0f, std, p);
    return p;
}

static cb_mem upload_f32(struct sam_model *m, const float *src, size_t n)
{
    cb_mem d;

    cb_fatal(m->cb, cb_upload(m->cb, src, n * sizeof(float), CB_F32, &d));
    return d;
}

static cb_mem upload_const(struct sam_model *m, float v, size_t n)
{
    float *h = malloc(n * sizeof(float));
    cb_mem d;
    size_t i;

    if (!h)
        G_fatal_error("%s%s", "out of host memory", "");
    for (i = 0; i < n; i++)
        h[i] = v;
    d = upload_f32(m, h, n);
    free(h);
    return d;
}

static cb_mem weight_bf16(struct sam_model *m, uint64_t seed, uint64_t stream, size_t n)
{
    float *h = host_normal(seed, stream, n, 0.02f);
    cb_mem d;

    cb_fatal(m->cb, cb_upload_weight(m->cb, h, n, CB_BF16, &d));
    free(h);
    return d;
}

static cb_mem alloc_f32(struct sam_model *m, size_t n)
{
    cb_mem d;

    cb_fatal(m->cb, cb_alloc(m->cb, n * sizeof(float), CB_F32, &d));
    return d;
}

int main(int argc, char **argv)
{
    struct sam_model m;
    struct vit_block blk;
    const int T = SAM_GRID * SAM_GRID;
    uint64_t seed, s0;
    int kind;
    size_t E;
    float *x, *tab;
    FILE *f;

    if (argc != 4) {
        fprintf(stderr, "usage: %s <out.f32> <seed> <0 windowed | 1 global>\n", argv[0]);
        return 2;
    }
    seed = strtoull(argv[2], NULL, 10);
    kind = atoi(argv[3]);
    m.embed = 1024;
    m.heads = 16;
    m.hd = 64;
    m.mlp = 4096;
    E = (size_t)m.embed;
    cb_fatal(NULL, cb_init(&m.cb, 0));

    /* the block's tensors, streams as in a 2-block trunk (block index kind) */
    s0 = SAM3_STREAM_BLOCK0 + 16 * (uint64_t)kind;
    blk.window = kind == 0 ? 24 : 0;
    blk.n1w = upload_const(&m, 1.0f, E);
    blk.n1b = upload_const(&m, 0.0f, E);
    blk.n2w = upload_const(&m, 1.0f, E);
    blk.n2b = upload_const(&m, 0.0f, E);
    blk.qkvb = upload_const(&m, 0.0f, 3 * E);
    blk.projb = upload_const(&m, 0.0f, E);
    blk.l1b = upload_const(&m, 0.0f, (size_t)m.mlp);
    blk.l2b = upload_const(&m, 0.0f, E);
    blk.qkvw = weight_bf16(&m, seed, s0 + SAM3_BT_QKV_W, 3 * E * E);
    blk.projw = weight_bf16(&m, seed, s0 + SAM3_BT_PROJ_W, E * E);
    blk.l1w = weight_bf16(&m, seed, s0 + SAM3_BT_FC1_W, (size_t)m.mlp * E);
    blk.l2w = weight_bf16(&m, seed, s0 + SAM3_BT_FC2_W, E * (size_t)m.mlp);

    /* RoPE tables (load_encoder, sam3_model.c:457-471) */
    tab = malloc((size_t)T * m.hd * sizeof(float));
    if (!tab)
        G_fatal_error("%s%s", "out of host memory", "");
    sam3_synth_rope_axial(24, m.hd, 10000.0, tab);
    m.rope_win = upload_f32(&m, tab, (size_t)576 * m.hd);
    sam3_synth_rope_axial(SAM_GRID, m.hd, 10000.0, tab);
    m.rope_glob = upload_f32(&m, tab, (size_t)T * m.hd);
    free(tab);

    /* alloc_buffers (sam3_model.c:815-916), fp32 as in the reference */
    x = host_normal(seed, 99, (size_t)T * E, 1.0f);
    m.x = upload_f32(&m, x, (size_t)T * E);
    m.xn = alloc_f32(&m, (size_t)T * E);
    m.xw = alloc_f32(&m, (size_t)T * E);
    m.qkv = alloc_f32(&m, (size_t)T * 3 * E);
    m.attn = alloc_f32(&m, (size_t)T * E);
    m.tmp = alloc_f32(&m, (size_t)T * E);
    m.mlpbuf = alloc_f32(&m, (size_t)T * m.mlp);

    vit_block(&m, &blk);

    cb_fatal(m.cb, cb_read(m.cb, m.x, 0, x, (size_t)T * E * sizeof(float)));
    cb_fatal(m.cb, cb_sync(m.cb));
    f = fopen(argv[1], "wb");
    if (!f || fwrite(x, sizeof(float), (size_t)T * E, f) != (size_t)T * E)
        G_fatal_error("cannot write %s%s", argv[1], "");
    fclose(f);
    free(x);
    cb_free(m.cb);
    return 0;
}
