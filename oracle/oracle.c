/* CPU restatement of the reference's hot-path kernels (see oracle.h).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
 *
 * Floating-point conventions shared with oracle/ocl_shim.hpp (which compiles
 * the reference kernels themselves): OpenCL mad() = fmaf; dot(float4) =
 * fmaf(w, fmaf(z, fmaf(y, x*x')))); built with -ffp-contract=off so that no
 * other multiply-add is fused. */
#include "oracle.h"
#include "sam3_synth.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* gelu_erf / apply_act: sam3_kernels.cl:43-55. */
static inline float gelu_erf(float x)
{
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

static inline float apply_act(float v, int act)
{
    if (act == OR_ACT_GELU)
        return gelu_erf(v);
    if (act == OR_ACT_RELU)
        return fmaxf(v, 0.0f);
    return v;
}

/* store_one: sam3_kernels.cl:307-319. */
static inline void store_one(float *C, const float *R, const float *bias,
                             int m, int n, int ldc, float alpha, int act,
                             float v)
{
    float x = alpha * v;

    if (bias)
        x += bias[n];
    x = apply_act(x, act);
    if (R)
        x += R[(long)m * ldc + n];
    C[(long)m * ldc + n] = x;
}

/* gemm_cpu_t (sam3_kernels.cl:334-391) for one 2 x 4 output block
 * (m0, n0): eight-lane partial sums along K in steps of 8 when the whole
 * block is inside C, hsum8 (lo + hi, then x + y + z + w), then the K tail. */
static void gemm_t_block(int M, int N, int K, const float *A, int lda,
                         const float *B, int ldb, float *C, int ldc,
                         const float *bias, const float *R, float alpha,
                         int act, int m0, int n0)
{
    float s[2][4][8];
    int i, j, k, l;

    memset(s, 0, sizeof(s));
    if (m0 + 1 < M && n0 + 3 < N) {
        const float *a0 = A + (long)m0 * lda, *a1 = A + (long)(m0 + 1) * lda;

        for (k = 0; k + 8 <= K; k += 8)
            for (j = 0; j < 4; j++) {
                const float *bv = B + (long)(n0 + j) * ldb + k;

                for (l = 0; l < 8; l++) {
                    s[0][j][l] = fmaf(a0[k + l], bv[l], s[0][j][l]);
                    s[1][j][l] = fmaf(a1[k + l], bv[l], s[1][j][l]);
                }
            }
    }
    else
        k = 0;
    for (i = 0; i < 2; i++)
        for (j = 0; j < 4; j++) {
            const int m = m0 + i, n = n0 + j;
            const float *t = s[i][j];
            float h0, h1, h2, h3, v;
            int kk;

            if (m >= M || n >= N)
                continue;
            h0 = t[0] + t[4];
            h1 = t[1] + t[5];
            h2 = t[2] + t[6];
            h3 = t[3] + t[7];
            v = h0 + h1 + h2 + h3;
            for (kk = k; kk < K; kk++)
                v = fmaf(A[(long)m * lda + kk], B[(long)n * ldb + kk], v);
            store_one(C, R, bias, m, n, ldc, alpha, act, v);
        }
}

/* gemm_cpu_n (sam3_kernels.cl:395-448): every output is one fmaf chain
 * along K starting from zero, in both the float8 and the scalar branch. */
static void gemm_n_row(int N, int K, const float *A, int lda, const float *B,
                       int ldb, float *C, int ldc, const float *bias,
                       const float *R, float alpha, int act, int m, float *acc)
{
    int n, k;

    for (n = 0; n < N; n++)
        acc[n] = 0.0f;
    for (k = 0; k < K; k++) {
        const float a = A[(long)m * lda + k];
        const float *b = B + (long)k * ldb;

        for (n = 0; n < N; n++)
            acc[n] = fmaf(a, b[n], acc[n]);
    }
    for (n = 0; n < N; n++)
        store_one(C, R, bias, m, n, ldc, alpha, act, acc[n]);
}

/* Batched GEMM with the reference's operand contract (sam3_kernels.cl:57-69,
 * host geometry sam3_model.c:289-296). */
void or_gemm(const struct or_gemm_args *a, int nb)
{
    int b;

    for (b = 0; b < nb; b++) {
        const long b0 = b / a->nb1, b1 = b % a->nb1;
        const float *A = a->A + a->aoff + b0 * a->sa0 + b1 * a->sa1;
        const float *B = a->B + a->boff + b0 * a->sb0 + b1 * a->sb1;
        float *C = a->C + a->coff + b0 * a->sc0 + b1 * a->sc1;
        const float *R = a->R ? a->R + a->roff + b0 * a->sc0 + b1 * a->sc1
                              : NULL;

        if (a->transb) {
            const int mb = (a->M + 1) / 2, nbk = (a->N + 3) / 4;
            long t;

#pragma omp parallel for schedule(dynamic, 8)
            for (t = 0; t < (long)mb * nbk; t++)
                gemm_t_block(a->M, a->N, a->K, A, a->lda, B, a->ldb, C,
                             a->ldc, a->bias, R, a->alpha, a->act,
                             (int)(t / nbk) * 2, (int)(t % nbk) * 4);
        }
        else {
#pragma omp parallel
            {
                float *acc = malloc(sizeof(float) * (size_t)a->N);
                int m;

#pragma omp for schedule(dynamic, 4)
                for (m = 0; m < a->M; m++)
                    gemm_n_row(a->N, a->K, A, a->lda, B, a->ldb, C, a->ldc,
                               a->bias, R, a->alpha, a->act, m, acc);
                free(acc);
            }
        }
    }
}

/* layernorm: sam3_kernels.cl:489-514 with one work-item per row. */
void or_layernorm(const float *X, float *Y, const float *g, const float *b,
                  long rows, int C, float eps, int act)
{
    long r;

#pragma omp parallel for schedule(static)
    for (r = 0; r < rows; r++) {
        const float *x = X + r * C;
        float *y = Y + r * C;
        float s = 0.0f, mean, var;
        int c;

        for (c = 0; c < C; c++)
            s += x[c];
        mean = s / C;
        s = 0.0f;
        for (c = 0; c < C; c++) {
            const float d = x[c] - mean;

            s += d * d;
        }
        var = s / C;
        s = 1.0f / sqrtf(var + eps);
        for (c = 0; c < C; c++)
            y[c] = apply_act((x[c] - mean) * s * g[c] + b[c], act);
    }
}

/* softmax_rows: sam3_kernels.cl:637-656 with one work-item per row. */
static void softmax_row(float *s, int L)
{
    float m = -INFINITY, sum = 0.0f, v;
    int j;

    for (j = 0; j < L; j++)
        m = fmaxf(m, s[j]);
    for (j = 0; j < L; j++) {
        v = expf(s[j] - m);
        s[j] = v;
        sum += v;
    }
    v = 1.0f / sum;
    for (j = 0; j < L; j++)
        s[j] *= v;
}

void or_softmax_rows(float *S, long rows, int L)
{
    long r;

#pragma omp parallel for schedule(static)
    for (r = 0; r < rows; r++)
        softmax_row(S + r * L, L);
}

/* rope_apply: sam3_kernels.cl:679-698 (row r uses table row r % npos). */
void or_rope_apply(float *qkv, long rows, int E, int hd, int npos,
                   const float *cs)
{
    const int nf = hd / 2;
    long r;

#pragma omp parallel for schedule(static)
    for (r = 0; r < rows; r++) {
        int qk, pr;

        for (qk = 0; qk < 2; qk++)
            for (pr = 0; pr < E / 2; pr++) {
                const int h = pr / nf, j = pr % nf;
                float *x = qkv + r * 3 * E + qk * E + h * hd + 2 * j;
                const float *rot = cs + ((r % npos) * nf + j) * 2;
                const float a = x[0], b = x[1];

                x[0] = a * rot[0] - b * rot[1];
                x[1] = a * rot[1] + b * rot[0];
            }
    }
}

/* add_bcast: sam3_kernels.cl:701-708. */
void or_add_bcast(float *out, const float *a, const float *b, long n,
                  long bmod)
{
    long i;

#pragma omp parallel for schedule(static)
    for (i = 0; i < n; i++)
        out[i] = a[i] + b[i % bmod];
}

/* window_partition: sam3_kernels.cl:712-724. */
void or_window_partition(const float *X, float *out, int H, int C, int ws,
                         int nwx)
{
    const long rows = (long)nwx * nwx * ws * ws;
    long r;

#pragma omp parallel for schedule(static)
    for (r = 0; r < rows; r++) {
        const int w = (int)(r / (ws * ws)), i = (int)(r % (ws * ws));
        const int y = (w / nwx) * ws + i / ws, x = (w % nwx) * ws + i % ws;
        int c;

        for (c = 0; c < C; c++)
            out[r * C + c] =
                (y < H && x < H) ? X[((long)y * H + x) * C + c] : 0.0f;
    }
}

/* window_unpartition_add: sam3_kernels.cl:728-741. */
void or_window_unpartition_add(float *X, const float *Wd, int H, int C,
                               int ws, int nwx)
{
    long t;

#pragma omp parallel for schedule(static)
    for (t = 0; t < (long)H * H; t++) {
        const int y = (int)(t / H), x = (int)(t % H);
        const int w = (y / ws) * nwx + x / ws, i = (y % ws) * ws + x % ws;
        int c;

        for (c = 0; c < C; c++)
            X[t * C + c] += Wd[((long)w * ws * ws + i) * C + c];
    }
}

/* patch_im2col: sam3_kernels.cl:661-672. */
void or_patch_im2col(const float *img, float *out, int side, int grid, int ps)
{
    const int k = 3 * ps * ps;
    long t;

#pragma omp parallel for schedule(static)
    for (t = 0; t < (long)grid * grid; t++) {
        const int ty = (int)(t / grid), tx = (int)(t % grid);
        int col;

        for (col = 0; col < k; col++) {
            const int c = col / (ps * ps), ky = (col % (ps * ps)) / ps,
                      kx = col % ps;

            out[t * k + col] =
                img[((long)c * side + ty * ps + ky) * side + tx * ps + kx];
        }
    }
}

/* image_encoder_input without resampling (image.c:346-369): uint8 HWC to
 * CHW floats (u / 255 - 0.5) / 0.5 (pixel_mean = pixel_std = 0.5,
 * image.c:28-29). */
void or_image_input(const uint8_t *rgb, int side, float *out)
{
    long i;

#pragma omp parallel for schedule(static)
    for (i = 0; i < (long)side * side; i++) {
        int c;

        for (c = 0; c < 3; c++)
            out[(long)c * side * side + i] = (rgb[i * 3 + c] / 255.0f - 0.5f) / 0.5f;
    }
}

/* float16 dot product of the decoder kernels (dot16,
 * sam3_kernels.cl:516-520): four float4 dots added left to right. */
static inline float dot4(const float *a, const float *b)
{
    return fmaf(a[3], b[3], fmaf(a[2], b[2], fmaf(a[1], b[1], a[0] * b[0])));
}

static inline float dot16(const float *a, const float *b)
{
    return dot4(a, b) + dot4(a + 4, b + 4) + dot4(a + 8, b + 8) +
           dot4(a + 12, b + 12);
}

/* attn_fewkeys: sam3_kernels.cl:527-569, one (prompt, head, query) item. */
static void attn_fewkeys_item(const float *Q, int sq, const float *K, int sk,
                              const float *V, int sv, float *O, int Nq, int Nk,
                              int dint, int c, float scale, int gid)
{
    const int heads = 8;
    const int i = gid % Nq, ph = gid / Nq;
    const int h = ph % heads, p = ph / heads;
    const float *q = Q + (long)p * sq + (long)i * dint + h * c;
    const float *kb = K + (long)p * sk + h * c;
    const float *vb = V + (long)p * sv + h * c;
    float o[32] = {0}, m = -INFINITY, sum = 0.0f;
    int j, l;

    for (j = 0; j < Nk; j++) {
        const float *kj = kb + (long)j * dint, *vj = vb + (long)j * dint;
        float s = dot16(q, kj), mn, corr, e;

        if (c > 16)
            s += dot16(q + 16, kj + 16);
        s *= scale;
        mn = fmaxf(m, s);
        corr = expf(m - mn);
        e = expf(s - mn);
        sum = sum * corr + e;
        for (l = 0; l < (c > 16 ? 32 : 16); l++)
            o[l] = o[l] * corr + e * vj[l];
        m = mn;
    }
    O += ((long)p * Nq + i) * dint + h * c;
    for (l = 0; l < (c > 16 ? 32 : 16); l++)
        O[l] = o[l] / sum;
}

/* attn_manykeys: sam3_kernels.cl:577-633 for one (prompt, head, query)
 * row: 256 item-partial online softmaxes, then the work-group tree
 * reductions (wg_max, wg_sum, and the 16 weighted-value sums). */
static void attn_manykeys_row(const float *Q, int sq, const float *K, int sk,
                              const float *V, int sv, float *O, int Nq, int Nk,
                              int dint, int c, float scale, int row,
                              float (*part)[257], float *mm, float *ss)
{
    const int heads = 8;
    const int i = row % Nq, ph = row / Nq;
    const int h = ph % heads, p = ph / heads;
    const float *kb = K + (long)p * sk + h * c;
    const float *vb = V + (long)p * sv + h * c;
    const float *q = Q + (long)p * sq + (long)i * dint + h * c;
    float scratch[256], mall, inv;
    int lid, j, s;

    for (lid = 0; lid < 256; lid++) {
        float o[16] = {0}, m = -INFINITY, sum = 0.0f;

        for (j = lid; j < Nk; j += 256) {
            const float sc = dot16(q, kb + (long)j * dint) * scale;
            const float mn = fmaxf(m, sc), corr = expf(m - mn),
                        e = expf(sc - mn);
            int l;

            sum = sum * corr + e;
            for (l = 0; l < 16; l++)
                o[l] = o[l] * corr + e * vb[(long)j * dint + l];
            m = mn;
        }
        mm[lid] = m;
        ss[lid] = sum;
        for (j = 0; j < 16; j++)
            part[j][lid] = o[j];
    }
    for (lid = 0; lid < 256; lid++)
        scratch[lid] = mm[lid];
    for (s = 128; s > 0; s >>= 1)
        for (lid = 0; lid < s; lid++)
            scratch[lid] = fmaxf(scratch[lid], scratch[lid + s]);
    mall = scratch[0];
    for (lid = 0; lid < 256; lid++) {
        const float f = mm[lid] == -INFINITY ? 0.0f : expf(mm[lid] - mall);

        for (j = 0; j < 16; j++)
            part[j][lid] *= f;
        scratch[lid] = ss[lid] * f;
    }
    for (s = 128; s > 0; s >>= 1)
        for (lid = 0; lid < s; lid++)
            scratch[lid] += scratch[lid + s];
    inv = 1.0f / scratch[0];
    for (s = 128; s > 0; s >>= 1)
        for (lid = 0; lid < s; lid++)
            for (j = 0; j < 16; j++)
                part[j][lid] += part[j][lid + s];
    for (j = 0; j < 16; j++)
        O[((long)p * Nq + i) * dint + h * c + j] = part[j][0] * inv;
}

/* mha: sam3_model.c:419-451 (8 heads, scale 1/sqrt(c), fewkeys for
 * Nk <= 64, manykeys otherwise, which needs c == 16). */
int or_mha(int P, int Nq, int Nk, int dint, const float *qp, long sq,
           const float *kp, long sk, const float *vp, long sv, float *o)
{
    const int heads = 8, c = dint / heads, total = P * heads * Nq;
    const float scale = 1.0f / sqrtf((float)c);
    int g;

    if (Nk > 64 && c != 16)
        return -1;
    if (Nk <= 64) {
#pragma omp parallel for schedule(static)
        for (g = 0; g < total; g++)
            attn_fewkeys_item(qp, (int)sq, kp, (int)sk, vp, (int)sv, o, Nq, Nk,
                              dint, c, scale, g);
        return 0;
    }
#pragma omp parallel
    {
        float(*part)[257] = malloc(sizeof(float) * 16 * 257);
        float *mm = malloc(sizeof(float) * 256), *ss = malloc(sizeof(float) * 256);

#pragma omp for schedule(dynamic, 4)
        for (g = 0; g < total; g++)
            attn_manykeys_row(qp, (int)sq, kp, (int)sk, vp, (int)sv, o, Nq, Nk,
                              dint, c, scale, g, part, mm, ss);
        free(part);
        free(mm);
        free(ss);
    }
    return 0;
}

/* Attention of vit_block, sam3_model.c:1000-1013, one query row at a time:
 * scores by the gemm_cpu_t arithmetic (2 x 4 blocks, eight lanes along the
 * head dimension, alpha applied in store_one), softmax_rows, then P.V by
 * the gemm_cpu_n arithmetic (one fmaf chain along the keys). Rows of the
 * score matrix are independent, so this gives the same bits as the
 * reference's batched, head-chunked launches. */
void or_attention(const float *qkv, int nseq, int N, int E, int heads, int hd,
                  float alpha, float *out)
{
    const long ld = 3L * E;
    const long total = (long)nseq * heads * N;
    long t;

#pragma omp parallel
    {
        float *s = malloc(sizeof(float) * (size_t)N);
        float *acc = malloc(sizeof(float) * (size_t)hd);

#pragma omp for schedule(dynamic, 16)
        for (t = 0; t < total; t++) {
            const int m = (int)(t % N), h = (int)((t / N) % heads);
            const long w = t / ((long)N * heads);
            const float *Q = qkv + w * N * ld + (long)h * hd;
            const float *K = qkv + w * N * ld + E + (long)h * hd;
            const float *V = qkv + w * N * ld + 2L * E + (long)h * hd;
            const float *q = Q + (long)m * ld;
            const int m0 = m & ~1;
            int n, k, l, d;

            for (n = 0; n < N; n++) {
                const int n0 = n & ~3;
                const float *kv = K + (long)n * ld;
                float v;

                k = 0;
                if (m0 + 1 < N && n0 + 3 < N) {
                    float lane[8] = {0};

                    for (k = 0; k + 8 <= hd; k += 8)
                        for (l = 0; l < 8; l++)
                            lane[l] = fmaf(q[k + l], kv[k + l], lane[l]);
                    v = (lane[0] + lane[4]) + (lane[1] + lane[5]) +
                        (lane[2] + lane[6]) + (lane[3] + lane[7]);
                }
                else
                    v = 0.0f;
                for (; k < hd; k++)
                    v = fmaf(q[k], kv[k], v);
                s[n] = alpha * v;
            }
            softmax_row(s, N);
            for (d = 0; d < hd; d++)
                acc[d] = 0.0f;
            for (k = 0; k < N; k++) {
                const float p = s[k];
                const float *vv = V + (long)k * ld;

                for (d = 0; d < hd; d++)
                    acc[d] = fmaf(p, vv[d], acc[d]);
            }
            for (d = 0; d < hd; d++)
                out[(w * N + m) * E + (long)h * hd + d] = 1.0f * acc[d];
        }
        free(s);
        free(acc);
    }
}

static void linear(int rows, int in, int out, const float *X, const float *W,
                   const float *b, float *Y, int act, int residual)
{
    struct or_gemm_args a;

    memset(&a, 0, sizeof(a));
    a.M = rows;
    a.N = out;
    a.K = in;
    a.A = X;
    a.lda = in;
    a.B = W;
    a.ldb = in;
    a.transb = 1;
    a.C = Y;
    a.ldc = out;
    a.nb1 = 1;
    a.bias = b;
    a.R = residual ? Y : NULL;
    a.alpha = 1.0f;
    a.act = act;
    or_gemm(&a, 1);
}

void or_vit_block(const struct or_trunk *t, const struct or_block *b, float *x)
{
    const int G = t->grid, T = G * G, E = t->E, hd = t->hd;
    const int s = b->window ? b->window : G;
    const int nwx = (G + s - 1) / s, nwin = nwx * nwx, N = s * s;
    const long rows = (long)nwin * N;
    const float eps = 1e-5f, scale = 1.0f / sqrtf((float)hd);
    float *xn = malloc(sizeof(float) * (size_t)T * E);
    float *xw = b->window ? malloc(sizeof(float) * (size_t)rows * E) : NULL;
    float *qkv = malloc(sizeof(float) * (size_t)rows * 3 * E);
    float *attn = malloc(sizeof(float) * (size_t)rows * E);
    float *mlp = malloc(sizeof(float) * (size_t)T * t->mlp);
    const float *A = xn;

    or_layernorm(x, xn, b->n1w, b->n1b, T, E, eps, OR_ACT_NONE);
    if (b->window) {
        or_window_partition(xn, xw, G, E, s, nwx);
        A = xw;
    }
    linear((int)rows, E, 3 * E, A, b->qkvw, b->qkvb, qkv, OR_ACT_NONE, 0);
    or_rope_apply(qkv, rows, E, hd, N, b->window ? t->rope_win : t->rope_glob);
    or_attention(qkv, nwin, N, E, E / hd, hd, scale, attn);
    if (b->window) {
        float *tmp = xw; /* free again: reuse as the projection output */

        linear((int)rows, E, E, attn, b->projw, b->projb, tmp, OR_ACT_NONE, 0);
        or_window_unpartition_add(x, tmp, G, E, s, nwx);
    }
    else
        linear(T, E, E, attn, b->projw, b->projb, x, OR_ACT_NONE, 1);
    or_layernorm(x, xn, b->n2w, b->n2b, T, E, eps, OR_ACT_NONE);
    linear(T, E, t->mlp, xn, b->l1w, b->l1b, mlp, OR_ACT_GELU, 0);
    linear(T, t->mlp, E, mlp, b->l2w, b->l2b, x, OR_ACT_NONE, 1);
    free(xn);
    free(xw);
    free(qkv);
    free(attn);
    free(mlp);
}

void or_encode_trunk(const struct or_trunk *t, const float *img, float *x,
                     int first, int last)
{
    const int G = t->grid, T = G * G, E = t->E;
    const int K = 3 * t->patch * t->patch;
    int i;

    if (img) {
        float *col = malloc(sizeof(float) * (size_t)T * K);

        or_patch_im2col(img, col, t->img, G, t->patch);
        linear(T, K, E, col, t->pe_w, NULL, x, OR_ACT_NONE, 0);
        or_add_bcast(x, x, t->pos, (long)T * E, (long)T * E);
        or_layernorm(x, x, t->lnpw, t->lnpb, T, E, 1e-5f, OR_ACT_NONE);
        free(col);
    }
    for (i = first; i < last; i++)
        or_vit_block(t, &t->blocks[i], x);
}

int or_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------ mask decoder */

/* Shape and init kind of decoder tensor i (include/sam3_synth.h). */
void or_dec_tensor(int i, int *rows, int *cols, int *init)
{
    sam3_dec_tensor(i, rows, cols, init);
}

/* convt_scatter: sam3_kernels.cl:766-781, one work-item per output value. */
void or_convt_scatter(const float *G, float *out, const float *bias,
                      const float *add, int P, int H, int W, int Co, int act)
{
    const long total = (long)P * 4 * H * W * Co;
    long gid;

#pragma omp parallel for schedule(static)
    for (gid = 0; gid < total; gid++) {
        const int co = (int)(gid % Co);
        const long pix = gid / Co;
        const int ox = (int)(pix % (2 * W));
        const long rest = pix / (2 * W);
        const int oy = (int)(rest % (2 * H));
        const long p = rest / (2 * H);
        const int y = oy >> 1, x = ox >> 1, dy = oy & 1, dx = ox & 1;
        float v = G[((p * H + y) * W + x) * (Co * 4) + co * 4 + dy * 2 + dx] + bias[co];

        if (add)
            v += add[gid % (4L * H * W * Co)];
        out[gid] = apply_act(v, act);
    }
}

/* mask_logits: sam3_kernels.cl:789-807. */
void or_mask_logits(const float *U, const float *hyper, float *out, int npix,
                    long total)
{
    long gid;

#pragma omp parallel for schedule(static)
    for (gid = 0; gid < total; gid++) {
        const long p = gid / npix;
        const int pix = (int)(gid % npix);
        const float *h = hyper + p * 96, *u = U + gid * 32;
        int m;

        for (m = 0; m < 3; m++)
            out[(p * 3 + m) * npix + pix] =
                dot16(u, h + 32 * m) + dot16(u + 16, h + 32 * m + 16);
    }
}

/* pe_encode: sam3_model.c:760-773. */
void or_pe_encode(const float *gauss, float x, float y, float *out)
{
    int i;

    x = 2.0f * x - 1.0f;
    y = 2.0f * y - 1.0f;
    for (i = 0; i < 128; i++) {
        float v = x * gauss[i] + y * gauss[128 + i];

        v *= 2.0f * (float)M_PI;
        out[i] = sinf(v);
        out[128 + i] = cosf(v);
    }
}

/* host_linear / host_mlp3: sam3_model.c:1188-1210. */
static void host_linear(const float *W, const float *b, const float *x, int nin,
                        int nout, int relu, float *y)
{
    int o, i;

    for (o = 0; o < nout; o++) {
        const float *w = W + (long)o * nin;
        double acc = b[o];

        for (i = 0; i < nin; i++)
            acc += (double)w[i] * x[i];
        y[o] = relu && acc < 0.0 ? 0.0f : (float)acc;
    }
}

static void host_mlp3(const float *const *wb, const float *x, int nout, float *y)
{
    float h1[256], h2[256];

    host_linear(wb[0], wb[1], x, 256, 256, 1, h1);
    host_linear(wb[2], wb[3], h1, 256, 256, 1, h2);
    host_linear(wb[4], wb[5], h2, 256, nout, 0, y);
}

#define DT(i) (w[(i)])
#define DATT(blk, t) (w[SAM3_DT_ATTN + 8 * (blk) + (t)])
#define DLAY(l, t) (w[SAM3_DT_LAYER + 12 * (l) + (t)])

/* t2i_attention: sam3_model.c:1212-1229. */
static void dec_t2i(const float *const *w, int blk, int P, float *qry,
                    const float *qpe, float *qin, float *keys, float *kin,
                    const float *pe_img, float *sq, float *bk, float *bv,
                    float *so)
{
    const long T = 5184, n = (long)P * 8 * 256;

    or_add_bcast(qin, qry, qpe, n, n);
    or_add_bcast(kin, keys, pe_img, P * T * 256, T * 256);
    linear(P * 8, 256, 128, qin, DATT(blk, 0), DATT(blk, 1), sq, OR_ACT_NONE, 0);
    linear((int)(P * T), 256, 128, kin, DATT(blk, 2), DATT(blk, 3), bk, OR_ACT_NONE, 0);
    linear((int)(P * T), 256, 128, keys, DATT(blk, 4), DATT(blk, 5), bv, OR_ACT_NONE, 0);
    or_mha(P, 8, (int)T, 128, sq, 8 * 128, bk, T * 128, bv, T * 128, so);
    linear(P * 8, 128, 256, so, DATT(blk, 6), DATT(blk, 7), qry, OR_ACT_NONE, 1);
}

/* token_mlp: sam3_model.c:1231-1237. */
static void dec_mlp(const float *const *w, int l, int P, float *qry, float *sh)
{
    linear(P * 8, 256, 2048, qry, DLAY(l, 8), DLAY(l, 9), sh, OR_ACT_RELU, 0);
    linear(P * 8, 2048, 256, sh, DLAY(l, 10), DLAY(l, 11), qry, OR_ACT_NONE, 1);
}

void or_sam_decode(const float *const *w, const float *emb, const float *s0,
                   const float *s1, int P, const float *points, float *iou,
                   float *lowres)
{
    const long T = 5184, n = (long)P * 8 * 256, L = 288;
    const float eps = 1e-5f;
    float *src = malloc(sizeof(float) * T * 256), *srcpe = malloc(sizeof(float) * T * 256);
    float *pe_img = malloc(sizeof(float) * T * 256);
    float *kp0 = malloc(sizeof(float) * T * 128), *vp0 = malloc(sizeof(float) * T * 128);
    float *qp0 = malloc(sizeof(float) * T * 128);
    float *tok = malloc(sizeof(float) * n), *qpe = malloc(sizeof(float) * n);
    float *qry = malloc(sizeof(float) * n), *qin = malloc(sizeof(float) * n);
    float *sq = malloc(sizeof(float) * n), *sk = malloc(sizeof(float) * n);
    float *sv = malloc(sizeof(float) * n), *so = malloc(sizeof(float) * n);
    float *sh = malloc(sizeof(float) * P * 8 * 2048);
    float *keys = malloc(sizeof(float) * P * T * 256), *kin = malloc(sizeof(float) * P * T * 256);
    float *bq = malloc(sizeof(float) * P * T * 128), *bk = malloc(sizeof(float) * P * T * 128);
    float *bv = malloc(sizeof(float) * P * T * 128), *bo = malloc(sizeof(float) * P * T * 128);
    float *u1 = malloc(sizeof(float) * P * 4 * T * 64);
    float *g2 = malloc(sizeof(float) * P * 4 * T * 128);
    float *u2 = malloc(sizeof(float) * P * 16 * T * 32);
    float *hyper = malloc(sizeof(float) * P * 96);
    struct or_gemm_args a;
    int p, i, x, y;

    /* decoder caches of sam_encode (sam3_model.c:1153-1170, 886-892) */
    or_add_bcast(src, emb, DT(SAM3_DT_NO_MASK), T * 256, 256);
    for (y = 0; y < 72; y++)
        for (x = 0; x < 72; x++)
            or_pe_encode(DT(SAM3_DT_GAUSS), (x + 0.5f) / 72, (y + 0.5f) / 72,
                         pe_img + ((long)y * 72 + x) * 256);
    or_add_bcast(srcpe, src, pe_img, T * 256, T * 256);
    linear((int)T, 256, 128, srcpe, DATT(1, 2), DATT(1, 3), kp0, OR_ACT_NONE, 0);
    linear((int)T, 256, 128, src, DATT(1, 4), DATT(1, 5), vp0, OR_ACT_NONE, 0);
    linear((int)T, 256, 128, srcpe, DATT(2, 0), DATT(2, 1), qp0, OR_ACT_NONE, 0);

    /* prompt tokens (sam3_model.c:1249-1263) */
    for (p = 0; p < P; p++) {
        float *t = tok + (long)p * 8 * 256;

        memcpy(t, DT(SAM3_DT_OBJ_TOKEN), 256 * sizeof(float));
        memcpy(t + 256, DT(SAM3_DT_IOU_TOKEN), 256 * sizeof(float));
        memcpy(t + 512, DT(SAM3_DT_MASK_TOKENS), 4 * 256 * sizeof(float));
        or_pe_encode(DT(SAM3_DT_GAUSS), (points[2 * p] + 0.5f) / 1008,
                     (points[2 * p + 1] + 0.5f) / 1008, t + 6 * 256);
        for (i = 0; i < 256; i++) {
            t[6 * 256 + i] += DT(SAM3_DT_POINT_EMB + 1)[i];
            t[7 * 256 + i] = DT(SAM3_DT_NOT_A_POINT)[i];
        }
    }
    memcpy(qpe, tok, sizeof(float) * n);
    memcpy(qry, tok, sizeof(float) * n);

    /* layer 0 (sam3_model.c:1269-1309) */
    linear(P * 8, 256, 256, qry, DATT(0, 0), DATT(0, 1), sq, OR_ACT_NONE, 0);
    linear(P * 8, 256, 256, qry, DATT(0, 2), DATT(0, 3), sk, OR_ACT_NONE, 0);
    linear(P * 8, 256, 256, qry, DATT(0, 4), DATT(0, 5), sv, OR_ACT_NONE, 0);
    or_mha(P, 8, 8, 256, sq, 8 * 256, sk, 8 * 256, sv, 8 * 256, so);
    linear(P * 8, 256, 256, so, DATT(0, 6), DATT(0, 7), qry, OR_ACT_NONE, 0);
    or_layernorm(qry, qry, DLAY(0, 0), DLAY(0, 1), P * 8, 256, eps, OR_ACT_NONE);
    or_add_bcast(qin, qry, qpe, n, n);
    linear(P * 8, 256, 128, qin, DATT(1, 0), DATT(1, 1), sq, OR_ACT_NONE, 0);
    or_mha(P, 8, (int)T, 128, sq, 8 * 128, kp0, 0, vp0, 0, so);
    linear(P * 8, 128, 256, so, DATT(1, 6), DATT(1, 7), qry, OR_ACT_NONE, 1);
    or_layernorm(qry, qry, DLAY(0, 2), DLAY(0, 3), P * 8, 256, eps, OR_ACT_NONE);
    dec_mlp(w, 0, P, qry, sh);
    or_layernorm(qry, qry, DLAY(0, 4), DLAY(0, 5), P * 8, 256, eps, OR_ACT_NONE);
    or_add_bcast(qin, qry, qpe, n, n);
    linear(P * 8, 256, 128, qin, DATT(2, 2), DATT(2, 3), sk, OR_ACT_NONE, 0);
    linear(P * 8, 256, 128, qry, DATT(2, 4), DATT(2, 5), sv, OR_ACT_NONE, 0);
    or_mha(P, (int)T, 8, 128, qp0, 0, sk, 8 * 128, sv, 8 * 128, bo);
    linear((int)(P * T), 128, 256, bo, DATT(2, 6), DATT(2, 7), keys, OR_ACT_NONE, 0);
    or_add_bcast(keys, keys, src, P * T * 256, T * 256);
    or_layernorm(keys, keys, DLAY(0, 6), DLAY(0, 7), P * T, 256, eps, OR_ACT_NONE);

    /* layer 1 (sam3_model.c:1311-1348) */
    or_add_bcast(qin, qry, qpe, n, n);
    linear(P * 8, 256, 256, qin, DATT(3, 0), DATT(3, 1), sq, OR_ACT_NONE, 0);
    linear(P * 8, 256, 256, qin, DATT(3, 2), DATT(3, 3), sk, OR_ACT_NONE, 0);
    linear(P * 8, 256, 256, qry, DATT(3, 4), DATT(3, 5), sv, OR_ACT_NONE, 0);
    or_mha(P, 8, 8, 256, sq, 8 * 256, sk, 8 * 256, sv, 8 * 256, so);
    linear(P * 8, 256, 256, so, DATT(3, 6), DATT(3, 7), qry, OR_ACT_NONE, 1);
    or_layernorm(qry, qry, DLAY(1, 0), DLAY(1, 1), P * 8, 256, eps, OR_ACT_NONE);
    dec_t2i(w, 4, P, qry, qpe, qin, keys, kin, pe_img, sq, bk, bv, so);
    or_layernorm(qry, qry, DLAY(1, 2), DLAY(1, 3), P * 8, 256, eps, OR_ACT_NONE);
    dec_mlp(w, 1, P, qry, sh);
    or_layernorm(qry, qry, DLAY(1, 4), DLAY(1, 5), P * 8, 256, eps, OR_ACT_NONE);
    or_add_bcast(qin, qry, qpe, n, n);
    linear((int)(P * T), 256, 128, kin, DATT(5, 0), DATT(5, 1), bq, OR_ACT_NONE, 0);
    linear(P * 8, 256, 128, qin, DATT(5, 2), DATT(5, 3), sk, OR_ACT_NONE, 0);
    linear(P * 8, 256, 128, qry, DATT(5, 4), DATT(5, 5), sv, OR_ACT_NONE, 0);
    or_mha(P, (int)T, 8, 128, bq, T * 128, sk, 8 * 128, sv, 8 * 128, bo);
    linear((int)(P * T), 128, 256, bo, DATT(5, 6), DATT(5, 7), keys, OR_ACT_NONE, 1);
    or_layernorm(keys, keys, DLAY(1, 6), DLAY(1, 7), P * T, 256, eps, OR_ACT_NONE);

    /* final token -> image attention (sam3_model.c:1350-1352) */
    dec_t2i(w, 6, P, qry, qpe, qin, keys, kin, pe_img, sq, bk, bv, so);
    or_layernorm(qry, qry, DT(SAM3_DT_NF_W), DT(SAM3_DT_NF_B), P * 8, 256, eps, OR_ACT_NONE);

    /* output upscaling (sam3_model.c:1353-1366) */
    memset(&a, 0, sizeof(a));
    a.M = (int)(P * T), a.N = 256, a.K = 256, a.A = keys, a.lda = 256;
    a.B = DT(SAM3_DT_UP0_W), a.ldb = 256, a.C = kin, a.ldc = 256, a.nb1 = 1;
    a.alpha = 1.0f;
    or_gemm(&a, 1);
    or_convt_scatter(kin, u1, DT(SAM3_DT_UP0_B), s1, P, 72, 72, 64, OR_ACT_NONE);
    or_layernorm(u1, u1, DT(SAM3_DT_UP1_W), DT(SAM3_DT_UP1_B), P * 4 * T, 64, 1e-6f,
                 OR_ACT_GELU);
    memset(&a, 0, sizeof(a));
    a.M = (int)(P * 4 * T), a.N = 128, a.K = 64, a.A = u1, a.lda = 64;
    a.B = DT(SAM3_DT_UP3_W), a.ldb = 128, a.C = g2, a.ldc = 128, a.nb1 = 1;
    a.alpha = 1.0f;
    or_gemm(&a, 1);
    or_convt_scatter(g2, u2, DT(SAM3_DT_UP3_B), s0, P, 144, 144, 32, OR_ACT_GELU);

    /* hypernetwork MLPs 1..3 and the IoU head (sam3_model.c:1368-1386) */
    for (p = 0; p < P; p++) {
        const float *t = qry + (long)p * 8 * 256;
        float out[4];

        for (i = 1; i <= 3; i++)
            host_mlp3(w + SAM3_DT_HYPER + 6 * i, t + (2 + i) * 256, 32,
                      hyper + (long)p * 96 + (i - 1) * 32);
        host_mlp3(w + SAM3_DT_IOU, t + 256, 4, out);
        for (i = 0; i < 3; i++)
            iou[p * 3 + i] = 1.0f / (1.0f + expf(-out[1 + i]));
    }
    or_mask_logits(u2, hyper, lowres, (int)(L * L), P * L * L);

    free(src), free(srcpe), free(pe_img), free(kp0), free(vp0), free(qp0);
    free(tok), free(qpe), free(qry), free(qin), free(sq), free(sk), free(sv), free(so);
    free(sh), free(keys), free(kin), free(bq), free(bk), free(bv), free(bo);
    free(u1), free(g2), free(u2), free(hyper);
}

/* ------------------------------------------------------------ neck */

/* im2col3x3: sam3_kernels.cl:746-760 (tokens t0 .. of an H x W x C map,
 * column c * 9 + ky * 3 + kx). */
void or_im2col3x3(const float *X, float *out, int H, int W, int C, int t0,
                  long total)
{
    long gid;

#pragma omp parallel for schedule(static)
    for (gid = 0; gid < total; gid++) {
        const int t = t0 + (int)(gid / (C * 9)), col = (int)(gid % (C * 9));
        const int c = col / 9, ky = (col % 9) / 3, kx = col % 3;
        const int y = t / W + ky - 1, x = t % W + kx - 1;

        out[gid] = (y >= 0 && y < H && x >= 0 && x < W) ? X[((long)y * W + x) * C + c] : 0.0f;
    }
}

void or_neck_tensor(int i, int E, int *rows, int *cols, int *init)
{
    sam3_neck_tensor(i, E, rows, cols, init);
}

/* conv3x3: sam3_model.c:1032-1054, im2col in bands of col_rows tokens
 * (128 MB of fp32 columns, sam3_model.c:849). */
static void neck_conv3x3(const float *X, int side, const float *w, const float *b, float *Y)
{
    const long T = (long)side * side, col_rows = (128L << 20) / (9 * 256 * 4);
    float *col = malloc(sizeof(float) * (size_t)(col_rows < T ? col_rows : T) * 9 * 256);
    long t0;

    for (t0 = 0; t0 < T; t0 += col_rows) {
        const long n = T - t0 < col_rows ? T - t0 : col_rows;

        or_im2col3x3(X, col, side, side, 256, (int)t0, n * 9 * 256);
        linear((int)n, 9 * 256, 256, col, w, b, Y + t0 * 256, OR_ACT_NONE, 0);
    }
    free(col);
}

/* convt2x2: sam3_model.c:1058-1065. */
static void neck_convt2x2(const float *X, int side, int cin, int cout, const float *w,
                          const float *b, float *G, float *Y, int act)
{
    struct or_gemm_args a;

    memset(&a, 0, sizeof(a));
    a.M = side * side, a.N = cout * 4, a.K = cin, a.A = X, a.lda = cin;
    a.B = w, a.ldb = cout * 4, a.C = G, a.ldc = cout * 4, a.nb1 = 1, a.alpha = 1.0f;
    or_gemm(&a, 1);
    or_convt_scatter(G, Y, b, NULL, 1, side, side, cout, act);
}

/* neck_level: sam3_model.c:1071-1095 (level l, scale 4 >> l). */
static void neck_level(const float *const *w, int l, int Gd, int E, const float *x, float *nka,
                       float *nkb, float *g, float *out)
{
    const float *const *t = w + 8 * l;
    const int scale = 4 >> l;

    if (scale == 4) {
        neck_convt2x2(x, Gd, E, E / 2, t[0], t[1], g, nkb, OR_ACT_GELU);
        neck_convt2x2(nkb, 2 * Gd, E / 2, E / 4, t[2], t[3], g, nka, OR_ACT_NONE);
        linear(16 * Gd * Gd, E / 4, 256, nka, t[4], t[5], nkb, OR_ACT_NONE, 0);
    }
    else if (scale == 2) {
        neck_convt2x2(x, Gd, E, E / 2, t[0], t[1], g, nka, OR_ACT_NONE);
        linear(4 * Gd * Gd, E / 2, 256, nka, t[4], t[5], nkb, OR_ACT_NONE, 0);
    }
    else
        linear(Gd * Gd, E, 256, x, t[4], t[5], nkb, OR_ACT_NONE, 0);
    neck_conv3x3(nkb, scale * Gd, t[6], t[7], out);
}

void or_point_neck(const float *const *w, int Gd, int E, const float *x, float *emb,
                   float *s0, float *s1)
{
    const long T = (long)Gd * Gd;
    float *nka = malloc(sizeof(float) * 16 * T * (E / 4 > 256 ? E / 4 : 256));
    float *nkb = malloc(sizeof(float) * 16 * T * (E / 4 > 256 ? E / 4 : 256));
    float *g = malloc(sizeof(float) * 4 * T * E);
    float *out = malloc(sizeof(float) * 16 * T * 256);

    /* point_neck: sam3_model.c:1098-1110 */
    neck_level(w, 0, Gd, E, x, nka, nkb, g, out);
    linear((int)(16 * T), 256, 32, out, w[SAM3_NT_S0_W], w[SAM3_NT_S0_B], s0, OR_ACT_NONE, 0);
    neck_level(w, 1, Gd, E, x, nka, nkb, g, out);
    linear((int)(4 * T), 256, 64, out, w[SAM3_NT_S1_W], w[SAM3_NT_S1_B], s1, OR_ACT_NONE, 0);
    neck_level(w, 2, Gd, E, x, nka, nkb, g, emb);
    or_add_bcast(emb, emb, w[SAM3_NT_NO_MEM], T * 256, 256);
    free(nka), free(nkb), free(g), free(out);
}

/* ------------------------------------------------------------ input path */

/* precompute_coeffs (image.c:219-276): per output pixel of one axis, the
 * window [xmin, xmin + cnt) and its fixed-point triangle weights, with the
 * axis' precision (the largest at which the biggest weight fits int16). */
struct or_coeffs {
    int ksize, prec;
    int *bounds, *kk;
};

static void or_precompute_coeffs(int in, int out, struct or_coeffs *c)
{
    const double scale = (double)in / out;
    const double filterscale = scale < 1.0 ? 1.0 : scale;
    const double support = 1.0 * filterscale, ss = 1.0 / filterscale;
    double *w, wt_max = 0.0;
    int xx, x;

    c->ksize = (int)ceil(support) * 2 + 1;
    c->bounds = malloc(2 * (size_t)out * sizeof(int));
    c->kk = calloc((size_t)out * c->ksize, sizeof(int));
    w = calloc((size_t)out * c->ksize, sizeof(double));
    for (xx = 0; xx < out; xx++) {
        const double center = (xx + 0.5) * scale;
        double ww = 0.0, *k = w + (size_t)xx * c->ksize;
        int xmin = (int)(center - support + 0.5), xmax = (int)(center + support + 0.5);

        if (xmin < 0)
            xmin = 0;
        if (xmax > in)
            xmax = in;
        xmax -= xmin;
        if (xmax > c->ksize)
            xmax = c->ksize;
        if (xmax < 0)
            xmax = 0;
        for (x = 0; x < xmax; x++) {
            const double t = fabs((x + xmin - center + 0.5) * ss);

            k[x] = t < 1.0 ? 1.0 - t : 0.0;
            ww += k[x];
        }
        if (ww != 0.0)
            for (x = 0; x < xmax; x++) {
                k[x] /= ww;
                if (k[x] > wt_max)
                    wt_max = k[x];
            }
        c->bounds[2 * xx] = xmin;
        c->bounds[2 * xx + 1] = xmax;
    }
    for (c->prec = 0; c->prec < 22; c->prec++)
        if ((int)(0.5 + wt_max * (1 << (c->prec + 1))) >= (1 << 15))
            break;
    for (xx = 0; xx < out * c->ksize; xx++) {
        const double v = w[xx] * (1 << c->prec);

        c->kk[xx] = v < 0 ? (int)(-0.5 + v) : (int)(0.5 + v);
    }
    free(w);
}

static unsigned char or_clip8(int64_t v, int prec)
{
    v >>= prec;
    return v < 0 ? 0 : v > 255 ? 255 : (unsigned char)v;
}

/* aa_resize (image.c:284-339): interleaved RGB w x h (row stride `stride`
 * pixels) -> nw x nh, horizontal pass first, each pass rounded and clipped
 * to 8 bits. */
void or_aa_resize(const uint8_t *src, int w, int h, int stride, int nw, int nh, uint8_t *dst)
{
    struct or_coeffs cx, cy;
    uint8_t *tmp = malloc((size_t)nw * h * 3);
    int y;

    or_precompute_coeffs(w, nw, &cx);
    or_precompute_coeffs(h, nh, &cy);
#pragma omp parallel for schedule(static)
    for (y = 0; y < h; y++) {
        int x, c, i;

        for (x = 0; x < nw; x++) {
            const int *k = cx.kk + (size_t)x * cx.ksize;
            const int xmin = cx.bounds[2 * x], cnt = cx.bounds[2 * x + 1];

            for (c = 0; c < 3; c++) {
                int64_t ss = (int64_t)1 << (cx.prec - 1);

                for (i = 0; i < cnt; i++)
                    ss += (int64_t)src[((size_t)y * stride + xmin + i) * 3 + c] * k[i];
                tmp[((size_t)y * nw + x) * 3 + c] = or_clip8(ss, cx.prec);
            }
        }
    }
#pragma omp parallel for schedule(static)
    for (y = 0; y < nh; y++) {
        const int *k = cy.kk + (size_t)y * cy.ksize;
        const int ymin = cy.bounds[2 * y], cnt = cy.bounds[2 * y + 1];
        int x, c, i;

        for (x = 0; x < nw; x++)
            for (c = 0; c < 3; c++) {
                int64_t ss = (int64_t)1 << (cy.prec - 1);

                for (i = 0; i < cnt; i++)
                    ss += (int64_t)tmp[((size_t)(ymin + i) * nw + x) * 3 + c] * k[i];
                dst[((size_t)y * nw + x) * 3 + c] = or_clip8(ss, cy.prec);
            }
    }
    free(tmp);
    free(cx.bounds), free(cx.kk), free(cy.bounds), free(cy.kk);
}

/* image_encoder_input (image.c:346-371): the crop (x0, y0, w, h) of an
 * interleaved RGB image `cols` pixels wide, resized to side x side unless it
 * has that size already, then out[c][y][x] = (u / 255 - 0.5) / 0.5. */
void or_image_encoder_input(const uint8_t *rgb, int cols, int x0, int y0, int w, int h, int side,
                            float *out)
{
    const uint8_t *src = rgb + ((size_t)y0 * cols + x0) * 3;
    uint8_t *rs = NULL;
    int stride = cols, c, y, x;

    if (w != side || h != side) {
        rs = malloc((size_t)side * side * 3);
        or_aa_resize(src, w, h, cols, side, side, rs);
        src = rs;
        stride = side;
    }
    for (c = 0; c < 3; c++)
        for (y = 0; y < side; y++)
            for (x = 0; x < side; x++)
                out[((size_t)c * side + y) * side + x] =
                    (src[((size_t)y * stride + x) * 3 + c] / 255.0f - 0.5f) / 0.5f;
    free(rs);
}

/* ------------------------------------------------------------ detector attention */

/* softmax_ext: sam3_kernels.cl:889-921 (serial sums, i.e. one work-item
 * per group). Rows r < rows, row = (head - h0) * Nq + query. */
void or_softmax_ext(float *S, long rows, int L, int Nq, int h0, int causal, const float *dy,
                    const float *dx, int W, int nh)
{
    long row;

#pragma omp parallel for schedule(static)
    for (row = 0; row < rows; row++) {
        const int i = (int)(row % Nq), h = h0 + (int)(row / Nq);
        const int H = W > 0 ? L / W : 0;
        float *s = S + row * L;
        float m = -INFINITY, sum = 0.0f, v;
        int j;

        for (j = 0; j < L; j++) {
            v = s[j];
            if (causal && j > i)
                v = -INFINITY;
            else if (dy)
                v += dy[((long)i * H + j / W) * nh + h] + dx[((long)i * W + j % W) * nh + h];
            s[j] = v;
            m = fmaxf(m, v);
        }
        for (j = 0; j < L; j++) {
            v = expf(s[j] - m);
            s[j] = v;
            sum += v;
        }
        v = 1.0f / sum;
        for (j = 0; j < L; j++)
            s[j] *= v;
    }
}

/* attend: sam3_text.c:305-343 (the GEMM-based detector attention), one head
 * at a time (the reference's head chunking does not change the result). */
void or_attend(int Nq, int Nk, int heads, int hd, const float *Q, int ldq, const float *K,
               int ldk, const float *V, int ldv, float *O, int ldo, int causal,
               const float *dy, const float *dx, int W)
{
    float *S = malloc(sizeof(float) * (size_t)Nq * Nk);
    struct or_gemm_args a;
    int h;

    for (h = 0; h < heads; h++) {
        memset(&a, 0, sizeof(a));
        a.M = Nq, a.N = Nk, a.K = hd;
        a.A = Q, a.aoff = (long)h * hd, a.lda = ldq;
        a.B = K, a.boff = (long)h * hd, a.ldb = ldk, a.transb = 1;
        a.C = S, a.ldc = Nk, a.nb1 = 1;
        a.alpha = 1.0f / sqrtf((float)hd);
        or_gemm(&a, 1);
        or_softmax_ext(S, Nq, Nk, Nq, h, causal, dy, dx, W, heads);
        memset(&a, 0, sizeof(a));
        a.M = Nq, a.N = hd, a.K = Nk;
        a.A = S, a.lda = Nk;
        a.B = V, a.boff = (long)h * hd, a.ldb = ldv;
        a.C = O, a.coff = (long)h * hd, a.ldc = ldo, a.nb1 = 1;
        a.alpha = 1.0f;
        or_gemm(&a, 1);
    }
    free(S);
}
