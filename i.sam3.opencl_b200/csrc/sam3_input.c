/* SPDX-License-Identifier: Unlicense */
/* The encoder's input path on the device: image_encoder_input
 * (image.c:346-371) with the uint8 antialiased resize of aa_resize
 * (image.c:209-339). The per-axis windows and fixed-point weights are
 * computed here on the host, exactly as the reference computes them
 * (precompute_coeffs, image.c:219-276: a triangle filter widened by the
 * downscale factor, normalised, then scaled by the largest power of two at
 * which the biggest weight still fits int16); the two integer passes and the
 * normalisation run on the GPU (input.cu). */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "backend_internal.h"

#define MAX_PRECISION_BITS 22

struct axis_coeffs {
    int ksize, prec;
    int *tab; /* bounds [2 out] then weights [out * ksize] */
};

static int axis_coeffs(int in, int out, struct axis_coeffs *c)
{
    const double scale = (double)in / out;
    const double filterscale = scale < 1.0 ? 1.0 : scale;
    const double support = filterscale, ss = 1.0 / filterscale;
    double *w, wt_max = 0.0;
    int *bounds, *kk;
    int o, x;

    c->ksize = (int)ceil(support) * 2 + 1;
    c->tab = calloc((size_t)out * (2 + c->ksize), sizeof(int));
    w = calloc((size_t)out * c->ksize, sizeof(double));
    if (!c->tab || !w) {
        free(c->tab);
        free(w);
        return CB_EALLOC;
    }
    bounds = c->tab;
    kk = c->tab + 2 * out;
    for (o = 0; o < out; o++) {
        const double center = (o + 0.5) * scale;
        double sum = 0.0, *k = w + (size_t)o * c->ksize;
        int lo = (int)(center - support + 0.5), hi = (int)(center + support + 0.5);

        if (lo < 0)
            lo = 0;
        if (hi > in)
            hi = in;
        hi -= lo; /* the window's width from here on */
        if (hi > c->ksize)
            hi = c->ksize; /* rounding can widen it by one */
        if (hi < 0)
            hi = 0;
        for (x = 0; x < hi; x++) {
            const double t = fabs((x + lo - center + 0.5) * ss);

            k[x] = t < 1.0 ? 1.0 - t : 0.0;
            sum += k[x];
        }
        if (sum != 0.0)
            for (x = 0; x < hi; x++) {
                k[x] /= sum;
                if (k[x] > wt_max)
                    wt_max = k[x];
            }
        bounds[2 * o] = lo;
        bounds[2 * o + 1] = hi;
    }
    for (c->prec = 0; c->prec < MAX_PRECISION_BITS; c->prec++)
        if ((int)(0.5 + wt_max * (1 << (c->prec + 1))) >= (1 << 15))
            break;
    for (o = 0; o < out * c->ksize; o++) {
        const double v = w[o] * (1 << c->prec);

        kk[o] = v < 0 ? (int)(-0.5 + v) : (int)(0.5 + v);
    }
    free(w);
    return CB_OK;
}

int cb_image_encoder_input(cb_backend *b, cb_mem img, int cols, int rows, int x0, int y0, int w,
                           int h, int side, cb_mem tiles, int tile, cb_mem chw)
{
    const size_t tile_bytes = (size_t)side * side * 3;
    struct axis_coeffs cx = {0, 0, NULL}, cy = {0, 0, NULL};
    const uint8_t *src;
    uint8_t *dst;
    char *s = NULL;
    size_t need, tab_x, tab_y, tmp_bytes;
    k_stream st;
    int rc;

    if (!b || !img || (!tiles && !chw))
        return CB_EARG;
    if (img->dtype != CB_U8 || cols <= 0 || rows <= 0 || side <= 0 || w <= 0 || h <= 0 ||
        x0 < 0 || y0 < 0 || x0 + w > cols || y0 + h > rows ||
        img->bytes < (size_t)cols * rows * 3 || tile < 0 ||
        (tiles && (tiles->dtype != CB_U8 || tiles->bytes < (size_t)(tile + 1) * tile_bytes)) ||
        (chw && (chw->dtype != CB_F32 || chw->bytes < tile_bytes * 4)))
        return cbi_fail(b, CB_EARG, "image_encoder_input");
    CB_TRY(cbi_enter(b));
    st = (k_stream)b->stream;
    src = (const uint8_t *)img->ptr + ((size_t)y0 * cols + x0) * 3;
    if (w == side && h == side) {
        /* no resampling (image.c:355) */
        if (tiles)
            dst = (uint8_t *)tiles->ptr + (size_t)tile * tile_bytes;
        else {
            CB_TRY(cbi_scratch(b, tile_bytes, (void **)&s));
            dst = (uint8_t *)s;
        }
        CB_TRY(cbi_kstatus(b, k_crop_copy_u8(src, (long)cols * 3, w, h, dst, st),
                           "image_encoder_input"));
    }
    else {
        CB_TRY(axis_coeffs(w, side, &cx));
        rc = axis_coeffs(h, side, &cy);
        if (rc != CB_OK) {
            free(cx.tab);
            return rc;
        }
        tab_x = (size_t)side * (2 + cx.ksize) * sizeof(int);
        tab_y = (size_t)side * (2 + cy.ksize) * sizeof(int);
        tmp_bytes = ((size_t)h * side * 3 + 255) / 256 * 256;
        need = tmp_bytes + (tiles ? 0 : (tile_bytes + 255) / 256 * 256) + tab_x + tab_y;
        rc = cbi_scratch(b, need, (void **)&s);
        if (rc == CB_OK) {
            char *tabs = s + tmp_bytes + (tiles ? 0 : (tile_bytes + 255) / 256 * 256);
            const int *bx = (const int *)tabs, *by = (const int *)(tabs + tab_x);

            dst = tiles ? (uint8_t *)tiles->ptr + (size_t)tile * tile_bytes
                        : (uint8_t *)(s + tmp_bytes);
            rc = cbi_kstatus(b,
                             (int)cudaMemcpyAsync(tabs, cx.tab, tab_x, cudaMemcpyHostToDevice,
                                                  b->stream),
                             "image_encoder_input");
            if (rc == CB_OK)
                rc = cbi_kstatus(b,
                                 (int)cudaMemcpyAsync(tabs + tab_x, cy.tab, tab_y,
                                                      cudaMemcpyHostToDevice, b->stream),
                                 "image_encoder_input");
            /* horizontal pass: each of the h crop rows, x -> side */
            if (rc == CB_OK)
                rc = cbi_kstatus(b,
                                 k_resize_pass_u8(src, (long)cols * 3, 3, (uint8_t *)s,
                                                  (long)side * 3, 3, h, side, 0, bx,
                                                  bx + 2 * side, cx.ksize, cx.prec, st),
                                 "image_encoder_input");
            /* vertical pass: each of the side columns, y -> side */
            if (rc == CB_OK)
                rc = cbi_kstatus(b,
                                 k_resize_pass_u8((const uint8_t *)s, 3, (long)side * 3, dst, 3,
                                                  (long)side * 3, side, side, 1, by,
                                                  by + 2 * side, cy.ksize, cy.prec, st),
                                 "image_encoder_input");
            /* copies from pageable host memory are staged before
             * cudaMemcpyAsync returns, so the tables can be freed now */
        }
        free(cx.tab);
        free(cy.tab);
        CB_TRY(rc);
    }
    if (chw)
        CB_TRY(cbi_kstatus(b, k_normalize_chw(dst, side, (float *)chw->ptr, st),
                           "image_encoder_input"));
    return CB_OK;
}
