/* SPDX-License-Identifier: Unlicense */
/* Operator layer of the C-ABI (include/sam3_cuda.h): the B200 versions of
 * the reference's sam3_ops.h operators and of the static helpers vit_block
 * calls (sam3_model.c:147-451, 965-1013). Every operator validates shapes,
 * dtypes and buffer extents, then enqueues one or two kernels on the
 * backend stream. */
#include <math.h>
#include <string.h>

#include "backend_internal.h"

struct cb_opnd cb_mat(cb_mem buf, int64_t off, int32_t ld)
{
    struct cb_opnd o = {buf, off, ld, 0, 0};

    return o;
}

struct cb_opnd cb_bmat(cb_mem buf, int64_t off, int32_t ld, int64_t s0,
                       int64_t s1)
{
    struct cb_opnd o = {buf, off, ld, s0, s1};

    return o;
}

/* Largest element index + 1 a strided batched operand touches. */
static int64_t opnd_span(const struct cb_opnd *o, int rows, int cols, int nb,
                         int nb1)
{
    const int64_t nb0 = (nb + nb1 - 1) / nb1;
    const int64_t b0 = nb0 > 0 ? nb0 - 1 : 0, b1 = (nb < nb1 ? nb : nb1) - 1;

    return o->off + b0 * o->s0 + b1 * o->s1 + (int64_t)(rows - 1) * o->ld + cols;
}

static int fits(cb_mem m, int64_t elems)
{
    return m && elems >= 0 &&
           (uint64_t)elems * cbi_dtype_size(m->dtype) <= (uint64_t)m->bytes;
}

static int is_float_dt(int dt)
{
    return dt == CB_F32 || dt == CB_BF16 || dt == CB_F16;
}

static void *elem_ptr(cb_mem m, int64_t off)
{
    return (char *)m->ptr + off * (int64_t)cbi_dtype_size(m->dtype);
}

static int aligned16(const void *p)
{
    return ((uintptr_t)p & 15) == 0;
}

int cb_gemm(cb_backend *b, int M, int N, int K, struct cb_opnd A,
            struct cb_opnd B, int transb, struct cb_opnd C, int nb, int nb1,
            cb_mem bias, cb_mem R, int64_t roff, float alpha, int act)
{
    int tc;

    if (!b || !A.buf || !B.buf || !C.buf || M <= 0 || N <= 0 || K <= 0 ||
        nb <= 0 || nb1 <= 0 || A.s0 < 0 || A.s1 < 0 || B.s0 < 0 || B.s1 < 0 ||
        C.s0 < 0 || C.s1 < 0)
        return cbi_fail(b, CB_EARG, "gemm");
    if (!is_float_dt(A.buf->dtype) || !is_float_dt(B.buf->dtype) ||
        (C.buf->dtype != CB_F32 && C.buf->dtype != CB_BF16) ||
        (bias && bias->dtype != CB_F32) || (R && R->dtype != CB_F32))
        return cbi_fail(b, CB_EDTYPE, "gemm");
    if (!fits(A.buf, opnd_span(&A, M, K, nb, nb1)) ||
        !fits(B.buf, transb ? opnd_span(&B, N, K, nb, nb1)
                            : opnd_span(&B, K, N, nb, nb1)) ||
        !fits(C.buf, opnd_span(&C, M, N, nb, nb1)) || (bias && !fits(bias, N)))
        return cbi_fail(b, CB_EARG, "gemm: operand extent");
    if (R) {
        struct cb_opnd r = C;

        r.buf = R;
        r.off = roff;
        if (!fits(R, opnd_span(&r, M, N, nb, nb1)))
            return cbi_fail(b, CB_EARG, "gemm: residual extent");
    }
    CB_TRY(cbi_enter(b));
    tc = nb == 1 && transb && A.buf->dtype == CB_BF16 && B.buf->dtype == CB_BF16 &&
         A.ld % 8 == 0 && B.ld % 8 == 0 && A.ld >= K && B.ld >= K &&
         aligned16(elem_ptr(A.buf, A.off)) && aligned16(elem_ptr(B.buf, B.off));
    if (tc)
        return cbi_kstatus(
            b,
            k_gemm_bf16_tc(M, N, K, elem_ptr(A.buf, A.off), A.ld,
                           elem_ptr(B.buf, B.off), B.ld, elem_ptr(C.buf, C.off),
                           C.ld, C.buf->dtype == CB_BF16,
                           bias ? (const float *)bias->ptr : NULL,
                           R ? (const float *)elem_ptr(R, roff) : NULL, C.ld, 0,
                           alpha, act, NULL, b->d_err, b->num_sms,
                           (k_stream)b->stream),
            "gemm (tcgen05)");
    if (C.buf->dtype != CB_F32)
        return cbi_fail(b, CB_EDTYPE, "gemm: bf16 output needs bf16 operands");
    return cbi_kstatus(
        b,
        k_gemm_simt(M, N, K, A.buf->ptr, A.buf->dtype, A.off, A.ld, A.s0, A.s1,
                    B.buf->ptr, B.buf->dtype, B.off, B.ld, B.s0, B.s1, transb,
                    (float *)C.buf->ptr, C.off, C.ld, C.s0, C.s1, nb, nb1,
                    bias ? (const float *)bias->ptr : NULL,
                    R ? (const float *)R->ptr : NULL, roff, alpha, act,
                    (k_stream)b->stream),
        "gemm (simt)");
}

int cb_linear(cb_backend *b, int rows, int in, int out, cb_mem X, int64_t xoff,
              cb_mem W, cb_mem bias, cb_mem Y, int64_t yoff, int act,
              int residual)
{
    struct cb_mem_s tmp;

    if (!b || !X || !W || !Y)
        return cbi_fail(b, CB_EARG, "linear");
    /* fp32 activations against bf16 weights: convert the rows once into
     * scratch so the product runs on the tensor cores. */
    if (X->dtype == CB_F32 && W->dtype == CB_BF16 && in % 8 == 0 &&
        fits(X, xoff + (int64_t)rows * in)) {
        void *s = NULL;

        CB_TRY(cbi_enter(b));
        CB_TRY(cbi_scratch(b, (size_t)rows * in * 2, &s));
        CB_TRY(cbi_kstatus(b, k_cast_f32_bf16((const float *)X->ptr + xoff, s,
                                             (long)rows * in, (k_stream)b->stream),
                          "linear: cast"));
        tmp.ptr = s;
        tmp.bytes = (size_t)rows * in * 2;
        tmp.dtype = CB_BF16;
        tmp.owned = 0;
        X = &tmp;
        xoff = 0;
    }
    return cb_gemm(b, rows, out, in, cb_mat(X, xoff, in), cb_mat(W, 0, in), 1,
                   cb_mat(Y, yoff, out), 1, 1, bias, residual ? Y : NULL, yoff,
                   1.0f, act);
}

int cb_layernorm(cb_backend *b, int64_t rows, int C, cb_mem X, cb_mem Y,
                 cb_mem g, cb_mem bias, float eps, int act)
{
    if (!b || !X || !Y || !g || !bias || rows < 0 || C <= 0 ||
        X->dtype != CB_F32 || (Y->dtype != CB_F32 && Y->dtype != CB_BF16) ||
        g->dtype != CB_F32 || bias->dtype != CB_F32 || !fits(X, rows * C) ||
        !fits(Y, rows * C) || !fits(g, C) || !fits(bias, C))
        return cbi_fail(b, CB_EARG, "layernorm");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_layernorm((const float *)X->ptr, Y->ptr,
                                  Y->dtype == CB_BF16, (const float *)g->ptr,
                                  (const float *)bias->ptr, (long)rows, C, eps,
                                  act, (k_stream)b->stream),
                      "layernorm");
}

int cb_add_bcast(cb_backend *b, cb_mem out, cb_mem a, cb_mem bb, int64_t n,
                 int64_t bmod)
{
    if (!b || !out || !a || !bb || n < 0 || bmod <= 0 || out->dtype != CB_F32 ||
        a->dtype != CB_F32 || bb->dtype != CB_F32 || !fits(out, n) ||
        !fits(a, n) || !fits(bb, n < bmod ? n : bmod))
        return cbi_fail(b, CB_EARG, "add_bcast");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_add_bcast((float *)out->ptr, (const float *)a->ptr,
                                  (const float *)bb->ptr, (long)n, (long)bmod,
                                  (k_stream)b->stream),
                      "add_bcast");
}

int cb_softmax_rows(cb_backend *b, cb_mem S, int64_t rows, int L)
{
    if (!b || !S || S->dtype != CB_F32 || rows < 0 || L <= 0 ||
        !fits(S, rows * L))
        return cbi_fail(b, CB_EARG, "softmax_rows");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b, k_softmax_rows((float *)S->ptr, (long)rows, L,
                                        (k_stream)b->stream),
                      "softmax_rows");
}

int cb_rope_apply(cb_backend *b, cb_mem qkv, int64_t rows, int E, int hd,
                  int npos, cb_mem cs)
{
    if (!b || !qkv || !cs || qkv->dtype != CB_F32 || cs->dtype != CB_F32 ||
        hd <= 0 || E % hd || npos <= 0 || !fits(qkv, rows * 3 * E) ||
        !fits(cs, (int64_t)npos * hd))
        return cbi_fail(b, CB_EARG, "rope_apply");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_rope_apply((float *)qkv->ptr, (long)rows, E, hd, npos,
                                   (const float *)cs->ptr, (k_stream)b->stream),
                      "rope_apply");
}

int cb_window_partition(cb_backend *b, cb_mem X, cb_mem out, int H, int C,
                        int ws, int nwx)
{
    if (!b || !X || !out || X->dtype != CB_F32 || out->dtype != CB_F32 ||
        H <= 0 || C <= 0 || ws <= 0 || nwx * ws < H ||
        !fits(X, (int64_t)H * H * C) ||
        !fits(out, (int64_t)nwx * nwx * ws * ws * C))
        return cbi_fail(b, CB_EARG, "window_partition");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_window_partition((const float *)X->ptr,
                                         (float *)out->ptr, H, C, ws, nwx,
                                         (k_stream)b->stream),
                      "window_partition");
}

int cb_window_unpartition_add(cb_backend *b, cb_mem X, cb_mem Wd, int H, int C,
                              int ws, int nwx)
{
    if (!b || !X || !Wd || X->dtype != CB_F32 || Wd->dtype != CB_F32 ||
        H <= 0 || C <= 0 || ws <= 0 || nwx * ws < H ||
        !fits(X, (int64_t)H * H * C) ||
        !fits(Wd, (int64_t)nwx * nwx * ws * ws * C))
        return cbi_fail(b, CB_EARG, "window_unpartition_add");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_window_unpartition_add((float *)X->ptr,
                                               (const float *)Wd->ptr, H, C, ws,
                                               nwx, (k_stream)b->stream),
                      "window_unpartition_add");
}

int cb_patch_im2col(cb_backend *b, cb_mem img, cb_mem out, int side, int grid,
                    int ps)
{
    if (!b || !img || !out || img->dtype != CB_F32 || out->dtype != CB_F32 ||
        grid * ps > side || !fits(img, 3LL * side * side) ||
        !fits(out, (int64_t)grid * grid * 3 * ps * ps))
        return cbi_fail(b, CB_EARG, "patch_im2col");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_patch_im2col((const float *)img->ptr, (float *)out->ptr,
                                     side, grid, ps, (k_stream)b->stream),
                      "patch_im2col");
}

int cb_attention(cb_backend *b, cb_mem qkv, int nseq, int N, int E, int heads,
                 int hd, cb_mem cs, int npos, float scale, int mode, cb_mem out)
{
    const int64_t rows = (int64_t)nseq * N;

    if (!b || !qkv || !out || nseq <= 0 || N <= 0 || hd != 64 ||
        E != heads * hd || !fits(qkv, rows * 3 * E) || !fits(out, rows * E))
        return cbi_fail(b, CB_EARG, "attention");
    if (cs && (cs->dtype != CB_F32 || npos <= 0 ||
               !fits(cs, (int64_t)npos * hd)))
        return cbi_fail(b, CB_EARG, "attention: rope table");
    CB_TRY(cbi_enter(b));
    if (mode == CB_ATTN_F32) {
        if (qkv->dtype != CB_F32 || out->dtype != CB_F32)
            return cbi_fail(b, CB_EDTYPE, "attention (fp32 mode)");
        if (cs)
            CB_TRY(cbi_kstatus(b,
                              k_rope_apply((float *)qkv->ptr, (long)rows, E, hd,
                                           npos, (const float *)cs->ptr,
                                           (k_stream)b->stream),
                              "attention: rope"));
        return cbi_kstatus(b,
                          k_attn_f32((const float *)qkv->ptr, nseq, N, E, heads,
                                     hd, scale, (float *)out->ptr,
                                     (k_stream)b->stream),
                          "attention (fp32)");
    }
    if (mode != CB_ATTN_TC || (out->dtype != CB_F32 && out->dtype != CB_BF16))
        return cbi_fail(b, CB_EARG, "attention: mode");
    if (qkv->dtype == CB_F32) {
        const size_t copy = ((size_t)rows * 3 * E * 2 + 255) & ~(size_t)255;
        const size_t wsb = k_attn_tc_workspace(nseq, N, heads);
        void *s = NULL;

        CB_TRY(cbi_scratch(b, copy + wsb, &s));
        if (cs)
            CB_TRY(cbi_kstatus(b,
                              k_rope_cast_bf16((const float *)qkv->ptr,
                                               (long)rows, E, hd, npos,
                                               (const float *)cs->ptr, s,
                                               (k_stream)b->stream),
                              "attention: rope+cast"));
        else
            CB_TRY(cbi_kstatus(b,
                              k_cast_f32_bf16((const float *)qkv->ptr, s,
                                              (long)rows * 3 * E,
                                              (k_stream)b->stream),
                              "attention: cast"));
        return cbi_kstatus(b,
                          k_attn_tc(s, nseq, N, E, heads, scale, out->ptr,
                                    out->dtype == CB_BF16, (char *)s + copy, wsb,
                                    b->d_err, (k_stream)b->stream),
                          "attention (tcgen05)");
    }
    if (qkv->dtype != CB_BF16 || cs)
        return cbi_fail(b, CB_EDTYPE, "attention: bf16 qkv must be pre-roped");
    {
        const size_t wsb = k_attn_tc_workspace(nseq, N, heads);
        void *ws = NULL;

        if (wsb)
            CB_TRY(cbi_scratch(b, wsb, &ws));
        return cbi_kstatus(b,
                          k_attn_tc(qkv->ptr, nseq, N, E, heads, scale, out->ptr,
                                    out->dtype == CB_BF16, ws, wsb, b->d_err,
                                    (k_stream)b->stream),
                          "attention (tcgen05)");
    }
}

int cb_mha(cb_backend *b, int P, int Nq, int Nk, int dint, cb_mem qp,
           int64_t sq, cb_mem kp, int64_t sk, cb_mem vp, int64_t sv, cb_mem o)
{
    if (!b || !qp || !kp || !vp || !o || P <= 0 || Nq <= 0 || Nk <= 0 ||
        dint <= 0 || sq < 0 || sk < 0 || sv < 0 || qp->dtype != CB_F32 ||
        kp->dtype != CB_F32 || vp->dtype != CB_F32 || o->dtype != CB_F32 ||
        !fits(qp, (P - 1) * sq + (int64_t)Nq * dint) ||
        !fits(kp, (P - 1) * sk + (int64_t)Nk * dint) ||
        !fits(vp, (P - 1) * sv + (int64_t)Nk * dint) ||
        !fits(o, (int64_t)P * Nq * dint))
        return cbi_fail(b, CB_EARG, "mha");
    if (Nk > 64 && dint != 128)
        return cbi_fail(b, CB_EARG, "mha: unsupported shape");
    CB_TRY(cbi_enter(b));
    {
        const size_t wsb = k_mha_workspace(P, Nq, Nk, dint, b->num_sms);
        void *ws = NULL;

        if (wsb)
            CB_TRY(cbi_scratch(b, wsb, &ws));
        return cbi_kstatus(b,
                          k_mha(P, Nq, Nk, dint, (const float *)qp->ptr, (long)sq,
                                (const float *)kp->ptr, (long)sk,
                                (const float *)vp->ptr, (long)sv, (float *)o->ptr, ws,
                                wsb, b->d_err, b->num_sms, (k_stream)b->stream),
                          "mha");
    }
}

int cb_convt_scatter(cb_backend *b, cb_mem G, cb_mem out, cb_mem bias,
                     cb_mem add, int P, int H, int W, int Co, int act)
{
    const int64_t n = (int64_t)P * H * W * Co;

    if (!b || !G || !out || !bias || P <= 0 || H <= 0 || W <= 0 || Co <= 0 ||
        G->dtype != CB_F32 || out->dtype != CB_F32 || bias->dtype != CB_F32 ||
        (add && add->dtype != CB_F32) || !fits(G, 4 * n) || !fits(out, 4 * n) ||
        !fits(bias, Co) || (add && !fits(add, 4 * (int64_t)H * W * Co)) ||
        !aligned16(G->ptr))
        return cbi_fail(b, CB_EARG, "convt_scatter");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_convt_scatter((const float *)G->ptr, (float *)out->ptr,
                                      (const float *)bias->ptr,
                                      add ? (const float *)add->ptr : NULL, P, H, W,
                                      Co, act, (k_stream)b->stream),
                      "convt_scatter");
}

int cb_mask_logits(cb_backend *b, cb_mem U, cb_mem hyper, cb_mem out, int P,
                   int npix)
{
    if (!b || !U || !hyper || !out || P <= 0 || npix <= 0 ||
        U->dtype != CB_F32 || hyper->dtype != CB_F32 || out->dtype != CB_F32 ||
        !fits(U, (int64_t)P * npix * 32) || !fits(hyper, (int64_t)P * 96) ||
        !fits(out, (int64_t)P * 3 * npix) || !aligned16(U->ptr) ||
        !aligned16(hyper->ptr))
        return cbi_fail(b, CB_EARG, "mask_logits");
    CB_TRY(cbi_enter(b));
    return cbi_kstatus(b,
                      k_mask_logits((const float *)U->ptr, (const float *)hyper->ptr,
                                    (float *)out->ptr, P, npix, (k_stream)b->stream),
                      "mask_logits");
}

static size_t al256(size_t n)
{
    return (n + 255) & ~(size_t)255;
}

int cb_attend(cb_backend *b, int Nq, int Nk, int heads, int hd, cb_mem Q, int ldq,
              cb_mem K, int ldk, cb_mem V, int ldv, cb_mem O, int ldo, int causal,
              cb_mem dy, cb_mem dx, int W, int mode)
{
    const int E = heads * hd;
    const k_stream st = (k_stream)(b ? b->stream : NULL);

    if (!b || !Q || !K || !V || !O || Nq <= 0 || Nk <= 0 || heads <= 0 ||
        (hd != 32 && hd != 64) || ldq < E || ldk < E || ldv < E || ldo < E ||
        Q->dtype != CB_F32 || K->dtype != CB_F32 || V->dtype != CB_F32 ||
        O->dtype != CB_F32 || !fits(Q, (int64_t)(Nq - 1) * ldq + E) ||
        !fits(K, (int64_t)(Nk - 1) * ldk + E) || !fits(V, (int64_t)(Nk - 1) * ldv + E) ||
        !fits(O, (int64_t)(Nq - 1) * ldo + E) || (!dy) != (!dx) ||
        (dy && (W <= 0 || Nk % W || dy->dtype != CB_F32 || dx->dtype != CB_F32 ||
                !fits(dy, (int64_t)Nq * (Nk / W) * heads) ||
                !fits(dx, (int64_t)Nq * W * heads))))
        return cbi_fail(b, CB_EARG, "attend");
    CB_TRY(cbi_enter(b));
    if (mode == CB_ATTN_TC && !causal && !dy && Nq == Nk && Nq >= 1024 &&
        ldq % 4 == 0 && ldk % 4 == 0 && ldv % 4 == 0 && ldo % 4 == 0 &&
        aligned16(Q->ptr) && aligned16(K->ptr) && aligned16(V->ptr) && aligned16(O->ptr)) {
        /* tensor cores: heads zero-padded to 64 columns in bf16; the kernel
         * writes each head's hd real columns into O */
        const size_t E64 = (size_t)heads * 64;
        const size_t packed = al256((size_t)Nq * 3 * E64 * 2);
        const size_t wsb = k_attn_tc_cross_workspace(1, Nq, Nq, heads);
        char *s = NULL;

        CB_TRY(cbi_scratch(b, packed + wsb, (void **)&s));
        CB_TRY(cbi_kstatus(b,
                           k_pack_qkv_pad64((const float *)Q->ptr, ldq, (const float *)K->ptr,
                                            ldk, (const float *)V->ptr, ldv, Nq, heads, hd, s,
                                            st),
                           "attend: pack"));
        return cbi_kstatus(b,
                           k_attn_tc_cross(s, (long)(3 * E64), s + E64 * 2, (long)(3 * E64),
                                           s + 2 * E64 * 2, (long)(3 * E64), 1, Nq, Nq, heads,
                                           1.0f / sqrtf((float)hd), NULL, O->ptr, (long)ldo, hd,
                                           0, wsb ? s + packed : NULL, wsb, b->d_err, st),
                           "attend");
    }
    /* (k_rpb_bias stages a row's Nk / W + W bias terms in 48 KB of shared
     * memory) */
    if (mode == CB_ATTN_TC && !causal && Nk >= 1024 && ldq % 4 == 0 && ldk % 4 == 0 &&
        ldv % 4 == 0 && ldo % 4 == 0 && aligned16(Q->ptr) && aligned16(K->ptr) &&
        aligned16(V->ptr) && aligned16(O->ptr) && (!dy || Nk / W + W <= 12288)) {
        /* tensor cores for queries over many keys, with or without the box
         * bias: Q, K, V padded to 64-column heads in bf16, the bias as a
         * dense [heads, Nq, Nk] term, keys split over CTAs when the query
         * tiles are few (the detector's 201 queries over the image) */
        const size_t E64 = (size_t)heads * 64;
        const size_t szq = al256((size_t)Nq * E64 * 2), szk = al256((size_t)Nk * E64 * 2);
        const size_t szb = dy ? al256((size_t)heads * Nq * Nk * 4) : 0;
        const size_t szw = k_attn_tc_cross_workspace(1, Nq, Nk, heads);
        char *s = NULL, *qp, *kp, *vp, *bp, *wp;

        CB_TRY(cbi_scratch(b, szq + 2 * szk + szb + szw, (void **)&s));
        qp = s;
        kp = qp + szq;
        vp = kp + szk;
        bp = vp + szk;
        wp = bp + szb;
        CB_TRY(cbi_kstatus(b, k_pad_heads64(Q->ptr, 0, ldq, Nq, heads, hd, qp, st), "attend: pack"));
        CB_TRY(cbi_kstatus(b, k_pad_heads64(K->ptr, 0, ldk, Nk, heads, hd, kp, st), "attend: pack"));
        CB_TRY(cbi_kstatus(b, k_pad_heads64(V->ptr, 0, ldv, Nk, heads, hd, vp, st), "attend: pack"));
        if (dy)
            CB_TRY(cbi_kstatus(b,
                               k_rpb_bias((const float *)dy->ptr, (const float *)dx->ptr, Nq, Nk,
                                          W, heads, (float *)bp, st),
                               "attend: bias"));
        return cbi_kstatus(b,
                           k_attn_tc_cross(qp, (long)E64, kp, (long)E64, vp, (long)E64, 1, Nq, Nk,
                                           heads, 1.0f / sqrtf((float)hd),
                                           dy ? (const float *)bp : NULL, O->ptr, (long)ldo, hd,
                                           0, szw ? wp : NULL, szw, b->d_err, st),
                           "attend");
    }
    {
        const size_t wsb = k_attend_workspace(Nq, Nk, heads, hd, b->num_sms);
        void *ws = NULL;

        CB_TRY(cbi_scratch(b, wsb, &ws));
        return cbi_kstatus(b,
                           k_attend_simt(Nq, Nk, heads, hd, (const float *)Q->ptr, ldq,
                                         (const float *)K->ptr, ldk, (const float *)V->ptr, ldv,
                                         (float *)O->ptr, ldo, causal,
                                         dy ? (const float *)dy->ptr : NULL,
                                         dx ? (const float *)dx->ptr : NULL, W, ws, wsb,
                                         b->num_sms, st),
                           "attend");
    }
}
