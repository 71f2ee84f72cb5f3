/* CPU restatement of the reference's hot-path kernels and their host-side
 * orchestration (i.sam3.opencl: sam3_kernels.cl, sam3_model.c).
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker and the timed CPU
 * baseline; the product never links, loads or calls it.
 *
 * Every function restates the cited reference code in plain C with the same
 * order of floating-point operations, so that it gives the same bits as the
 * reference kernels compiled from their own source (oracle/_ref, built by
 * oracle/Makefile) on the same inputs. Work-group reductions
 * (layernorm, softmax_rows) are restated as serial sums, which equals the
 * reference kernels run with one work-item per group. */
#ifndef SAM3_ORACLE_H
#define SAM3_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_ACT_NONE 0
#define OR_ACT_GELU 1
#define OR_ACT_RELU 2

/* Arguments of the reference gemm kernels (sam3_kernels.cl:57-77). */
struct or_gemm_args {
    int M, N, K;
    const float *A;
    long aoff;
    int lda;
    long sa0, sa1;
    const float *B;
    long boff;
    int ldb;
    long sb0, sb1;
    int transb;
    float *C;
    long coff;
    int ldc;
    long sc0, sc1;
    int nb1;
    const float *bias, *R;
    long roff;
    float alpha;
    int act;
};

void or_gemm(const struct or_gemm_args *a, int nb);
void or_layernorm(const float *X, float *Y, const float *g, const float *b,
                  long rows, int C, float eps, int act);
void or_softmax_rows(float *S, long rows, int L);
void or_rope_apply(float *qkv, long rows, int E, int hd, int npos,
                   const float *cs);
void or_add_bcast(float *out, const float *a, const float *b, long n,
                  long bmod);
void or_window_partition(const float *X, float *out, int H, int C, int ws,
                         int nwx);
void or_window_unpartition_add(float *X, const float *Wd, int H, int C,
                               int ws, int nwx);
void or_patch_im2col(const float *img, float *out, int side, int grid, int ps);
void or_image_input(const uint8_t *rgb, int side, float *out);
int or_mha(int P, int Nq, int Nk, int dint, const float *qp, long sq,
           const float *kp, long sk, const float *vp, long sv, float *o);

/* Attention core of vit_block (sam3_model.c:1000-1013) on roped qkv rows:
 * nseq sequences of N tokens, qkv [nseq * N, 3E], out [nseq * N, E]. */
void or_attention(const float *qkv, int nseq, int N, int E, int heads, int hd,
                  float alpha, float *out);

/* Backbone weights (fp32). */
struct or_block {
    const float *n1w, *n1b, *qkvw, *qkvb, *projw, *projb, *n2w, *n2b;
    const float *l1w, *l1b, *l2w, *l2b;
    int window; /* window side, 0 = global */
};
struct or_trunk {
    int E, heads, hd, mlp, depth, grid, patch, img;
    const float *pe_w, *pos, *lnpw, *lnpb;
    const struct or_block *blocks;
    const float *rope_win, *rope_glob;
};

/* One pre-norm block, x [grid^2, E] updated in place
 * (sam3_model.c:981-1028). Work buffers are allocated inside. */
void or_vit_block(const struct or_trunk *t, const struct or_block *b, float *x);

/* sam_encode_trunk (sam3_model.c:1112-1144) on a normalised CHW image;
 * x [grid^2, E] receives the output tokens. first/last select blocks
 * [first, last) (0, depth for the whole trunk). With img == NULL the
 * prologue (patch embedding, pos_embed, ln_pre) is skipped and x is the
 * input of block `first`. */
void or_encode_trunk(const struct or_trunk *t, const float *img, float *x,
                     int first, int last);

int or_num_threads(void);

/* Mask decoder kernels: convt_scatter (sam3_kernels.cl:766-781),
 * mask_logits (sam3_kernels.cl:789-807; total = P * npix), pe_encode
 * (sam3_model.c:760-773). */
void or_convt_scatter(const float *G, float *out, const float *bias,
                      const float *add, int P, int H, int W, int Co, int act);
void or_mask_logits(const float *U, const float *hyper, float *out, int npix,
                    long total);
void or_pe_encode(const float *gauss, float x, float y, float *out);
void or_dec_tensor(int i, int *rows, int *cols, int *init);

/* The decoder caches of sam_encode (sam3_model.c:1153-1170) and sam_decode
 * (sam3_model.c:1239-1399) for P prompts: w holds the decoder tensors in
 * include/sam3_synth.h order (SAM3_DT_*) and checkpoint layout; emb
 * [5184, 256], s0 [288 * 288, 32], s1 [144 * 144, 64]; points [2P] (x, y)
 * in input pixels; iou [3P] and lowres [P, 3, 288, 288] receive the
 * outputs. Work buffers are allocated inside. */
void or_sam_decode(const float *const *w, const float *emb, const float *s0,
                   const float *s1, int P, const float *points, float *iou,
                   float *lowres);

/* Neck: im2col3x3 (sam3_kernels.cl:746-760, total = n * 9 * C values from
 * token t0), and point_neck (sam3_model.c:1098-1110 with neck_level,
 * conv3x3, convt2x2) on the trunk output x [Gd^2, E]: w holds the neck
 * tensors in include/sam3_synth.h order (SAM3_NT_*); emb [Gd^2, 256],
 * s0 [16 Gd^2, 32], s1 [4 Gd^2, 64]. */
void or_im2col3x3(const float *X, float *out, int H, int W, int C, int t0,
                  long total);
void or_neck_tensor(int i, int E, int *rows, int *cols, int *init);
void or_point_neck(const float *const *w, int Gd, int E, const float *x,
                   float *emb, float *s0, float *s1);

/* Input path: aa_resize (image.c:284-339, torchvision's uint8 antialiased
 * bilinear) and image_encoder_input (image.c:346-371). */
void or_aa_resize(const uint8_t *src, int w, int h, int stride, int nw, int nh,
                  uint8_t *dst);
void or_image_encoder_input(const uint8_t *rgb, int cols, int x0, int y0,
                            int w, int h, int side, float *out);

/* Detector attention: softmax_ext (sam3_kernels.cl:889-921; rows =
 * heads * Nq score rows of L keys, optional causal mask or box relative
 * position bias dy / dx over a key grid W wide) and attend
 * (sam3_text.c:305-343: Q.K^T / sqrt(hd), softmax_ext, P.V per head). */
void or_softmax_ext(float *S, long rows, int L, int Nq, int h0, int causal,
                    const float *dy, const float *dx, int W, int nh);
void or_attend(int Nq, int Nk, int heads, int hd, const float *Q, int ldq,
               const float *K, int ldk, const float *V, int ldv, float *O,
               int ldo, int causal, const float *dy, const float *dx, int W);

#ifdef __cplusplus
}
#endif
#endif
