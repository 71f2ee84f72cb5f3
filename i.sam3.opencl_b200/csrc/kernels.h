/* SPDX-License-Identifier: Unlicense */
/* Internal launch entry points of the CUDA kernels (C linkage), called by
 * the C host layer (cuda_backend.c, sam3_ops.c, sam3_backbone.c). Every
 * launcher enqueues on the given stream and returns a cudaError_t value
 * (0 on success) or one of the SAM3_E* argument errors below. Device-side
 * failures (bounded waits that ran out) are written to *err. */
#ifndef SAM3_CUDA_KERNELS_H
#define SAM3_CUDA_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *k_stream;

#define K_ACT_NONE 0
#define K_ACT_GELU 1
#define K_ACT_RELU 2

/* Argument errors (distinct from cudaError_t values, which are < 1000). */
#define K_EARG 1001   /* shape, stride or alignment not supported */
#define K_ETMAP 1002  /* cuTensorMapEncodeTiled failed */

/* RoPE epilogue of the QKV projection: rotate the (2j, 2j+1) column pairs
 * of the q and k blocks (columns [0, 2E)) by the (cos, sin) table row of
 * each output row (sam3_kernels.cl:679-698). mode 0: off; 1: table row =
 * row % npos (the reference's indexing, rows in window order); 2: rows in
 * window-major order over a grid x grid image of ws-wide windows, table row
 * = raster position of the token (global attention on window-major rows). */
struct k_rope {
    const float *cs;
    int mode, E, hd, npos, ws, nwx, grid;
};

/* C[M,N] = epi(alpha * A[M,K] . B[N,K]^T); A, B bf16 row-major (lda, ldb in
 * elements, multiples of 8); epilogue: + bias[n], act, + R[m', n] with
 * m' = m % rmod (rmod 0: m' = m; fp32, ldr; may alias C), RoPE; C fp32 or
 * bf16 (c_bf16), ldc in elements. */
int k_gemm_bf16_tc(int M, int N, int K, const void *A, int lda, const void *B,
                   int ldb, void *C, int ldc, int c_bf16, const float *bias,
                   const float *R, int ldr, int rmod, float alpha, int act,
                   const struct k_rope *rope, int *err, int num_sms,
                   k_stream s);

/* 2x2 / stride-2 ConvTranspose as a tcgen05 GEMM with the scatter in its
 * epilogue: X bf16 [nimg, H, W, cin], Wt bf16 [4 * cout, cin] in
 * sub-pixel-major rows (d * cout + co), out bf16 [nimg, 2H, 2W, cout] =
 * act(convt + bias[co]). cin % 8 == 0, cout % 64 == 0. */
int k_convt2x2_bf16_tc(const void *X, int nimg, int H, int W, int cin,
                       const void *Wt, int cout, const float *bias, int act,
                       void *out, int *err, int num_sms, k_stream s);

/* 3x3 / pad-1 convolution as an implicit tcgen05 GEMM: X bf16 [nimg, H, W, C]
 * (C % 64 == 0), Wt bf16 [N, 9C] in tap-major column order ((ky*3 + kx)*C +
 * c), out [nimg, H, W, N] fp32 or bf16 (out_bf16) = conv + bias[n]
 * (+ R[n], one fp32 row added to every pixel, when R != NULL). N % 64 == 0,
 * 16-byte aligned buffers. */
int k_conv3x3_bf16_tc(const void *X, int nimg, int H, int W, int C,
                      const void *Wt, int N, const float *bias, const float *R,
                      void *out, int out_bf16, int *err, int num_sms,
                      k_stream s);

/* Reference-contract GEMM on CUDA cores (any strides/offsets, fp32 math):
 * C = act(alpha * A op(B) + bias) + R, batched with the two-level strides of
 * sam3_kernels.cl:57-69. Operand dtypes: 0 fp32, 1 bf16, 2 fp16. */
int k_gemm_simt(int M, int N, int K, const void *A, int adt, long aoff, int lda,
                long sa0, long sa1, const void *B, int bdt, long boff, int ldb,
                long sb0, long sb1, int transb, float *C, long coff, int ldc,
                long sc0, long sc1, int nb, int nb1, const float *bias,
                const float *R, long roff, float alpha, int act, k_stream s);

/* Fused windowed/global self-attention on tensor cores. qkv: bf16
 * [nseq * N, 3E] rows (q | k | v, head h at column h * hd, RoPE already
 * applied), out: [nseq * N, E] fp32 or bf16. scale multiplies the scores
 * (1/sqrt(hd)). hd must be 64; E % 64 == 0. */
int k_attn_tc(const void *qkv, int nseq, int N, int E, int heads, float scale,
              void *out, int out_bf16, void *ws, size_t ws_bytes, int *err,
              k_stream s);
/* Workspace with which k_attn_tc splits the KV range of the items that do
 * not fill the last wave of CTAs (0: no split planned; launches of many
 * waves never split). With a smaller ws, or NULL, the kernel runs whole
 * items: same results up to rounding, slower tail. */
size_t k_attn_tc_workspace(int nseq, int N, int heads);

/* The same kernel for cross-attention: nseq sequences of Nq query rows of
 * Q and Nk key / value rows of K and V (bf16, leading dimensions ldq / ldk /
 * ldv in elements, head h at column 64 h, 16-byte aligned rows), out rows
 * seq * Nq + q with leading dimension ldo, the first ohd (16, 32 or 64)
 * columns of head h at column ohd h (heads narrower than 64 given
 * zero-padded: their real columns written straight to the caller's
 * layout), fp32 (bf16 only without a bias). bias: NULL, or fp32 [nseq,
 * heads, Nq, Nk] added to the scaled scores, in log2 units (natural-log
 * bias x log2 e). */
int k_attn_tc_cross(const void *Q, long ldq, const void *K, long ldk, const void *V,
                    long ldv, int nseq, int Nq, int Nk, int heads, float scale,
                    const float *bias, void *out, long ldo, int ohd, int out_bf16, void *ws,
                    size_t ws_bytes, int *err, k_stream s);
/* Device workspace k_attn_tc_cross needs to split the keys of its items
 * over CTAs and merge the partial results (0: no split planned); with less,
 * the items run whole. */
size_t k_attn_tc_cross_workspace(int nseq, int Nq, int Nk, int heads);

/* The same attention in fp32 on CUDA cores (reference mode): qkv fp32. */
int k_attn_f32(const float *qkv, int nseq, int N, int E, int heads, int hd,
               float scale, float *out, k_stream s);

/* fp32 qkv -> bf16 qkv with RoPE on q and k (table row = row % npos). */
int k_rope_cast_bf16(const float *qkv, long rows, int E, int hd, int npos,
                     const float *cs, void *out, k_stream s);

/* In-place RoPE on fp32 qkv rows (rope_apply, sam3_kernels.cl:679-698). */
int k_rope_apply(float *qkv, long rows, int E, int hd, int npos,
                 const float *cs, k_stream s);

/* Row LayerNorm (sam3_kernels.cl:489-514): fp32 X [rows, C] -> Y (fp32 or
 * bf16); Y may alias X when fp32. */
int k_layernorm(const float *X, void *Y, int y_bf16, const float *g,
                const float *b, long rows, int C, float eps, int act,
                k_stream s);

int k_softmax_rows(float *S, long rows, int L, k_stream s);
int k_add_bcast(float *out, const float *a, const float *b, long n, long bmod,
                k_stream s);
/* out bf16 [n] = a + b (fp32 sum, one rounding). */
int k_add_bf16(const float *a, const float *b, void *out, long n, k_stream s);
int k_window_partition(const float *X, float *out, int H, int C, int ws,
                       int nwx, k_stream s);
int k_window_unpartition_add(float *X, const float *Wd, int H, int C, int ws,
                             int nwx, k_stream s);
int k_patch_im2col(const float *img, float *out, int side, int grid, int ps,
                   k_stream s);
int k_cast_f32_bf16(const float *x, void *y, long n, k_stream s);
int k_cast_bf16_f32(const void *x, float *y, long n, k_stream s);

/* Decoder attention (sam3_kernels.cl:527-633): 8 heads, scale 1/sqrt(c).
 * Nk > 64 (c = 16 only) splits the keys over CTAs and needs a device
 * workspace of k_mha_workspace(...) bytes (0 otherwise) and the device
 * error word err (a pipeline wait that times out records kErrWaitTimeout
 * there instead of hanging). */
size_t k_mha_workspace(int P, int Nq, int Nk, int dint, int num_sms);
int k_mha(int P, int Nq, int Nk, int dint, const float *qp, long sq,
          const float *kp, long sk, const float *vp, long sv, float *o,
          void *ws, size_t ws_bytes, int *err, int num_sms, k_stream s);
/* The decoder's image -> token attention (dint 128, at most 8 keys) with its
 * queries qp read as bf16 (rows of 128 channels, prompt stride sq and row
 * stride ldq in elements; as the Q projection writes them) and its output o
 * written as bf16 [P * Nq, 128] (the operand of the following Linear);
 * otherwise the arithmetic of k_mha. */
int k_mha_i2t_bf16(int P, int Nq, int Nk, const void *qp, long sq, long ldq,
                   const float *kp, long sk, const float *vp, long sv, void *o, int num_sms,
                   k_stream s);
/* The decoder's token -> image attention (dint 128, more than 64 keys) with
 * its keys and values kp / vp read as bf16 rows of 128 channels (as their
 * projections write them; prompt strides sk / sv and row strides kld / vld
 * in elements) and o written as bf16 when out_bf16 (the operand of the
 * output projection), else fp32; otherwise k_mha (same workspace). */
int k_mha_t2i_bf16kv(int P, int Nq, int Nk, const float *qp, long sq, const void *kp,
                     long sk, long kld, const void *vp, long sv, long vld, void *o,
                     int out_bf16, void *ws, size_t ws_bytes, int *err, int num_sms,
                     k_stream s);

/* Mask decoder (decoder.cu). convt_scatter: G [P*H*W, Co*4] (16-byte
 * aligned) -> out [P, 2H, 2W, Co], + bias, + add (shared, may be NULL),
 * act. mask_logits: U [P, npix, 32], hyper [P, 96] -> out [P, 3, npix].
 * dec_heads: hypernetwork MLPs w/b[0..2] on token rows 3..5 and the IoU
 * head w/b[3] on row 1 of tok [P, 8, 256] -> hyper [P, 96], iou [P, 3]
 * (sigmoid). transpose_cast: fp32 [rows, cols] -> bf16 [cols, rows]. */
int k_convt_scatter(const float *G, float *out, const float *bias,
                    const float *add, int P, int H, int W, int Co, int act,
                    k_stream s);
int k_mask_logits(const float *U, const float *hyper, float *out, int P,
                  int npix, k_stream s);
struct k_dec_heads_w {
    const float *w[4][3], *b[4][3];
};
int k_dec_heads(const float *tok, int P, const struct k_dec_heads_w *hw,
                float *hyper, float *iou, k_stream s);
int k_transpose_cast_bf16(const float *src, int rows, int cols, int dmajor,
                          void *dst, k_stream s);
/* Decoder fusions. ln_keys: LayerNorm of 256-wide rows X (+ R[row % T]
 * first when R is given), Y fp32 (may alias X), Yb = bf16(Y), Yk =
 * bf16(Y + pe[row % T]); each output NULL = skipped, at least one given. up1:
 * ConvT 256 -> 64 scatter of G [P*H*W, 256] + bias + feat [4HW, 64],
 * LayerNorm2d (g, b, eps), GELU -> bf16 [P, 2H, 2W, 64]. up2_logits: ConvT
 * 64 -> 32 scatter of G [P*H*W, 128] (sub-pixel-major columns d*32 + co)
 * + bias + feat [4HW, 32], GELU, dotted with hyper [P, 96] -> out
 * [P, 3, 2H * 2W]. transpose_cast with dmajor: source column co*4 + d
 * becomes row d * cols/4 + co. */
int k_dec_ln_keys(const float *X, const float *R, float *Y, const float *g,
                  const float *b, long rows, float eps, const float *pe, int T,
                  void *Yb, void *Yk, k_stream s);
/* feat_subpix: an upscaling stage's residual feat fp32 [(2H)*(2W), C] (one
 * image, NHWC) -> out fp32 [4][C][H*W], out[(d*C + c)*H*W + y*W + x] =
 * feat[pixel (2y + d/2, 2x + d%2)][c] (ConvTranspose input pixel (y, x),
 * sub-pixel d); C a multiple of 32. The layout the two epilogues below
 * read. */
int k_dec_feat_subpix(const float *feat, int H, int W, int C, float *out, k_stream s);
/* Last output-upscaling stage + mask logits on the tensor cores (gemm_tc.cu):
 * X bf16 [P*H*W, 64] (the first stage's output), Wt bf16 [128, 64] (the
 * ConvTranspose 64 -> 32 weight in sub-pixel-major rows d*32 + co), bias
 * [32], feat = feat_s0 [(2H)*(2W), 32] through k_dec_feat_subpix (fp32
 * [4][32][H*W]), hyper [P, 3, 32] -> out fp32 [P, 3, 2H, 2W] =
 * sum_c hyper[p][k][c] * GELU(convt + bias + feat). */
int k_dec_convt_logits(const void *X, int P, int H, int W, const void *Wt,
                       const float *bias, const float *feat, const float *hyper,
                       float *out, int *err, int num_sms, k_stream s);
/* First output-upscaling stage on the tensor cores (gemm_tc.cu): X bf16
 * [P*H*W, 256] (the keys), Wt bf16 [256, 256] (the ConvTranspose 256 -> 64
 * weight in sub-pixel-major rows d*64 + co), bias [64], feat = feat_s1
 * [(2H)*(2W), 64] through k_dec_feat_subpix (fp32 [4][64][H*W]),
 * LayerNorm2d lnw / lnb [64] -> out bf16 [P, 2H, 2W, 64] =
 * GELU(LN(convt + bias + feat)). */
int k_dec_convt_ln2d(const void *X, int P, int H, int W, const void *Wt,
                     const float *bias, const float *feat, const float *lnw,
                     const float *lnb, float eps, void *out, int *err, int num_sms,
                     k_stream s);

/* SimpleFPN neck (neck.cu). permute_conv3x3_bf16: fp32 [cout, cin, 3, 3]
 * -> bf16 [cout, 9 cin], columns (ky*3 + kx)*cin + c (k_conv3x3_bf16_tc's
 * K order). */
int k_permute_conv3x3_bf16(const float *src, int cout, int cin, void *dst,
                           k_stream s);

/* Input path (input.cu). resize_pass_u8: one axis of the uint8 antialiased
 * resize over `lines` lines of interleaved RGB, source / destination
 * strides in bytes between lines (s_line, d_line) and between pixels along
 * the axis (s_step, d_step); bounds [2 nout] (first, count), kk [nout,
 * ksize] fixed-point weights with `prec` fraction bits; line_fastest:
 * consecutive threads take consecutive lines. crop_copy_u8: w x h
 * RGB crop (row pitch in bytes) -> packed. normalize_chw: uint8 HWC side^2
 * tile -> fp32 CHW (u / 255 - 0.5) / 0.5. */
int k_resize_pass_u8(const uint8_t *src, long s_line, long s_step,
                     uint8_t *dst, long d_line, long d_step, int lines,
                     int nout, int line_fastest, const int *bounds,
                     const int *kk, int ksize, int prec, k_stream s);
int k_crop_copy_u8(const uint8_t *src, long pitch, int w, int h, uint8_t *dst,
                   k_stream s);
int k_normalize_chw(const uint8_t *tile, int side, float *out, k_stream s);

/* Detector attention (detector.cu). pack_qkv_pad64: fp32 q, k, v [N, ld]
 * (head h at column h * hd) -> bf16 [N, 3 * heads * 64] with heads
 * zero-padded to 64 columns (the tcgen05 attention's layout);
 * unpack_heads64: fp32 [N, heads * 64] -> O [N, ldo], first hd columns of
 * each head. attend_simt: fp32 flash attention (hd 32 or 64) with an
 * optional causal mask or box relative position bias dy / dx (key grid W
 * wide), keys split over CTAs; workspace k_attend_workspace bytes. */
int k_pack_qkv_pad64(const float *q, int ldq, const float *k, int ldk,
                     const float *v, int ldv, long N, int heads, int hd,
                     void *out, k_stream s);
int k_unpack_heads64(const float *in, long N, int heads, int hd, float *O,
                     int ldo, k_stream s);
int k_attend_splits(int Nq, int Nk, int heads, int num_sms);
/* pad_heads64: one attention operand, fp32 or bf16 (src_bf16) [rows, ld],
 * head h at column h * hd -> bf16 [rows, heads * 64], columns hd..63 of
 * each head zero. rpb_bias: the box relative position bias of softmax_ext
 * as fp32 [heads, Nq, Nk] in log2 units (k_attn_tc_cross's bias);
 * K_EARG unless W divides Nk and Nk / W + W <= 12288. */
int k_pad_heads64(const void *src, int src_bf16, long ld, long rows, int heads, int hd,
                  void *out, k_stream s);
int k_rpb_bias(const float *dy, const float *dx, int Nq, int Nk, int W, int heads,
               float *bias, k_stream s);
size_t k_attend_workspace(int Nq, int Nk, int heads, int hd, int num_sms);
int k_attend_simt(int Nq, int Nk, int heads, int hd, const float *Q, int ldq,
                  const float *K, int ldk, const float *V, int ldv, float *O,
                  int ldo, int causal, const float *dy, const float *dx,
                  int W, void *ws, size_t ws_bytes, int num_sms, k_stream s);

/* uint8 HWC tiles -> bf16 patch rows in window-major token order:
 * out[ntile * grid^2, kpad], column c*ps*ps + ky*ps + kx (the Conv2d weight
 * order), value (u/255 - 0.5)/0.5 (image.c:360-366), zero for columns >= 3
 * ps^2. Row order: token r of a tile is window w = r / ws^2, in-window
 * index i = r % ws^2 (ws = grid gives raster order). */
int k_patch_embed_in(const uint8_t *rgb, int ntile, int side, int grid, int ps,
                     int ws, int kpad, void *out, k_stream s);

/* Seeded generator on the device (bit-identical to include/sam3_synth.h). */
int k_synth_normal(uint64_t seed, uint64_t stream, long n, float mean,
                   float std, void *out, int out_bf16, k_stream s);

/* x (window-major rows) -> y (raster rows) for ntile tiles. */
int k_unpermute_rows(const float *x, float *y, int ntile, int grid, int ws,
                     int C, k_stream s);
/* pos [T, C] raster -> window-major rows. */
int k_permute_rows(const float *x, float *y, int ntile, int grid, int ws,
                   int C, k_stream s);

#ifdef __cplusplus
}
#endif
#endif
