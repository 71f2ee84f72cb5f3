/* SPDX-License-Identifier: Unlicense */
/* C-ABI of the B200 backend for the SAM 3 Perception Encoder hot path.
 *
 * Drop-in for the reference's OpenCL backend and operator layer
 * (i.sam3.opencl: ocl_backend.h, sam3_ops.h). Plain C types only: opaque
 * handles, pointers, sizes and int status codes (0 = success, see
 * cb_errstr). Every call that enqueues device work runs on the backend's
 * stream; results are visible after cb_sync() or a blocking cb_read().
 *
 * Per-device state lives in the cb_backend handle (no globals), so one
 * process may drive several GPUs from several host threads, one backend
 * per thread. */
#ifndef SAM3_CUDA_H
#define SAM3_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status */
#define CB_OK 0
#define CB_ENODEV 1   /* no CUDA device / bad ordinal / not sm_100 */
#define CB_EALLOC 2   /* device or host allocation failed */
#define CB_EARG 3     /* invalid argument, shape, stride or alignment */
#define CB_ECUDA 4    /* CUDA runtime error (cb_last_error has the text) */
#define CB_ETIMEOUT 5 /* a kernel's bounded wait ran out (device error word) */
#define CB_EDTYPE 6   /* operand dtype not supported by this op */

/* Buffer element types. */
#define CB_F32 0
#define CB_BF16 1
#define CB_F16 2
#define CB_U8 3

/* Activations, as sam3_ops.h:11-13. */
#define CB_ACT_NONE 0
#define CB_ACT_GELU 1
#define CB_ACT_RELU 2

typedef struct cb_backend cb_backend;
typedef struct cb_mem_s *cb_mem;

/* ------------------------------------------------------------ backend
 * Replaces ocl_backend.h:57-104. */

/* ocl_init (ocl_backend.h:57-59): select CUDA device `device` (ordinal),
 * create a stream and the device error word. Fails with CB_ENODEV when the
 * device is absent or is not compute capability 10.x. */
int cb_init(cb_backend **out, int device);
/* ocl_free (ocl_backend.h:79). */
void cb_free(cb_backend *b);
/* ocl_errstr (ocl_backend.h:82): text of a status code. */
const char *cb_errstr(int status);
/* Detail of the last failure on this backend (CUDA error text etc.). */
const char *cb_last_error(const cb_backend *b);
int cb_device(const cb_backend *b);
int cb_num_sms(const cb_backend *b);

/* ocl_alloc (ocl_backend.h:88): device buffer of `bytes`, tagged dtype. */
int cb_alloc(cb_backend *b, size_t bytes, int dtype, cb_mem *out);
/* Borrow an existing device pointer (not freed by cb_release). */
int cb_wrap(cb_backend *b, void *dptr, size_t bytes, int dtype, cb_mem *out);
/* ocl_upload (ocl_backend.h:91): allocate and fill from host memory. */
int cb_upload(cb_backend *b, const void *src, size_t bytes, int dtype,
              cb_mem *out);
/* ocl_upload_weight (ocl_backend.h:65): count fp32 values stored as dtype
 * (CB_BF16 for tensor-core GEMM operands, CB_F16 or CB_F32), rounded to
 * nearest even. */
int cb_upload_weight(cb_backend *b, const float *src, size_t count, int dtype,
                     cb_mem *out);
/* ocl_write / ocl_read (ocl_backend.h:94-97): blocking copies, byte
 * offsets. */
int cb_write(cb_backend *b, cb_mem dst, size_t off, const void *src, size_t n);
int cb_read(cb_backend *b, cb_mem src, size_t off, void *dst, size_t n);
/* ocl_release (ocl_backend.h:104): free and set *m to NULL. */
int cb_release(cb_mem *m);
void *cb_ptr(cb_mem m);
size_t cb_bytes(cb_mem m);
int cb_dtype(cb_mem m);
/* clFinish (sam3_model.c:1140 etc.): wait for the stream, then report a
 * device-side failure (CB_ETIMEOUT) if a kernel recorded one. */
int cb_sync(cb_backend *b);
/* Use an external CUDA stream (cudaStream_t as void*); NULL = own stream. */
int cb_set_stream(cb_backend *b, void *stream);
void *cb_stream(const cb_backend *b);
/* Device error word: 0 when no kernel has failed. cb_clear_error resets it. */
int cb_device_error(cb_backend *b);
int cb_clear_error(cb_backend *b);

/* Per-kernel profile, the counterpart of the reference's
 * I_SAM3_OPENCL_PROFILE table (sam3_model.c:149-207, printed in sam_free):
 * with profiling on, every kernel the backend launches is bracketed by CUDA
 * events on its stream (no host synchronisation is added) and accounted
 * under a name with its algorithmic FLOPs and bytes. cb_profile(b, 1)
 * clears the table and starts; cb_profile(b, 0) stops. cb_profile_entry
 * synchronises the stream, folds pending events in, and returns entry i
 * (CB_EARG past the end). */
int cb_profile(cb_backend *b, int on);
int cb_profile_entry(cb_backend *b, int i, const char **name, long *calls,
                     double *ms, double *flops, double *bytes);

/* ------------------------------------------------------------ operators
 * Replaces sam3_ops.h:17-65. Offsets, leading dimensions and batch strides
 * are in elements, as in the reference. */

/* struct opnd (sam3_ops.h:19-24). */
struct cb_opnd {
    cb_mem buf;
    int64_t off;
    int32_t ld;
    int64_t s0, s1;
};

/* mat / bmat (sam3_ops.h:48-49). */
struct cb_opnd cb_mat(cb_mem buf, int64_t off, int32_t ld);
struct cb_opnd cb_bmat(cb_mem buf, int64_t off, int32_t ld, int64_t s0,
                       int64_t s1);

/* gemm (sam3_ops.h:51-54, kernel contract sam3_kernels.cl:57-69): batched
 * C = act(alpha * A op(B) + bias) + R. transb != 0: B is N x K (Linear
 * weight layout). Batch b = (b / nb1, b % nb1) with per-operand strides s0,
 * s1; R has C's layout (offset roff) and may alias C. A, B: F32, BF16 or
 * F16; C, bias, R: F32, except that C may be BF16 on the tensor-core path.
 * nb == 1, transb, bf16 A and B with 16-byte aligned rows run on tcgen05
 * tensor cores (fp32 accumulation); other operands on CUDA cores (fp32). */
int cb_gemm(cb_backend *b, int M, int N, int K, struct cb_opnd A,
            struct cb_opnd B, int transb, struct cb_opnd C, int nb, int nb1,
            cb_mem bias, cb_mem R, int64_t roff, float alpha, int act);

/* linear (sam3_ops.h:56-58): Y[rows, out] = act(X[rows, in] W^T + b)
 * (+ Y when residual). An F32 X with a BF16 W is converted to bf16 in the
 * backend's scratch buffer first. */
int cb_linear(cb_backend *b, int rows, int in, int out, cb_mem X, int64_t xoff,
              cb_mem W, cb_mem bias, cb_mem Y, int64_t yoff, int act,
              int residual);

/* layernorm (sam3_ops.h:60-61): X F32 [rows, C] -> Y F32 or BF16; Y may
 * alias X (F32). */
int cb_layernorm(cb_backend *b, int64_t rows, int C, cb_mem X, cb_mem Y,
                 cb_mem g, cb_mem bias, float eps, int act);

/* add_bcast (sam3_ops.h:63-65): out[i] = a[i] + b[i % bmod]. */
int cb_add_bcast(cb_backend *b, cb_mem out, cb_mem a, cb_mem bb, int64_t n,
                 int64_t bmod);

/* The static helpers of sam3_model.c that vit_block calls, exported so a
 * caller can keep the reference's unfused sequence:
 * softmax_rows (sam3_model.c:332-341), rope_apply (:965-978, table row =
 * row % npos, on F32 qkv), window_partition / window_unpartition_add
 * (:360-392), patch_im2col (sam3_model.c:1120-1130). */
int cb_softmax_rows(cb_backend *b, cb_mem S, int64_t rows, int L);
int cb_rope_apply(cb_backend *b, cb_mem qkv, int64_t rows, int E, int hd,
                  int npos, cb_mem cs);
int cb_window_partition(cb_backend *b, cb_mem X, cb_mem out, int H, int C,
                        int ws, int nwx);
int cb_window_unpartition_add(cb_backend *b, cb_mem X, cb_mem Wd, int H, int C,
                              int ws, int nwx);
int cb_patch_im2col(cb_backend *b, cb_mem img, cb_mem out, int side, int grid,
                    int ps);

/* Attention core of vit_block: the one additive operator. It replaces the
 * inline sequence rope_apply -> QK^T gemm -> softmax_rows -> P.V gemm of
 * sam3_model.c:998-1013 (the reference has no attention op in sam3_ops.h).
 *
 * qkv: [nseq * N, 3E] rows (q | k | v, head h at column h * hd), as the
 * QKV linear leaves them. cs: RoPE table [npos, hd/2] (cos, sin) applied to
 * q and k with table row = row % npos (cs == NULL: RoPE already applied).
 * out: [nseq * N, E]. scale: 1/sqrt(hd) in vit_block.
 *   mode CB_ATTN_TC:  bf16 operands, fp32 accumulation, tcgen05 tensor
 *                     cores; qkv F32 (roped + cast into scratch) or BF16
 *                     (already roped, cs must be NULL); out F32 or BF16.
 *   mode CB_ATTN_F32: fp32 on CUDA cores (reference precision); qkv F32,
 *                     out F32. With cs != NULL, qkv is roped IN PLACE, as
 *                     the reference's rope_apply does.
 * hd must be 64 (as load_encoder requires, sam3_model.c:511-513). */
#define CB_ATTN_TC 0
#define CB_ATTN_F32 1
int cb_attention(cb_backend *b, cb_mem qkv, int nseq, int N, int E, int heads,
                 int hd, cb_mem cs, int npos, float scale, int mode,
                 cb_mem out);

/* Allocation-free variant of cb_attention (mode CB_ATTN_TC, fp32 qkv in,
 * fp32 out). No counterpart in the reference: it exists for callers that
 * cannot let a library call cudaMalloc -- code that hands all device memory
 * to its own pool or arena (an inference server's allocator, PyTorch's
 * caching allocator) and must not see allocations behind its back, and code
 * on a latency path where cudaMalloc/cudaFree and the synchronisation they
 * imply are not acceptable. cb_attention stages the bf16 copy of qkv in the
 * backend's scratch buffer, which it grows with cudaMalloc; this entry point
 * stages it in a fixed 32 MiB array compiled into the library instead, and
 * calls no cudaMalloc, cudaFree or allocating routine.
 *
 * Plain device pointers, no backend: qkv [nseq * N, 3E] fp32, cs the RoPE
 * table of (cos, sin) pairs, [npos, 32] float2 = npos * 64 fp32, or NULL (no
 * RoPE), out [nseq * N, E] fp32, stream a cudaStream_t (NULL = default
 * stream); runs on the current device and is asynchronous on `stream`.
 * err: a caller-owned device int, zeroed by the caller, that receives
 * CB_ETIMEOUT-style device codes (nonzero = a kernel wait ran out). With
 * err == NULL the kernels report into a word inside the library that is
 * cleared on each call and never read back: a device-side timeout then
 * cannot be observed (the call still returns CB_OK and out may hold partial
 * results), so callers that need to see it pass their own err.
 *
 * Limits: hd 64 (E = 64 * heads); nseq * N * 3E * 2 bytes must fit the
 * 32 MiB array (at E = 1024: at most 5461 rows, which covers the 9 x 576
 * windows and the 5184-token global grid of one tile); larger inputs return
 * CB_EARG before any work is queued.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture. The looked-up address is cached per device
 * ordinal for the life of the process: after cudaDeviceReset the cache is
 * stale, so do not call this entry point again on a device that was reset.
 * Every call shares the one array, which keeps the previous call's
 * contents: calls that overlap on the GPU (different streams, or different
 * host threads on one device) race on it. Each GPU that loads the library
 * holds the 32 MiB until the process exits. */
int cb_attention_noalloc(const float *qkv, int nseq, int N, int E, int heads,
                         const float *cs, int npos, float scale, float *out,
                         int *err, void *stream);

/* mha (sam3_model.c:413-451): mask-decoder attention, 8 heads, scale
 * 1/sqrt(dint/8); qp/kp/vp hold P prompts of Nq/Nk rows of dint channels
 * with per-prompt strides sq/sk/sv in elements (0 = shared); o receives
 * P * Nq rows. Nk > 64 requires dint == 128 (CB_EARG otherwise, as the
 * reference's "mha: unsupported shape"). All F32. */
int cb_mha(cb_backend *b, int P, int Nq, int Nk, int dint, cb_mem qp,
           int64_t sq, cb_mem kp, int64_t sk, cb_mem vp, int64_t sv, cb_mem o);

/* ------------------------------------------------------------ encoder
 * The PE ViT trunk of sam3_model.c (load_encoder :473-581, alloc_buffers
 * :815-916, vit_block :981-1028, sam_encode_trunk :1112-1144) on the
 * tensor-core path, batched over image tiles. */
typedef struct cb_encoder cb_encoder;

struct cb_encoder_config {
    int embed;         /* E, 1024 */
    int depth;         /* blocks, 32 */
    int heads;         /* 16 (head width E / heads must be 64) */
    int mlp;           /* 4096 */
    int grid;          /* tokens per side, 72 */
    int patch;         /* 14 */
    int window;        /* window side of windowed blocks, 24 */
    int max_tiles;     /* work buffers sized for this many tiles at once */
    uint64_t global_mask; /* bit i set: block i uses global attention */
};

/* Default SAM 3 geometry: 1024 wide, 32 blocks, global blocks 7/15/23/31. */
void cb_encoder_default_config(struct cb_encoder_config *cfg);

/* Allocate weights (bf16 matrices, fp32 vectors) and work buffers. */
int cb_encoder_create(cb_backend *b, const struct cb_encoder_config *cfg,
                      cb_encoder **out);
void cb_encoder_free(cb_encoder *e);

/* Random-init weights drawn on the device from include/sam3_synth.h
 * streams: matrices N(0, std), biases 0, LayerNorm gamma 1 / beta 0,
 * pos_embed N(0, std) on the 72 x 72 grid, 2D axial RoPE tables with
 * `theta`. */
int cb_encoder_init_random(cb_encoder *e, uint64_t seed, float std,
                           double theta);

/* Set one tensor from host fp32 data (a checkpoint loader's entry point).
 * which: see CB_W_* below; block is ignored for trunk-level tensors.
 * Shapes follow the PyTorch checkpoint (load_encoder, sam3_model.c:519-577):
 * PATCH_W [E, 3, p, p], POS [grid^2, E] (already tiled to the grid, as
 * sam3_model.c:492-498 does), LN_PRE_W/B [E], ROPE_WIN [window^2, hd/2, 2],
 * ROPE_GLOB [grid^2, hd/2, 2], and per block N1_W/B, N2_W/B [E], QKV_W
 * [3E, E], QKV_B [3E], PROJ_W [E, E], PROJ_B [E], FC1_W [mlp, E], FC1_B
 * [mlp], FC2_W [E, mlp], FC2_B [E]. */
#define CB_W_PATCH_W 0
#define CB_W_POS 1
#define CB_W_LN_PRE_W 2
#define CB_W_LN_PRE_B 3
#define CB_W_ROPE_WIN 4
#define CB_W_ROPE_GLOB 5
#define CB_W_N1_W 10
#define CB_W_N1_B 11
#define CB_W_QKV_W 12
#define CB_W_QKV_B 13
#define CB_W_PROJ_W 14
#define CB_W_PROJ_B 15
#define CB_W_N2_W 16
#define CB_W_N2_B 17
#define CB_W_FC1_W 18
#define CB_W_FC1_B 19
#define CB_W_FC2_W 20
#define CB_W_FC2_B 21
int cb_encoder_set_weight(cb_encoder *e, int which, int block,
                          const float *src, size_t count);

/* sam_encode_trunk on ntile uint8 HWC tiles (grid*patch square, RGB) in a
 * device buffer `tiles` (CB_U8): patch embedding with the image
 * normalisation of image.c:360-366, + pos_embed, ln_pre, all blocks.
 * out: F32 [ntile, grid^2, E], tokens in raster order (the reference's
 * m->x). ntile <= max_tiles. Asynchronous on the backend stream. */
int cb_encode_tiles(cb_encoder *e, cb_mem tiles, int ntile, cb_mem out);

/* Run blocks [first, last) on a raster-order F32 token buffer x [ntile,
 * grid^2, E] in place (the prologue is skipped). For block-level tests. */
int cb_encode_blocks(cb_encoder *e, cb_mem x, int ntile, int first, int last);

/* Host-to-host convenience: tiles from host memory, tokens back to host
 * memory out [ntile, grid^2, E]. Blocking. Runs as a pipeline over chunks
 * (about ntile / 4 tiles, at least 4, at most max_tiles; a batch of more
 * than two chunks plus 4 tiles ends with a chunk of 4, whose read-back is
 * the copy nothing overlaps): the copy of the next chunk in and of the
 * previous chunk out overlap the encode of the current one (page-locked
 * host buffers let the copies run asynchronously). */
int cb_encode_tiles_host(cb_encoder *e, const uint8_t *tiles, int ntile,
                         float *out);

/* ------------------------------------------------------------ decoder ops
 * Kernels of the mask decoder's output upscaling (sam3_kernels.cl:762-807).
 *
 * convt_scatter (sam3_model.c:394-410, sam3_kernels.cl:762-781): the GEMM
 * form G [P * H * W, Co * 4] (column co * 4 + dy * 2 + dx) of a 2x2 /
 * stride-2 ConvTranspose2d scattered into out [P, 2H, 2W, Co], + bias[co],
 * + add[(2H * 2W * Co) index] when add != NULL (shared by all P), then act.
 * All F32. */
int cb_convt_scatter(cb_backend *b, cb_mem G, cb_mem out, cb_mem bias,
                     cb_mem add, int P, int H, int W, int Co, int act);

/* mask_logits (sam3_model.c:1387-1399, sam3_kernels.cl:787-807):
 * out[p, m, pix] = hyper[p, m, :] . U[p, pix, :] for m < 3 over 32
 * channels; U [P, npix, 32], hyper [P, 96], out [P, 3, npix]. All F32. */
int cb_mask_logits(cb_backend *b, cb_mem U, cb_mem hyper, cb_mem out, int P,
                   int npix);

/* ------------------------------------------------------------ decoder
 * The point-prompt mask decoder of sam3_model.c: prompt encoding
 * (pe_encode :760-773), the image-side caches of sam_encode (:1153-1170),
 * sam_decode (:1239-1399: two-way transformer, final token-to-image
 * attention, output upscaling, hypernetwork and IoU heads, mask_logits).
 * Tensors and their order: include/sam3_synth.h (SAM3_DT_*). */
typedef struct cb_decoder cb_decoder;

/* Weights and work buffers for up to `batch` prompts per decode. */
int cb_decoder_create(cb_backend *b, int batch, cb_decoder **out);
void cb_decoder_free(cb_decoder *d);

/* Random init of every decoder tensor from the sam3_synth.h streams
 * (SAM3_STREAM_DECW + index; init kinds SAM3_INIT_*, std for the W and B
 * kinds). */
int cb_decoder_init_random(cb_decoder *d, uint64_t seed, float std);

/* Set decoder tensor `which` (SAM3_DT_*) from host fp32 data in the
 * checkpoint's layout and shape (sam3_dec_tensor gives rows x cols). */
int cb_decoder_set_weight(cb_decoder *d, int which, const float *src,
                          size_t count);

/* Image-side inputs of the decodes that follow (the outputs of the neck,
 * sam3_model.c:1098-1110): emb [72 * 72, 256] (with no_mem_embed added),
 * feat_s0 [288 * 288, 32], feat_s1 [144 * 144, 64], all F32 device
 * buffers, copied. Computes src = emb + no_mask_embed, the dense
 * positional encoding and the layer-0 projections that every prompt
 * shares (sam3_model.c:1153-1170). */
int cb_decoder_set_image(cb_decoder *d, cb_mem emb, cb_mem feat_s0,
                         cb_mem feat_s1);

/* sam_decode for P <= batch prompts, one positive point each: points [2P]
 * host (x, y) in input-image pixels; iou [3P] host receives the IoU
 * predictions of the three multimask outputs; lowres F32 device [P, 3,
 * 288, 288] receives their low-resolution mask logits. Blocking (iou is
 * read back at the end). */
int cb_decode(cb_decoder *d, int P, const float *points, float *iou,
              cb_mem lowres);

/* ------------------------------------------------------------ neck
 * The SimpleFPN neck of the point-prompt head and the decoder's
 * high-resolution projections (sam3_model.c: load_neck :585-622,
 * load_point_neck :642-654, conv3x3 :1032-1054, convt2x2 :1058-1065,
 * neck_level :1071-1095, point_neck :1098-1110), batched over tiles.
 * Tensors and their order: include/sam3_synth.h (SAM3_NT_*). */
typedef struct cb_neck cb_neck;

/* Weights and work buffers for maps of grid x grid tokens of width embed
 * (72 and 1024 for SAM 3; embed % 64 == 0), up to max_tiles per call. */
int cb_neck_create(cb_backend *b, int grid, int embed, int max_tiles,
                   cb_neck **out);
void cb_neck_free(cb_neck *n);

/* Random init from the sam3_synth.h streams (SAM3_STREAM_NECKW + index),
 * weights and biases N(0, std). */
int cb_neck_init_random(cb_neck *n, uint64_t seed, float std);

/* Set neck tensor `which` (SAM3_NT_*) from host fp32 data in the
 * checkpoint's layout (sam3_neck_tensor gives rows x cols; tensors a level
 * does not have are rejected). */
int cb_neck_set_weight(cb_neck *n, int which, const float *src, size_t count);

/* point_neck on ntile trunk outputs x F32 [ntile, grid^2, embed] (raster
 * tokens, as cb_encode_tiles writes them): emb F32 [ntile, grid^2, 256]
 * (no_mem_embed added), feat_s0 F32 [ntile, (4 grid)^2, 32], feat_s1 F32
 * [ntile, (2 grid)^2, 64] -- the inputs of cb_decoder_set_image.
 * Asynchronous on the backend stream. */
int cb_neck_run(cb_neck *n, cb_mem x, int ntile, cb_mem emb, cb_mem feat_s0,
                cb_mem feat_s1);

/* ------------------------------------------------------------ detector attention
 * attend (sam3_text.c:305-343): O = softmax(Q K^T / sqrt(hd) [+ mask or
 * bias]) V per head, Nq queries over Nk keys, heads of hd columns (32 or
 * 64), Q/K/V/O F32 rows with their own leading dimensions (elements), head h
 * at column h * hd. causal != 0 excludes keys j > query i; dy / dx (F32,
 * both or neither) add SAM 3's box relative position bias dy[(i * (Nk / W)
 * + y) * heads + h] + dx[(i * W + x) * heads + h] for key j = y * W + x
 * (softmax_ext, sam3_kernels.cl:889-921). mode CB_ATTN_TC runs every
 * call without the causal mask over at least 1024 keys on the tcgen05 flash
 * kernel with bf16 operands (heads zero-padded to 64 columns): the fusion
 * encoder's 5184-token self-attention, and queries over the image with or
 * without the box bias (the detector decoder's 201 queries; the bias enters
 * as a dense per-score term, the keys are split over CTAs when the query
 * tiles are few); everything else runs on the CUDA cores in fp32 (a flash
 * kernel with the keys split over CTAs). CB_ATTN_F32 always uses the fp32
 * kernel. */
int cb_attend(cb_backend *b, int Nq, int Nk, int heads, int hd, cb_mem Q,
              int ldq, cb_mem K, int ldk, cb_mem V, int ldv, cb_mem O, int ldo,
              int causal, cb_mem dy, cb_mem dx, int W, int mode);

/* ------------------------------------------------------------ input path
 * image_encoder_input (image.c:346-371) on the device: the crop (x0, y0, w,
 * h) of an interleaved 8-bit RGB image cols x rows in device buffer img
 * (CB_U8), resized to side x side with torchvision's uint8 antialiased
 * bilinear (aa_resize, image.c:209-339; bit-exact: integer arithmetic,
 * weights computed as the reference computes them) unless it has that size
 * already. Outputs (either may be NULL, not both): tiles (CB_U8) receives
 * the uint8 tile at byte offset tile * side * side * 3 -- the input of
 * cb_encode_tiles, which fuses the normalisation; chw (CB_F32 [3, side,
 * side]) receives the reference's float output (u / 255 - 0.5) / 0.5.
 * Asynchronous on the backend stream (the resize tables are computed on the
 * host and copied in the call). */
int cb_image_encoder_input(cb_backend *b, cb_mem img, int cols, int rows,
                           int x0, int y0, int w, int h, int side,
                           cb_mem tiles, int tile, cb_mem chw);

/* Diagnostics: the two exponential paths of the attention softmax on n
 * (even) device values x <= 0: y_poly = the FMA-pipe polynomial 2^x,
 * y_mufu = ex2.approx, for accuracy tests against the CUDA math library. */
int cb_diag_exp2(const float *x, float *y_poly, float *y_mufu, int n,
                 void *stream);

/* Diagnostics: the kernels' bounded pipeline wait on an mbarrier that
 * nothing arrives on, limited to limit_us (1 .. 1e6) microseconds. On the
 * device: *err (int, device memory) receives the wait-timeout code 1 unless
 * it already holds a code; status (2 device ints) = {wait returned
 * success, abort flag raised}. Tests that a wait gives up with a status
 * instead of hanging the GPU. */
int cb_diag_wait_timeout(int *err, int *status, int limit_us, void *stream);

/* Generator: fill a device buffer with normal(seed, stream, i) values
 * (include/sam3_synth.h) as F32 or BF16 (the buffer's dtype). */
int cb_synth_normal(cb_backend *b, uint64_t seed, uint64_t stream, float mean,
                    float std, cb_mem out, size_t count);

#ifdef __cplusplus
}
#endif
#endif
