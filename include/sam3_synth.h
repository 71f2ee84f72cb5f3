/* SPDX-License-Identifier: Unlicense */
/* Seeded synthetic data for the SAM 3 PE backbone path: random-init weights,
 * uint8 image tiles, activations and 2D axial RoPE tables.
 *
 * The reference reads weights from the gated sam3.pt checkpoint
 * (sam3_model.c:473-581) and images through GRASS (image.c). Neither is
 * available, so every benchmark and parity test draws its inputs from this
 * counter-based generator. Value i of stream s under seed k depends only on
 * (k, s, i), so the host and the GPU produce the same bits in any order:
 *
 *   normal(k, s, i)  = mean + std * z,  z = (sum of 12 uniform 16-bit
 *                      integers - 393210) / 65536   (Irwin-Hall(12): mean 0,
 *                      variance 1 - 2^-32, bounded to |z| < 6)
 *   u8(k, s, i)      = one byte of the same hash stream.
 *
 * All arithmetic is exact or a single IEEE-rounded float multiply and add,
 * so results are bit-identical between C on the host and CUDA on the GPU.
 */
#ifndef SAM3_SYNTH_H
#define SAM3_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifdef __CUDACC__
#define SAM3_HD __host__ __device__
#else
#define SAM3_HD
#endif

/* splitmix64 finalizer. */
static inline SAM3_HD uint64_t sam3_mix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

static inline SAM3_HD uint64_t sam3_stream_base(uint64_t seed, uint64_t stream)
{
    return sam3_mix64(seed * 0xD1B54A32D192ED03ULL ^ sam3_mix64(stream));
}

/* Irwin-Hall(12) draw number i of a stream; see the file comment. */
static inline SAM3_HD float sam3_normal_at(uint64_t base, uint64_t i)
{
    int64_t s = 0;
    for (int k = 0; k < 3; k++) {
        uint64_t h = sam3_mix64(base + 3 * i + (uint64_t)k);
        s += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) +
             (int64_t)((h >> 32) & 0xFFFF) + (int64_t)(h >> 48);
    }
    return (float)(s - 393210) * (1.0f / 65536.0f);
}

static inline SAM3_HD uint8_t sam3_u8_at(uint64_t base, uint64_t i)
{
    return (uint8_t)(sam3_mix64(base + (i >> 3)) >> (8 * (i & 7)));
}

/* out[i] = mean + std * normal(seed, stream, i), i < n (OpenMP-parallel). */
void sam3_synth_normal(uint64_t seed, uint64_t stream, size_t n, float mean,
                       float std, float *out);

/* out[i] = u8(seed, stream, i), i < n. */
void sam3_synth_u8(uint64_t seed, uint64_t stream, size_t n, uint8_t *out);

/* 2D axial RoPE table of a side x side token grid, head width hd (hd % 4 ==
 * 0), as (cos, sin) float pairs: cs[(p * hd/2 + j) * 2 + {0, 1}] for
 * position p = y * side + x. Frequencies f_k = theta^(-4k / hd), k < hd/4;
 * pairs j < hd/4 rotate by x * f_j, pairs j >= hd/4 by y * f_(j - hd/4).
 * This is the layout the reference uploads from the checkpoint's complex
 * freqs_cis (sam3_model.c:455-471) and indexes in rope_apply
 * (sam3_kernels.cl:693). */
void sam3_synth_rope_axial(int side, int hd, double theta, float *cs);

/* Stream numbers of the backbone's random-init tensors (any fixed
 * assignment works; this one is shared by the GPU path and the oracle). */
enum {
    SAM3_STREAM_PATCH_W = 1,   /* [E, 3, 14, 14] */
    SAM3_STREAM_POS = 2,       /* [T, E], already tiled to the 72 x 72 grid */
    SAM3_STREAM_IMAGE = 3,     /* uint8 tiles, HWC, stream + tile index */
    SAM3_STREAM_QKV_IN = 4,    /* fp32 Q/K/V activations of configs 1-2 */
    SAM3_STREAM_DEC = 8,       /* decoder activations, + tensor index */
    SAM3_STREAM_BLOCK0 = 1024  /* + 16 * block + tensor (see below) */
};
enum {
    SAM3_BT_QKV_W = 0,
    SAM3_BT_PROJ_W = 1,
    SAM3_BT_FC1_W = 2,
    SAM3_BT_FC2_W = 3
};
#define SAM3_IMAGE_STREAM_TILE(t) ((uint64_t)SAM3_STREAM_IMAGE * 1000003ULL + (uint64_t)(t))

/* ------------------------------------------------ point-prompt mask decoder
 * The tensors of the decoder (sam3_model.c load_decoder :656-755 and the
 * decoder's share of load_point_neck :642-654) in one fixed order, with the
 * reference's shapes ([rows, cols], cols 1 for vectors; 4-D ConvTranspose
 * weights [cin, cout, 2, 2] as [cin, cout * 4]). Random init of tensor i
 * draws stream SAM3_STREAM_DECW + i:
 *   SAM3_INIT_W     N(0, std)      Linear / ConvTranspose weights
 *   SAM3_INIT_B     N(0, std)      their biases
 *   SAM3_INIT_LNW   N(1, 0.1)      LayerNorm weights
 *   SAM3_INIT_LNB   N(0, 0.1)      LayerNorm biases
 *   SAM3_INIT_EMB   N(0, 1)        tokens, prompt embeddings, the gaussian
 *                                  matrix of the positional encoding
 * The image-side inputs of a decode (image embedding [T, 256], feat_s0
 * [16T, 32], feat_s1 [4T, 64]) draw N(0, 1) from SAM3_STREAM_DECIMG + 0, 1,
 * 2 when a test or benchmark synthesises them. */
enum {
    SAM3_INIT_W = 0,
    SAM3_INIT_B = 1,
    SAM3_INIT_LNW = 2,
    SAM3_INIT_LNB = 3,
    SAM3_INIT_EMB = 4
};
#define SAM3_STREAM_DECW 8192ULL
#define SAM3_STREAM_DECIMG 9216ULL

/* Attention blocks of the decoder, 8 tensors each (q, k, v, out projection
 * weight and bias: q_w [d, 256], q_b [d], k_w, k_b, v_w, v_b, o_w [256, d],
 * o_b [256]) with inner width d = 256 (self) or 128 (cross). */
enum {
    SAM3_DA_L0_SELF = 0,
    SAM3_DA_L0_T2I = 1,
    SAM3_DA_L0_I2T = 2,
    SAM3_DA_L1_SELF = 3,
    SAM3_DA_L1_T2I = 4,
    SAM3_DA_L1_I2T = 5,
    SAM3_DA_FINAL_T2I = 6,
    SAM3_DA_COUNT = 7
};
/* Tensor indices. */
enum {
    SAM3_DT_ATTN = 0,                       /* + 8 * block + {q_w, q_b, k_w, k_b, v_w, v_b, o_w, o_b} */
    SAM3_DT_LAYER = 8 * SAM3_DA_COUNT,      /* + 12 * layer + {n1w, n1b, n2w, n2b, n3w, n3b, n4w, n4b, m1w, m1b, m2w, m2b} */
    SAM3_DT_NF_W = SAM3_DT_LAYER + 24,      /* norm_final_attn */
    SAM3_DT_NF_B,
    SAM3_DT_UP0_W,                          /* output_upscaling.0: [256, 64 * 4] */
    SAM3_DT_UP0_B,                          /* [64] */
    SAM3_DT_UP1_W,                          /* output_upscaling.1 (LayerNorm2d) [64] */
    SAM3_DT_UP1_B,
    SAM3_DT_UP3_W,                          /* output_upscaling.3: [64, 32 * 4] */
    SAM3_DT_UP3_B,                          /* [32] */
    SAM3_DT_HYPER,                          /* + 6 * mlp + {w0, b0, w1, b1, w2, b2}, 4 MLPs */
    SAM3_DT_IOU = SAM3_DT_HYPER + 24,       /* + {w0, b0, w1, b1, w2, b2} */
    SAM3_DT_GAUSS = SAM3_DT_IOU + 6,        /* [2, 128] */
    SAM3_DT_POINT_EMB,                      /* + 4: point_embeddings.0..3 [256] */
    SAM3_DT_NOT_A_POINT = SAM3_DT_POINT_EMB + 4,
    SAM3_DT_NO_MASK,
    SAM3_DT_OBJ_TOKEN,
    SAM3_DT_IOU_TOKEN,
    SAM3_DT_MASK_TOKENS,                    /* [4, 256] */
    SAM3_DT_COUNT
};

/* Shape and init kind of decoder tensor i (0 <= i < SAM3_DT_COUNT). */
static inline void sam3_dec_tensor(int i, int *rows, int *cols, int *init)
{
    int r = 256, c = 1, k = SAM3_INIT_EMB;

    if (i < SAM3_DT_LAYER) {
        const int blk = i / 8, t = i % 8;
        const int d = (blk == SAM3_DA_L0_SELF || blk == SAM3_DA_L1_SELF) ? 256 : 128;

        r = t < 6 ? d : 256;
        c = (t & 1) ? 1 : (t < 6 ? 256 : d);
        k = (t & 1) ? SAM3_INIT_B : SAM3_INIT_W;
    }
    else if (i < SAM3_DT_NF_W) {
        const int t = (i - SAM3_DT_LAYER) % 12;

        if (t < 8) {
            k = (t & 1) ? SAM3_INIT_LNB : SAM3_INIT_LNW;
        }
        else if (t == 8 || t == 9) {
            r = 2048;
            c = t == 8 ? 256 : 1;
            k = t == 8 ? SAM3_INIT_W : SAM3_INIT_B;
        }
        else {
            c = t == 10 ? 2048 : 1;
            k = t == 10 ? SAM3_INIT_W : SAM3_INIT_B;
        }
    }
    else if (i == SAM3_DT_NF_W || i == SAM3_DT_NF_B) {
        k = i == SAM3_DT_NF_W ? SAM3_INIT_LNW : SAM3_INIT_LNB;
    }
    else if (i == SAM3_DT_UP0_W) {
        c = 256, k = SAM3_INIT_W;
    }
    else if (i == SAM3_DT_UP0_B || i == SAM3_DT_UP1_W || i == SAM3_DT_UP1_B) {
        r = 64;
        k = i == SAM3_DT_UP0_B ? SAM3_INIT_B : (i == SAM3_DT_UP1_W ? SAM3_INIT_LNW : SAM3_INIT_LNB);
    }
    else if (i == SAM3_DT_UP3_W) {
        r = 64, c = 128, k = SAM3_INIT_W;
    }
    else if (i == SAM3_DT_UP3_B) {
        r = 32, k = SAM3_INIT_B;
    }
    else if (i < SAM3_DT_GAUSS) {
        /* hypernetwork MLPs (output 32) and the IoU head (output 4) */
        const int t = (i - SAM3_DT_HYPER) % 6, last = t >= 4;
        const int nout = i >= SAM3_DT_IOU ? 4 : 32;

        r = last ? nout : 256;
        c = (t & 1) ? 1 : 256;
        k = (t & 1) ? SAM3_INIT_B : SAM3_INIT_W;
    }
    else if (i == SAM3_DT_GAUSS) {
        r = 2, c = 128;
    }
    else if (i == SAM3_DT_MASK_TOKENS) {
        r = 4, c = 256;
    }
    *rows = r;
    *cols = c;
    *init = k;
}

/* ------------------------------------------------ SimpleFPN neck
 * The neck of the point-prompt head (sam3_model.c load_neck :585-622 with
 * E = 1024, SAM_DIM = 256) and the decoder's high-resolution projections
 * and no-memory embedding (load_point_neck :642-654). Level l = 0, 1, 2
 * (scale 4, 2, 1) has 8 tensors {d0_w, d0_b, d1_w, d1_b, c1_w, c1_b, c3_w,
 * c3_b}; the ones a level does not have are empty (0 rows). Shapes in the
 * checkpoint layout, ConvTranspose weights [cin, cout, 2, 2] as
 * [cin, cout * 4], convolution weights [cout, cin, kh, kw] as
 * [cout, cin * kh * kw]. Random init of tensor i draws stream
 * SAM3_STREAM_NECKW + i: weights and biases N(0, std) (SAM3_INIT_W / _B). */
#define SAM3_STREAM_NECKW 10240ULL
enum {
    SAM3_NT_LEVEL = 0,           /* + 8 * level + {d0w, d0b, d1w, d1b, c1w, c1b, c3w, c3b} */
    SAM3_NT_S0_W = 24,           /* conv_s0 [32, 256] */
    SAM3_NT_S0_B,                /* [32] */
    SAM3_NT_S1_W,                /* conv_s1 [64, 256] */
    SAM3_NT_S1_B,                /* [64] */
    SAM3_NT_NO_MEM,              /* no_mem_embed [256] */
    SAM3_NT_COUNT
};

/* Shape and init kind of neck tensor i for backbone width E. */
static inline void sam3_neck_tensor(int i, int E, int *rows, int *cols, int *init)
{
    int r = 0, c = 1, k = SAM3_INIT_B;

    if (i < SAM3_NT_S0_W) {
        const int l = i / 8, t = i % 8;
        const int cin = l == 0 ? E / 4 : (l == 1 ? E / 2 : E);

        switch (t) {
        case 0: /* ConvTranspose 0: E -> E / 2 (levels 0 and 1) */
            if (l < 2)
                r = E, c = (E / 2) * 4;
            break;
        case 1:
            if (l < 2)
                r = E / 2;
            break;
        case 2: /* ConvTranspose 1: E / 2 -> E / 4 (level 0) */
            if (l == 0)
                r = E / 2, c = (E / 4) * 4;
            break;
        case 3:
            if (l == 0)
                r = E / 4;
            break;
        case 4:
            r = 256, c = cin;
            break;
        case 6:
            r = 256, c = 256 * 9;
            break;
        default: /* c1_b, c3_b */
            r = 256;
        }
        k = (t & 1) ? SAM3_INIT_B : SAM3_INIT_W;
    }
    else if (i == SAM3_NT_S0_W || i == SAM3_NT_S1_W) {
        r = i == SAM3_NT_S0_W ? 32 : 64, c = 256, k = SAM3_INIT_W;
    }
    else if (i == SAM3_NT_S0_B || i == SAM3_NT_S1_B) {
        r = i == SAM3_NT_S0_B ? 32 : 64;
    }
    else if (i == SAM3_NT_NO_MEM) {
        r = 256;
    }
    *rows = r;
    *cols = r ? c : 0;
    *init = k;
}

#ifdef __cplusplus
}
#endif
#endif
