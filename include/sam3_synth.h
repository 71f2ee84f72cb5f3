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

#ifdef __cplusplus
}
#endif
#endif
