/* SPDX-License-Identifier: Unlicense */
/* Host side of the seeded synthetic-data generator (include/sam3_synth.h). */
#include "sam3_synth.h"

#include <math.h>

void sam3_synth_normal(uint64_t seed, uint64_t stream, size_t n, float mean,
                       float std, float *out)
{
    const uint64_t base = sam3_stream_base(seed, stream);
    long i;

#pragma omp parallel for schedule(static)
    for (i = 0; i < (long)n; i++) {
        /* One rounded multiply, one rounded add: the CUDA generator uses
         * __fmul_rn/__fadd_rn to give the same bits. */
        volatile float p = std * sam3_normal_at(base, (uint64_t)i);
        out[i] = mean + p;
    }
}

void sam3_synth_u8(uint64_t seed, uint64_t stream, size_t n, uint8_t *out)
{
    const uint64_t base = sam3_stream_base(seed, stream);
    long i;

#pragma omp parallel for schedule(static)
    for (i = 0; i < (long)n; i++)
        out[i] = sam3_u8_at(base, (uint64_t)i);
}

void sam3_synth_rope_axial(int side, int hd, double theta, float *cs)
{
    const int nf = hd / 2, q = hd / 4;
    int p, j;

    for (p = 0; p < side * side; p++) {
        const int y = p / side, x = p % side;

        for (j = 0; j < nf; j++) {
            const int k = j < q ? j : j - q;
            const double f = pow(theta, -4.0 * k / hd);
            const double a = (j < q ? x : y) * f;

            cs[((size_t)p * nf + j) * 2 + 0] = (float)cos(a);
            cs[((size_t)p * nf + j) * 2 + 1] = (float)sin(a);
        }
    }
}
