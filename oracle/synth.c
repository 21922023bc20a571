/*
 * synth.c -- the reference's fixture generator (TEST INFRASTRUCTURE).
 *
 *  - orc_xorshift_f32: the reference's own fixture generator, xorshift32 with
 *    unit = seed / u32::MAX and value (unit*2 - 1)*scale (main.rs:18-28,
 *    kernels.rs:425-435, transformer.rs:959-969).
 */

#include "oracle.h"

void orc_xorshift_f32(float *out, size_t n, uint32_t seed, float scale) {
    for (size_t i = 0; i < n; i++) {
        seed ^= seed << 13;
        seed ^= seed >> 17;
        seed ^= seed << 5;
        float unit = (float)seed / 4294967296.0f; /* u32::MAX as f32 == 2^32 */
        out[i] = (unit * 2.0f - 1.0f) * scale;
    }
}
