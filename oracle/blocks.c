/*
 * blocks.c -- Q4_0 / Q8_0 block formats and quantizers (TEST INFRASTRUCTURE).
 * Restates static-lm src/quant/blocks.rs and the `half` 2.7.1 f16 conversion.
 */
#include <math.h>
#include <string.h>

#include "oracle.h"

/* half::f16::from_f32 (half 2.7.1): IEEE binary16, round to nearest even,
 * overflow to infinity, gradual underflow to subnormals. */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {
        if (man) return (uint16_t)(sign | 0x7e00u | (man >> 13));
        return (uint16_t)(sign | 0x7c00u);
    }
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t m = man | 0x800000u;
        int shift = 14 - e;
        uint32_t hm = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t man = (uint32_t)h & 0x3ffu;
    uint32_t x;
    float f;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {
            f = (float)man * 5.9604644775390625e-08f; /* 2^-24, exact */
            memcpy(&x, &f, 4);
            x |= sign;
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (man << 13);
    }
    memcpy(&f, &x, 4);
    return f;
}

/* Rust `f32 as i32`: saturating, NaN -> 0 */
static int sat_f32_to_i32(float v) {
    if (v != v) return 0;
    if (v >= 2147483647.0f) return 2147483647;
    if (v <= -2147483648.0f) return (-2147483647 - 1);
    return (int)v;
}

static float rust_max(float a, float b) { /* f32::max: NaN-ignoring */
    if (a != a) return b;
    if (b != b) return a;
    return a > b ? a : b;
}

/* blocks.rs:50-82 */
void orc_quantize_row_q4_0(const float *src, orc_block_q4_0 *dst, size_t n) {
    size_t nb = n / ORC_QK;
    for (size_t b = 0; b < nb; b++) {
        const float *chunk = src + b * ORC_QK;
        float min_val = 0.0f, max_val = 0.0f;
        for (int j = 0; j < ORC_QK; j++) {
            float v = chunk[j];
            if (v < min_val) min_val = v;
            if (v > max_val) max_val = v;
        }
        float d_pos = rust_max(-min_val / 8.0f, max_val / 7.0f);
        float d_neg = rust_max(max_val / 8.0f, -min_val / 7.0f);
        float d = (d_pos <= d_neg) ? d_pos : -d_neg;
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        dst[b].d = orc_f32_to_f16(d);
        for (int j = 0; j < ORC_QK / 2; j++) {
            float x0 = chunk[j] * id;
            float x1 = chunk[j + ORC_QK / 2] * id;
            int q0 = sat_f32_to_i32(roundf(x0)) + 8;
            int q1 = sat_f32_to_i32(roundf(x1)) + 8;
            q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
            q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
            dst[b].qs[j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

/* blocks.rs:85-99 */
void orc_dequantize_row_q4_0(const orc_block_q4_0 *src, float *dst, size_t n) {
    size_t nb = n / ORC_QK;
    for (size_t b = 0; b < nb; b++) {
        float d = orc_f16_to_f32(src[b].d);
        for (int j = 0; j < ORC_QK / 2; j++) {
            uint8_t packed = src[b].qs[j];
            int q0 = (int)(packed & 0x0F) - 8;
            int q1 = (int)(packed >> 4) - 8;
            dst[b * ORC_QK + j] = (float)q0 * d;
            dst[b * ORC_QK + j + ORC_QK / 2] = (float)q1 * d;
        }
    }
}

/* blocks.rs:102-123 */
void orc_quantize_row_q8_0(const float *src, orc_block_q8_0 *dst, size_t n) {
    size_t nb = n / ORC_QK;
    for (size_t b = 0; b < nb; b++) {
        const float *chunk = src + b * ORC_QK;
        float amax = 0.0f;
        for (int j = 0; j < ORC_QK; j++) {
            float av = fabsf(chunk[j]);
            if (av > amax) amax = av;
        }
        float d = amax / 127.0f;
        float id = (amax != 0.0f) ? 127.0f / amax : 0.0f;
        dst[b].d = orc_f32_to_f16(d);
        for (int j = 0; j < ORC_QK; j++) {
            float r = roundf(chunk[j] * id);
            /* f32::clamp(-127, 127) then `as i8` */
            if (r < -127.0f) r = -127.0f;
            if (r > 127.0f) r = 127.0f;
            dst[b].qs[j] = (r != r) ? 0 : (int8_t)r;
        }
    }
}

/* blocks.rs:126-135 */
void orc_dequantize_row_q8_0(const orc_block_q8_0 *src, float *dst, size_t n) {
    size_t nb = n / ORC_QK;
    for (size_t b = 0; b < nb; b++) {
        float d = orc_f16_to_f32(src[b].d);
        for (int j = 0; j < ORC_QK; j++) dst[b * ORC_QK + j] = (float)src[b].qs[j] * d;
    }
}
