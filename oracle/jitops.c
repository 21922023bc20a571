/*
 * jitops.c -- the JIT vector operators (TEST INFRASTRUCTURE).
 *
 * Restates the semantics of the Cranelift code static-lm generates from its
 * FuseGraph op graphs (src/jit/graph.rs:130-193) through lower_fuse_graph
 * (src/jit/lower.rs:212-480):
 *   - every reduction is its own pass: four F32X4 lane accumulators over
 *     indices [0, len & ~3) (lane l sees i = l, l+4, ...), the horizontal
 *     combine (l0 op l1) op (l2 op l3), then a sequential scalar tail over
 *     [len & ~3, len)  (lower.rs:252-389);
 *   - values a pass needs are recomputed per element, with IEEE fmul/fadd/
 *     fdiv/sqrt rounded individually (no fused multiply-add);
 *   - exp is the polynomial of lower.rs:22-65; SiLU is v / (1 + exp(-v))
 *     (lower.rs:87-93); Recip is 1/v (lower.rs:82-85).
 * ORC_MODE_SCALAR gives the scalar forms of bench.rs:15-39 and
 * transformer.rs:246-262 instead (sequential sums, libm expf).
 */
#include <math.h>
#include <string.h>

#include "oracle.h"

/* Cranelift fmax/fmin: NaN-propagating, -0 < +0 */
static float cl_fmax(float a, float b) {
    if (a != a || b != b) return a + b;
    if (a == b) return signbit(a) ? b : a;
    return a > b ? a : b;
}
static float cl_fmin(float a, float b) {
    if (a != a || b != b) return a + b;
    if (a == b) return signbit(a) ? a : b;
    return a < b ? a : b;
}

static float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* lower.rs:22-65 */
float orc_exp_poly(float x) {
    float xc = cl_fmin(cl_fmax(x, -87.3f), 88.3f);
    float fx = xc * 1.44269504088896340736f; /* std::f32::consts::LOG2_E */
    float n = rintf(fx);                       /* Cranelift `nearest`: ties to even */
    float n_hi = n * 0.69314575f;
    float n_lo = n * 1.4286068e-6f;
    float r = (xc - n_hi) - n_lo;
    float p = r * (1.0f / 120.0f);
    p = p + (1.0f / 24.0f);
    p = r * p;
    p = p + (1.0f / 6.0f);
    p = r * p;
    p = p + 0.5f;
    p = r * p;
    p = p + 1.0f;
    p = r * p;
    float poly = p + 1.0f;
    int ni = (int)n; /* fcvt_to_sint_sat; n is integral and within [-126, 127] */
    uint32_t pow2_bits = (uint32_t)(ni + 127) << 23;
    return poly * bits_f32(pow2_bits);
}

/* Sum reduction in the lowered order: 4 lanes, (l0+l1)+(l2+l3), scalar tail. */
static float lane4_sum(const float *v, size_t len) {
    size_t vl = len & ~(size_t)3;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (size_t i = 0; i < vl; i += 4) {
        a0 = a0 + v[i];
        a1 = a1 + v[i + 1];
        a2 = a2 + v[i + 2];
        a3 = a3 + v[i + 3];
    }
    float s = (a0 + a1) + (a2 + a3);
    for (size_t i = vl; i < len; i++) s = s + v[i];
    return s;
}

static float lane4_sumsq(const float *x, size_t len) {
    size_t vl = len & ~(size_t)3;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (size_t i = 0; i < vl; i += 4) {
        a0 = a0 + x[i] * x[i];
        a1 = a1 + x[i + 1] * x[i + 1];
        a2 = a2 + x[i + 2] * x[i + 2];
        a3 = a3 + x[i + 3] * x[i + 3];
    }
    float s = (a0 + a1) + (a2 + a3);
    for (size_t i = vl; i < len; i++) s = s + x[i] * x[i];
    return s;
}

/* graph.rs:168-179; in place allowed (out == x) */
void orc_softmax(const float *x, float *out, size_t len, int mode) {
    if (len == 0) return;
    if (mode == ORC_MODE_SCALAR) {
        /* transformer.rs:246-262 */
        float mx = -INFINITY;
        for (size_t i = 0; i < len; i++)
            if (x[i] > mx) mx = x[i];
        float s = 0.0f;
        for (size_t i = 0; i < len; i++) {
            float e = expf(x[i] - mx);
            out[i] = e;
            s = s + e;
        }
        float inv = 1.0f / s;
        for (size_t i = 0; i < len; i++) out[i] = out[i] * inv;
        return;
    }
    size_t vl = len & ~(size_t)3;
    float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
    for (size_t i = 0; i < vl; i += 4) {
        m0 = cl_fmax(m0, x[i]);
        m1 = cl_fmax(m1, x[i + 1]);
        m2 = cl_fmax(m2, x[i + 2]);
        m3 = cl_fmax(m3, x[i + 3]);
    }
    float mx = cl_fmax(cl_fmax(m0, m1), cl_fmax(m2, m3));
    for (size_t i = vl; i < len; i++) mx = cl_fmax(mx, x[i]);
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (size_t i = 0; i < vl; i += 4) {
        a0 = a0 + orc_exp_poly(x[i] - mx);
        a1 = a1 + orc_exp_poly(x[i + 1] - mx);
        a2 = a2 + orc_exp_poly(x[i + 2] - mx);
        a3 = a3 + orc_exp_poly(x[i + 3] - mx);
    }
    float s = (a0 + a1) + (a2 + a3);
    for (size_t i = vl; i < len; i++) s = s + orc_exp_poly(x[i] - mx);
    float inv = 1.0f / s;
    for (size_t i = 0; i < len; i++) out[i] = orc_exp_poly(x[i] - mx) * inv;
}

/* graph.rs:141-155: rms = 1/sqrt(sum(x^2) * (1/n) + eps); out = (x*rms)*w.
 * The graph is compiled with n = the layer dim and run with len = n. */
void orc_rmsnorm(const float *x, const float *w, float *out, size_t len, float eps, int mode) {
    if (len == 0) return;
    if (mode == ORC_MODE_SCALAR) {
        /* bench.rs:15-24 */
        float s = 0.0f;
        for (size_t i = 0; i < len; i++) s = s + x[i] * x[i];
        float rms = 1.0f / sqrtf(s / (float)len + eps);
        for (size_t i = 0; i < len; i++) out[i] = (x[i] * rms) * w[i];
        return;
    }
    float inv_n = 1.0f / (float)len;
    float s = lane4_sumsq(x, len);
    float mean = s * inv_n;
    float var = mean + eps;
    float sd = sqrtf(var);
    float rms = 1.0f / sd;
    for (size_t i = 0; i < len; i++) out[i] = (x[i] * rms) * w[i];
}

/* graph.rs:131-138 */
void orc_swiglu(const float *g, const float *u, float *out, size_t len, int mode) {
    for (size_t i = 0; i < len; i++) {
        float v = g[i];
        float e = (mode == ORC_MODE_SCALAR) ? expf(-v) : orc_exp_poly(-v);
        float silu = v / (1.0f + e);
        out[i] = silu * u[i];
    }
}

/* graph.rs:158-164 */
void orc_residual_add(const float *a, const float *b, float *out, size_t len) {
    for (size_t i = 0; i < len; i++) out[i] = a[i] + b[i];
}

/* graph.rs:182-193: out = x * (1/sqrt(sum(x^2) + eps)) */
void orc_l2_norm(const float *x, float *out, size_t len, float eps) {
    if (len == 0) return;
    float s = lane4_sumsq(x, len);
    float norm = sqrtf(s + eps);
    float inv = 1.0f / norm;
    for (size_t i = 0; i < len; i++) out[i] = x[i] * inv;
}

/* exported for the attention restatement */
float orc__lane4_sum(const float *v, size_t len) { return lane4_sum(v, len); }
