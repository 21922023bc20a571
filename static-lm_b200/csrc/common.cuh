// common.cuh -- shared device helpers for the sm_100a hot path.
//
// Every kernel here reproduces the reference's f32 arithmetic operation by
// operation.  The library is compiled with --fmad=false so that no multiply
// and add are ever contracted behind our back; the one fused multiply-add the
// reference itself performs (the AVX2 vec-dot accumulation,
// src/quant/kernels.rs:200) is written as an explicit __fmaf_rn.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace slm {

constexpr int QK = 32;             // elements per Q4_0 / Q8_0 block
constexpr int TILE_ROWS = 32;      // rows per repacked weight tile (one warp)
constexpr int TILE_BYTES = 576;    // 32 rows x (16 B nibbles) + 32 x f16 scale
constexpr int MAGIC_I = 0x4B400000;  // bits of 12582912.0f = 1.5 * 2^23
constexpr float MAGIC_F = 12582912.0f;

// ---------------------------------------------------------------------------
// Repacked Q4_0 weights ("row tiles").  A rows x cols matrix of the reference's
// 18-byte BlockQ4_0 (src/quant/blocks.rs:11-16) is stored as
// ceil(rows/32) x (cols/32) tiles of 576 bytes:
//     bytes [0, 512):   16-byte nibble payload of block j for rows 32t .. 32t+31
//     bytes [512, 576): the 32 f16 scales of those blocks
// so that a warp reading block j of 32 consecutive rows issues one fully
// coalesced 128-bit load per lane.  Same 18 bytes per block as the reference.
// ---------------------------------------------------------------------------
__host__ __device__ inline size_t tile_offset(size_t row_tile, size_t nb, size_t j) {
    return (row_tile * nb + j) * (size_t)TILE_BYTES;
}

// ---------------------------------------------------------------------------
// Device activation format "Q8X" (the arena's q8 scratch).  For each 32-element
// block of an activation row: 32 int8 values (clamped to >= -127 as
// kernels.rs:189-191 does), 8 int32 "lane constants" c_k = MAGIC_I - 8*sum of
// the 4 values of lane k, and the f16-rounded scale widened to f32.  With
// these, one dp4a of the unsigned weight nibbles yields MAGIC_I + isum_k
// directly, i.e. the f32 bit pattern of 12582912 + isum_k.
// Planar layout for `rows` rows of `nb` blocks:
//     qs: int8 [rows*nb*32] | c: int32 [rows*nb*8] | d: f32 [rows*nb]
// ---------------------------------------------------------------------------
struct Q8X {
    int8_t *qs;
    int32_t *c;
    float *d;
};

__host__ __device__ inline size_t q8x_bytes(size_t blocks) { return blocks * 68; }

__host__ __device__ inline Q8X q8x_view(void *base, size_t blocks) {
    Q8X v;
    v.qs = (int8_t *)base;
    v.c = (int32_t *)((char *)base + blocks * 32);
    v.d = (float *)((char *)base + blocks * 64);
    return v;
}

// dp4a with unsigned bytes in `a` and signed bytes in `b`.
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// ---------------------------------------------------------------------------
// Cranelift float semantics used by the JIT vector ops (src/jit/lower.rs).
// ---------------------------------------------------------------------------
// fmax/fmin: NaN when either input is NaN (as a + b), +0 over -0 for max and
// -0 over +0 for min, else the larger / smaller.  Written as selects: the
// early-return form compiles to branches that cost ~70 cycles per call.
// For a == b the two bit patterns differ at most in the sign of a zero, so
// AND (max) / OR (min) of the bits picks the right zero.
__device__ __forceinline__ float cl_fmax(float a, float b) {
    const float nan = __fadd_rn(a, b);
    const float eq = __int_as_float(__float_as_int(a) & __float_as_int(b));
    float r = a > b ? a : b;
    r = a == b ? eq : r;
    return (a != a || b != b) ? nan : r;
}
__device__ __forceinline__ float cl_fmin(float a, float b) {
    const float nan = __fadd_rn(a, b);
    const float eq = __int_as_float(__float_as_int(a) | __float_as_int(b));
    float r = a < b ? a : b;
    r = a == b ? eq : r;
    return (a != a || b != b) ? nan : r;
}

// Maximum over the warp of a float, NaN if any lane holds NaN (sm_100a
// redux.sync on f32).  Zeros of either sign compare equal.
__device__ __forceinline__ float warp_max_nan(float v) {
    float r;
    asm volatile("redux.sync.max.NaN.f32 %0, %1, 0xffffffff;\n" : "=f"(r) : "f"(v));
    return r;
}

// The reference's polynomial exp (src/jit/lower.rs:22-65): clamp to
// [-87.3, 88.3], n = nearest(x*log2 e), Cody-Waite split of n*ln2,
// degree-5 Horner polynomial with separately rounded mul/add, times 2^n built
// from exponent bits.
__device__ __forceinline__ float exp_poly(float x) {
    // cl_fmin(cl_fmax(x, -87.3), 88.3) for constant, non-zero bounds
    float xc = x > -87.3f ? x : -87.3f;
    xc = xc < 88.3f ? xc : 88.3f;
    xc = x != x ? __fadd_rn(__fadd_rn(x, -87.3f), 88.3f) : xc;
    float fx = __fmul_rn(xc, 1.44269504088896340736f);
    float n = rintf(fx);
    float n_hi = __fmul_rn(n, 0.69314575f);
    float n_lo = __fmul_rn(n, 1.4286068e-6f);
    float r = __fsub_rn(__fsub_rn(xc, n_hi), n_lo);
    float p = __fmul_rn(r, 1.0f / 120.0f);
    p = __fadd_rn(p, 1.0f / 24.0f);
    p = __fmul_rn(r, p);
    p = __fadd_rn(p, 1.0f / 6.0f);
    p = __fmul_rn(r, p);
    p = __fadd_rn(p, 0.5f);
    p = __fmul_rn(r, p);
    p = __fadd_rn(p, 1.0f);
    p = __fmul_rn(r, p);
    float poly = __fadd_rn(p, 1.0f);
    int ni = (int)n;
    float pow2 = __int_as_float((ni + 127) << 23);
    return __fmul_rn(poly, pow2);
}

// SiLU(v) * u as the SwiGLU graph lowers it (graph.rs:131-138, lower.rs:87-93)
__device__ __forceinline__ float swiglu1(float g, float u) {
    float e = exp_poly(-g);
    float silu = __fdiv_rn(g, __fadd_rn(1.0f, e));
    return __fmul_rn(silu, u);
}

// Rust f32::round (ties away from zero), then clamp(-127, 127) and `as i8`
// (src/quant/blocks.rs:120).
__device__ __forceinline__ int q8_round(float v) {
    float r = roundf(v);
    if (r != r) return 0;
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return (int)r;
}

__device__ __forceinline__ float warp_max_abs(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Quantize one 32-element block held one element per lane into Q8X block
// `blk` (blocks.rs:102-123 numerics).  All 32 lanes must call it.
__device__ __forceinline__ void q8x_store_block(float v, Q8X out, size_t blk, int lane) {
    float amax = warp_max_abs(fabsf(v));
    float d = __fdiv_rn(amax, 127.0f);
    float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    int q = q8_round(__fmul_rn(v, id));
    out.qs[blk * 32 + lane] = (int8_t)q;
    int s = q;
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((lane & 3) == 0) out.c[blk * 8 + (lane >> 2)] = MAGIC_I - 8 * s;
    if (lane == 0) out.d[blk] = __half2float(__float2half_rn(d));
}

// One thread quantizes a whole block: v(i) gives element i of the block
// (i = 0..31; called twice per element), the result lands in Q8X block blk.
// Same bytes as q8x_store_block: amax over |v| (order-free), d = amax/127,
// id = 127/amax (0 for amax == 0), q = clamp(round(v*id)), lane constant k
// from elements 4k..4k+3, f16-rounded d.  The 16-byte groups are visited
// starting at `rot` (0..7) so that threads of a warp working on different
// blocks spread over the shared-memory banks.
template <typename F>
__device__ __forceinline__ void q8x_store_block_thread(F v, Q8X out, size_t blk, int rot) {
    float amax = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const int g = (u + rot) & 7;
#pragma unroll
        for (int e = 0; e < 4; e++) amax = fmaxf(amax, fabsf(v(4 * g + e)));
    }
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const int g = (u + rot) & 7;
        int q[4];
#pragma unroll
        for (int e = 0; e < 4; e++) q[e] = q8_round(__fmul_rn(v(4 * g + e), id));
        const unsigned word = (unsigned)(q[0] & 0xff) | ((unsigned)(q[1] & 0xff) << 8) |
                              ((unsigned)(q[2] & 0xff) << 16) | ((unsigned)(q[3] & 0xff) << 24);
        reinterpret_cast<unsigned *>(out.qs + blk * 32)[g] = word;
        out.c[blk * 8 + g] = MAGIC_I - 8 * (q[0] + q[1] + q[2] + q[3]);
    }
    out.d[blk] = __half2float(__float2half_rn(d));
}

}  // namespace slm
