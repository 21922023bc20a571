// kernels_vec.cu -- RMSNorm+Q8 quantize, Q8 quantizers, embedding lookup,
// argmax and the standalone equivalents of the JIT vector ops.
//
// Reductions follow the order of the Cranelift lowering the reference runs
// (src/jit/lower.rs:252-389): four lane accumulators over [0, len & ~3)
// where lane l sees elements l, l+4, l+8, ..., then (l0+l1)+(l2+l3), then a
// sequential tail.  These are serial chains by construction; the kernels
// keep them on four threads and parallelise everything around them.
#include <float.h>
#include <limits.h>

#include "async.cuh"
#include "kernels.h"

namespace slm {

namespace {

constexpr unsigned FULL = 0xffffffffu;

// One CTA (8 warps) per row: the row and the weights are staged in shared
// memory with coalesced loads; lanes 0..3 of warp 0 run the four
// sum-of-squares chains; rms = 1/sqrt(sum(x^2) * (1/n) + eps); then the
// warps share the 32-element blocks of y = (x*rms)*w, each quantized to Q8X.
constexpr int NORM_THREADS = 256;

__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_q8_kernel(
    const float *__restrict__ x, size_t ldx, const float *__restrict__ w, int n, float eps,
    float inv_n, float *__restrict__ y, size_t ldy, Q8X q8, int rows, int do_q8) {
    extern __shared__ __align__(16) float s_x[];  // [n] row, then [n] weights
    __shared__ float s_rms;
    float *s_w = s_x + ((n + 3) & ~3);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = blockIdx.x;
    if (r >= rows) return;
    const float *xr = x + (size_t)r * ldx;
    pdl_wait();  // x is the previous kernel's output (no-op without programmatic launch)
    if ((n & 3) == 0 && (((uintptr_t)xr | (uintptr_t)w) & 15) == 0) {
        for (int i = tid; i < n / 4; i += NORM_THREADS) {
            reinterpret_cast<float4 *>(s_x)[i] = __ldg(reinterpret_cast<const float4 *>(xr) + i);
            reinterpret_cast<float4 *>(s_w)[i] = __ldg(reinterpret_cast<const float4 *>(w) + i);
        }
    } else {
        for (int i = tid; i < n; i += NORM_THREADS) {
            s_x[i] = xr[i];
            s_w[i] = w[i];
        }
    }
    __syncthreads();
    if (warp == 0) {
        const int vl = n & ~3;
        float acc = 0.0f;
        if (lane < 4) {
            int i = lane;
            for (; i + 28 < vl; i += 32) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; u++) v[u] = s_x[i + 4 * u];
#pragma unroll
                for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, __fmul_rn(v[u], v[u]));
            }
            for (; i < vl; i += 4) acc = __fadd_rn(acc, __fmul_rn(s_x[i], s_x[i]));
        }
        float a1 = __shfl_sync(FULL, acc, 1);
        float a2 = __shfl_sync(FULL, acc, 2);
        float a3 = __shfl_sync(FULL, acc, 3);
        if (lane == 0) {
            float sum = __fadd_rn(__fadd_rn(acc, a1), __fadd_rn(a2, a3));
            for (int i = vl; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(s_x[i], s_x[i]));
            float mean = __fmul_rn(sum, inv_n);
            float var = __fadd_rn(mean, eps);
            s_rms = __fdiv_rn(1.0f, __fsqrt_rn(var));
        }
    }
    __syncthreads();
    const float rms = s_rms;
    const int nb = n >> 5;
    for (int j = warp; j < nb; j += NORM_THREADS / 32) {
        const int i = j * 32 + lane;
        const float o = __fmul_rn(__fmul_rn(s_x[i], rms), s_w[i]);
        if (y) y[(size_t)r * ldy + i] = o;
        if (do_q8) q8x_store_block(o, q8, (size_t)r * nb + j, lane);
    }
    for (int i = nb * 32 + tid; i < n; i += NORM_THREADS)
        if (y) y[(size_t)r * ldy + i] = __fmul_rn(__fmul_rn(s_x[i], rms), s_w[i]);
}

// One warp per (row, block).
__global__ void quantize_q8x_kernel(const float *__restrict__ x, size_t ldx, int nb, Q8X q8,
                                    int rows) {
    size_t gw = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (gw >= (size_t)rows * nb) return;
    size_t r = gw / nb, j = gw % nb;
    q8x_store_block(x[r * ldx + j * 32 + lane], q8, gw, lane);
}

// One warp per block, reference 34-byte BlockQ8_0 output (blocks.rs:102-123).
__global__ void quantize_q8_ref_kernel(const float *__restrict__ x, uint8_t *__restrict__ dst,
                                       size_t nblocks) {
    size_t b = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (b >= nblocks) return;
    float v = x[b * 32 + lane];
    float amax = warp_max_abs(fabsf(v));
    float d = __fdiv_rn(amax, 127.0f);
    float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    int q = q8_round(__fmul_rn(v, id));
    uint8_t *blk = dst + b * 34;
    blk[2 + lane] = (uint8_t)(int8_t)q;
    if (lane == 0) *(unsigned short *)blk = __half_as_ushort(__float2half_rn(d));
}

__global__ void q8_ref_to_q8x_kernel(const uint8_t *__restrict__ src, Q8X q8, size_t nblocks) {
    size_t b = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (b >= nblocks) return;
    const uint8_t *blk = src + b * 34;
    int a = (int)(int8_t)blk[2 + lane];
    a = a < -127 ? -127 : a;
    q8.qs[b * 32 + lane] = (int8_t)a;
    int s = a;
    s += __shfl_xor_sync(FULL, s, 1);
    s += __shfl_xor_sync(FULL, s, 2);
    if ((lane & 3) == 0) q8.c[b * 8 + (lane >> 2)] = MAGIC_I - 8 * s;
    if (lane == 0) q8.d[b] = __half2float(__ushort_as_half(*(const unsigned short *)blk));
}

// x[r][e] = (nibble - 8) * d of token_embd row tokens[r] (blocks.rs:85-99).
__global__ void embed_kernel(const uint8_t *__restrict__ tiles, int nb,
                             const int32_t *__restrict__ tokens, int vocab,
                             float *__restrict__ x, size_t ldx, int rows, int32_t *err) {
    int r = blockIdx.y;
    int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows || e >= nb * 32) return;
    int tok = tokens[r];
    if (tok < 0 || tok >= vocab) {
        if (e == 0 && err) atomicExch(err, 1);
        x[(size_t)r * ldx + e] = 0.0f;
        return;
    }
    int j = e >> 5, m = e & 31;
    const uint8_t *t = tiles + tile_offset((size_t)tok / TILE_ROWS, nb, j);
    int lane = tok % TILE_ROWS;
    uint8_t byte = t[lane * 16 + (m & 15)];
    int q = (m < 16 ? (byte & 0x0F) : (byte >> 4)) - 8;
    float d = __half2float(__ushort_as_half(*(const unsigned short *)(t + 512 + lane * 2)));
    x[(size_t)r * ldx + e] = __fmul_rn((float)q, d);
}

__global__ void argmax_kernel(const float *__restrict__ logits, size_t ld, int n,
                              int32_t *__restrict__ out) {
    const float *l = logits + (size_t)blockIdx.x * ld;
    float best = -FLT_MAX;
    int idx = INT_MAX;
    bool init = false;
    // eight independent loads in flight per thread, then compared in index order
    constexpr int U = 8;
    const int step = (int)blockDim.x;
    int i0 = threadIdx.x;
    for (; i0 + (U - 1) * step < n; i0 += U * step) {
        float v[U];
#pragma unroll
        for (int u = 0; u < U; u++) v[u] = l[i0 + u * step];
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (v[u] != v[u]) continue;
            if (!init || v[u] > best) {
                best = v[u];
                idx = i0 + u * step;
                init = true;
            }
        }
    }
    for (int i = i0; i < n; i += step) {
        float v = l[i];
        if (v != v) continue;
        if (!init || v > best) {
            best = v;
            idx = i;
            init = true;
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(FULL, best, o);
        int oi = __shfl_xor_sync(FULL, idx, o);
        if (oi != INT_MAX && (idx == INT_MAX || ov > best || (ov == best && oi < idx))) {
            best = ov;
            idx = oi;
        }
    }
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
        int nw = blockDim.x >> 5;
        best = lane < nw ? sv[lane] : -FLT_MAX;
        idx = lane < nw ? si[lane] : INT_MAX;
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(FULL, best, o);
            int oi = __shfl_xor_sync(FULL, idx, o);
            if (oi != INT_MAX && (idx == INT_MAX || ov > best || (ov == best && oi < idx))) {
                best = ov;
                idx = oi;
            }
        }
        if (lane == 0) {
            float l0 = l[0];
            // logits[0] NaN: the reference's strict `>` never moves off index 0
            out[blockIdx.x] = (l0 != l0 || idx == INT_MAX) ? 0 : idx;
        }
    }
}

// ---- standalone JIT-op equivalents (one CTA, any length)

__device__ float block_max_cl(float v, float *sh) {
    for (int o = 16; o > 0; o >>= 1) v = cl_fmax(v, __shfl_xor_sync(FULL, v, o));
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    if (warp == 0) {
        int nw = blockDim.x >> 5;
        v = lane < nw ? sh[lane] : -INFINITY;
        for (int o = 16; o > 0; o >>= 1) v = cl_fmax(v, __shfl_xor_sync(FULL, v, o));
        if (lane == 0) sh[0] = v;
    }
    __syncthreads();
    float r = sh[0];
    __syncthreads();
    return r;
}

// Lane-ordered sum of v[0..len) by threads 0..3; result broadcast through sh.
__device__ float block_lane4_sum(const float *v, size_t len, float *sh) {
    size_t vl = len & ~(size_t)3;
    if (threadIdx.x < 4) {
        float acc = 0.0f;
        for (size_t i = threadIdx.x; i < vl; i += 4) acc = __fadd_rn(acc, v[i]);
        sh[threadIdx.x] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = __fadd_rn(__fadd_rn(sh[0], sh[1]), __fadd_rn(sh[2], sh[3]));
        for (size_t i = vl; i < len; i++) s = __fadd_rn(s, v[i]);
        sh[4] = s;
    }
    __syncthreads();
    float r = sh[4];
    __syncthreads();
    return r;
}

__device__ float block_lane4_sumsq(const float *x, size_t len, float *sh) {
    size_t vl = len & ~(size_t)3;
    if (threadIdx.x < 4) {
        float acc = 0.0f;
        for (size_t i = threadIdx.x; i < vl; i += 4) acc = __fadd_rn(acc, __fmul_rn(x[i], x[i]));
        sh[threadIdx.x] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = __fadd_rn(__fadd_rn(sh[0], sh[1]), __fadd_rn(sh[2], sh[3]));
        for (size_t i = vl; i < len; i++) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
        sh[4] = s;
    }
    __syncthreads();
    float r = sh[4];
    __syncthreads();
    return r;
}

// graph.rs:168-179; out may alias x
__global__ void softmax_vec_kernel(const float *x, float *out, size_t len) {
    __shared__ float sh[32];
    float m = -INFINITY;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) m = cl_fmax(m, x[i]);
    float mx = block_max_cl(m, sh);
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) out[i] = exp_poly(__fsub_rn(x[i], mx));
    __syncthreads();
    float s = block_lane4_sum(out, len, sh);
    float inv = __fdiv_rn(1.0f, s);
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) out[i] = __fmul_rn(out[i], inv);
}

// graph.rs:141-155 compiled with n = len
__global__ void rmsnorm_vec_kernel(const float *x, const float *w, float *out, size_t len,
                                   float eps, float inv_n) {
    __shared__ float sh[32];
    float s = block_lane4_sumsq(x, len, sh);
    float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(s, inv_n), eps)));
    for (size_t i = threadIdx.x; i < len; i += blockDim.x)
        out[i] = __fmul_rn(__fmul_rn(x[i], rms), w[i]);
}

// graph.rs:182-193
__global__ void l2norm_vec_kernel(const float *x, float *out, size_t len, float eps) {
    __shared__ float sh[32];
    float s = block_lane4_sumsq(x, len, sh);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s, eps)));
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) out[i] = __fmul_rn(x[i], inv);
}

__global__ void swiglu_vec_kernel(const float *g, const float *u, float *out, size_t len) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < len) out[i] = swiglu1(g[i], u[i]);
}

__global__ void residual_vec_kernel(const float *a, const float *b, float *out, size_t len) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < len) out[i] = __fadd_rn(a[i], b[i]);
}

// transformer.rs:178-194; one thread per (head, pair)
__global__ void rope_vec_kernel(float *vec, size_t len, const float *cos_row,
                                const float *sin_row, int head_dim) {
    size_t p = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    int half = head_dim / 2;
    size_t heads = len / (size_t)head_dim;
    if (p >= heads * half) return;
    size_t h = p / half;
    int j = (int)(p % half);
    float *hs = vec + h * head_dim;
    float c = cos_row[j], s = sin_row[j];
    float v0 = hs[2 * j], v1 = hs[2 * j + 1];
    hs[2 * j] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    hs[2 * j + 1] = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
}

__global__ void mean_pool_kernel(const float *y, size_t ldy, int rows, int n, float inv_batch,
                                 float *accum) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float acc = 0.0f;
    for (int b = 0; b < rows; b++) acc = __fadd_rn(acc, __fmul_rn(y[(size_t)b * ldy + i], inv_batch));
    accum[i] = acc;
}

__global__ void advance_kernel(int32_t *tokens, int32_t *pos, const int32_t *next, int rows) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows) return;
    tokens[i] = next[i];
    pos[i] = pos[i] + 1;
}

inline unsigned cdiv(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

}  // namespace

void set_rmsnorm_smem_limit(int bytes) {
    cudaFuncSetAttribute(rmsnorm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

void launch_rmsnorm_q8(const float *x, size_t ldx, const float *w, int n, float eps, float *y,
                       size_t ldy, Q8X q8, int rows, cudaStream_t s, bool pdl) {
    if (rows <= 0) return;
    float inv_n = 1.0f / (float)n;
    size_t smem = sizeof(float) * (2 * (size_t)((n + 3) & ~3));
    launch_kernel(rmsnorm_q8_kernel, dim3(rows), dim3(NORM_THREADS), smem, s, pdl, x, ldx, w, n, eps, inv_n, y,
                  ldy, q8, rows, (int)(q8.qs != nullptr));
}

void launch_quantize_q8x(const float *x, size_t ldx, int n, Q8X q8, int rows, cudaStream_t s) {
    size_t warps = (size_t)rows * (n / 32);
    if (!warps) return;
    quantize_q8x_kernel<<<cdiv(warps, 8), 256, 0, s>>>(x, ldx, n / 32, q8, rows);
}

void launch_quantize_q8_ref(const float *x, void *blocks, size_t n, cudaStream_t s) {
    size_t nb = n / 32;
    if (!nb) return;
    quantize_q8_ref_kernel<<<cdiv(nb, 8), 256, 0, s>>>(x, (uint8_t *)blocks, nb);
}

void launch_q8_ref_to_q8x(const void *blocks, Q8X q8, size_t nblocks, cudaStream_t s) {
    if (!nblocks) return;
    q8_ref_to_q8x_kernel<<<cdiv(nblocks, 8), 256, 0, s>>>((const uint8_t *)blocks, q8, nblocks);
}

void launch_embed(const uint8_t *tiles, int nb, const int32_t *tokens, int vocab, float *x,
                  size_t ldx, int rows, int32_t *err, cudaStream_t s) {
    if (rows <= 0) return;
    dim3 grid(cdiv((size_t)nb * 32, 256), rows);
    embed_kernel<<<grid, 256, 0, s>>>(tiles, nb, tokens, vocab, x, ldx, rows, err);
}

void launch_argmax(const float *logits, size_t ld, int n, int32_t *out, int rows,
                   cudaStream_t s) {
    if (rows <= 0) return;
    argmax_kernel<<<rows, 1024, 0, s>>>(logits, ld, n, out);
}

void launch_softmax_vec(const float *x, float *out, size_t len, cudaStream_t s) {
    if (!len) return;
    softmax_vec_kernel<<<1, 1024, 0, s>>>(x, out, len);
}

void launch_rmsnorm_vec(const float *x, const float *w, float *out, size_t len, float eps,
                        cudaStream_t s) {
    if (!len) return;
    // 1/n as FuseGraph::rmsnorm(n, eps) computes it (graph.rs:147): one IEEE
    // single-precision division, identical on the host
    rmsnorm_vec_kernel<<<1, 1024, 0, s>>>(x, w, out, len, eps, 1.0f / (float)len);
}

void launch_rmsnorm_vec_inv_n(const float *x, const float *w, float *out, size_t len, float eps,
                              float inv_n, cudaStream_t s) {
    if (!len) return;
    rmsnorm_vec_kernel<<<1, 1024, 0, s>>>(x, w, out, len, eps, inv_n);
}

void launch_swiglu_vec(const float *g, const float *u, float *out, size_t len, cudaStream_t s) {
    if (!len) return;
    swiglu_vec_kernel<<<cdiv(len, 256), 256, 0, s>>>(g, u, out, len);
}

void launch_residual_add_vec(const float *a, const float *b, float *out, size_t len,
                             cudaStream_t s) {
    if (!len) return;
    residual_vec_kernel<<<cdiv(len, 256), 256, 0, s>>>(a, b, out, len);
}

void launch_l2norm_vec(const float *x, float *out, size_t len, float eps, cudaStream_t s) {
    if (!len) return;
    l2norm_vec_kernel<<<1, 1024, 0, s>>>(x, out, len, eps);
}

void launch_mean_pool(const float *y, size_t ldy, int rows, int n, float inv_batch,
                      float *accum, cudaStream_t s) {
    if (n <= 0) return;
    mean_pool_kernel<<<cdiv(n, 128), 128, 0, s>>>(y, ldy, rows, n, inv_batch, accum);
}

void launch_advance(int32_t *tokens, int32_t *pos, const int32_t *next, int rows,
                    cudaStream_t s) {
    if (rows <= 0) return;
    advance_kernel<<<cdiv(rows, 128), 128, 0, s>>>(tokens, pos, next, rows);
}

// BlockQ4_0 rows (18 bytes per block, as GgufFile::tensor_q4_0 returns them,
// src/memory/loader.rs:496-500) -> the 576-byte row tiles of common.cuh:
// rows [row0, row0+nrows) of a matrix of nb blocks per row.  One thread per
// (row, block); a block is 2-byte aligned, so it moves as nine 16-bit words.
__global__ void repack_q4_kernel(const uint16_t *raw, uint64_t nrows, int nb, uint64_t row0,
                                 uint8_t *tiles) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nrows * (uint64_t)nb) return;
    const uint64_t r = row0 + i / (uint64_t)nb;
    const int j = (int)(i % (uint64_t)nb);
    const uint16_t *src = raw + i * 9;
    uint8_t *dst = tiles + tile_offset(r / TILE_ROWS, (size_t)nb, (size_t)j);
    const int lane = (int)(r % TILE_ROWS);
    reinterpret_cast<uint16_t *>(dst + 512)[lane] = src[0];
    uint16_t *nib = reinterpret_cast<uint16_t *>(dst + lane * 16);
#pragma unroll
    for (int k = 0; k < 8; k++) nib[k] = src[1 + k];
}

void launch_repack_q4(const void *raw, uint64_t nrows, int nb, uint64_t row0, uint8_t *tiles,
                      cudaStream_t s) {
    const uint64_t n = nrows * (uint64_t)nb;
    if (!n) return;
    repack_q4_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<const uint16_t *>(raw), nrows, nb,
                                                                  row0, tiles);
}

// Self-test of the bounded mbarrier wait every TMA pipeline uses: thread 0
// sets up a barrier that nothing ever arrives on, every thread waits on it
// with the given limit; the first to give up sets the shared abort flag (the
// others then leave at once) and the error flag (3).  Always ends.
__global__ void wait_selftest_kernel(long long limit, int32_t *err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int s_abort;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    mbar_wait_limit(&bar, 0u, &s_abort, err, limit);
}

void launch_wait_selftest(long long limit_cycles, int32_t *err, cudaStream_t s) {
    wait_selftest_kernel<<<1, 64, 0, s>>>(limit_cycles, err);
}

void launch_rope_vec(float *vec, size_t len, const float *cos_row, const float *sin_row,
                     int head_dim, cudaStream_t s) {
    size_t pairs = len / (size_t)head_dim * (size_t)(head_dim / 2);
    if (!pairs) return;
    rope_vec_kernel<<<cdiv(pairs, 256), 256, 0, s>>>(vec, len, cos_row, sin_row, head_dim);
}

}  // namespace slm
