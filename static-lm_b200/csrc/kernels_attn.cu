// kernels_attn.cu -- causal GQA attention with the reference's f32 numerics
// (causal_multi_head_attention_jit, src/model/transformer.rs:273-321).
//
// For query row r at position p (L = p+1 keys) and head h with KV head
// h / kv_mul:
//   score_t = (sum_i q_i*k_t,i, sequential in i, mul and add rounded
//              separately) * (1/sqrt(hd))                      t = 0..p
//   softmax over the L scores with the Cranelift-lowered order: max; four
//   lane sums of exp_poly(s - max), (l0+l1)+(l2+l3), sequential tail; times
//   1/sum                                          (graph.rs:168-179)
//   out_i = sum_t p_t*v_t,i, sequential in t starting from 0.0
//
// The only freedom the numerics leave is which thread runs which chain, so
// the work is split into three launches that each expose the parallelism of
// their phase:
//   scores : one thread per (row, key position), kv_mul query heads per
//            thread so every K row is loaded once per KV head group
//   softmax: one CTA per (row, head); max in parallel, exp in parallel, the
//            four lane chains on four threads over a shared-memory copy
//   pv     : one thread per (row, head, dim) chain over t; a warp covers 32
//            consecutive dims so each V row segment is one coalesced load
// Decode is the case of one row per sequence; prefill is rows = tokens with
// p = start_pos + i, which reproduces the reference's per-token loop
// (transformer.rs:563-593) exactly.
#include "kernels.h"

namespace slm {

namespace {

constexpr int SCORE_T = 128;  // key positions per scores CTA

// keys attended by row r: pos+1, never beyond the cache nor the launch's
// max_len (which sizes the grid and the softmax's shared memory)
__device__ __forceinline__ int row_len(const AttnArgs &a, int r) {
    int p = a.pos ? a.pos[r] : a.pos_const;
    int L = p + 1;
    L = L < a.max_seq ? L : a.max_seq;
    return L < a.max_len ? L : a.max_len;
}
__device__ __forceinline__ size_t row_slot(const AttnArgs &a, int r) {
    return a.slot ? (size_t)a.slot[r] : 0;
}

__global__ void __launch_bounds__(SCORE_T) attn_scores_kernel(AttnArgs a) {
    extern __shared__ float s_q[];  // [kv_mul][head_dim]
    const int r = blockIdx.z, g = blockIdx.y;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    const int hd = a.head_dim;
    const float *qr = a.q + (size_t)r * a.ldq + (size_t)g * kv_mul * hd;
    for (int i = threadIdx.x; i < kv_mul * hd; i += blockDim.x) s_q[i] = qr[i];
    __syncthreads();
    const int L = row_len(a, r);
    const int t = blockIdx.x * SCORE_T + threadIdx.x;
    if (t >= L) return;
    const float *kt = a.k_base + row_slot(a, r) * a.slot_stride + a.layer_off +
                      (size_t)t * a.kv_dim + (size_t)g * hd;
    float dot[8];
    for (int h = 0; h < kv_mul; h += 8) {
        const int nh = kv_mul - h < 8 ? kv_mul - h : 8;
#pragma unroll
        for (int u = 0; u < 8; u++) dot[u] = 0.0f;
        for (int i0 = 0; i0 < hd; i0 += 16) {
            float k[16];
            const int ni = hd - i0 < 16 ? hd - i0 : 16;
            if (ni == 16 && (hd & 3) == 0) {
#pragma unroll
                for (int v = 0; v < 4; v++) {
                    float4 f = __ldg(reinterpret_cast<const float4 *>(kt + i0) + v);
                    k[4 * v] = f.x;
                    k[4 * v + 1] = f.y;
                    k[4 * v + 2] = f.z;
                    k[4 * v + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int v = 0; v < 16; v++) k[v] = v < ni ? kt[i0 + v] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                if (u < nh) {
                    const float *qh = s_q + (h + u) * hd + i0;
#pragma unroll
                    for (int v = 0; v < 16; v++)
                        if (v < ni) dot[u] = __fadd_rn(dot[u], __fmul_rn(qh[v], k[v]));
                }
            }
        }
        for (int u = 0; u < nh; u++) {
            const int head = g * kv_mul + h + u;
            a.att[((size_t)r * a.num_heads + head) * a.att_ld + t] = __fmul_rn(dot[u], a.scale);
        }
    }
}

__global__ void __launch_bounds__(256) attn_softmax_kernel(AttnArgs a) {
    extern __shared__ float s_e[];  // [L]
    __shared__ float sh[40];
    const int r = blockIdx.y, h = blockIdx.x;
    const int L = row_len(a, r);
    float *row = a.att + ((size_t)r * a.num_heads + h) * a.att_ld;
    // max: order-free
    float m = -INFINITY;
    for (int i = threadIdx.x; i < L; i += blockDim.x) m = cl_fmax(m, row[i]);
    for (int o = 16; o > 0; o >>= 1) m = cl_fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sh[warp] = m;
    __syncthreads();
    if (warp == 0) {
        m = lane < (int)(blockDim.x >> 5) ? sh[lane] : -INFINITY;
        for (int o = 16; o > 0; o >>= 1) m = cl_fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) sh[32] = m;
    }
    __syncthreads();
    const float mx = sh[32];
    for (int i = threadIdx.x; i < L; i += blockDim.x) s_e[i] = exp_poly(__fsub_rn(row[i], mx));
    __syncthreads();
    // four lane chains over [0, L & ~3), then the combine and the tail
    const int vl = L & ~3;
    if (threadIdx.x < 4) {
        float acc = 0.0f;
        int i = threadIdx.x;
        for (; i + 28 < vl; i += 32) {
            float e0 = s_e[i], e1 = s_e[i + 4], e2 = s_e[i + 8], e3 = s_e[i + 12];
            float e4 = s_e[i + 16], e5 = s_e[i + 20], e6 = s_e[i + 24], e7 = s_e[i + 28];
            acc = __fadd_rn(acc, e0);
            acc = __fadd_rn(acc, e1);
            acc = __fadd_rn(acc, e2);
            acc = __fadd_rn(acc, e3);
            acc = __fadd_rn(acc, e4);
            acc = __fadd_rn(acc, e5);
            acc = __fadd_rn(acc, e6);
            acc = __fadd_rn(acc, e7);
        }
        for (; i < vl; i += 4) acc = __fadd_rn(acc, s_e[i]);
        sh[33 + threadIdx.x] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = __fadd_rn(__fadd_rn(sh[33], sh[34]), __fadd_rn(sh[35], sh[36]));
        for (int i = vl; i < L; i++) s = __fadd_rn(s, s_e[i]);
        sh[37] = __fdiv_rn(1.0f, s);
    }
    __syncthreads();
    const float inv = sh[37];
    for (int i = threadIdx.x; i < L; i += blockDim.x) row[i] = __fmul_rn(s_e[i], inv);
}

__global__ void __launch_bounds__(1024) attn_pv_kernel(AttnArgs a) {
    const int r = blockIdx.z, g = blockIdx.y;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    const int hl = threadIdx.x >> 5;
    const int i = blockIdx.x * 32 + (threadIdx.x & 31);
    if (hl >= kv_mul || i >= a.head_dim) return;
    const int head = g * kv_mul + hl;
    const int L = row_len(a, r);
    const float *p = a.att + ((size_t)r * a.num_heads + head) * a.att_ld;
    const float *vt = a.v_base + row_slot(a, r) * a.slot_stride + a.layer_off +
                      (size_t)g * a.head_dim + i;
    const size_t ld = (size_t)a.kv_dim;
    float acc = 0.0f;
    int t = 0;
    for (; t + 8 <= L; t += 8) {
        float pv[8], vv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            pv[u] = p[t + u];
            vv[u] = __ldg(vt + (size_t)(t + u) * ld);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, __fmul_rn(pv[u], vv[u]));
    }
    for (; t < L; t++) acc = __fadd_rn(acc, __fmul_rn(p[t], __ldg(vt + (size_t)t * ld)));
    a.out[(size_t)r * a.ldo + (size_t)head * a.head_dim + i] = acc;
}

}  // namespace

void set_attention_smem_limit(int bytes) {
    cudaFuncSetAttribute(attn_softmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

void launch_attn_scores(const AttnArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    dim3 g((a.max_len + SCORE_T - 1) / SCORE_T, a.num_kv_heads, a.rows);
    attn_scores_kernel<<<g, SCORE_T, sizeof(float) * kv_mul * a.head_dim, s>>>(a);
}

void launch_attn_softmax(const AttnArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return;
    dim3 g(a.num_heads, a.rows);
    attn_softmax_kernel<<<g, 256, sizeof(float) * a.max_len, s>>>(a);
}

void launch_attn_pv(const AttnArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    dim3 g((a.head_dim + 31) / 32, a.num_kv_heads, a.rows);
    attn_pv_kernel<<<g, 32 * kv_mul, 0, s>>>(a);
}

void launch_attention(const AttnArgs &a, cudaStream_t s) {
    launch_attn_scores(a, s);
    launch_attn_softmax(a, s);
    launch_attn_pv(a, s);
}

}  // namespace slm
