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
constexpr int FUSED_STAGES = 4;
constexpr size_t FUSED_SMEM_MAX = 200 * 1024;

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
    // the whole K row (up to 64 floats per pass) is loaded before the dot
    // chains start, so a thread has all its loads in flight at once
    float dot[8];
    for (int h = 0; h < kv_mul; h += 8) {
        const int nh = kv_mul - h < 8 ? kv_mul - h : 8;
#pragma unroll
        for (int u = 0; u < 8; u++) dot[u] = 0.0f;
        for (int i0 = 0; i0 < hd; i0 += 64) {
            float k[64];
            const int ni = hd - i0 < 64 ? hd - i0 : 64;
            if ((hd & 3) == 0) {
#pragma unroll
                for (int v = 0; v < 16; v++) {
                    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (4 * v < ni) f = __ldg(reinterpret_cast<const float4 *>(kt + i0) + v);
                    k[4 * v] = f.x;
                    k[4 * v + 1] = f.y;
                    k[4 * v + 2] = f.z;
                    k[4 * v + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int v = 0; v < 64; v++) k[v] = v < ni ? kt[i0 + v] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                if (u < nh) {
                    const float *qh = s_q + (h + u) * hd + i0;
#pragma unroll
                    for (int v = 0; v < 64; v++)
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
    // 32 independent loads of V (and of p) in flight per thread before the
    // 32 dependent adds of the chain consume them
    constexpr int U = 32;
    float acc = 0.0f;
    int t = 0;
    for (; t + U <= L; t += U) {
        float pv[U], vv[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            pv[u] = __ldg(p + t + u);
            vv[u] = __ldg(vt + (size_t)(t + u) * ld);
        }
#pragma unroll
        for (int u = 0; u < U; u++) acc = __fadd_rn(acc, __fmul_rn(pv[u], vv[u]));
    }
    for (; t < L; t++) acc = __fadd_rn(acc, __fmul_rn(__ldg(p + t), __ldg(vt + (size_t)t * ld)));
    a.out[(size_t)r * a.ldo + (size_t)head * a.head_dim + i] = acc;
}


// ---------------------------------------------------------------------------
// Fused attention: one CTA per (row, KV head).  K and then V rows of the KV
// head stream through a multi-stage cp.async shared-memory ring (rows padded
// to hd+4 floats, so the 16-byte reads of 8 consecutive rows by a
// quarter-warp hit 8 different bank groups); the scores of the kv_mul query
// heads stay in shared memory; the softmax runs between the two streams while
// the first V tiles are already in flight.  Chains and orders are those of
// the three-kernel path above, so results are identical.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gsrc));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

struct FusedShape {
    int tt;      // key rows per stage
    int lp;      // scores row stride (floats)
    int rs;      // ring row stride (floats)
    size_t smem; // bytes
};

__host__ __device__ inline FusedShape fused_shape(int kv_mul, int hd, int max_len, int tt) {
    FusedShape f;
    f.tt = tt;
    f.lp = (max_len + 31) / 32 * 32 + 4;
    f.rs = hd + 4;
    f.smem = sizeof(float) * ((size_t)kv_mul * f.lp + (size_t)FUSED_STAGES * tt * f.rs +
                              (size_t)kv_mul * hd + 64);
    return f;
}

// Copy `nrows` rows of hd floats (global stride ld floats) into shared
// memory rows of stride rs with 16-byte cp.async, all threads of the CTA.
// When the thread count is a multiple of the 16-byte chunks per row, each
// thread keeps its column and walks rows without any division.
__device__ __forceinline__ void stage_rows(float *dst, int rs, const float *src, size_t ld,
                                           int nrows, int cpr, int tid, int nth) {
    if (nth % cpr == 0) {
        const int rstep = nth / cpr;
        const int cc = tid % cpr;
        for (int rr = tid / cpr; rr < nrows; rr += rstep)
            cp_async16(dst + rr * rs + cc * 4, src + (size_t)rr * ld + cc * 4);
    } else {
        for (int c = tid; c < nrows * cpr; c += nth) {
            const int rr = c / cpr, cc = c - rr * cpr;
            cp_async16(dst + rr * rs + cc * 4, src + (size_t)rr * ld + cc * 4);
        }
    }
}

// (A) scores: one CTA per (128 keys, KV head, row).  The 128 K rows are
// copied with coalesced 16-byte cp.async into shared memory (rows padded to
// hd+4 floats); thread t then runs the kv_mul query-head dot chains of key t
// side by side (kv_mul-way ILP), each chain sequential in i.
constexpr int TILE_KEYS = 128;

__global__ void __launch_bounds__(TILE_KEYS) attn_scores_tiled_kernel(AttnArgs a) {
    extern __shared__ __align__(16) float smem[];
    const int r = blockIdx.z, g = blockIdx.y;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    const int hd = a.head_dim, rs = hd + 4, cpr = hd >> 2;
    const int L = row_len(a, r);
    const int t0 = blockIdx.x * TILE_KEYS;
    if (t0 >= L) return;  // CTA-uniform
    const int nrows = L - t0 < TILE_KEYS ? L - t0 : TILE_KEYS;
    float *s_k = smem;                          // [TILE_KEYS][rs]
    float *s_q = smem + TILE_KEYS * rs;         // [kv_mul][hd]
    const float *kb = a.k_base + row_slot(a, r) * a.slot_stride + a.layer_off +
                      (size_t)t0 * a.kv_dim + (size_t)g * hd;
    stage_rows(s_k, rs, kb, (size_t)a.kv_dim, nrows, cpr, threadIdx.x, TILE_KEYS);
    cp_async_commit();
    const float *qr = a.q + (size_t)r * a.ldq + (size_t)g * kv_mul * hd;
    for (int i = threadIdx.x; i < kv_mul * hd; i += TILE_KEYS) s_q[i] = qr[i];
    cp_async_wait<0>();
    __syncthreads();
    const int t = threadIdx.x;
    if (t >= nrows) return;
    const float4 *k4 = reinterpret_cast<const float4 *>(s_k + t * rs);
    float *att = a.att + ((size_t)r * a.num_heads + (size_t)g * kv_mul) * a.att_ld + t0 + t;
    for (int h0 = 0; h0 < kv_mul; h0 += 4) {
        const int nh = kv_mul - h0 < 4 ? kv_mul - h0 : 4;
        float dot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float4 *q4 = reinterpret_cast<const float4 *>(s_q + h0 * hd);
        for (int v = 0; v < cpr; v++) {
            const float4 kk = k4[v];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (u < nh) {
                    const float4 qq = q4[u * cpr + v];
                    dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.x, kk.x));
                    dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.y, kk.y));
                    dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.z, kk.z));
                    dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.w, kk.w));
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (u < nh) att[(size_t)(h0 + u) * a.att_ld] = __fmul_rn(dot[u], a.scale);
    }
}

// (B) softmax + PV: one CTA per (row, KV head).  The first V tiles are put
// in flight through a multi-stage cp.async ring (rows padded to hd+4 floats)
// before anything else; meanwhile the kv_mul score rows come from the scores
// kernel's output into shared memory and the softmax runs there; then the PV
// chains consume the V tiles, two dims per thread (two independent chains).
// When q8_out is given, the output block that this CTA owns is quantized for
// the Wo GEMV in the same kernel.
__global__ void __launch_bounds__(1024) attn_softmax_pv_kernel(AttnArgs a, int tt, int lp) {
    extern __shared__ __align__(16) float smem[];
    const int g = blockIdx.x, r = blockIdx.y;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    const int hd = a.head_dim, rs = hd + 4;
    const int tid = threadIdx.x, nth = blockDim.x;
    float *s_sc = smem;                          // [kv_mul][lp]
    float *s_ring = s_sc + (size_t)kv_mul * lp;  // [STAGES][tt][rs]
    float *s_out = s_ring + (size_t)FUSED_STAGES * tt * rs;  // [kv_mul*hd]
    float *s_red = s_out + (size_t)kv_mul * hd;  // 64 floats
    const int L = row_len(a, r);
    const int ntiles = (L + tt - 1) / tt;
    const float *vb = a.v_base + row_slot(a, r) * a.slot_stride + a.layer_off + (size_t)g * hd;
    const size_t ld = (size_t)a.kv_dim;
    const int cpr = hd >> 2;

    auto issue = [&](int tile) {
        if (tile < ntiles) {
            const int t0 = tile * tt;
            const int nrows = L - t0 < tt ? L - t0 : tt;
            stage_rows(s_ring + (size_t)(tile % FUSED_STAGES) * tt * rs, rs, vb + (size_t)t0 * ld,
                       ld, nrows, cpr, tid, nth);
        }
        cp_async_commit();
    };
#pragma unroll 1
    for (int s = 0; s < FUSED_STAGES - 1; s++) issue(s);

    // scores of the kv_mul heads of this group
    const float *att = a.att + ((size_t)r * a.num_heads + (size_t)g * kv_mul) * a.att_ld;
    for (int h = 0; h < kv_mul; h++)
        for (int t = tid; t < L; t += nth) s_sc[h * lp + t] = att[(size_t)h * a.att_ld + t];
    __syncthreads();

    // ---- softmax per query head (graph.rs:168-179 order)
    const int warp = tid >> 5, lane = tid & 31, nw = nth >> 5;
    for (int h = 0; h < kv_mul; h++) {
        float m = -INFINITY;
        for (int t = tid; t < L; t += nth) m = cl_fmax(m, s_sc[h * lp + t]);
        for (int o = 16; o > 0; o >>= 1) m = cl_fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_red[warp] = m;
        __syncthreads();
        if (tid == 0) {
            float mm = s_red[0];
            for (int w = 1; w < nw; w++) mm = cl_fmax(mm, s_red[w]);
            s_red[32 + h] = mm;
        }
        __syncthreads();
    }
    for (int h = 0; h < kv_mul; h++) {
        const float mx = s_red[32 + h];
        for (int t = tid; t < L; t += nth)
            s_sc[h * lp + t] = exp_poly(__fsub_rn(s_sc[h * lp + t], mx));
    }
    __syncthreads();
    const int vl = L & ~3;
    if (tid < 4 * kv_mul) {
        const int h = tid >> 2, l = tid & 3;
        const float *e = s_sc + h * lp;
        float acc = 0.0f;
        int i = l;
        for (; i + 28 < vl; i += 32) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = e[i + 4 * u];
#pragma unroll
            for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, v[u]);
        }
        for (; i < vl; i += 4) acc = __fadd_rn(acc, e[i]);
        s_red[tid] = acc;  // [0, 4*kv_mul) with kv_mul <= 8 stays below 32
    }
    __syncthreads();
    if (tid < kv_mul) {
        const float *e = s_sc + tid * lp;
        float sum = __fadd_rn(__fadd_rn(s_red[4 * tid], s_red[4 * tid + 1]),
                              __fadd_rn(s_red[4 * tid + 2], s_red[4 * tid + 3]));
        for (int i = vl; i < L; i++) sum = __fadd_rn(sum, e[i]);
        s_red[48 + tid] = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    for (int h = 0; h < kv_mul; h++) {
        const float inv = s_red[48 + h];
        float *prow = a.write_probs
                          ? a.att + ((size_t)r * a.num_heads + g * kv_mul + h) * a.att_ld
                          : nullptr;
        for (int t = tid; t < L; t += nth) {
            const float pr = __fmul_rn(s_sc[h * lp + t], inv);
            s_sc[h * lp + t] = pr;
            if (prow) prow[t] = pr;
        }
    }

    // ---- out = sum_t p_t * v_t (sequential in t from 0.0); thread = (head,
    // pair of dims): two independent chains
    const int half = hd >> 1;
    const int hl = tid / half, i2 = tid - (tid / half) * half;
    const bool active = tid < kv_mul * half;
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 1
    for (int tile = 0; tile < ntiles; tile++) {
        cp_async_wait<FUSED_STAGES - 2>();
        __syncthreads();
        issue(tile + FUSED_STAGES - 1);
        if (active) {
            const float *vt = s_ring + (size_t)(tile % FUSED_STAGES) * tt * rs + 2 * i2;
            const float *pp = s_sc + hl * lp + tile * tt;
            const int t0 = tile * tt;
            const int nrows = L - t0 < tt ? L - t0 : tt;
            int tl = 0;
            for (; tl + 4 <= nrows; tl += 4) {
                const float4 p4 = *reinterpret_cast<const float4 *>(pp + tl);
                const float2 v0 = *reinterpret_cast<const float2 *>(vt + (tl + 0) * rs);
                const float2 v1 = *reinterpret_cast<const float2 *>(vt + (tl + 1) * rs);
                const float2 v2 = *reinterpret_cast<const float2 *>(vt + (tl + 2) * rs);
                const float2 v3 = *reinterpret_cast<const float2 *>(vt + (tl + 3) * rs);
                acc0 = __fadd_rn(acc0, __fmul_rn(p4.x, v0.x));
                acc1 = __fadd_rn(acc1, __fmul_rn(p4.x, v0.y));
                acc0 = __fadd_rn(acc0, __fmul_rn(p4.y, v1.x));
                acc1 = __fadd_rn(acc1, __fmul_rn(p4.y, v1.y));
                acc0 = __fadd_rn(acc0, __fmul_rn(p4.z, v2.x));
                acc1 = __fadd_rn(acc1, __fmul_rn(p4.z, v2.y));
                acc0 = __fadd_rn(acc0, __fmul_rn(p4.w, v3.x));
                acc1 = __fadd_rn(acc1, __fmul_rn(p4.w, v3.y));
            }
            for (; tl < nrows; tl++) {
                const float2 vv = *reinterpret_cast<const float2 *>(vt + tl * rs);
                acc0 = __fadd_rn(acc0, __fmul_rn(pp[tl], vv.x));
                acc1 = __fadd_rn(acc1, __fmul_rn(pp[tl], vv.y));
            }
        }
    }
    cp_async_wait<0>();
    if (active) {
        s_out[hl * hd + 2 * i2] = acc0;
        s_out[hl * hd + 2 * i2 + 1] = acc1;
    }
    __syncthreads();
    float *orow = a.out + (size_t)r * a.ldo + (size_t)g * kv_mul * hd;
    for (int k = tid; k < kv_mul * hd; k += nth) orow[k] = s_out[k];
    // Q8_0 of the attention output for the Wo GEMV: this CTA owns the
    // kv_mul*hd consecutive dims from g*kv_mul*hd, one 32-element block per
    // warp when kv_mul*hd is a multiple of 32 (checked by the host)
    if (a.q8_out.qs) {
        const int nbr = a.dim / 32;
        for (int blk = warp; blk < (kv_mul * hd) / 32; blk += nw)
            q8x_store_block(s_out[blk * 32 + lane], a.q8_out,
                            (size_t)r * nbr + (size_t)(g * kv_mul * hd) / 32 + blk, lane);
    }
}

}  // namespace

bool attention_fused_ok(const AttnArgs &a) {
    const int kv_mul = a.num_heads / a.num_kv_heads;
    if (a.head_dim % 4 || kv_mul > 8 || kv_mul * a.head_dim > 1024) return false;
    if (((uintptr_t)a.k_base | (uintptr_t)a.v_base) & 15) return false;
    if (!a.att) return false;  // the scores go through att
    if ((a.slot_stride | a.layer_off) & 3) return false;
    return fused_shape(kv_mul, a.head_dim, a.max_len, 64).smem <= FUSED_SMEM_MAX ||
           fused_shape(kv_mul, a.head_dim, a.max_len, 16).smem <= FUSED_SMEM_MAX;
}

void launch_attn_fused(const AttnArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    const size_t sk = sizeof(float) * ((size_t)TILE_KEYS * (a.head_dim + 4) + (size_t)kv_mul * a.head_dim);
    dim3 g1((a.max_len + TILE_KEYS - 1) / TILE_KEYS, a.num_kv_heads, a.rows);
    attn_scores_tiled_kernel<<<g1, TILE_KEYS, sk, s>>>(a);
    int tt = 64;
    FusedShape f = fused_shape(kv_mul, a.head_dim, a.max_len, tt);
    while (f.smem > FUSED_SMEM_MAX && tt > 16) {
        tt >>= 1;
        f = fused_shape(kv_mul, a.head_dim, a.max_len, tt);
    }
    int nth = (kv_mul * (a.head_dim / 2) + 31) / 32 * 32;
    nth = nth < 256 ? 256 : nth;
    dim3 grid(a.num_kv_heads, a.rows);
    attn_softmax_pv_kernel<<<grid, nth, f.smem, s>>>(a, tt, f.lp);
}

void set_attention_smem_limit(int bytes) {
    cudaFuncSetAttribute(attn_softmax_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_scores_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
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
    if (attention_fused_ok(a)) {
        launch_attn_fused(a, s);
        return;
    }
    launch_attn_scores(a, s);
    launch_attn_softmax(a, s);
    launch_attn_pv(a, s);
}

}  // namespace slm
