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
// The only freedom the numerics leave is which thread runs which chain.
// Two paths give identical results:
//   fused (two launches): (A) tiled scores, K rows through the TMA engine,
//            one thread per key running the kv_mul head chains; (B) per
//            (row, KV head): softmax in shared memory, then PV with V tiles
//            streamed by a 3-D tensor map into an mbarrier-guarded ring
//   three-phase fallback (any shape):
//   scores : one thread per (row, key position), kv_mul query heads per
//            thread so every K row is loaded once per KV head group
//   softmax: one CTA per (row, head); max in parallel, exp in parallel, the
//            four lane chains on four threads over a shared-memory copy
//   pv     : one thread per (row, head, dim) chain over t; a warp covers 32
//            consecutive dims so each V row segment is one coalesced load
// Packed f32x2 arithmetic is not used: measured on B200 it does not round
// like separate mul.rn / add.rn.
// Decode is the case of one row per sequence; prefill is rows = tokens with
// p = start_pos + i, which reproduces the reference's per-token loop
// (transformer.rs:563-593) exactly.
#include "async.cuh"
#include "attn_rows.cuh"
#include "kernels.h"

namespace slm {

namespace {

constexpr int SCORE_T = 128;  // key positions per scores CTA
constexpr int FUSED_STAGES = 4;
constexpr size_t FUSED_SMEM_MAX = 200 * 1024;

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

// Fused path: V comes through a 3-D tensor map over the cache planes
// (x = kv_dim floats, y = positions, z = plane), one TMA box of TT_V rows x
// head_dim floats per stage.
constexpr int TT_V = V_BOX_POSITIONS;
constexpr int PV_THREADS = 256;

struct FusedShape {
    int tt;      // V rows per stage (one TMA box)
    int lp;      // scores row stride (floats)
    int nst;     // stages of the V ring
    size_t smem; // dynamic shared memory bytes (with 128 B of alignment slack)
};

// Shared memory of a softmax + PV CTA over `hpc` query heads with an
// `nst`-stage V ring.
__host__ __device__ inline FusedShape fused_shape(int hpc, int hd, int max_len, int nst = FUSED_STAGES,
                                                  int tt = TT_V) {
    FusedShape f;
    f.tt = tt;
    f.lp = (max_len + 31) / 32 * 32 + 4;
    f.nst = nst;
    f.smem = sizeof(float) * ((size_t)nst * tt * hd + (size_t)hpc * f.lp +
                              (size_t)hpc * hd + 64 + 8 * 32) +
             128;
    return f;
}
constexpr int PV_MAX_STAGES = 32;
#ifndef SLM_PV_MIN_STAGES
#define SLM_PV_MIN_STAGES 2
#endif
constexpr int PV_MIN_STAGES = SLM_PV_MIN_STAGES;

// (A) scores: one CTA per (128 keys, KV head, row).  The 128 K rows go
// global -> shared through the TMA engine, one bulk copy per row (rows padded
// to hd+4 floats), all completing on one mbarrier; thread t then runs the
// kv_mul query-head dot chains of key t side by side (kv_mul-way ILP), each
// chain sequential in i.
constexpr int TILE_KEYS = K_BOX_KEYS;

__global__ void __launch_bounds__(TILE_KEYS) attn_scores_tiled_kernel(AttnArgs a) {
    extern __shared__ __align__(16) float smem[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ int s_abort;
    const int r = blockIdx.z, g = blockIdx.y;
    if (!unit_owned(a, r, g)) return;  // CTA-uniform
    const int kv_mul = a.num_heads / a.num_kv_heads;
    const int hd = a.head_dim, rs = hd + 4;
    const int L = row_len(a, r);
    const int t0 = blockIdx.x * TILE_KEYS;
    if (t0 >= L) return;  // CTA-uniform
    const int nrows = L - t0 < TILE_KEYS ? L - t0 : TILE_KEYS;
    float *s_k = smem;                          // [TILE_KEYS][rs]
    float *s_q = smem + TILE_KEYS * rs;         // [kv_mul][hd]
    const float *kb = a.k_base + row_slot(a, r) * a.slot_stride + a.layer_off +
                      (size_t)t0 * a.kv_dim + (size_t)g * hd;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    // the K rows of this tile go through the TMA engine, one bulk copy per row
    if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar, (unsigned)nrows * (unsigned)hd * 4u);
    if ((int)threadIdx.x < nrows)
        bulk_copy(s_k + threadIdx.x * rs, kb + (size_t)threadIdx.x * a.kv_dim, (unsigned)hd * 4u, &bar);
    const float *qr = a.q + (size_t)r * a.ldq + (size_t)g * kv_mul * hd;
    for (int i = threadIdx.x; i < kv_mul * hd; i += TILE_KEYS) s_q[i] = qr[i];
    const bool ok = mbar_wait(&bar, 0, &s_abort, a.err);
    __syncthreads();
    if (!ok || s_abort) {
        // bounded drain of the copies in flight before the shared memory goes away
        if (threadIdx.x == 0) {
            const long long tw = clock64();
            while (!mbar_test(&bar, 0) && clock64() - tw < WAIT_LIMIT) {
            }
        }
        __syncthreads();
        return;
    }
    const int cpr = hd >> 2;
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

// (A') scores with K through a tensor map: the same CTA shape and chains as
// (A), but the 128 K rows x head_dim floats arrive as head_dim/32 TMA boxes of
// [128 rows][32 floats] in the 128-byte swizzled layout (16-byte chunk c of
// row t stored at chunk c ^ (t & 7)), one instruction per box instead of one
// bulk copy per row.  Thread t reads its row's chunks through the same XOR,
// so the eight rows of a quarter-warp hit eight different bank groups.
__global__ void __launch_bounds__(TILE_KEYS)
    attn_scores_tma_kernel(AttnArgs a, const __grid_constant__ CUtensorMap kmap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ int s_abort;
    // swizzled TMA destinations must be 1024-byte aligned (1 KB of slack)
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int r = blockIdx.z, g = blockIdx.y;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    const int hd = a.head_dim, nbox = hd >> 5;
    const int L = row_len(a, r);
    const int t0 = blockIdx.x * TILE_KEYS;
    if (t0 >= L) return;  // CTA-uniform
    const int nrows = L - t0 < TILE_KEYS ? L - t0 : TILE_KEYS;
    const unsigned char *s_k = base;                                          // [nbox][128][128 B]
    float *s_q = reinterpret_cast<float *>(base + (size_t)nbox * TILE_KEYS * 128);  // [kv_mul][hd]
    const int kz = (int)((long long)row_slot(a, r) * a.z_slot + a.z_layer);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();  // q and the K row at pos come from the QKV kernel
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, (unsigned)nbox * TILE_KEYS * 128u);
        for (int b = 0; b < nbox; b++)
            tma_load_3d(const_cast<unsigned char *>(s_k) + (size_t)b * TILE_KEYS * 128, &kmap,
                        g * hd + 32 * b, t0, kz, &bar);
    }
    const float *qr = a.q + (size_t)r * a.ldq + (size_t)g * kv_mul * hd;
    for (int i = threadIdx.x; i < kv_mul * hd; i += TILE_KEYS) s_q[i] = qr[i];
    const bool ok = mbar_wait(&bar, 0, &s_abort, a.err);
    __syncthreads();
    if (!ok || s_abort) {
        // bounded drain of the copies in flight before the shared memory goes away
        if (threadIdx.x == 0) {
            const long long tw = clock64();
            while (!mbar_test(&bar, 0) && clock64() - tw < WAIT_LIMIT) {
            }
        }
        __syncthreads();
        return;
    }
    pdl_release();
    const int t = threadIdx.x;
    if (t >= nrows) return;
    const unsigned sw = (unsigned)(t & 7);
    float *att = a.att + ((size_t)r * a.num_heads + (size_t)g * kv_mul) * a.att_ld + t0 + t;
    for (int h0 = 0; h0 < kv_mul; h0 += 4) {
        const int nh = kv_mul - h0 < 4 ? kv_mul - h0 : 4;
        float dot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float4 *q4 = reinterpret_cast<const float4 *>(s_q + h0 * hd);
        for (int b = 0; b < nbox; b++) {
            const unsigned char *row = s_k + (size_t)b * TILE_KEYS * 128 + (size_t)t * 128;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const float4 kk = *reinterpret_cast<const float4 *>(row + ((c ^ sw) << 4));
                const int v = b * 8 + c;  // float4 index within the head
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (u < nh) {
                        const float4 qq = q4[u * (hd >> 2) + v];
                        dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.x, kk.x));
                        dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.y, kk.y));
                        dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.z, kk.z));
                        dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.w, kk.w));
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (u < nh) att[(size_t)(h0 + u) * a.att_ld] = __fmul_rn(dot[u], a.scale);
    }
}

// (A'') scores, pipelined: a fixed grid of a few CTAs per SM walks the
// (row, KV head, 128-key tile) items.  One producer warp loads each item's
// row position and slot, then puts its K tile (head_dim/32 swizzled TMA boxes
// as in (A')) and its query vectors (one bulk copy) into one of two stages;
// four consumer warps compute the previous item meanwhile (thread t = key t,
// kv_mul chains), so copy latency and the per-item set-up overlap compute
// instead of being paid once per CTA.  FULL/EMPTY mbarriers per stage, all
// waits bounded; an item with info.r < 0 ends the consumers' loop.
#ifndef SLM_SCORE_STAGES
#define SLM_SCORE_STAGES 2
#endif
constexpr int SCORE_STAGES = SLM_SCORE_STAGES;
constexpr int SCORE_CONS_WARPS = TILE_KEYS / 32;

struct ScoreItem {
    int r, g, t0, nrows;
};

__host__ __device__ inline size_t score_stage_bytes(int kv_mul, int hd) {
    // K boxes, then the query vectors, 1 KB aligned
    return ((size_t)(hd / 32) * TILE_KEYS * 128 + sizeof(float) * kv_mul * hd + 1023) / 1024 * 1024;
}

__global__ void __launch_bounds__(TILE_KEYS + 32)
    attn_scores_pipe_kernel(AttnArgs a, int ntile_max, const __grid_constant__ CUtensorMap kmap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_full[SCORE_STAGES], bar_empty[SCORE_STAGES];
    __shared__ ScoreItem s_item[SCORE_STAGES];
    __shared__ int s_abort, s_issued;
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int kv_mul = a.num_heads / a.num_kv_heads;
    const int hd = a.head_dim, nbox = hd >> 5;
    const size_t stage_bytes = score_stage_bytes(kv_mul, hd);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long n_items = (long long)a.rows * a.num_kv_heads * ntile_max;
    if (tid == 0) {
        for (int st = 0; st < SCORE_STAGES; st++) {
            mbar_init(&bar_full[st], 1);
            mbar_init(&bar_empty[st], SCORE_CONS_WARPS);
        }
        s_abort = 0;
        s_issued = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();  // q and the K row at pos come from the QKV kernel
    pdl_release();

    if (warp == SCORE_CONS_WARPS) {
        // ---- producer
        int n = 0;  // items handed to the consumers
        for (long long it = blockIdx.x; ; it += gridDim.x) {
            ScoreItem item{-1, 0, 0, 0};
            if (it < n_items) {
                // KV head fastest: CTAs next to each other in the grid read
                // the kv_heads slices of the same K rows at about the same
                // time, so each row of the position-major cache is fetched
                // from HBM whole
                item.g = (int)(it % a.num_kv_heads);
                const long long rk = it / a.num_kv_heads;
                const int k = (int)(rk % ntile_max);
                item.r = (int)(rk / ntile_max);
                if (!unit_owned(a, item.r, item.g)) continue;  // another rank's unit
                const int L = row_len(a, item.r);
                item.t0 = k * TILE_KEYS;
                if (item.t0 >= L) continue;  // past this row's keys
                item.nrows = L - item.t0 < TILE_KEYS ? L - item.t0 : TILE_KEYS;
            }
            const int st = n % SCORE_STAGES;
            if (n >= SCORE_STAGES &&
                !mbar_wait(&bar_empty[st], (unsigned)((n / SCORE_STAGES) - 1) & 1u, &s_abort, a.err))
                break;
            if (lane == 0) {
                s_item[st] = item;
                if (item.r < 0) {
                    mbar_arrive(&bar_full[st]);  // end marker, no bytes
                } else {
                    unsigned char *dst = base + (size_t)st * stage_bytes;
                    float *q_dst = reinterpret_cast<float *>(dst + (size_t)nbox * TILE_KEYS * 128);
                    const int kz = (int)((long long)row_slot(a, item.r) * a.z_slot + a.z_layer);
                    mbar_arrive_expect_tx(&bar_full[st],
                                          (unsigned)nbox * TILE_KEYS * 128u + (unsigned)(kv_mul * hd) * 4u);
                    for (int b = 0; b < nbox; b++)
                        tma_load_3d(dst + (size_t)b * TILE_KEYS * 128, &kmap, item.g * hd + 32 * b,
                                    item.t0, kz, &bar_full[st]);
                    bulk_copy(q_dst, a.q + (size_t)item.r * a.ldq + (size_t)item.g * kv_mul * hd,
                              (unsigned)(kv_mul * hd) * 4u, &bar_full[st]);
                }
                s_issued = n + 1;
            }
            __syncwarp();
            n++;
            if (item.r < 0) break;
        }
    } else {
        // ---- consumers: thread t = key t0 + t of the current item
        const unsigned sw = (unsigned)(tid & 7);
        for (int n = 0; ; n++) {
            const int st = n % SCORE_STAGES;
            if (!mbar_wait(&bar_full[st], (unsigned)(n / SCORE_STAGES) & 1u, &s_abort, a.err)) break;
            const ScoreItem item = s_item[st];
            if (item.r < 0) break;
            const unsigned char *s_k = base + (size_t)st * stage_bytes;
            const float *s_q = reinterpret_cast<const float *>(s_k + (size_t)nbox * TILE_KEYS * 128);
            if (tid < item.nrows) {
                float *att = a.att + ((size_t)item.r * a.num_heads + (size_t)item.g * kv_mul) * a.att_ld +
                             item.t0 + tid;
                for (int h0 = 0; h0 < kv_mul; h0 += 4) {
                    const int nh = kv_mul - h0 < 4 ? kv_mul - h0 : 4;
                    float dot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    const float4 *q4 = reinterpret_cast<const float4 *>(s_q + h0 * hd);
                    for (int b = 0; b < nbox; b++) {
                        const unsigned char *row = s_k + (size_t)b * TILE_KEYS * 128 + (size_t)tid * 128;
#pragma unroll
                        for (int c = 0; c < 8; c++) {
                            const float4 kk = *reinterpret_cast<const float4 *>(row + ((c ^ sw) << 4));
                            const int v = b * 8 + c;  // float4 index within the head
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                if (u < nh) {
                                    const float4 qq = q4[u * (hd >> 2) + v];
                                    dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.x, kk.x));
                                    dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.y, kk.y));
                                    dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.z, kk.z));
                                    dot[u] = __fadd_rn(dot[u], __fmul_rn(qq.w, kk.w));
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 4; u++)
                        if (u < nh) att[(size_t)(h0 + u) * a.att_ld] = __fmul_rn(dot[u], a.scale);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_empty[st]);
        }
    }
    __syncthreads();
    if (s_abort && tid == 0) {
        // a wait gave up: let the copies already issued land (bounded)
        const int n_iss = s_issued;
        for (int k = n_iss - SCORE_STAGES < 0 ? 0 : n_iss - SCORE_STAGES; k < n_iss; k++) {
            const long long t0 = clock64();
            while (!mbar_test(&bar_full[k % SCORE_STAGES], (unsigned)(k / SCORE_STAGES) & 1u) &&
                   clock64() - t0 < WAIT_LIMIT) {
            }
        }
    }
}

// (P1) prefill scores, query-tiled: rows come in runs of consecutive
// positions (the tokens of one prompt); an item is (run, PQT query rows,
// KV head, 128-key tile) of the causal triangle.  A producer warp fetches the
// K tile (swizzled boxes as in (A')) and the tile's query vectors (one bulk
// copy per row) into one of two stages; consumer thread t loads key t's K row
// into registers once and runs every (row, head) dot of the tile against it,
// sequential in i as in (A), so each K tile crosses the memory system once
// per PQT query rows instead of once per row.
constexpr int PQT = 16;

struct PrefillItem {
    int r0, nr, p0, g, t0;
};

__host__ __device__ inline size_t prefill_stage_bytes(int kv_mul, int hd) {
    return ((size_t)(hd / 32) * TILE_KEYS * 128 + sizeof(float) * PQT * kv_mul * hd + 1023) / 1024 * 1024;
}

template <int KVM, int HD>
__global__ void __launch_bounds__(TILE_KEYS + 32)
    attn_prefill_scores_kernel(AttnArgs a, int run, int nqt, int nkt,
                               const __grid_constant__ CUtensorMap kmap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_full[SCORE_STAGES], bar_empty[SCORE_STAGES];
    __shared__ PrefillItem s_item[SCORE_STAGES];
    __shared__ int s_abort, s_issued;
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr int nbox = HD / 32, QW = KVM * HD;  // floats of one row's query vectors
    const size_t stage_bytes = prefill_stage_bytes(KVM, HD);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long n_items = (long long)(a.rows / run) * nqt * a.num_kv_heads * nkt;
    if (tid == 0) {
        for (int st = 0; st < SCORE_STAGES; st++) {
            mbar_init(&bar_full[st], 1);
            mbar_init(&bar_empty[st], SCORE_CONS_WARPS);
        }
        s_abort = 0;
        s_issued = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();  // q and the K rows of this prompt come from the QKV kernel
    pdl_release();

    if (warp == SCORE_CONS_WARPS) {
        // ---- producer
        int n = 0;
        for (long long it = blockIdx.x; ; it += gridDim.x) {
            PrefillItem item{-1, 0, 0, 0, 0};
            if (it < n_items) {
                const int kt = (int)(it % nkt);
                long long rest = it / nkt;
                item.g = (int)(rest % a.num_kv_heads);
                rest /= a.num_kv_heads;
                const int qt = (int)(rest % nqt);
                const int run_i = (int)(rest / nqt);
                item.r0 = run_i * run + qt * PQT;
                item.nr = run - qt * PQT < PQT ? run - qt * PQT : PQT;
                if (!unit_owned(a, item.r0, item.g)) continue;  // another rank's unit
                item.p0 = a.pos ? a.pos[item.r0] : a.pos_const;
                int lmax = item.p0 + item.nr;  // keys of the tile's last row
                lmax = lmax < a.max_seq ? lmax : a.max_seq;
                lmax = lmax < a.max_len ? lmax : a.max_len;
                item.t0 = kt * TILE_KEYS;
                if (item.t0 >= lmax) continue;  // above the causal triangle
            }
            const int st = n % SCORE_STAGES;
            if (n >= SCORE_STAGES &&
                !mbar_wait(&bar_empty[st], (unsigned)((n / SCORE_STAGES) - 1) & 1u, &s_abort, a.err))
                break;
            unsigned char *dst = base + (size_t)st * stage_bytes;
            if (lane == 0) {
                s_item[st] = item;
                if (item.r0 < 0) {
                    mbar_arrive(&bar_full[st]);  // end marker, no bytes
                } else {
                    const int kz = (int)((long long)row_slot(a, item.r0) * a.z_slot + a.z_layer);
                    mbar_arrive_expect_tx(&bar_full[st],
                                          (unsigned)nbox * TILE_KEYS * 128u + (unsigned)(item.nr * QW) * 4u);
                    for (int b = 0; b < nbox; b++)
                        tma_load_3d(dst + (size_t)b * TILE_KEYS * 128, &kmap, item.g * HD + 32 * b,
                                    item.t0, kz, &bar_full[st]);
                }
                s_issued = n + 1;
            }
            __syncwarp();
            if (item.r0 >= 0 && lane < item.nr) {
                float *q_dst = reinterpret_cast<float *>(dst + (size_t)nbox * TILE_KEYS * 128) + lane * QW;
                bulk_copy(q_dst, a.q + (size_t)(item.r0 + lane) * a.ldq + (size_t)item.g * QW,
                          (unsigned)QW * 4u, &bar_full[st]);
            }
            __syncwarp();
            n++;
            if (item.r0 < 0) break;
        }
    } else {
        // ---- consumers: thread t = key t0 + t
        const unsigned sw = (unsigned)(tid & 7);
        for (int n = 0; ; n++) {
            const int st = n % SCORE_STAGES;
            if (!mbar_wait(&bar_full[st], (unsigned)(n / SCORE_STAGES) & 1u, &s_abort, a.err)) break;
            const PrefillItem item = s_item[st];
            if (item.r0 < 0) break;
            const unsigned char *s_k = base + (size_t)st * stage_bytes;
            const float *s_q = reinterpret_cast<const float *>(s_k + (size_t)nbox * TILE_KEYS * 128);
            float kr[HD];
#pragma unroll
            for (int b = 0; b < nbox; b++) {
                const unsigned char *row = s_k + (size_t)b * TILE_KEYS * 128 + (size_t)tid * 128;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const float4 kk = *reinterpret_cast<const float4 *>(row + ((c ^ sw) << 4));
                    kr[b * 32 + c * 4 + 0] = kk.x;
                    kr[b * 32 + c * 4 + 1] = kk.y;
                    kr[b * 32 + c * 4 + 2] = kk.z;
                    kr[b * 32 + c * 4 + 3] = kk.w;
                }
            }
            const int key = item.t0 + tid, wkey = item.t0 + warp * 32;
            auto row_keys = [&](int i) {  // keys of row r0+i (0 past the tile)
                int L = item.p0 + i + 1;
                L = L < a.max_seq ? L : a.max_seq;
                L = L < a.max_len ? L : a.max_len;
                return i < item.nr ? L : 0;
            };
            // two query rows at a time: 2*KVM independent sequential chains
            for (int i = 0; i < item.nr; i += 2) {
                const int L0 = row_keys(i), L1 = row_keys(i + 1);
                if (wkey >= (L0 > L1 ? L0 : L1)) continue;  // the causal mask, whole warp
                float dot[2][KVM];
#pragma unroll
                for (int h = 0; h < KVM; h++) dot[0][h] = dot[1][h] = 0.0f;
                // row i+1 past the tile reads stale q; its results are dropped
                const float4 *q4 = reinterpret_cast<const float4 *>(s_q + i * QW);
#pragma unroll
                for (int v = 0; v < HD / 4; v++) {
#pragma unroll
                    for (int j = 0; j < 2; j++) {
#pragma unroll
                        for (int h = 0; h < KVM; h++) {
                            const float4 qq = q4[j * (QW / 4) + h * (HD / 4) + v];
                            dot[j][h] = __fadd_rn(dot[j][h], __fmul_rn(qq.x, kr[4 * v + 0]));
                            dot[j][h] = __fadd_rn(dot[j][h], __fmul_rn(qq.y, kr[4 * v + 1]));
                            dot[j][h] = __fadd_rn(dot[j][h], __fmul_rn(qq.z, kr[4 * v + 2]));
                            dot[j][h] = __fadd_rn(dot[j][h], __fmul_rn(qq.w, kr[4 * v + 3]));
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int L = j ? L1 : L0;
                    if (wkey >= L) continue;  // warp-uniform
                    const size_t prow = (size_t)(item.r0 + i + j) * a.num_heads + (size_t)item.g * KVM;
                    float *att = a.att + prow * a.att_ld + key;
                    const bool live = key < L;  // lanes past the mask computed on whatever the tile held
#pragma unroll
                    for (int h = 0; h < KVM; h++) {
                        const float sc = __fmul_rn(dot[j][h], a.scale);
                        if (live) att[(size_t)h * a.att_ld] = sc;
                        if (a.tmax) {
                            // maximum of this warp's 32 scores, masked keys left
                            // out; NaN propagates.  The sign of a zero maximum
                            // does not matter to the softmax: exp(x - (+0)) and
                            // exp(x - (-0)) are equal for every x.
                            const float m = warp_max_nan(live ? sc : -INFINITY);
                            if (lane == 0) a.tmax[(prow + h) * a.tmax_ld + wkey / 32] = m;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_empty[st]);
        }
    }
    __syncthreads();
    if (s_abort && tid == 0) {
        // a wait gave up: let the copies already issued land (bounded)
        const int n_iss = s_issued;
        for (int k = n_iss - SCORE_STAGES < 0 ? 0 : n_iss - SCORE_STAGES; k < n_iss; k++) {
            const long long t0 = clock64();
            while (!mbar_test(&bar_full[k % SCORE_STAGES], (unsigned)(k / SCORE_STAGES) & 1u) &&
                   clock64() - t0 < WAIT_LIMIT) {
            }
        }
    }
}

// (P2) prefill softmax + PV, query-tiled: one CTA per (run, PQT query rows,
// KV head).  The softmax of the tile's PQT x kv_mul (row, head) score rows
// runs over att (L2-resident) in the reference's order -- max, exp, four lane
// chains + tail, 1/sum, p = e * inv written back -- then a producer warp
// streams, per 64-key stage, the V tile (tensor map over the V planes) and
// the probability tile [PQT rows][kv_mul heads][64 keys] (tensor map over
// att) into a ring; consumer thread (dim pair, row group) runs the PV chains
// of its rows and heads, sequential in t, masking each row's keys past its
// own position.  The probabilities are written with ordinary stores and read
// by TMA (the async proxy): every thread fences before the barrier that
// precedes the first TMA issue.
constexpr int PPV_TT = 64;
static_assert(PPV_TT == TT_V, "the V tensor map's box holds PPV_TT positions");
constexpr int PPV_STAGES = 3;
constexpr int PPV_CONS = 256;  // consumer threads

__host__ __device__ inline size_t ppv_stage_bytes(int kv_mul, int hd) {
    return ((size_t)PPV_TT * hd * 4 + (size_t)PQT * kv_mul * PPV_TT * 4 + 127) / 128 * 128;
}

template <int KVM, int HD>
__global__ void __launch_bounds__(PPV_CONS + 32)
    attn_prefill_softmax_pv_kernel(AttnArgs a, int run, const __grid_constant__ CUtensorMap vmap,
                                   const __grid_constant__ CUtensorMap amap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_full[PPV_STAGES], bar_empty[PPV_STAGES];
    __shared__ int s_abort, s_issued;
    __shared__ float s_max[PQT * KVM], s_inv[PQT * KVM], s_chain[4 * PQT * KVM];
    unsigned char *base = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
    constexpr int DP = HD / 2;               // dim pairs
    constexpr int RG = PPV_CONS / DP;        // row groups
    constexpr int RPG = PQT / RG;            // rows per group
    static_assert(RPG * RG == PQT && RPG >= 1, "tile shape");
    const int qt = blockIdx.x, g = blockIdx.y, run_i = blockIdx.z;
    const int r0 = run_i * run + qt * PQT;
    const int nr = run - qt * PQT < PQT ? run - qt * PQT : PQT;
    if (!unit_owned(a, r0, g)) return;  // CTA-uniform: another rank's unit
    const int tid = threadIdx.x, nth = blockDim.x, warp = tid >> 5, lane = tid & 31;
    const int nw = nth >> 5;
    const int p0 = a.pos ? a.pos[r0] : a.pos_const;
    auto row_L = [&](int i) {
        int L = p0 + i + 1;
        L = L < a.max_seq ? L : a.max_seq;
        return L < a.max_len ? L : a.max_len;
    };
    const int npairs = nr * KVM;
    auto prow = [&](int pr) {  // score / probability row of pair pr = i*KVM + h
        return a.att + ((size_t)(r0 + pr / KVM) * a.num_heads + (size_t)g * KVM + pr % KVM) * a.att_ld;
    };
    const size_t stage_bytes = ppv_stage_bytes(KVM, HD);
    if (tid == 0) {
        for (int st = 0; st < PPV_STAGES; st++) {
            mbar_init(&bar_full[st], 1);
            mbar_init(&bar_empty[st], PPV_CONS / 32);
        }
        s_abort = 0;
        s_issued = 0;
        mbar_fence_init();
    }
    pdl_wait();  // the score rows come from the scores kernel
    __syncthreads();

    // ---- softmax of every pair (graph.rs:168-179 order)
    for (int pr = warp; pr < npairs; pr += nw) {
        const int L = row_L(pr / KVM);
        float m = -INFINITY;
        if (a.tmax) {  // from the scores kernel's per-32-key maxima
            const float *tm = a.tmax + ((size_t)(r0 + pr / KVM) * a.num_heads + (size_t)g * KVM + pr % KVM) *
                                           a.tmax_ld;
            for (int j = lane; j < (L + 31) / 32; j += 32) m = cl_fmax(m, tm[j]);
        } else {
            const float *row = prow(pr);
            for (int t = lane; t < L; t += 32) m = cl_fmax(m, row[t]);
        }
        for (int o = 16; o > 0; o >>= 1) m = cl_fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_max[pr] = m;
    }
    __syncthreads();
    if (tid < 4 * npairs) {
        // lane chain l of pair pr over [0, L & ~3): this thread also forms the
        // exps of its lane (off the dependent chain) and stores them; the
        // scores are loaded eight steps ahead
        const int pr = tid >> 2, l = tid & 3;
        float *e = prow(pr);
        const float mx = s_max[pr];
        const int L = row_L(pr / KVM), vl = L & ~3;
        float acc = 0.0f;
        int i = l;
        for (; i + 28 < vl; i += 32) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = e[i + 4 * u];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                v[u] = exp_poly(__fsub_rn(v[u], mx));
                e[i + 4 * u] = v[u];
            }
#pragma unroll
            for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, v[u]);
        }
        for (; i < vl; i += 4) {
            const float ev = exp_poly(__fsub_rn(e[i], mx));
            e[i] = ev;
            acc = __fadd_rn(acc, ev);
        }
        s_chain[tid] = acc;
        if (l == 0)
            for (int t = vl; t < L; t++) e[t] = exp_poly(__fsub_rn(e[t], mx));  // the tail
    }
    __syncthreads();
    if (tid < npairs) {
        const float *e = prow(tid);
        const int L = row_L(tid / KVM), vl = L & ~3;
        float sum = __fadd_rn(__fadd_rn(s_chain[4 * tid], s_chain[4 * tid + 1]),
                              __fadd_rn(s_chain[4 * tid + 2], s_chain[4 * tid + 3]));
        for (int i = vl; i < L; i++) sum = __fadd_rn(sum, e[i]);
        s_inv[tid] = __fdiv_rn(1.0f, sum);
    }
    // the exps are read next by TMA (async proxy); p = e * inv is formed in
    // shared memory when each tile lands
    __threadfence();
    asm volatile("fence.proxy.async.global;\n" ::: "memory");
    __syncthreads();

    // ---- out = sum_t p_t * v_t per (row, head, dim), sequential in t
    const int Lmax = row_L(nr - 1);
    const int ntiles = (Lmax + PPV_TT - 1) / PPV_TT;
    const unsigned tile_tx = (unsigned)(PPV_TT * HD * 4 + PQT * KVM * PPV_TT * 4);
    if (warp == PPV_CONS / 32) {
        // ---- producer
        const int vz = (int)((long long)row_slot(a, r0) * a.z_slot + a.z_layer);
        for (int k = 0; k < ntiles; k++) {
            const int st = k % PPV_STAGES;
            if (k >= PPV_STAGES &&
                !mbar_wait(&bar_empty[st], (unsigned)((k / PPV_STAGES) - 1) & 1u, &s_abort, a.err))
                break;
            if (lane == 0) {
                unsigned char *dst = base + (size_t)st * stage_bytes;
                mbar_arrive_expect_tx(&bar_full[st], tile_tx);
                tma_load_3d(dst, &vmap, g * HD, k * PPV_TT, vz, &bar_full[st]);
                tma_load_3d(dst + (size_t)PPV_TT * HD * 4, &amap, k * PPV_TT, g * KVM, r0, &bar_full[st]);
                s_issued = k + 1;
            }
            __syncwarp();
        }
    } else {
        // ---- consumers: dims 2*dp, 2*dp+1 of rows rg*RPG .. rg*RPG+RPG-1, all heads
        const int dp = tid % DP, rg = tid / DP;
        int Lr[RPG];
#pragma unroll
        for (int ii = 0; ii < RPG; ii++) Lr[ii] = rg * RPG + ii < nr ? row_L(rg * RPG + ii) : 0;
        float acc[RPG][KVM][2];
#pragma unroll
        for (int ii = 0; ii < RPG; ii++)
#pragma unroll
            for (int h = 0; h < KVM; h++) acc[ii][h][0] = acc[ii][h][1] = 0.0f;
        for (int k = 0; k < ntiles; k++) {
            const int st = k % PPV_STAGES;
            const bool ok = mbar_wait(&bar_full[st], (unsigned)(k / PPV_STAGES) & 1u, &s_abort, a.err);
            unsigned char *stg = base + (size_t)st * stage_bytes;
            const float2 *vt = reinterpret_cast<const float2 *>(stg) + dp;  // row stride DP pairs
            float *ptw = reinterpret_cast<float *>(stg + (size_t)PPV_TT * HD * 4);
            // p = e * (1/sum) of the tile's [PQT][KVM][64] entries, once, by
            // all consumers; the barrier over the consumer warps also makes the
            // give-up decision the same for all of them
            if (ok)
                for (int j = tid; j < PQT * KVM * PPV_TT; j += PPV_CONS) {
                    const int pr = j / PPV_TT;
                    if (pr < npairs) ptw[j] = __fmul_rn(ptw[j], s_inv[pr]);
                }
            if (named_bar_or(1, PPV_CONS, !ok)) break;
            const float *pt = ptw;
            const int t0 = k * PPV_TT;
            bool full = true;
#pragma unroll
            for (int ii = 0; ii < RPG; ii++) full = full && (Lr[ii] >= t0 + PPV_TT || Lr[ii] == 0);
            if (full) {
#pragma unroll 4
                for (int u0 = 0; u0 < PPV_TT; u0 += 4) {
                    float2 vv[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) vv[u] = vt[(u0 + u) * DP];
#pragma unroll
                    for (int ii = 0; ii < RPG; ii++) {
#pragma unroll
                        for (int h = 0; h < KVM; h++) {
                            const float4 p4 = *reinterpret_cast<const float4 *>(
                                pt + ((rg * RPG + ii) * KVM + h) * PPV_TT + u0);
                            acc[ii][h][0] = __fadd_rn(acc[ii][h][0], __fmul_rn(p4.x, vv[0].x));
                            acc[ii][h][1] = __fadd_rn(acc[ii][h][1], __fmul_rn(p4.x, vv[0].y));
                            acc[ii][h][0] = __fadd_rn(acc[ii][h][0], __fmul_rn(p4.y, vv[1].x));
                            acc[ii][h][1] = __fadd_rn(acc[ii][h][1], __fmul_rn(p4.y, vv[1].y));
                            acc[ii][h][0] = __fadd_rn(acc[ii][h][0], __fmul_rn(p4.z, vv[2].x));
                            acc[ii][h][1] = __fadd_rn(acc[ii][h][1], __fmul_rn(p4.z, vv[2].y));
                            acc[ii][h][0] = __fadd_rn(acc[ii][h][0], __fmul_rn(p4.w, vv[3].x));
                            acc[ii][h][1] = __fadd_rn(acc[ii][h][1], __fmul_rn(p4.w, vv[3].y));
                        }
                    }
                }
            } else {
                for (int u = 0; u < PPV_TT; u++) {
                    const float2 v = vt[u * DP];
#pragma unroll
                    for (int ii = 0; ii < RPG; ii++) {
                        if (t0 + u < Lr[ii]) {
#pragma unroll
                            for (int h = 0; h < KVM; h++) {
                                const float pv = pt[((rg * RPG + ii) * KVM + h) * PPV_TT + u];
                                acc[ii][h][0] = __fadd_rn(acc[ii][h][0], __fmul_rn(pv, v.x));
                                acc[ii][h][1] = __fadd_rn(acc[ii][h][1], __fmul_rn(pv, v.y));
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_empty[st]);
        }
        if (!s_abort) {
#pragma unroll
            for (int ii = 0; ii < RPG; ii++) {
                const int i = rg * RPG + ii;
                if (i < nr) {
#pragma unroll
                    for (int h = 0; h < KVM; h++)
                        *reinterpret_cast<float2 *>(a.out + (size_t)(r0 + i) * a.ldo + (size_t)(g * KVM + h) * HD +
                                                    2 * dp) = make_float2(acc[ii][h][0], acc[ii][h][1]);
                }
            }
        }
    }
    pdl_release();
    __syncthreads();
    if (s_abort && tid == 0) {
        // a wait gave up: let the copies already issued land (bounded)
        const int n_iss = s_issued;
        for (int k = n_iss - PPV_STAGES < 0 ? 0 : n_iss - PPV_STAGES; k < n_iss; k++) {
            const long long t0 = clock64();
            while (!mbar_test(&bar_full[k % PPV_STAGES], (unsigned)(k / PPV_STAGES) & 1u) &&
                   clock64() - t0 < WAIT_LIMIT) {
            }
        }
    }
}

// (B) softmax + PV: one CTA per (row, KV head), warp-specialized.  One
// producer thread owns every copy of V: each stage is one TMA box (TT_V
// positions x head_dim floats of this KV head) of a 3-D tensor map over the
// cache planes, landing densely in a ring of FUSED_STAGES stages guarded by
// FULL/EMPTY mbarriers.  The first stages are issued before the softmax.  The
// KVM score rows come from the scores kernel's output; the softmax runs in
// shared memory with all warps; then consumer thread (head h, dims 2j, 2j+1)
// runs its two chains side by side on float2 loads of V, each probability
// load covering four positions.  When q8_out is
// given, the output block this CTA owns is quantized for the Wo GEMV in the
// same kernel.  Every mbarrier wait is bounded (mbar_wait).
// PV consumer thread shape: NH query heads x ND consecutive dims of chains
// per thread.  The launch uses (1, 2), a thread per (head, dim pair); (KVM, 1)
// and (1, 1) were measured slower on B200.
template <int ND>
struct PvVec {
    float v[ND];
    __device__ __forceinline__ static PvVec load(const float *p) {
        PvVec r;
        if constexpr (ND == 2) {
            const float2 t = *reinterpret_cast<const float2 *>(p);
            r.v[0] = t.x;
            r.v[1] = t.y;
        } else {
            r.v[0] = *p;
        }
        return r;
    }
};

// KVM here is the number of query heads of one CTA (HPC): all kv_mul heads
// of a KV head (grid.x = num_kv_heads), or one query head (grid.x =
// num_heads; the kv_mul CTAs of a KV head then each stream its V rows, mostly
// from L2).  NST is the depth of the V ring (<= PV_MAX_STAGES), chosen by the
// launch from the CTAs each SM holds.
// DS: the head_dim split -- with DS = 2 a CTA covers half of every head's dims
// (grid.x = num_kv_heads * 2, V from a tensor map whose box is head_dim / 2
// wide), so each V tile is half as large and is staged once for all KVM heads.
// TTV: V positions per stage.  TT_V is one box of the standard map; other
// sizes (16, 32) come from a map whose box is V_FINE_POSITIONS positions, as
// TTV / V_FINE_POSITIONS boxes per stage: smaller stages give a deeper ring
// in the same shared memory, so more of each CTA's V stream is in flight.
template <int KVM, int NH, int ND, int HDT = 0, int DS = 1, int TTV = TT_V>
__global__ void __launch_bounds__(512)
    attn_softmax_pv_kernel(AttnArgs a, int lp, int NST, const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_full[PV_MAX_STAGES], bar_empty[PV_MAX_STAGES];
    __shared__ int s_abort, s_issued;
    // TMA destinations 128-byte aligned (the launch adds 128 B of slack)
    float *smem = reinterpret_cast<float *>(smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u));
    constexpr int tt = TTV;
    constexpr int box_pos = TTV == TT_V ? TT_V : V_FINE_POSITIONS;  // positions per TMA box
    static_assert(TTV % box_pos == 0, "a stage is whole boxes");
    constexpr int nld = TTV / box_pos;
    const int nth = blockDim.x;
    const int h0 = (blockIdx.x / DS) * KVM, r = blockIdx.y;  // first query head of this CTA
    const int dsp = blockIdx.x % DS;                          // which part of the head's dims
    const int g = h0 / (a.num_heads / a.num_kv_heads);  // its KV head
    if (!unit_owned(a, r, g)) return;  // CTA-uniform: another rank's unit
    // HDT: head_dim fixed at compile time (V rows at immediate offsets), or 0;
    // hd is this CTA's part of it (the V tile width and the dims it computes)
    const int hdf = HDT ? HDT : a.head_dim;
    const int hd = hdf / DS;
    const int tid = threadIdx.x;
    float *s_ring = smem;                                   // [NST][tt][hd]
    float *s_sc = s_ring + (size_t)NST * tt * hd;           // [KVM][lp]
    float *s_out = s_sc + (size_t)KVM * lp;                 // [KVM*hd]
    float *s_red = s_out + (size_t)KVM * hd;                // 64 + 8*32 floats
    const int L = row_len(a, r);
    const int ntiles = (L + tt - 1) / tt;
    const int vx = g * hdf + dsp * hd;
    const int vz = (int)((long long)row_slot(a, r) * a.z_slot + a.z_layer);
    const int n_thr = KVM * hd / (NH * ND);  // consumer threads: (NH heads, ND dims)
    const int n_cons = (n_thr + 31) >> 5;  // consumer warps
    const int warp = tid >> 5, lane = tid & 31;
    const int nw = nth >> 5;
    const bool producer = warp == n_cons;  // the launch has n_cons + 1 warps or more
    const unsigned tile_bytes = (unsigned)tt * (unsigned)hd * 4u;

    if (tid == 0) {
        for (int st = 0; st < NST; st++) {
            mbar_init(&bar_full[st], 1);
            mbar_init(&bar_empty[st], (unsigned)n_cons);
        }
        s_abort = 0;
        s_issued = 0;
        mbar_fence_init();
    }
    __syncthreads();
    if (producer && lane == 0) {
        int k = 0;
        for (; k < NST && k < ntiles; k++) {
            mbar_arrive_expect_tx(&bar_full[k], tile_bytes);
#pragma unroll
            for (int j = 0; j < nld; j++)
                tma_load_3d(s_ring + ((size_t)k * tt + j * box_pos) * hd, &vmap, vx, k * tt + j * box_pos, vz,
                            &bar_full[k]);
        }
        s_issued = k;
    }
    // V rows were written two kernels back (QKV), the scores by the previous one
    pdl_wait();

    // scores of the KVM heads of this group (cp.async, awaited before the softmax)
    const float *att = a.att + ((size_t)r * a.num_heads + (size_t)h0) * a.att_ld;
    const bool vec = (a.att_ld & 3) == 0 && ((uintptr_t)att & 15) == 0;
    if (vec) {
        const int c4 = (L + 3) >> 2;
        for (int h = 0; h < KVM; h++)
            for (int c = tid; c < c4; c += nth)
                cp_async16(s_sc + h * lp + 4 * c, att + (size_t)h * a.att_ld + 4 * c);
    } else {
        for (int h = 0; h < KVM; h++)
            for (int t = tid; t < L; t += nth) s_sc[h * lp + t] = att[(size_t)h * a.att_ld + t];
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();

    // ---- softmax per query head (graph.rs:168-179 order)
    {
        // maxima of all KVM heads with one pass and two barriers
        float m[KVM];
#pragma unroll
        for (int h = 0; h < KVM; h++) m[h] = -INFINITY;
        // the maximum of a set does not depend on the order it is taken in:
        // four independent running maxima per thread
#pragma unroll
        for (int h = 0; h < KVM; h++) {
            const float *row = s_sc + h * lp;
            float m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
            int t = tid;
            for (; t + 3 * nth < L; t += 4 * nth) {
                m[h] = cl_fmax(m[h], row[t]);
                m1 = cl_fmax(m1, row[t + nth]);
                m2 = cl_fmax(m2, row[t + 2 * nth]);
                m3 = cl_fmax(m3, row[t + 3 * nth]);
            }
            for (; t < L; t += nth) m[h] = cl_fmax(m[h], row[t]);
            m[h] = cl_fmax(cl_fmax(m[h], m1), cl_fmax(m2, m3));
        }
#pragma unroll
        for (int h = 0; h < KVM; h++) {
            for (int o = 16; o > 0; o >>= 1) m[h] = cl_fmax(m[h], __shfl_xor_sync(0xffffffffu, m[h], o));
            if (lane == 0) s_red[64 + h * 32 + warp] = m[h];
        }
        __syncthreads();
        if (tid < KVM) {
            float mm = s_red[64 + tid * 32];
            for (int w = 1; w < nw; w++) mm = cl_fmax(mm, s_red[64 + tid * 32 + w]);
            s_red[32 + tid] = mm;
        }
        __syncthreads();
    }
    // exp(s - max) of every position by all threads, then the four lane sums
    // of each head (graph.rs:168-179 order): lane 4h + l of warp 0 adds
    // e[l], e[l+4], ... over [0, L & ~3) in order, its loads one group of 16
    // ahead of the adds; the tail [L & ~3, L) is added after.
    const int vl = L & ~3;
#pragma unroll
    for (int h = 0; h < KVM; h++) {
        const float mx = s_red[32 + h];
        float *row = s_sc + h * lp;
        int t = tid;
        for (; t + 3 * nth < L; t += 4 * nth) {
            const float x0 = row[t], x1 = row[t + nth], x2 = row[t + 2 * nth], x3 = row[t + 3 * nth];
            const float e0 = exp_poly(__fsub_rn(x0, mx)), e1 = exp_poly(__fsub_rn(x1, mx));
            const float e2 = exp_poly(__fsub_rn(x2, mx)), e3 = exp_poly(__fsub_rn(x3, mx));
            row[t] = e0;
            row[t + nth] = e1;
            row[t + 2 * nth] = e2;
            row[t + 3 * nth] = e3;
        }
        for (; t < L; t += nth) row[t] = exp_poly(__fsub_rn(row[t], mx));
    }
    __syncthreads();
    float chain = 0.0f;
    if (warp == 0 && tid < 4 * KVM) {
        const int h = tid >> 2, l = tid & 3;
        const unsigned e0 = smem_addr(s_sc + h * lp + l);
        const int n4 = vl >> 2;  // this lane's positions l, l+4, ... below vl
        constexpr int G = 16;
        float cur[G], nxt[G];
        auto load = [&](int i, float (&v)[G]) {
#pragma unroll
            for (int u = 0; u < G; u++)
                asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v[u]) : "r"(e0 + 16u * (unsigned)(i + u)) : "memory");
        };
        int i = 0;
        if (n4 >= G) load(0, cur);
        for (; i + 2 * G <= n4; i += 2 * G) {
            load(i + G, nxt);
#pragma unroll
            for (int u = 0; u < G; u++) chain = __fadd_rn(chain, cur[u]);
            if (i + 3 * G <= n4) load(i + 2 * G, cur);
#pragma unroll
            for (int u = 0; u < G; u++) chain = __fadd_rn(chain, nxt[u]);
        }
        if (i + G <= n4) {
#pragma unroll
            for (int u = 0; u < G; u++) chain = __fadd_rn(chain, cur[u]);
            i += G;
        }
        const float *e = s_sc + h * lp + l;
        for (; i < n4; i++) chain = __fadd_rn(chain, e[4 * i]);
    }
    if (tid < 4 * KVM) s_red[tid] = chain;  // [0, 4*KVM) with KVM <= 8 stays below 32
    __syncthreads();
    if (tid < KVM) {
        const float *e = s_sc + tid * lp;
        float sum = __fadd_rn(__fadd_rn(s_red[4 * tid], s_red[4 * tid + 1]),
                              __fadd_rn(s_red[4 * tid + 2], s_red[4 * tid + 3]));
        for (int i = vl; i < L; i++) sum = __fadd_rn(sum, e[i]);
        s_red[48 + tid] = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    // p = e * (1/sum), in place (and into att when the caller wants the
    // probabilities)
    for (int h = 0; h < KVM; h++) {
        const float inv = s_red[48 + h];
        float *row = s_sc + h * lp;
        float *prow = a.write_probs ? a.att + ((size_t)r * a.num_heads + h0 + h) * a.att_ld : nullptr;
        int t = tid;
        for (; t + 3 * nth < L; t += 4 * nth) {
            const float p0 = __fmul_rn(row[t], inv), p1 = __fmul_rn(row[t + nth], inv);
            const float p2 = __fmul_rn(row[t + 2 * nth], inv), p3 = __fmul_rn(row[t + 3 * nth], inv);
            row[t] = p0;
            row[t + nth] = p1;
            row[t + 2 * nth] = p2;
            row[t + 3 * nth] = p3;
            if (prow) {
                prow[t] = p0;
                prow[t + nth] = p1;
                prow[t + 2 * nth] = p2;
                prow[t + 3 * nth] = p3;
            }
        }
        for (; t < L; t += nth) {
            const float pr = __fmul_rn(row[t], inv);
            row[t] = pr;
            if (prow) prow[t] = pr;
        }
    }

    // ---- out = sum_t p_t * v_t (sequential in t from 0.0)
    __syncthreads();  // probabilities complete
    if (producer) {
#pragma unroll 1
        for (int k = NST; k < ntiles; k++) {
            // the stage is free once every consumer warp released tile k - STAGES
            if (!mbar_wait(&bar_empty[k % NST], (unsigned)((k / NST) - 1) & 1u,
                           &s_abort, a.err))
                break;
            if (lane == 0) {
                const int st = k % NST;
                mbar_arrive_expect_tx(&bar_full[st], tile_bytes);
#pragma unroll
                for (int j = 0; j < nld; j++)
                    tma_load_3d(s_ring + ((size_t)st * tt + j * box_pos) * hd, &vmap, vx, k * tt + j * box_pos, vz,
                                &bar_full[st]);
                s_issued = k + 1;
            }
            __syncwarp();
        }
    } else if (warp < n_cons) {
        const bool active = tid < n_thr;
        const int dgrp = hd / ND;  // threads per head group
        const int hl = (tid / dgrp) * NH, jc = ND * (tid % dgrp);  // first head (of this CTA's), dim
        float acc[NH][ND];  // out[hl + h][jc + c]
#pragma unroll
        for (int h = 0; h < NH; h++)
#pragma unroll
            for (int c = 0; c < ND; c++) acc[h][c] = 0.0f;
        // Full tiles: a register pipeline of CH-position chunks, one chunk
        // ahead, that runs across stage boundaries -- a stage is released
        // as soon as its last chunk is in registers and the next stage's
        // first chunk is loaded before the current chunk is added, so the
        // only serial work per position is the add of each chain.  The
        // loads are volatile so that they stay ahead of the adds.
        constexpr int CH0 = NH > 1 ? 8 : 16, CH = CH0 < tt / 2 ? CH0 : tt / 2, NCH = tt / CH;
        static_assert(tt % CH == 0 && NCH % 2 == 0 && CH % 4 == 0, "an even number of whole chunks per stage");
        const int nfull = L / tt;
        const unsigned ring0 = smem_addr(s_ring) + 4u * (unsigned)jc;
        const unsigned prob0 = smem_addr(s_sc) + 4u * (unsigned)(hl * lp);
        float va[CH][ND], vb[CH][ND], pa[NH][CH], pb[NH][CH];
        // chunk ch of tile k into (v, p)
        auto load = [&](int k, int ch, float (&v)[CH][ND], float (&pr)[NH][CH]) {
            const unsigned vs = ring0 + 4u * (unsigned)(((k % NST) * tt + ch * CH) * hd);
            const unsigned ps = prob0 + 4u * (unsigned)(k * tt + ch * CH);
#pragma unroll
            for (int u = 0; u < CH; u++) {
                if constexpr (ND == 2)
                    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v[u][0]), "=f"(v[u][1])
                                 : "r"(vs + 4u * (unsigned)(u * hd)));
                else
                    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v[u][0]) : "r"(vs + 4u * (unsigned)(u * hd)));
            }
#pragma unroll
            for (int h = 0; h < NH; h++)
#pragma unroll
                for (int u = 0; u < CH; u += 4)
                    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                 : "=f"(pr[h][u]), "=f"(pr[h][u + 1]), "=f"(pr[h][u + 2]), "=f"(pr[h][u + 3])
                                 : "r"(ps + 4u * (unsigned)(h * lp + u)));
        };
        auto add = [&](const float (&v)[CH][ND], const float (&pr)[NH][CH]) {
#pragma unroll
            for (int u = 0; u < CH; u++)
#pragma unroll
                for (int h = 0; h < NH; h++)
#pragma unroll
                    for (int c = 0; c < ND; c++) acc[h][c] = __fadd_rn(acc[h][c], __fmul_rn(pr[h][u], v[u][c]));
        };
        auto release = [&](int k) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_empty[k % NST]);
        };
        bool ok = true;
        if (nfull > 0) {
            ok = mbar_wait(&bar_full[0], 0u, &s_abort, a.err);
            if (ok && active) load(0, 0, va, pa);
        }
#pragma unroll 1
        for (int k = 0; ok && k < nfull; k++) {
#pragma unroll
            for (int ch = 0; ch < NCH; ch += 2) {
                // chunk ch is in (va, pa); bring chunk ch + 1 into (vb, pb)
                if (active) load(k, ch + 1, vb, pb);
                if (active) add(va, pa);
                // chunk ch + 2, or the next tile's chunk 0, into (va, pa)
                if (ch + 2 < NCH) {
                    if (active) load(k, ch + 2, va, pa);
                } else {
                    release(k);  // every chunk of tile k is in registers
                    if (k + 1 < nfull) {
                        ok = mbar_wait(&bar_full[(k + 1) % NST], (unsigned)((k + 1) / NST) & 1u, &s_abort, a.err);
                        if (ok && active) load(k + 1, 0, va, pa);
                    }
                }
                if (active) add(vb, pb);
            }
        }
        // the ragged last tile, position by position
        if (ok && nfull < ntiles) {
            const int k = nfull;
            ok = mbar_wait(&bar_full[k % NST], (unsigned)(k / NST) & 1u, &s_abort, a.err);
            if (ok && active) {
                const float *vt = s_ring + (size_t)(k % NST) * tt * hd + jc;  // row stride hd
                const float *pp = s_sc + hl * lp + k * tt;                    // head stride lp
                const int nrows = L - k * tt;
                for (int tl = 0; tl < nrows; tl++) {
                    const PvVec<ND> vv = PvVec<ND>::load(vt + (size_t)tl * hd);
#pragma unroll
                    for (int h = 0; h < NH; h++) {
                        const float pr = pp[(size_t)h * lp + tl];
#pragma unroll
                        for (int c = 0; c < ND; c++) acc[h][c] = __fadd_rn(acc[h][c], __fmul_rn(pr, vv.v[c]));
                    }
                }
            }
            if (ok) release(k);
        }
        if (active)
#pragma unroll
            for (int h = 0; h < NH; h++)
#pragma unroll
                for (int c = 0; c < ND; c++) s_out[(hl + h) * hd + jc + c] = acc[h][c];
    }
    __syncthreads();
    if (s_abort) {
        // a wait gave up: let the copies already issued land (bounded) before
        // the shared memory is released, and leave the outputs untouched
        if (tid == 0) {
            // the last tile issued into each stage is the one whose phase is pending
            const int n_iss = s_issued;
            for (int k = n_iss - NST < 0 ? 0 : n_iss - NST; k < n_iss; k++) {
                const long long t0 = clock64();
                while (!mbar_test(&bar_full[k % NST], (unsigned)(k / NST) & 1u) &&
                       clock64() - t0 < WAIT_LIMIT) {
                }
            }
        }
        __syncthreads();
        return;
    }
    pdl_release();  // the successor may start while the outputs are written
    // this CTA's dims: [dsp*hd, (dsp+1)*hd) of each of its KVM heads
    float *orow = a.out + (size_t)r * a.ldo + (size_t)h0 * hdf + (size_t)dsp * hd;
    for (int k = tid; k < KVM * hd; k += nth) orow[(k / hd) * hdf + k % hd] = s_out[k];
    // Q8_0 of the attention output for the Wo GEMV: this CTA owns whole
    // 32-element blocks (hd a multiple of 32, checked by the host), one per
    // warp
    if (a.q8_out.qs) {
        const int nbr = a.dim / 32, bph = hd / 32;  // blocks per head part
        for (int blk = warp; blk < (KVM * hd) / 32; blk += nw)
            q8x_store_block(s_out[blk * 32 + lane], a.q8_out,
                            (size_t)r * nbr + (size_t)((h0 + blk / bph) * hdf + dsp * hd) / 32 + blk % bph, lane);
    }
}

// The (row, KV head) form: kv_mul heads per CTA, a 4-stage V ring.
template <int KVM>
void launch_softmax_pv(const AttnArgs &a, const CUtensorMap &vmap, cudaStream_t s) {
    const FusedShape f = fused_shape(KVM, a.head_dim, a.max_len);
    dim3 grid(a.num_kv_heads, a.rows);
    // consumer warps plus the producer warp, at least PV_THREADS
    auto threads = [&](int cons) {
        const int n = (cons + 31) / 32 * 32 + 32;
        return n < PV_THREADS ? PV_THREADS : n;
    };
    // a thread per (head, dim pair): measured faster than a thread per dim
    // running every head (fewer warps) or per (head, dim) (more warps)
    launch_kernel(attn_softmax_pv_kernel<KVM, 1, 2>, grid, dim3(threads(KVM * a.head_dim / 2)), f.smem, s,
                  a.pdl, a, f.lp, (int)FUSED_STAGES, vmap);
}

int sm_count() {
    static int sms = [] {
        int dev = 0, n = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        return n;
    }();
    return sms;
}

#define KVM_GROUP_OK(k) ((k) >= 1 && (k) <= 4)

// Depth of the V ring of a softmax + PV CTA over `hpc` query heads: the
// shared memory an SM has, shared by the CTAs it holds when the grid is
// spread evenly, in whole stages (2 to PV_MAX_STAGES).  Few CTAs per SM (small batches)
// get deep rings, so that each CTA keeps enough bytes in flight to stream its
// V rows at a useful rate on its own.
FusedShape pv_shape(const AttnArgs &a, int hpc, int tt = TT_V) {
    const long long ctas = (long long)a.rows * (a.num_heads / hpc);
    const long long per_sm = (ctas + sm_count() - 1) / sm_count();
    const size_t budget = (size_t)(FUSED_SMEM_MAX / (per_sm < 1 ? 1 : per_sm));
    const size_t fixed = fused_shape(hpc, a.head_dim, a.max_len, 0, tt).smem;
    const size_t stage = (size_t)tt * a.head_dim * sizeof(float);
    long long nst = budget > fixed ? (long long)((budget - fixed) / stage) : 0;
    nst = nst < PV_MIN_STAGES ? PV_MIN_STAGES : nst > PV_MAX_STAGES ? PV_MAX_STAGES : nst;
    return fused_shape(hpc, a.head_dim, a.max_len, (int)nst, tt);
}
FusedShape per_head_shape(const AttnArgs &a, int tt = TT_V) { return pv_shape(a, 1, tt); }

// The (row, KV head) form with a thread per (head, dim), head_dim fixed at
// compile time where it is 64 or 128 and a ring sized like the per-head one:
// each V tile is staged once for all kv_mul heads.
// Thread shape (NH heads x ND dims of chains per thread) for head_dim 64/128.
template <int KVM, int NH, int ND>
void launch_pv_group_shape(const AttnArgs &a, const FusedShape &f, const CUtensorMap &vmap, cudaStream_t s) {
    const int cons = (KVM * a.head_dim / (NH * ND) + 31) / 32 * 32;
    const dim3 grid(a.num_kv_heads, a.rows), block(cons + 32);
    if (a.head_dim == 64)
        launch_kernel(attn_softmax_pv_kernel<KVM, NH, ND, 64>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst, vmap);
    else if (a.head_dim == 128)
        launch_kernel(attn_softmax_pv_kernel<KVM, NH, ND, 128>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst, vmap);
    else
        launch_kernel(attn_softmax_pv_kernel<KVM, NH, ND>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst, vmap);
}

// The (row, KV head, head_dim half) form: grid.x = num_kv_heads * 2, V
// through vmap_half (box head_dim / 2 wide); mode 6: a thread per (head,
// dim), 7: a thread per (head, dim pair).
template <int KVM, int ND>
void launch_softmax_pv_split(const AttnArgs &a, const CUtensorMap &vmap_half, cudaStream_t s) {
    const int hdv = a.head_dim / 2;
    const long long ctas = (long long)a.rows * a.num_kv_heads * 2;
    const long long per_sm = (ctas + sm_count() - 1) / sm_count();
    const size_t budget = (size_t)(FUSED_SMEM_MAX / (per_sm < 1 ? 1 : per_sm));
    const size_t fixed = fused_shape(KVM, hdv, a.max_len, 0).smem;
    const size_t stage = (size_t)TT_V * hdv * sizeof(float);
    long long nst = budget > fixed ? (long long)((budget - fixed) / stage) : 0;
    nst = nst < PV_MIN_STAGES ? PV_MIN_STAGES : nst > PV_MAX_STAGES ? PV_MAX_STAGES : nst;
    const FusedShape f = fused_shape(KVM, hdv, a.max_len, (int)nst);
    const int cons = (KVM * hdv / ND + 31) / 32 * 32;
    const dim3 grid(a.num_kv_heads * 2, a.rows), block(cons + 32);
    if (a.head_dim == 64)
        launch_kernel(attn_softmax_pv_kernel<KVM, 1, ND, 64, 2>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst,
                      vmap_half);
    else
        launch_kernel(attn_softmax_pv_kernel<KVM, 1, ND, 128, 2>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst,
                      vmap_half);
}

// The (row, query head, half of head_dim) form (mode 10): grid.x =
// num_heads * 2, V through vmap_half, a thread per dim of the half; twice
// the CTAs of the per-head form, each streaming half of its head's V rows.
void launch_softmax_pv_per_head_split(const AttnArgs &a, const CUtensorMap &vmap_half, cudaStream_t s) {
    const int hdv = a.head_dim / 2;
    const long long ctas = (long long)a.rows * a.num_heads * 2;
    const long long per_sm = (ctas + sm_count() - 1) / sm_count();
    const size_t budget = (size_t)(FUSED_SMEM_MAX / (per_sm < 1 ? 1 : per_sm));
    const size_t fixed = fused_shape(1, hdv, a.max_len, 0).smem;
    const size_t stage = (size_t)TT_V * hdv * sizeof(float);
    long long nst = budget > fixed ? (long long)((budget - fixed) / stage) : 0;
    nst = nst < PV_MIN_STAGES ? PV_MIN_STAGES : nst > PV_MAX_STAGES ? PV_MAX_STAGES : nst;
    const FusedShape f = fused_shape(1, hdv, a.max_len, (int)nst);
    const int cons = (hdv + 31) / 32 * 32;
    const dim3 grid(a.num_heads * 2, a.rows), block(cons + 32);
    if (a.head_dim == 64)
        launch_kernel(attn_softmax_pv_kernel<1, 1, 1, 64, 2>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst,
                      vmap_half);
    else
        launch_kernel(attn_softmax_pv_kernel<1, 1, 1, 128, 2>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst,
                      vmap_half);
}

template <int KVM>
void set_softmax_pv_split_smem(int bytes) {
    cudaFuncSetAttribute(attn_softmax_pv_kernel<KVM, 1, 1, 64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<KVM, 1, 1, 128, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<KVM, 1, 2, 64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<KVM, 1, 2, 128, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// mode 3: a thread per (head, dim); 4: a thread per dim running every head
// of the group; 5: a thread per (head, dim pair)
template <int KVM>
void launch_softmax_pv_group(const AttnArgs &args, const CUtensorMap &vmap, cudaStream_t s) {
    AttnArgs a = args;
    const FusedShape f = pv_shape(a, KVM);
    const bool q8_after = a.q8_out.qs && (KVM * a.head_dim) % 32 != 0;
    if (q8_after) a.q8_out.qs = nullptr;
    if (a.pv_per_head == 4)
        launch_pv_group_shape<KVM, KVM, 1>(a, f, vmap, s);
    else if (a.pv_per_head == 5 && a.head_dim % 2 == 0)
        launch_pv_group_shape<KVM, 1, 2>(a, f, vmap, s);
    else
        launch_pv_group_shape<KVM, 1, 1>(a, f, vmap, s);
    if (q8_after) launch_quantize_q8x(a.out, a.ldo, a.dim, args.q8_out, a.rows, s);
}

template <int KVM, int NH, int ND>
void set_pv_shape_smem(int bytes) {
    cudaFuncSetAttribute(attn_softmax_pv_kernel<KVM, NH, ND, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<KVM, NH, ND, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<KVM, NH, ND>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}
template <int KVM>
void set_softmax_pv_group_smem(int bytes) {
    set_pv_shape_smem<KVM, 1, 1>(bytes);
    set_pv_shape_smem<KVM, KVM, 1>(bytes);
    set_pv_shape_smem<KVM, 1, 2>(bytes);
}

// The (row, query head) form: one head per CTA, a thread per dim (ND = 1) or
// per dim pair (ND = 2); kv_mul times the CTAs of the (row, KV head) form.
template <int ND, int TTV = TT_V>
void launch_softmax_pv_per_head(const AttnArgs &args, const CUtensorMap &vmap, cudaStream_t s) {
    AttnArgs a = args;
    const FusedShape f = per_head_shape(a, TTV);
    // the in-kernel Q8_0 of the output needs whole 32-element blocks per CTA
    const bool q8_after = a.q8_out.qs && a.head_dim % 32 != 0;
    if (q8_after) a.q8_out.qs = nullptr;
    const int cons = (a.head_dim / ND + 31) / 32 * 32;
    const dim3 grid(a.num_heads, a.rows), block(cons + 32);
    if (a.head_dim == 64)
        launch_kernel(attn_softmax_pv_kernel<1, 1, ND, 64, 1, TTV>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst,
                      vmap);
    else if (a.head_dim == 128)
        launch_kernel(attn_softmax_pv_kernel<1, 1, ND, 128, 1, TTV>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst,
                      vmap);
    else
        launch_kernel(attn_softmax_pv_kernel<1, 1, ND, 0, 1, TTV>, grid, block, f.smem, s, a.pdl, a, f.lp, f.nst,
                      vmap);
    if (q8_after) launch_quantize_q8x(a.out, a.ldo, a.dim, args.q8_out, a.rows, s);
}

template <int KVM>
void set_softmax_pv_smem(int bytes) {
    cudaFuncSetAttribute(attn_softmax_pv_kernel<KVM, 1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         bytes);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver the runtime loaded (no -lcuda)
EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (EncodeTiledFn) nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

}  // namespace

bool encode_v_map(CUtensorMap *map, const float *base, int kv_dim, int max_seq,
                  uint64_t planes, int head_dim, int box_pos) {
    const EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || !base || ((uintptr_t)base & 15) || (kv_dim & 3) || (head_dim & 3) ||
        head_dim > 256 || head_dim > kv_dim || max_seq <= 0 || planes == 0 ||
        planes > 0x7fffffffULL || box_pos < 1 || box_pos > 256)
        return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kv_dim, (cuuint64_t)max_seq, (cuuint64_t)planes};
    const cuuint64_t strides[2] = {(cuuint64_t)kv_dim * 4, (cuuint64_t)kv_dim * 4 * (cuuint64_t)max_seq};
    const cuuint32_t box[3] = {(cuuint32_t)head_dim, (cuuint32_t)box_pos, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_k_map(CUtensorMap *map, const float *base, int kv_dim, int max_seq,
                  uint64_t planes, int head_dim, int box_keys) {
    const EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || !base || ((uintptr_t)base & 15) || (kv_dim & 3) || (head_dim & 31) ||
        head_dim > kv_dim || max_seq <= 0 || planes == 0 || planes > 0x7fffffffULL)
        return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kv_dim, (cuuint64_t)max_seq, (cuuint64_t)planes};
    const cuuint64_t strides[2] = {(cuuint64_t)kv_dim * 4, (cuuint64_t)kv_dim * 4 * (cuuint64_t)max_seq};
    if (box_keys < 8 || box_keys > 256 || box_keys % 8) return false;
    const cuuint32_t box[3] = {32, (cuuint32_t)box_keys, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_att_map(CUtensorMap *map, const float *att, int att_ld, int heads, uint64_t rows,
                    int kv_mul) {
    const EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || !att || ((uintptr_t)att & 15) || (att_ld & 3) || att_ld < PPV_TT || kv_mul < 1 ||
        kv_mul > heads || heads > 256 || rows == 0 || rows > 0x7fffffffULL)
        return false;
    const cuuint64_t dims[3] = {(cuuint64_t)att_ld, (cuuint64_t)heads, (cuuint64_t)rows};
    const cuuint64_t strides[2] = {(cuuint64_t)att_ld * 4, (cuuint64_t)att_ld * 4 * (cuuint64_t)heads};
    const cuuint32_t box[3] = {(cuuint32_t)PPV_TT, (cuuint32_t)kv_mul, (cuuint32_t)PQT};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(att), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool attention_fused_ok(const AttnArgs &a) {
    const int kv_mul = a.num_heads / a.num_kv_heads;
    // the softmax+PV CTA: kv_mul*head_dim/2 consumer threads plus a producer warp, <= 512
    if (a.head_dim % 4 || kv_mul > 8 || kv_mul * a.head_dim > 960) return false;
    if (((uintptr_t)a.k_base | (uintptr_t)a.v_base) & 15) return false;
    if (!a.att) return false;  // the scores go through att
    if ((a.slot_stride | a.layer_off) & 3) return false;
    const size_t sk = sizeof(float) * ((size_t)TILE_KEYS * (a.head_dim + 4) + (size_t)kv_mul * a.head_dim);
    // the softmax + PV form that will run: per query head (modes 1, 2) with
    // its smallest ring, or the (row, KV head) forms
    const int pvm = a.pv_per_head;
    const size_t spv = (pvm == 1 || pvm == 2 || pvm == 10)
                           ? fused_shape(1, a.head_dim, a.max_len, PV_MIN_STAGES).smem
                       : pvm == 8             ? fused_shape(1, a.head_dim, a.max_len, PV_MIN_STAGES, 32).smem
                       : pvm == 9             ? fused_shape(1, a.head_dim, a.max_len, PV_MIN_STAGES, 16).smem
                       : pvm >= 3             ? fused_shape(kv_mul, a.head_dim, a.max_len, PV_MIN_STAGES).smem
                                              : fused_shape(kv_mul, a.head_dim, a.max_len).smem;
    return spv <= FUSED_SMEM_MAX && sk <= FUSED_SMEM_MAX;
}

void launch_attn_fused(const AttnArgs &args, const CUtensorMap &vmap, const CUtensorMap *kmap,
                       const CUtensorMap *amap, cudaStream_t s, const CUtensorMap *vmap_half,
                       const CUtensorMap *vmap_fine) {
    if (args.rows <= 0) return;
    if (args.prefill_tc && attn_prefill_tc_ok(args)) {
        launch_attn_prefill_tc(args, s);
        return;
    }
    AttnArgs a = args;
    const int kv_mul = a.num_heads / a.num_kv_heads;
    dim3 g1((a.max_len + TILE_KEYS - 1) / TILE_KEYS, a.num_kv_heads, a.rows);
    // the pipelined kernel bulk-copies the query vectors: 16-byte aligned rows
    const bool q_bulk = ((uintptr_t)a.q & 15) == 0 && (a.ldq & 3) == 0;
    const bool pipe = kmap && a.head_dim % 32 == 0 && q_bulk;
    const bool prefill_tiles = pipe && a.prefill_run > 0 && a.rows % a.prefill_run == 0 &&
                               (a.head_dim == 32 || a.head_dim == 64) && kv_mul <= 4;
    // the per-32-key maxima are made and used only by the two prefill kernels
    if (!(prefill_tiles && amap) || a.tmax_ld < (a.max_len + 31) / 32) a.tmax = nullptr;
    if (prefill_tiles) {
        // query-tiled: one K tile per PQT rows of a prompt
        const int run = a.prefill_run, nqt = (run + PQT - 1) / PQT;
        const int nkt = (a.max_len + TILE_KEYS - 1) / TILE_KEYS;
        const long long items = (long long)(a.rows / run) * nqt * a.num_kv_heads * nkt;
        const size_t sk = SCORE_STAGES * prefill_stage_bytes(kv_mul, a.head_dim) + 1024;
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int per_sm = (int)((200 * 1024) / sk) < 2 ? (int)((200 * 1024) / sk) : 2;
        long long grid = (long long)sms * (per_sm > 0 ? per_sm : 1);
        if (grid > items) grid = items;
        auto go = [&](auto kern) {
            launch_kernel(kern, dim3((unsigned)grid), dim3(TILE_KEYS + 32), sk, s, a.pdl, a, run, nqt,
                          nkt, *kmap);
        };
        if (a.head_dim == 32) {
            switch (kv_mul) {
                case 1: go(attn_prefill_scores_kernel<1, 32>); break;
                case 2: go(attn_prefill_scores_kernel<2, 32>); break;
                case 3: go(attn_prefill_scores_kernel<3, 32>); break;
                default: go(attn_prefill_scores_kernel<4, 32>); break;
            }
        } else {
            switch (kv_mul) {
                case 1: go(attn_prefill_scores_kernel<1, 64>); break;
                case 2: go(attn_prefill_scores_kernel<2, 64>); break;
                case 3: go(attn_prefill_scores_kernel<3, 64>); break;
                default: go(attn_prefill_scores_kernel<4, 64>); break;
            }
        }
    } else if (pipe) {
        // pipelined: a few CTAs per SM walk all (row, KV head, tile) items
        const int ntile_max = (a.max_len + TILE_KEYS - 1) / TILE_KEYS;
        const long long items = (long long)a.rows * a.num_kv_heads * ntile_max;
        const size_t sk = SCORE_STAGES * score_stage_bytes(kv_mul, a.head_dim) + 1024;
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        // as many CTAs as the SM's 228 KB of shared memory holds (1 KB of it
        // reserved per CTA), up to 3
        const int fit = (int)((228 * 1024) / (sk + 1024));
        const int per_sm = fit < 3 ? fit : 3;
        long long grid = (long long)sms * (per_sm > 0 ? per_sm : 1);
        if (grid > items) grid = items;
        launch_kernel(attn_scores_pipe_kernel, dim3((unsigned)grid), dim3(TILE_KEYS + 32), sk, s, a.pdl,
                      a, ntile_max, *kmap);
    } else {
        const size_t sk = sizeof(float) * ((size_t)TILE_KEYS * (a.head_dim + 4) + (size_t)kv_mul * a.head_dim);
        attn_scores_tiled_kernel<<<g1, TILE_KEYS, sk, s>>>(a);
    }
    if (prefill_tiles && amap) {
        // query-tiled softmax + PV, then the Q8_0 of the output if asked for
        // (the scores kernel above wrote the per-32-key maxima when a.tmax)
        const int run = a.prefill_run, nqt = (run + PQT - 1) / PQT;
        const size_t sp = PPV_STAGES * ppv_stage_bytes(kv_mul, a.head_dim) + 128;
        const dim3 grid((unsigned)nqt, (unsigned)a.num_kv_heads, (unsigned)(a.rows / run));
        auto go = [&](auto kern) {
            launch_kernel(kern, grid, dim3(PPV_CONS + 32), sp, s, a.pdl, a, run, vmap, *amap);
        };
        if (a.head_dim == 32) {
            switch (kv_mul) {
                case 1: go(attn_prefill_softmax_pv_kernel<1, 32>); break;
                case 2: go(attn_prefill_softmax_pv_kernel<2, 32>); break;
                case 3: go(attn_prefill_softmax_pv_kernel<3, 32>); break;
                default: go(attn_prefill_softmax_pv_kernel<4, 32>); break;
            }
        } else {
            switch (kv_mul) {
                case 1: go(attn_prefill_softmax_pv_kernel<1, 64>); break;
                case 2: go(attn_prefill_softmax_pv_kernel<2, 64>); break;
                case 3: go(attn_prefill_softmax_pv_kernel<3, 64>); break;
                default: go(attn_prefill_softmax_pv_kernel<4, 64>); break;
            }
        }
        if (a.q8_out.qs) launch_quantize_q8x(a.out, a.ldo, a.dim, a.q8_out, a.rows, s);
        return;
    }
    if ((a.pv_per_head == 6 || a.pv_per_head == 7) && vmap_half && KVM_GROUP_OK(kv_mul) && (a.head_dim == 64 || a.head_dim == 128) &&
        kv_mul * a.head_dim / 2 <= 480) {
        const bool nd2 = a.pv_per_head == 7;
        switch (kv_mul) {
            case 1: nd2 ? launch_softmax_pv_split<1, 2>(a, *vmap_half, s) : launch_softmax_pv_split<1, 1>(a, *vmap_half, s); break;
            case 2: nd2 ? launch_softmax_pv_split<2, 2>(a, *vmap_half, s) : launch_softmax_pv_split<2, 1>(a, *vmap_half, s); break;
            case 3: nd2 ? launch_softmax_pv_split<3, 2>(a, *vmap_half, s) : launch_softmax_pv_split<3, 1>(a, *vmap_half, s); break;
            default: nd2 ? launch_softmax_pv_split<4, 2>(a, *vmap_half, s) : launch_softmax_pv_split<4, 1>(a, *vmap_half, s); break;
        }
        return;
    }
    if (a.pv_per_head >= 3 && a.pv_per_head <= 5 && KVM_GROUP_OK(kv_mul) && kv_mul * a.head_dim <= 480) {
        switch (kv_mul) {
            case 1: launch_softmax_pv_group<1>(a, vmap, s); break;
            case 2: launch_softmax_pv_group<2>(a, vmap, s); break;
            case 3: launch_softmax_pv_group<3>(a, vmap, s); break;
            default: launch_softmax_pv_group<4>(a, vmap, s); break;
        }
        return;
    }
    if (a.pv_per_head == 10 && vmap_half && (a.head_dim == 64 || a.head_dim == 128)) {
        launch_softmax_pv_per_head_split(a, *vmap_half, s);
        return;
    }
    if ((a.pv_per_head == 8 || a.pv_per_head == 9) && vmap_fine) {
        // per query head, a thread per dim, 32- or 16-position stages
        if (a.pv_per_head == 8)
            launch_softmax_pv_per_head<1, 32>(a, *vmap_fine, s);
        else
            launch_softmax_pv_per_head<1, 16>(a, *vmap_fine, s);
        return;
    }
    if (a.pv_per_head) {
        if (a.pv_per_head == 2)
            launch_softmax_pv_per_head<2>(a, vmap, s);
        else
            launch_softmax_pv_per_head<1>(a, vmap, s);
        return;
    }
    switch (kv_mul) {
        case 1: launch_softmax_pv<1>(a, vmap, s); break;
        case 2: launch_softmax_pv<2>(a, vmap, s); break;
        case 3: launch_softmax_pv<3>(a, vmap, s); break;
        case 4: launch_softmax_pv<4>(a, vmap, s); break;
        case 5: launch_softmax_pv<5>(a, vmap, s); break;
        case 6: launch_softmax_pv<6>(a, vmap, s); break;
        case 7: launch_softmax_pv<7>(a, vmap, s); break;
        default: launch_softmax_pv<8>(a, vmap, s); break;
    }
}

void set_attention_smem_limit(int bytes) {
    set_attn_prefill_tc_smem();
    set_flash_decode_smem();
    set_attn_decode_cluster_smem();
    set_softmax_pv_smem<1>(bytes);
    set_softmax_pv_smem<2>(bytes);
    set_softmax_pv_smem<3>(bytes);
    set_softmax_pv_smem<4>(bytes);
    set_softmax_pv_smem<5>(bytes);
    set_softmax_pv_smem<6>(bytes);
    set_softmax_pv_smem<7>(bytes);
    set_softmax_pv_smem<8>(bytes);
    set_softmax_pv_split_smem<1>(bytes);
    set_softmax_pv_split_smem<2>(bytes);
    set_softmax_pv_split_smem<3>(bytes);
    set_softmax_pv_split_smem<4>(bytes);
    set_softmax_pv_group_smem<1>(bytes);
    set_softmax_pv_group_smem<2>(bytes);
    set_softmax_pv_group_smem<3>(bytes);
    set_softmax_pv_group_smem<4>(bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<1, 1, 1, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<1, 1, 1, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<1, 1, 2, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<1, 1, 2, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<1, 1, 1, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_softmax_pv_kernel<1, 1, 2, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    for (auto fn : {attn_softmax_pv_kernel<1, 1, 1, 64, 1, 32>, attn_softmax_pv_kernel<1, 1, 1, 128, 1, 32>,
                    attn_softmax_pv_kernel<1, 1, 1, 0, 1, 32>, attn_softmax_pv_kernel<1, 1, 1, 64, 1, 16>,
                    attn_softmax_pv_kernel<1, 1, 1, 128, 1, 16>, attn_softmax_pv_kernel<1, 1, 1, 0, 1, 16>})
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_scores_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_scores_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_scores_pipe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_softmax_pv_kernel<1, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_softmax_pv_kernel<2, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_softmax_pv_kernel<3, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_softmax_pv_kernel<4, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_softmax_pv_kernel<1, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_softmax_pv_kernel<2, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_softmax_pv_kernel<3, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_softmax_pv_kernel<4, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_scores_kernel<1, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_scores_kernel<2, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_scores_kernel<3, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_scores_kernel<4, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_scores_kernel<1, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_scores_kernel<2, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_scores_kernel<3, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(attn_prefill_scores_kernel<4, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
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

void launch_attention(const AttnArgs &a, const CUtensorMap *vmap, const CUtensorMap *kmap,
                      cudaStream_t s) {
    if (vmap && attention_fused_ok(a)) {
        launch_attn_fused(a, *vmap, kmap, nullptr, s);
        return;
    }
    launch_attn_scores(a, s);
    launch_attn_softmax(a, s);
    launch_attn_pv(a, s);
}

// ---- KV-head-sharded prefill: exchange layout ------------------------------

namespace {

__global__ void shard_pack_kernel(const float *x, size_t ldx, float *send, int nranks, int rank,
                                  int kvh, int kd, int n) {
    const int row = blockIdx.x, i = blockIdx.y;
    const int u = i * nranks + rank, s = u / kvh, g = u - s * kvh;
    const float *src = x + (size_t)(s * n + row) * ldx + (size_t)g * kd;
    float *dst = send + ((size_t)i * n + row) * kd;
    for (int c = threadIdx.x; c < kd; c += blockDim.x) dst[c] = src[c];
}

__global__ void shard_unpack_kernel(const float *recv, float *x, size_t ldx, int upr, int nranks,
                                    int kvh, int kd, int n) {
    const int row = blockIdx.x, i = blockIdx.y, q = blockIdx.z;
    const int u = i * nranks + q, s = u / kvh, g = u - s * kvh;
    const float *src = recv + (((size_t)q * upr + i) * n + row) * kd;
    float *dst = x + (size_t)(s * n + row) * ldx + (size_t)g * kd;
    for (int c = threadIdx.x; c < kd; c += blockDim.x) dst[c] = src[c];
}

}  // namespace

void launch_shard_pack(const float *x, size_t ldx, float *send, int units_per_rank, int nranks,
                       int rank, int kvh, int kd, int n, cudaStream_t s) {
    if (units_per_rank <= 0 || n <= 0) return;
    shard_pack_kernel<<<dim3((unsigned)n, (unsigned)units_per_rank), 128, 0, s>>>(x, ldx, send, nranks,
                                                                                 rank, kvh, kd, n);
}

void launch_shard_unpack(const float *recv, float *x, size_t ldx, int units_per_rank, int nranks,
                         int kvh, int kd, int n, cudaStream_t s) {
    if (units_per_rank <= 0 || n <= 0) return;
    shard_unpack_kernel<<<dim3((unsigned)n, (unsigned)units_per_rank, (unsigned)nranks), 128, 0, s>>>(
        recv, x, ldx, units_per_rank, nranks, kvh, kd, n);
}

}  // namespace slm
