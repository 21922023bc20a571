// kernels_attn_flash.cu -- opt-in split-K flash-decode attention for decode
// rows (one query row per sequence at position pos, keys 0..pos), the
// tolerance-based counterpart of the exact decode path for
// causal_multi_head_attention_jit (src/model/transformer.rs:273-321).
//
// The exact path must run every PV sum as one sequential chain over all keys
// (the reference's order), so a (row, head) costs at least L dependent adds.
// Here the keys of each (row, KV head) are split into chunks of FD_ITEM_KEYS;
// for each chunk and each of the kv_mul query heads of the KV head
//   s_t = (q . k_t) * scale               (fused multiply-adds)
//   m   = max_t s_t,  e_t = exp(s_t - m),  l = sum_t e_t
//   o   = sum_t e_t * v_t
// is written as a partial (o, m, l); a second kernel combines the chunks of
// each (row, KV head):
//   M = max_c m_c,  w_c = exp(m_c - M),  out = sum_c w_c o_c / sum_c w_c l_c,
// and quantizes the output block to Q8_0 for the Wo GEMV.  The result
// differs from the exact path by rounding only (about 1e-6 relative).
//
// Chunk kernel, persistent and pipelined: a grid of a few CTAs per SM walks
// the (row, KV head, chunk) items.  In each CTA one producer thread fills a
// ring of FD_STAGES stages -- per item the K rows (hd/32 swizzled TMA boxes of
// 32 floats x 64 keys), the V rows (one TMA box of hd floats x 64 positions)
// and the kv_mul query vectors (one bulk copy) -- while two consumer warps
// compute the item a stage holds (thread t = key t for the scores, thread t =
// dims t, t+64, .. for the PV).  Every mbarrier wait is bounded.  The two
// kernels are ordered by the stream (programmatic dependent launch), so the
// chunk kernel needs no counters or fences of its own.
#include <cstdlib>

#include "async.cuh"
#include "attn_rows.cuh"
#include "kernels.h"

namespace slm {

namespace {

// maximum that returns NaN when either input is NaN
__device__ __forceinline__ float fmax_nan(float x, float y) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(x), "f"(y));
    return r;
}

constexpr int FD_KEYS = FD_ITEM_KEYS;  // keys per chunk (= V box positions)
constexpr int FD_CONS = 64;            // consumer threads: one per key of a chunk
constexpr int FD_THREADS = FD_CONS + 32;
#ifndef SLM_FD_STAGES
#define SLM_FD_STAGES 2
#endif
constexpr int FD_STAGES = SLM_FD_STAGES;
constexpr int FD_BAR_CONS = 1;         // named barrier of the consumer warps
constexpr int FD_CLUSTER_MAX = 8;      // splits merged inside a cluster (portable cluster size)

template <int KVM, int HD>
struct FdSmem {
    static constexpr size_t k = (size_t)(HD / 32) * FD_KEYS * 128;  // swizzled K boxes
    static constexpr size_t v = (size_t)FD_KEYS * HD * 4;           // [key][dim]
    static constexpr size_t stage = (k + v + 1023) / 1024 * 1024;   // K boxes 1024-aligned
    static constexpr size_t q = (size_t)KVM * HD * 4;
    static constexpr size_t e = (size_t)KVM * FD_KEYS * 4;
    static constexpr size_t o = (size_t)KVM * HD * 4;
    static constexpr size_t red = (size_t)KVM * 4 * 4;
    static constexpr size_t total = 1024 + FD_STAGES * stage + q + e + o + red;
};

// One CTA per (split s, KV head g, row r): chunks [c0, c1) of the row's keys,
// one after another through the ring, with the running maximum m, sum l and
// output o of every query head kept across chunks (online softmax: when a
// chunk raises m, l and o are scaled by exp(m_old - m_new)).  With one split
// the CTA writes the row's output and its Q8_0 directly; otherwise (o, m, l)
// goes to the partial buffer for the combine kernel -- or, with CL, the
// splits of a (row, KV head) are one thread-block cluster: each leaves its
// (o, m, l) in its own shared memory and rank 0 merges them through
// distributed shared memory (the combine kernel's arithmetic, in the same
// order) and writes the output and its Q8_0, so no second kernel runs.
template <int KVM, int HD, bool CL = false>
__global__ void __launch_bounds__(FD_THREADS)
    attn_flash_decode_kernel(AttnArgs a, int nsplit, const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap) {
    using SM = FdSmem<KVM, HD>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_full[FD_STAGES], bar_empty[FD_STAGES];
    __shared__ int s_abort, s_issued;
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    float *s_q = reinterpret_cast<float *>(base + FD_STAGES * SM::stage);  // [KVM][HD]
    float *s_e = s_q + KVM * HD;                                            // [KVM][FD_KEYS]
    float *s_o = s_e + KVM * FD_KEYS;                                       // [KVM*HD]
    float *s_red = s_o + KVM * HD;                                          // [KVM][2] max, [KVM][2] sum
    const int sp = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L = row_len(a, r);
    const int nch = (L + FD_KEYS - 1) / FD_KEYS;
    const int cps = (nch + nsplit - 1) / nsplit;  // chunks per split
    const int c0 = sp * cps, c1 = c0 + cps < nch ? c0 + cps : nch;
    // CTA-uniform: an empty split (the combine skips it; in a cluster it
    // takes part with an empty partial)
    if (!CL && c0 >= c1) return;
    const int nc = c1 > c0 ? c1 - c0 : 0;
    const int z = (int)((long long)row_slot(a, r) * a.z_slot + a.z_layer);
    constexpr unsigned stage_tx = (unsigned)(SM::k + SM::v);
    constexpr size_t stride = (size_t)KVM * (HD + 2);  // one partial: o[KVM][HD], m[KVM], l[KVM]

    if (tid == 0) {
        for (int st = 0; st < FD_STAGES; st++) {
            mbar_init(&bar_full[st], 1);
            mbar_init(&bar_empty[st], FD_CONS / 32);
        }
        s_abort = 0;
        s_issued = 0;
        mbar_fence_init();
    }
    __syncthreads();
    auto issue = [&](int i) {  // chunk c0 + i into stage i % FD_STAGES
        unsigned char *dst = base + (size_t)(i % FD_STAGES) * SM::stage;
        const int t0 = (c0 + i) * FD_KEYS;
        mbar_arrive_expect_tx(&bar_full[i % FD_STAGES], stage_tx);
#pragma unroll
        for (int b = 0; b < HD / 32; b++)
            tma_load_3d(dst + (size_t)b * FD_KEYS * 128, &kmap, g * HD + 32 * b, t0, z, &bar_full[i % FD_STAGES]);
        tma_load_3d(dst + SM::k, &vmap, g * HD, t0, z, &bar_full[i % FD_STAGES]);
    };
    if (warp == FD_CONS / 32 && lane == 0) {
        // chunks before the row's last were written by earlier steps: their
        // copies may start before the wait; the last one holds the row at pos
        int i = 0;
        for (; i < FD_STAGES && i < nc && c0 + i < nch - 1; i++) issue(i);
        s_issued = i;
    }
    pdl_wait();  // q and the row at pos come from the QKV kernel
    if (warp == FD_CONS / 32) {
        // ---- producer
        if (lane == 0) {
            int i = s_issued;
            for (; i < FD_STAGES && i < nc; i++) issue(i);
            for (; i < nc; i++) {
                if (!mbar_wait(&bar_empty[i % FD_STAGES], (unsigned)((i / FD_STAGES) - 1) & 1u, &s_abort, a.err))
                    break;
                issue(i);
            }
            s_issued = i;
        }
        __syncwarp();
    } else {
        // ---- consumers
        const float *qg = a.q + (size_t)r * a.ldq + (size_t)g * KVM * HD;
        for (int i = tid; i < KVM * HD; i += FD_CONS) s_q[i] = qg[i];
        named_bar_or(FD_BAR_CONS, FD_CONS, false);
        const float4 *q4 = reinterpret_cast<const float4 *>(s_q);
        constexpr int DPT = HD / FD_CONS;  // output dims per thread: tid, tid + 64, ...
        float mrun[KVM], lrun[KVM], o[KVM][DPT];
#pragma unroll
        for (int h = 0; h < KVM; h++) {
            mrun[h] = -INFINITY;
            lrun[h] = 0.0f;
#pragma unroll
            for (int j = 0; j < DPT; j++) o[h][j] = 0.0f;
        }
        for (int i = 0; i < nc; i++) {
            const int st = i % FD_STAGES;
            if (!mbar_wait(&bar_full[st], (unsigned)(i / FD_STAGES) & 1u, &s_abort, a.err)) break;
            const unsigned char *s_k = base + (size_t)st * SM::stage;
            const float *s_v = reinterpret_cast<const float *>(s_k + SM::k);
            const int nk = L - (c0 + i) * FD_KEYS < FD_KEYS ? L - (c0 + i) * FD_KEYS : FD_KEYS;
            // scores of key tid (four partial sums per head: 4*KVM FMA chains)
            float s[KVM];
            {
                float acc[KVM][4];
#pragma unroll
                for (int h = 0; h < KVM; h++)
#pragma unroll
                    for (int u = 0; u < 4; u++) acc[h][u] = 0.0f;
                const unsigned sw = (unsigned)(tid & 7);
#pragma unroll
                for (int b = 0; b < HD / 32; b++) {
                    const unsigned char *row = s_k + (size_t)b * FD_KEYS * 128 + (size_t)tid * 128;
#pragma unroll
                    for (int cc = 0; cc < 8; cc++) {
                        const float4 kk = *reinterpret_cast<const float4 *>(row + ((cc ^ sw) << 4));
#pragma unroll
                        for (int h = 0; h < KVM; h++) {
                            const float4 qq = q4[h * (HD / 4) + b * 8 + cc];
                            acc[h][0] = __fmaf_rn(qq.x, kk.x, acc[h][0]);
                            acc[h][1] = __fmaf_rn(qq.y, kk.y, acc[h][1]);
                            acc[h][2] = __fmaf_rn(qq.z, kk.z, acc[h][2]);
                            acc[h][3] = __fmaf_rn(qq.w, kk.w, acc[h][3]);
                        }
                    }
                }
#pragma unroll
                for (int h = 0; h < KVM; h++) {
                    const float d = (acc[h][0] + acc[h][1]) + (acc[h][2] + acc[h][3]);
                    s[h] = tid < nk ? d * a.scale : -INFINITY;
                }
            }
            // chunk maximum -> new running maximum (NaN scores propagate)
#pragma unroll
            for (int h = 0; h < KVM; h++) {
                const float wm = warp_max_nan(s[h]);
                if (lane == 0) s_red[h * 2 + warp] = wm;
            }
            named_bar_or(FD_BAR_CONS, FD_CONS, false);
            float scale[KVM];
#pragma unroll
            for (int h = 0; h < KVM; h++) {
                const float mn = fmax_nan(mrun[h], fmax_nan(s_red[h * 2], s_red[h * 2 + 1]));
                scale[h] = i == 0 ? 0.0f : __expf(mrun[h] - mn);
                mrun[h] = mn;
                const float e = tid < nk ? __expf(s[h] - mn) : 0.0f;
                s_e[h * FD_KEYS + tid] = e;
                float sum = e;
#pragma unroll
                for (int o2 = 16; o2 > 0; o2 >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o2);
                if (lane == 0) s_red[KVM * 2 + h * 2 + warp] = sum;
            }
            named_bar_or(FD_BAR_CONS, FD_CONS, false);
            // o = o * scale + sum_t e_t v_t (two partial sums: even / odd keys)
            float o2[KVM][DPT];
#pragma unroll
            for (int h = 0; h < KVM; h++) {
                lrun[h] = __fmaf_rn(lrun[h], scale[h], s_red[KVM * 2 + h * 2] + s_red[KVM * 2 + h * 2 + 1]);
#pragma unroll
                for (int j = 0; j < DPT; j++) {
                    o[h][j] *= scale[h];
                    o2[h][j] = 0.0f;
                }
            }
            const int nk4 = nk & ~3;
            for (int t = 0; t < nk4; t += 4) {
                float v[4][DPT];
#pragma unroll
                for (int u = 0; u < 4; u++)
#pragma unroll
                    for (int j = 0; j < DPT; j++) v[u][j] = s_v[(size_t)(t + u) * HD + tid + FD_CONS * j];
#pragma unroll
                for (int h = 0; h < KVM; h++) {
                    const float4 e4 = *reinterpret_cast<const float4 *>(s_e + h * FD_KEYS + t);
#pragma unroll
                    for (int j = 0; j < DPT; j++) {
                        o[h][j] = __fmaf_rn(e4.x, v[0][j], o[h][j]);
                        o2[h][j] = __fmaf_rn(e4.y, v[1][j], o2[h][j]);
                        o[h][j] = __fmaf_rn(e4.z, v[2][j], o[h][j]);
                        o2[h][j] = __fmaf_rn(e4.w, v[3][j], o2[h][j]);
                    }
                }
            }
            for (int t = nk4; t < nk; t++) {
#pragma unroll
                for (int h = 0; h < KVM; h++) {
                    const float e = s_e[h * FD_KEYS + t];
#pragma unroll
                    for (int j = 0; j < DPT; j++)
                        o[h][j] = __fmaf_rn(e, s_v[(size_t)t * HD + tid + FD_CONS * j], o[h][j]);
                }
            }
#pragma unroll
            for (int h = 0; h < KVM; h++)
#pragma unroll
                for (int j = 0; j < DPT; j++) o[h][j] += o2[h][j];
            // the stage is no longer read: hand it back to the producer
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_empty[st]);
            // s_e and s_red are written again only after the next chunk's first barrier
            named_bar_or(FD_BAR_CONS, FD_CONS, false);
        }
        if constexpr (CL) {
            // this split's partial, left in this CTA's shared memory
#pragma unroll
            for (int h = 0; h < KVM; h++)
#pragma unroll
                for (int j = 0; j < DPT; j++) s_o[h * HD + tid + FD_CONS * j] = o[h][j];
#pragma unroll
            for (int h = 0; h < KVM; h++)
                if (tid == h) {
                    s_red[h] = mrun[h];
                    s_red[KVM + h] = lrun[h];
                }
        } else if (!s_abort) {
            if (nsplit == 1) {
                float *orow = a.out + (size_t)r * a.ldo + (size_t)g * KVM * HD;
#pragma unroll
                for (int h = 0; h < KVM; h++)
#pragma unroll
                    for (int j = 0; j < DPT; j++) {
                        const int idx = h * HD + tid + FD_CONS * j;
                        const float res = o[h][j] / lrun[h];
                        s_o[idx] = res;
                        orow[idx] = res;
                    }
                if (a.q8_out.qs) {
                    named_bar_or(FD_BAR_CONS, FD_CONS, false);
                    const int nbr = a.dim / 32;
                    for (int blk = warp; blk < (KVM * HD) / 32; blk += FD_CONS / 32)
                        q8x_store_block(s_o[blk * 32 + lane], a.q8_out,
                                        (size_t)r * nbr + (size_t)(g * KVM * HD) / 32 + blk, lane);
                }
            } else {
                float *part = a.fd_part + (((size_t)r * a.num_kv_heads + g) * a.fd_nch + sp) * stride;
#pragma unroll
                for (int h = 0; h < KVM; h++)
#pragma unroll
                    for (int j = 0; j < DPT; j++) part[h * HD + tid + FD_CONS * j] = o[h][j];
#pragma unroll
                for (int h = 0; h < KVM; h++)
                    if (tid == h) {
                        part[KVM * HD + h] = mrun[h];
                        part[KVM * HD + KVM + h] = lrun[h];
                    }
            }
        }
    }
    if constexpr (CL) {
        __syncthreads();
        cluster_sync_all();  // every split's partial is in place
        if (cluster_rank() == 0) {
            const unsigned o_addr = smem_addr(s_o), r_addr = smem_addr(s_red);
            float *s_res = reinterpret_cast<float *>(base);  // the ring is no longer read
            for (int idx = tid; idx < KVM * HD; idx += FD_THREADS) {
                const int h = idx / HD;
                float M = -INFINITY;
                for (int c = 0; c < nsplit; c++) M = fmax_nan(M, cluster_ld(cluster_map(r_addr + 4u * h, c)));
                float num = 0.0f, den = 0.0f;
                for (int c = 0; c < nsplit; c++) {
                    const float w = __expf(cluster_ld(cluster_map(r_addr + 4u * h, c)) - M);
                    num = __fmaf_rn(w, cluster_ld(cluster_map(o_addr + 4u * idx, c)), num);
                    den = __fmaf_rn(w, cluster_ld(cluster_map(r_addr + 4u * (KVM + h), c)), den);
                }
                const float res = num / den;
                s_res[idx] = res;
                if (!s_abort) a.out[(size_t)r * a.ldo + (size_t)g * KVM * HD + idx] = res;
            }
            __syncthreads();
            if (a.q8_out.qs && !s_abort) {
                const int nbr = a.dim / 32;
                for (int blk = warp; blk < (KVM * HD) / 32; blk += FD_THREADS / 32)
                    q8x_store_block(s_res[blk * 32 + lane], a.q8_out,
                                    (size_t)r * nbr + (size_t)(g * KVM * HD) / 32 + blk, lane);
            }
        }
        cluster_sync_all();  // rank 0 has read every split's shared memory
    }
    pdl_release();
    __syncthreads();
    if (s_abort && tid == 0) {
        // a wait gave up: let the copies already issued land (bounded); the
        // error flag is set and this row's output is left as it was
        const int n_iss = s_issued;
        for (int k = n_iss - FD_STAGES < 0 ? 0 : n_iss - FD_STAGES; k < n_iss; k++) {
            const long long t0 = clock64();
            while (!mbar_test(&bar_full[k % FD_STAGES], (unsigned)(k / FD_STAGES) & 1u) &&
                   clock64() - t0 < WAIT_LIMIT) {
            }
        }
    }
}

// Combine of the splits of one (row, KV head): thread (head h, dim d)
//   M = max_s m_s[h],  out = sum_s exp(m_s - M) o_s[h][d] / sum_s exp(m_s - M) l_s[h]
// then the Q8_0 of the KVM*HD output block (one 32-element block per warp).
template <int KVM, int HD>
__global__ void __launch_bounds__(KVM * HD)
    attn_flash_combine_kernel(AttnArgs a, int nsplit) {
    __shared__ float s_out[KVM * HD];
    constexpr size_t stride = (size_t)KVM * (HD + 2);
    const int g = blockIdx.x, r = blockIdx.y;
    const int tid = threadIdx.x, h = tid / HD, warp = tid >> 5, lane = tid & 31;
    const int nch = (row_len(a, r) + FD_KEYS - 1) / FD_KEYS;
    const int cps = (nch + nsplit - 1) / nsplit;
    const int ns = (nch + cps - 1) / cps;  // splits that hold chunks
    const float *p0 = a.fd_part + ((size_t)r * a.num_kv_heads + g) * a.fd_nch * stride;
    const float *pm = p0 + KVM * HD + h, *pl = pm + KVM;
    pdl_wait();  // the partials come from the split kernel
    float M = -INFINITY;
    for (int c = 0; c < ns; c++) M = fmax_nan(M, pm[c * stride]);
    float num = 0.0f, den = 0.0f;
    for (int c = 0; c < ns; c++) {
        const float w = __expf(pm[c * stride] - M);
        num = __fmaf_rn(w, p0[c * stride + tid], num);
        den = __fmaf_rn(w, pl[c * stride], den);
    }
    const float res = num / den;
    pdl_release();
    a.out[(size_t)r * a.ldo + (size_t)g * KVM * HD + tid] = res;
    if (a.q8_out.qs) {
        s_out[tid] = res;
        __syncthreads();
        const int nbr = a.dim / 32;
        q8x_store_block(s_out[tid], a.q8_out, (size_t)r * nbr + (size_t)(g * KVM * HD) / 32 + warp, lane);
    }
}

int sm_count_flash() {
    static int sms = [] {
        int dev = 0, n = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        return n;
    }();
    return sms;
}

// SLM_FD_CLUSTER: 1 (default) merges 2..8 splits inside a cluster, 2 also caps
// the splits at 8 to do so, 0 always uses the combine kernel
int fd_cluster_mode() {
    const char *e = getenv("SLM_FD_CLUSTER");
    return e && e[0] >= '0' && e[0] <= '2' ? e[0] - '0' : 1;
}
bool fd_cluster(int ns) { return fd_cluster_mode() > 0 && ns > 1 && ns <= FD_CLUSTER_MAX; }

// Splits per (row, KV head): as many as the resident CTA slots allow (one CTA
// per (row, KV head) when those alone fill the GPU).
template <int KVM, int HD>
int fd_splits(const AttnArgs &a) {
    using SM = FdSmem<KVM, HD>;
    const int nchm = (a.max_len + FD_KEYS - 1) / FD_KEYS;
    const long long units = (long long)a.rows * a.num_kv_heads;
    const int fit = (int)((228 * 1024) / (SM::total + 1024));
    const long long slots = (long long)sm_count_flash() * (fit > 0 ? fit : 1);
    long long ns = units > 0 ? slots / units : 1;
    ns = ns < 1 ? 1 : ns > nchm ? nchm : ns;
    if (ns > a.fd_nch) ns = a.fd_nch;
    if (fd_cluster_mode() == 2 && ns > FD_CLUSTER_MAX) ns = FD_CLUSTER_MAX;
    return (int)ns;
}

template <int KVM, int HD>
void launch_fd(const AttnArgs &a, const CUtensorMap &kmap, const CUtensorMap &vmap, cudaStream_t s) {
    using SM = FdSmem<KVM, HD>;
    const int ns = fd_splits<KVM, HD>(a);
    const dim3 grid((unsigned)ns, (unsigned)a.num_kv_heads, (unsigned)a.rows);
    if (fd_cluster(ns)) {
        launch_kernel_cluster(attn_flash_decode_kernel<KVM, HD, true>, grid, dim3(FD_THREADS), SM::total, s, a.pdl,
                              (unsigned)ns, a, (int)ns, kmap, vmap);
        return;
    }
    launch_kernel(attn_flash_decode_kernel<KVM, HD>, grid, dim3(FD_THREADS), SM::total, s, a.pdl, a, (int)ns,
                  kmap, vmap);
    if (ns > 1)
        launch_kernel(attn_flash_combine_kernel<KVM, HD>, dim3((unsigned)a.num_kv_heads, (unsigned)a.rows),
                      dim3(KVM * HD), 0, s, a.pdl, a, (int)ns);
}

template <int HD>
void launch_fd_hd(const AttnArgs &a, const CUtensorMap &kmap, const CUtensorMap &vmap, cudaStream_t s) {
    switch (a.num_heads / a.num_kv_heads) {
        case 1: launch_fd<1, HD>(a, kmap, vmap, s); break;
        case 2: launch_fd<2, HD>(a, kmap, vmap, s); break;
        case 3: launch_fd<3, HD>(a, kmap, vmap, s); break;
        case 4: launch_fd<4, HD>(a, kmap, vmap, s); break;
        case 6: launch_fd<6, HD>(a, kmap, vmap, s); break;
        default: launch_fd<8, HD>(a, kmap, vmap, s); break;
    }
}

template <int KVM, int HD>
void set_fd_smem_one() {
    cudaFuncSetAttribute(attn_flash_decode_kernel<KVM, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)FdSmem<KVM, HD>::total);
    cudaFuncSetAttribute(attn_flash_decode_kernel<KVM, HD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)FdSmem<KVM, HD>::total);
}

template <int HD>
void set_fd_smem_hd() {
    set_fd_smem_one<1, HD>();
    set_fd_smem_one<2, HD>();
    set_fd_smem_one<3, HD>();
    set_fd_smem_one<4, HD>();
    set_fd_smem_one<6, HD>();
    set_fd_smem_one<8, HD>();
}

}  // namespace

int flash_decode_chunks(int max_seq) { return (max_seq + FD_KEYS - 1) / FD_KEYS; }

template <int HD>
int fd_splits_hd(const AttnArgs &a) {
    switch (a.num_heads / a.num_kv_heads) {
        case 1: return fd_splits<1, HD>(a);
        case 2: return fd_splits<2, HD>(a);
        case 3: return fd_splits<3, HD>(a);
        case 4: return fd_splits<4, HD>(a);
        case 6: return fd_splits<6, HD>(a);
        default: return fd_splits<8, HD>(a);
    }
}

int flash_decode_launches(const AttnArgs &a) {
    const int ns = a.head_dim == 64 ? fd_splits_hd<64>(a) : fd_splits_hd<128>(a);
    // the split kernel, and the combine when splits are not merged in a cluster
    return ns > 1 && !fd_cluster(ns) ? 2 : 1;
}

bool flash_decode_ok(const AttnArgs &a) {
    const int kvm = a.num_heads / a.num_kv_heads;
    const bool kvm_ok = kvm == 1 || kvm == 2 || kvm == 3 || kvm == 4 || kvm == 6 || kvm == 8;
    return kvm_ok && (a.head_dim == 64 || a.head_dim == 128) && a.fd_part &&
           a.fd_nch >= flash_decode_chunks(a.max_len) && (a.kv_dim & 3) == 0 && (a.ldq & 3) == 0 &&
           ((uintptr_t)a.q & 15) == 0 && ((uintptr_t)a.k_base & 15) == 0 && ((uintptr_t)a.v_base & 15) == 0 &&
           (kvm * a.head_dim) % 32 == 0 && a.shard_n <= 1;
}

void launch_flash_decode(const AttnArgs &a, const CUtensorMap &kmap64, const CUtensorMap &vmap, cudaStream_t s) {
    if (a.rows <= 0) return;
    if (a.head_dim == 64)
        launch_fd_hd<64>(a, kmap64, vmap, s);
    else
        launch_fd_hd<128>(a, kmap64, vmap, s);
}

void set_flash_decode_smem() {
    set_fd_smem_hd<64>();
    set_fd_smem_hd<128>();
}

}  // namespace slm
