// kernels_attn_cluster.cu -- exact decode attention in one launch: one
// thread-block cluster of C CTAs per (row, KV head), bit for bit the
// reference's causal_multi_head_attention_jit (src/model/transformer.rs:
// 273-321; softmax order graph.rs:168-179).
//
// The reference's numerics fix every chain: score_t is a sequential dot over
// the head's dims, the softmax a max / four lane sums / 1/sum, and out_d a
// sequential sum over t of p_t*v_t,d.  What is free is who runs each chain,
// and that is what the cluster splits:
//   scores: CTA c of the cluster computes the scores of its share of the keys
//           (32-key K tiles [c*nkt/C, (c+1)*nkt/C)) for the kv_mul query
//           heads of the KV head, a key per lane, and stores each score into
//           the score rows of every CTA of the cluster (distributed shared
//           memory), so after one cluster barrier every CTA holds all L
//           scores of every head without a trip through global memory;
//   softmax: each CTA runs it on its own copy (max, exp, the four lane
//           chains, 1/sum, p = e*inv) -- the same values in every CTA;
//   PV:     CTA c runs the chains of dims [c*HD/C, (c+1)*HD/C) of every head
//           over all L positions, V streamed as tiles of 32*C positions x
//           HD/C dims.
// K is read once (each CTA its keys) and V once (each CTA its dims), so one
// layer moves the algorithmic K+V bytes, and a row's chains are spread over C
// SMs: at 8 rows per GPU the 2049-step chains of a row run on 8 CTAs each.
//
// One producer warp streams K tiles (hd/32 boxes of 32 floats x 32 keys,
// 128-byte swizzle) and then V tiles through a single ring of equal stages;
// eight consumer warps take the K tiles (warp w the tiles w, w+wk, ..., so a
// stage always returns to the warp that last read it) and the PV warps the V
// tiles in order.  Every mbarrier wait is bounded; every thread of every CTA
// takes part in every cluster barrier, also after a wait gave up, so no CTA
// of a cluster can be left waiting for another.
#include <cstdlib>

#include "async.cuh"
#include "attn_rows.cuh"
#include "common.cuh"
#include "kernels.h"

namespace slm {

namespace {

constexpr int CL_KEYS = CL_BOX_KEYS;              // keys per K stage: a key per lane of a warp
static_assert(CL_KEYS == 32, "a K tile is one warp's keys");
constexpr int CL_WARPS = 8;                       // consumer warps
constexpr int CL_THREADS = CL_WARPS * 32 + 32;    // + the producer warp
constexpr int CL_MAX_STAGES = 16;
constexpr int CL_MAX = 8;                         // portable cluster size
constexpr int CL_BAR = 1;                         // named barrier of the consumer warps
constexpr size_t CL_SMEM_SM = 224 * 1024;         // shared memory an SM shares among its CTAs
constexpr size_t CL_SCORES_MAX = 96 * 1024;       // the score rows of one CTA, at most
// dynamic shared memory of one CTA, at most: the opt-in limit (227 KB) less
// the kernel's static shared memory, rounded down
constexpr size_t CL_SMEM_CTA = 200 * 1024;

struct ClShape {
    int lp;      // score row stride (floats)
    int nst;     // ring stages
    size_t smem; // dynamic shared memory (with 1 KB of alignment slack)
};

// stage bytes: one K tile (32 keys x hd floats) = one V tile (32*C positions x hd/C floats)
__host__ __device__ inline size_t cl_stage_bytes(int hd) { return (size_t)CL_KEYS * hd * 4; }

// floats of one products buffer of cluster size C (products mode): a row of
// 32*C + 4 positions per chain, kvm * hd / C chains
__host__ __device__ inline size_t cl_prod_floats(int kvm, int hd, int C) {
    return (size_t)kvm * (hd / C) * (CL_KEYS * C + 4);
}

__host__ __device__ inline ClShape cl_shape(int kvm, int hd, int max_len, int nst, size_t prod_floats = 0) {
    ClShape f;
    f.lp = (max_len + 31) / 32 * 32 + 4;
    f.nst = nst;
    f.smem = 1024 + (size_t)nst * cl_stage_bytes(hd) +
             sizeof(float) * ((size_t)kvm * f.lp + 2 * (size_t)kvm * hd + 64 + 2 * prod_floats);
    return f;
}

// K tile i of a CTA's share (i < nk) or V tile i - nk: is position L-1 in it?
// That row was written by the QKV kernel this launch follows.
__device__ __forceinline__ bool cl_tile_has_last(int i, int nk, int kt0, int ttv, int L) {
    return i < nk ? (kt0 + i + 1) * CL_KEYS >= L : (i - nk + 1) * ttv >= L;
}

// PM (products mode, ND = NH = 1): the consumer warps past the chain warps
// form the products p_t * v_t,d of each V tile into one of two buffers
// [chain][32*C + 4] and release the ring stage; a chain thread then only adds
// its row of products, four per 16-byte load, so its adds follow each other
// at the add latency.  The products are the same rounded values the direct
// form multiplies, added in the same order.
template <int KVM, int HD, int ND, int NH, bool PM = false>
__global__ void __launch_bounds__(CL_THREADS, 3)
    attn_decode_cluster_kernel(AttnArgs a, int lp, int nst, const __grid_constant__ CUtensorMap kmap,
                               const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_full[CL_MAX_STAGES], bar_empty[CL_MAX_STAGES];
    __shared__ __align__(8) uint64_t bar_pfull[2], bar_pempty[2];  // products buffers (PM)
    __shared__ int s_abort, s_issued;
    __shared__ float s_red[CL_WARPS * KVM + 8 * KVM];
    __shared__ float s_cmax[CL_MAX * KVM];  // maxima of each CTA's scores, by cluster rank
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr int SB = CL_KEYS * HD * 4;
    float *s_sc = reinterpret_cast<float *>(base + (size_t)nst * SB);  // [KVM][lp] scores, then p
    float *s_q = s_sc + (size_t)KVM * lp;                               // [KVM][HD]
    float *s_o = s_q + KVM * HD;                                        // [KVM][HD] outputs
    float *s_pr = s_o + KVM * HD + 64;                                  // PM: [2][chains][TTV + 4]
    const int C = (int)gridDim.x, c = (int)cluster_rank();
    const int g = blockIdx.y, r = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L = row_len(a, r);
    const int DC = HD / C;            // dims of this CTA's PV chains
    const int TTV = CL_KEYS * C;      // V positions per stage (DC * TTV floats = SB bytes)
    const int nkt = (L + CL_KEYS - 1) / CL_KEYS;
    const int kt0 = (int)((long long)nkt * c / C), kt1 = (int)((long long)nkt * (c + 1) / C);
    const int nk = kt1 - kt0;          // K tiles of this CTA
    const int nv = (L + TTV - 1) / TTV;  // V tiles
    const int ntot = nk + nv;
    const int wk = nst < CL_WARPS ? nst : CL_WARPS;  // K warps (nst <= 8 or a multiple of 8)
    const int npv = KVM * DC / (ND * NH);            // PV threads: (NH heads, ND dims) each
    const int npvw = (npv + 31) >> 5;                // PV warps (PM: the chain warps)
    const int nhw = PM ? CL_WARPS - npvw : 0;        // PM: the products warps
    const int nrel = PM ? nhw : npvw;                // arrivals that free a ring stage
    const int prow_ld = TTV + 4;                     // PM: products row stride (floats)
    const bool own_blocks = DC % 32 == 0;            // this CTA's outputs are whole Q8_0 blocks
    const int z = (int)((long long)row_slot(a, r) * a.z_slot + a.z_layer);

    if (tid == 0) {
        for (int st = 0; st < nst; st++) {
            mbar_init(&bar_full[st], 1);
            mbar_init(&bar_empty[st], (unsigned)nrel);
        }
        if (PM)
            for (int b = 0; b < 2; b++) {
                mbar_init(&bar_pfull[b], (unsigned)(nhw * 32));
                mbar_init(&bar_pempty[b], (unsigned)(npvw * 32));
            }
        s_abort = 0;
        s_issued = 0;
        mbar_fence_init();
    }
    __syncthreads();
    cluster_arrive_relaxed();  // (#0) this CTA runs: peers may store into its score rows after #0

    if (warp == CL_WARPS) {
        // ---- producer: the K tiles of this CTA's keys, then every V tile of its dims
        bool waited = false, crossed = false;
        for (int i = 0; i < ntot; i++) {
            if (i == nk) {
                // every K tile is issued: (#0) wait, (#1) arrive -- before any
                // wait on a stage that a PV warp frees, which happens after #1
                cluster_wait();
                cluster_arrive();
                crossed = true;
            }
            const int st = i % nst;
            if (i >= nst && !mbar_wait(&bar_empty[st], (unsigned)((i / nst) - 1) & 1u, &s_abort, a.err)) break;
            if (lane == 0) {
                if (!waited && cl_tile_has_last(i, nk, kt0, TTV, L)) {
                    pdl_wait();
                    waited = true;
                }
                unsigned char *dst = base + (size_t)st * SB;
                mbar_arrive_expect_tx(&bar_full[st], (unsigned)SB);
                if (i < nk) {
                    const int t0 = (kt0 + i) * CL_KEYS;
#pragma unroll
                    for (int b = 0; b < HD / 32; b++)
                        tma_load_3d(dst + (size_t)b * CL_KEYS * 128, &kmap, g * HD + 32 * b, t0, z, &bar_full[st]);
                } else {
                    tma_load_3d(dst, &vmap, g * HD + c * DC, (i - nk) * TTV, z, &bar_full[st]);
                }
                s_issued = i + 1;
            }
            __syncwarp();
        }
        if (!crossed) {
            cluster_wait();
            cluster_arrive();
        }
        cluster_wait();  // (#1)
        if (!own_blocks) {
            cluster_arrive();  // (#2)
            cluster_wait();
        }
    } else {
        // ---- consumers
        constexpr int nth = CL_WARPS * 32;
        pdl_wait();  // q comes from the QKV kernel
        const float *qg = a.q + (size_t)r * a.ldq + (size_t)g * KVM * HD;
        for (int j = tid; j < KVM * HD; j += nth) s_q[j] = qg[j];
        named_bar_sync(CL_BAR, nth);
        pdl_release();

        // scores of this CTA's keys, stored into the score rows of every CTA
        // of the cluster; key t = lane of a K tile, the kv_mul dot chains side
        // by side, each sequential over the head's dims
        bool synced0 = false;
        float wmax[KVM];  // this thread's largest score of each head (the max is order-free)
#pragma unroll
        for (int h = 0; h < KVM; h++) wmax[h] = -INFINITY;
        if (warp < wk) {
            const unsigned q_a = smem_addr(s_q);
            const unsigned sw = (unsigned)(lane & 7);
            for (int i = warp; i < nk; i += wk) {
                const int st = i % nst;
                if (!mbar_wait(&bar_full[st], (unsigned)(i / nst) & 1u, &s_abort, a.err)) break;
                const unsigned row = smem_addr(base) + (unsigned)(st * SB) + 128u * (unsigned)lane;
                float dot[KVM];
#pragma unroll
                for (int h = 0; h < KVM; h++) dot[h] = 0.0f;
#pragma unroll
                for (int b = 0; b < HD / 32; b++) {
#pragma unroll
                    for (int cc = 0; cc < 8; cc++) {
                        const float4 kk = lds_f32x4(row + (unsigned)(b * CL_KEYS * 128) + (((unsigned)cc ^ sw) << 4));
#pragma unroll
                        for (int h = 0; h < KVM; h++) {
                            const float4 qq = lds_f32x4(q_a + 16u * (unsigned)(h * (HD / 4) + b * 8 + cc));
                            dot[h] = __fadd_rn(dot[h], __fmul_rn(qq.x, kk.x));
                            dot[h] = __fadd_rn(dot[h], __fmul_rn(qq.y, kk.y));
                            dot[h] = __fadd_rn(dot[h], __fmul_rn(qq.z, kk.z));
                            dot[h] = __fadd_rn(dot[h], __fmul_rn(qq.w, kk.w));
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive_cnt(&bar_empty[st], (unsigned)nrel);  // the stage is free
                if (!synced0) {
                    cluster_wait();  // (#0): every CTA of the cluster runs
                    synced0 = true;
                }
                const int t = (kt0 + i) * CL_KEYS + lane;
                if (t < L) {
#pragma unroll
                    for (int h = 0; h < KVM; h++) {
                        const float sc = __fmul_rn(dot[h], a.scale);
                        wmax[h] = cl_fmax(wmax[h], sc);
                        const unsigned ad = smem_addr(s_sc + (size_t)h * lp + t);
                        for (int q = 0; q < C; q++) cluster_st(cluster_map(ad, (unsigned)q), sc);
                    }
                }
            }
        }
        if (!synced0) cluster_wait();  // (#0)
        // this CTA's maximum of each head, to every CTA of the cluster
        constexpr int MX = CL_WARPS * KVM, CH = MX + KVM, INV = CH + 4 * KVM;
#pragma unroll
        for (int h = 0; h < KVM; h++) {
            for (int o = 16; o > 0; o >>= 1) wmax[h] = cl_fmax(wmax[h], __shfl_xor_sync(0xffffffffu, wmax[h], o));
            if (lane == 0) s_red[h * CL_WARPS + warp] = wmax[h];
        }
        named_bar_sync(CL_BAR, nth);
        if (tid < KVM) {
            float mm = s_red[tid * CL_WARPS];
            for (int w = 1; w < CL_WARPS; w++) mm = cl_fmax(mm, s_red[tid * CL_WARPS + w]);
            const unsigned ad = smem_addr(s_cmax + c * KVM + tid);
            for (int q = 0; q < C; q++) cluster_st(cluster_map(ad, (unsigned)q), mm);
        }
        cluster_arrive();  // (#1): this CTA's scores and maxima are in every CTA
        cluster_wait();    // (#1): every CTA's are here

        // ---- softmax of every head on the full score rows (graph.rs:168-179)
        if (tid < KVM) {
            float mm = s_cmax[tid];
            for (int q = 1; q < C; q++) mm = cl_fmax(mm, s_cmax[q * KVM + tid]);
            s_red[MX + tid] = mm;
        }
        named_bar_sync(CL_BAR, nth);
#pragma unroll
        for (int h = 0; h < KVM; h++) {
            const float mx = s_red[MX + h];
            const unsigned row = smem_addr(s_sc) + 4u * (unsigned)(h * lp);
            constexpr unsigned s1 = 4u * nth;
            int t = tid;
            for (; t + 3 * nth < L; t += 4 * nth) {
                const unsigned at = row + 4u * (unsigned)t;
                const float x0 = lds_f32(at), x1 = lds_f32(at + s1), x2 = lds_f32(at + 2 * s1), x3 = lds_f32(at + 3 * s1);
                const float e0 = exp_poly(__fsub_rn(x0, mx)), e1 = exp_poly(__fsub_rn(x1, mx));
                const float e2 = exp_poly(__fsub_rn(x2, mx)), e3 = exp_poly(__fsub_rn(x3, mx));
                sts_f32(at, e0);
                sts_f32(at + s1, e1);
                sts_f32(at + 2 * s1, e2);
                sts_f32(at + 3 * s1, e3);
            }
            for (; t < L; t += nth) {
                const unsigned at = row + 4u * (unsigned)t;
                sts_f32(at, exp_poly(__fsub_rn(lds_f32(at), mx)));
            }
        }
        named_bar_sync(CL_BAR, nth);
        // lane chain l of head h (thread 4h + l of warp 0): e[l], e[l+4], ...
        // over [0, L & ~3) in order, its loads a group of 16 ahead of the adds
        const int vl = L & ~3;
        if (tid < 4 * KVM) {
            const int h = tid >> 2, l = tid & 3;
            const unsigned e0 = smem_addr(s_sc + (size_t)h * lp + l);
            const int n4 = vl >> 2;
            constexpr int G = 16;
            float cur[G], nxt[G];
            auto load = [&](int i, float (&v)[G]) {
#pragma unroll
                for (int u = 0; u < G; u++)
                    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v[u]) : "r"(e0 + 16u * (unsigned)(i + u)) : "memory");
            };
            float chain = 0.0f;
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
            const float *e = s_sc + (size_t)h * lp + l;
            for (; i < n4; i++) chain = __fadd_rn(chain, e[4 * i]);
            s_red[CH + tid] = chain;
        }
        named_bar_sync(CL_BAR, nth);
        if (tid < KVM) {
            const float *e = s_sc + (size_t)tid * lp;
            float sum = __fadd_rn(__fadd_rn(s_red[CH + 4 * tid], s_red[CH + 4 * tid + 1]),
                                  __fadd_rn(s_red[CH + 4 * tid + 2], s_red[CH + 4 * tid + 3]));
            for (int i = vl; i < L; i++) sum = __fadd_rn(sum, e[i]);
            s_red[INV + tid] = __fdiv_rn(1.0f, sum);
        }
        named_bar_sync(CL_BAR, nth);
#pragma unroll
        for (int h = 0; h < KVM; h++) {
            const float inv = s_red[INV + h];
            const unsigned row = smem_addr(s_sc) + 4u * (unsigned)(h * lp);
            constexpr unsigned s1 = 4u * nth;
            int t = tid;
            for (; t + 3 * nth < L; t += 4 * nth) {
                const unsigned at = row + 4u * (unsigned)t;
                const float x0 = lds_f32(at), x1 = lds_f32(at + s1), x2 = lds_f32(at + 2 * s1), x3 = lds_f32(at + 3 * s1);
                sts_f32(at, __fmul_rn(x0, inv));
                sts_f32(at + s1, __fmul_rn(x1, inv));
                sts_f32(at + 2 * s1, __fmul_rn(x2, inv));
                sts_f32(at + 3 * s1, __fmul_rn(x3, inv));
            }
            for (; t < L; t += nth) {
                const unsigned at = row + 4u * (unsigned)t;
                sts_f32(at, __fmul_rn(lds_f32(at), inv));
            }
        }
        named_bar_sync(CL_BAR, nth);

        // ---- out_d = sum_t p_t * v_t,d, sequential in t from 0.0: thread
        // (heads h0 .. h0+NH-1, dims d0 .. d0+ND-1 of this CTA's DC).  Within
        // a full tile the p and v values of the next G positions are loaded
        // before the adds of the current G, so the adds of a chain follow each
        // other at the add latency.
        const int dg = DC / ND;  // threads per head group
        const bool active = tid < npv;
        const int h0 = active ? (tid / dg) * NH : 0, d0 = (tid % dg) * ND;
        const unsigned ring_a = smem_addr(base), sc_a = smem_addr(s_sc);
        if (PM && warp >= npvw) {
            // products warps: tile j's products into buffer j & 1; items
            // (group of 4 positions, chain), chain fastest, so the stores of a
            // warp go to rows 16 bytes apart and the V loads to consecutive dims
            const int chains = KVM * DC, hthr = nhw * 32, ht = tid - npvw * 32;
            const int dlog = 31 - __clz(DC);                       // DC is a power of two
            const int dq = hthr / chains, dr = hthr - dq * chains;  // step between a thread's items
            const unsigned vs = 4u * (unsigned)DC;
            for (int j = 0; j < nv; j++) {
                const int i = nk + j, st = i % nst, b = j & 1;
                if (!mbar_wait(&bar_full[st], (unsigned)(i / nst) & 1u, &s_abort, a.err)) break;
                if (j >= 2 && !mbar_wait(&bar_pempty[b], (unsigned)((j >> 1) - 1) & 1u, &s_abort, a.err)) break;
                const unsigned vt = ring_a + (unsigned)(st * SB);  // [TTV][DC]
                const unsigned pr = smem_addr(s_pr) + 4u * (unsigned)(b * chains * prow_ld);
                const int t0 = j * TTV;
                const int n = L - t0 < TTV ? L - t0 : TTV;
                const int ng = (n + 3) >> 2;  // groups of 4 positions (reads stay below L + 3 <= lp)
                int gi = ht / chains, ch = ht - gi * chains;
                while (gi < ng) {
                    const int hh = ch >> dlog, d = ch & (DC - 1), u = 4 * gi;
                    const float4 p4 = lds_f32x4(sc_a + 4u * (unsigned)(hh * lp + t0 + u));
                    const unsigned va = vt + 4u * (unsigned)(u * DC + d);
                    float4 o;
                    o.x = __fmul_rn(p4.x, lds_f32(va));
                    o.y = __fmul_rn(p4.y, lds_f32(va + vs));
                    o.z = __fmul_rn(p4.z, lds_f32(va + 2u * vs));
                    o.w = __fmul_rn(p4.w, lds_f32(va + 3u * vs));
                    sts_f32x4(pr + 4u * (unsigned)(ch * prow_ld + u), o);
                    gi += dq;
                    ch += dr;
                    if (ch >= chains) {
                        ch -= chains;
                        gi++;
                    }
                }
                mbar_arrive(&bar_pfull[b]);
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar_empty[st]);  // the V stage is free
            }
        } else if (PM) {
            // chain warps: thread = (head, dim), its row of products in order,
            // the loads of the next 16 before the adds of the current 16
            const bool act = tid < npv;
            const int chains = KVM * DC;
            float acc = 0.0f;
            for (int j = 0; j < nv; j++) {
                const int b = j & 1;
                if (!mbar_wait(&bar_pfull[b], (unsigned)(j >> 1) & 1u, &s_abort, a.err)) break;
                const int n = L - j * TTV < TTV ? L - j * TTV : TTV;
                if (act) {
                    const unsigned row = smem_addr(s_pr) + 4u * (unsigned)((b * chains + tid) * prow_ld);
                    const int n16 = n & ~15;
                    float cur[16], nxt[16];
                    auto ld = [&](int u, float (&v)[16]) {
#pragma unroll
                        for (int k = 0; k < 16; k += 4) {
                            const float4 x = lds_f32x4(row + 4u * (unsigned)(u + k));
                            v[k] = x.x, v[k + 1] = x.y, v[k + 2] = x.z, v[k + 3] = x.w;
                        }
                    };
                    int u = 0;
                    if (n16 > 0) ld(0, cur);
                    for (; u + 32 <= n16; u += 32) {
                        ld(u + 16, nxt);
#pragma unroll
                        for (int k = 0; k < 16; k++) acc = __fadd_rn(acc, cur[k]);
                        if (u + 48 <= n16) ld(u + 32, cur);
#pragma unroll
                        for (int k = 0; k < 16; k++) acc = __fadd_rn(acc, nxt[k]);
                    }
                    if (u + 16 <= n16) {
#pragma unroll
                        for (int k = 0; k < 16; k++) acc = __fadd_rn(acc, cur[k]);
                        u += 16;
                    }
                    for (; u < n; u++) acc = __fadd_rn(acc, lds_f32(row + 4u * (unsigned)u));
                }
                mbar_arrive(&bar_pempty[b]);
            }
            if (act) {
                const int hh = tid / DC, d = tid - hh * DC;
                if (own_blocks)
                    s_o[hh * DC + d] = acc;
                else
                    cluster_st(cluster_map(smem_addr(s_o + hh * HD + c * DC + d), 0u), acc);
            }
        } else if (warp < npvw) {
            float acc[NH][ND];
#pragma unroll
            for (int hh = 0; hh < NH; hh++)
#pragma unroll
                for (int cc = 0; cc < ND; cc++) acc[hh][cc] = 0.0f;
            const unsigned pbase = sc_a + 4u * (unsigned)(h0 * lp);  // head h0 + hh at + 4 * hh * lp
            const unsigned vs = 4u * (unsigned)DC;
            for (int j = 0; j < nv; j++) {
                const int i = nk + j, st = i % nst;
                if (!mbar_wait(&bar_full[st], (unsigned)(i / nst) & 1u, &s_abort, a.err)) break;
                const unsigned vt = ring_a + (unsigned)(st * SB) + 4u * (unsigned)d0;  // row stride DC
                const int t0 = j * TTV;
                const unsigned pt = pbase + 4u * (unsigned)t0;
                const int n = L - t0 < TTV ? L - t0 : TTV;
                if (active) {
                    if (n == TTV) {
                        // G positions per register group: 8 with one head per
                        // thread, 4 with several (registers)
                        constexpr int G = NH > 1 ? 4 : 8;
                        float pa[NH][G], va[G][ND], pb[NH][G], vb[G][ND];
                        auto ld = [&](int u, float (&pp)[NH][G], float (&vv)[G][ND]) {
#pragma unroll
                            for (int hh = 0; hh < NH; hh++)
#pragma unroll
                                for (int k = 0; k < G; k += 4) {
                                    const float4 x = lds_f32x4(pt + 4u * (unsigned)(hh * lp + u + k));
                                    pp[hh][k] = x.x, pp[hh][k + 1] = x.y, pp[hh][k + 2] = x.z, pp[hh][k + 3] = x.w;
                                }
                            const unsigned v0 = vt + (unsigned)u * vs;
#pragma unroll
                            for (int k = 0; k < G; k++) {
                                if constexpr (ND == 2) {
                                    const float2 t2 = lds_f32x2(v0 + (unsigned)k * vs);
                                    vv[k][0] = t2.x;
                                    vv[k][1] = t2.y;
                                } else {
                                    vv[k][0] = lds_f32(v0 + (unsigned)k * vs);
                                }
                            }
                        };
                        auto add = [&](const float (&pp)[NH][G], const float (&vv)[G][ND]) {
#pragma unroll
                            for (int k = 0; k < G; k++)
#pragma unroll
                                for (int hh = 0; hh < NH; hh++)
#pragma unroll
                                    for (int cc = 0; cc < ND; cc++)
                                        acc[hh][cc] = __fadd_rn(acc[hh][cc], __fmul_rn(pp[hh][k], vv[k][cc]));
                        };
                        ld(0, pa, va);
                        // TTV = 32 * C is a multiple of 2 * G
                        for (int u = 0; u < TTV; u += 2 * G) {
                            ld(u + G, pb, vb);
                            add(pa, va);
                            if (u + 2 * G < TTV) ld(u + 2 * G, pa, va);
                            add(pb, vb);
                        }
                    } else {
                        for (int u = 0; u < n; u++) {
                            float vv[ND];
#pragma unroll
                            for (int cc = 0; cc < ND; cc++) vv[cc] = lds_f32(vt + (unsigned)u * vs + 4u * (unsigned)cc);
#pragma unroll
                            for (int hh = 0; hh < NH; hh++) {
                                const float pu = lds_f32(pt + 4u * (unsigned)(hh * lp + u));
#pragma unroll
                                for (int cc = 0; cc < ND; cc++) acc[hh][cc] = __fadd_rn(acc[hh][cc], __fmul_rn(pu, vv[cc]));
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar_empty[st]);
            }
            if (active) {
#pragma unroll
                for (int hh = 0; hh < NH; hh++)
#pragma unroll
                    for (int cc = 0; cc < ND; cc++) {
                        if (own_blocks)  // [KVM][DC]
                            s_o[(h0 + hh) * DC + d0 + cc] = acc[hh][cc];
                        else             // rank 0's [KVM][HD]
                            cluster_st(cluster_map(smem_addr(s_o + (h0 + hh) * HD + c * DC + d0 + cc), 0u),
                                       acc[hh][cc]);
                    }
            }
        }
        // ---- the output rows, and their Q8_0 blocks for the Wo GEMV
        const int nbr = a.dim / 32;
        if (own_blocks) {
            named_bar_sync(CL_BAR, nth);
            if (!s_abort) {
                float *orow = a.out + (size_t)r * a.ldo + (size_t)g * KVM * HD + (size_t)c * DC;
                for (int k = tid; k < KVM * DC; k += nth) orow[(size_t)(k / DC) * HD + k % DC] = s_o[k];
                if (a.q8_out.qs) {
                    const int bpc = DC / 32;  // blocks of a head in this CTA
                    for (int blk = warp; blk < KVM * bpc; blk += CL_WARPS)
                        q8x_store_block(s_o[blk * 32 + lane], a.q8_out,
                                        (size_t)r * nbr + ((size_t)(g * KVM + blk / bpc) * HD + (size_t)c * DC) / 32 +
                                            blk % bpc,
                                        lane);
                }
            }
        } else {
            // a CTA that gave up tells rank 0, which then leaves the outputs untouched
            if (s_abort && tid == 0)
                asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_map(smem_addr(&s_abort), 0u)), "r"(1)
                             : "memory");
            cluster_arrive();  // (#2): every CTA's outputs are in rank 0
            cluster_wait();
            if (c == 0 && !s_abort) {
                float *orow = a.out + (size_t)r * a.ldo + (size_t)g * KVM * HD;
                for (int k = tid; k < KVM * HD; k += nth) orow[k] = s_o[k];
                if (a.q8_out.qs)
                    for (int blk = warp; blk < KVM * HD / 32; blk += CL_WARPS)
                        q8x_store_block(s_o[blk * 32 + lane], a.q8_out,
                                        (size_t)r * nbr + (size_t)g * KVM * HD / 32 + blk, lane);
            }
        }
    }
    __syncthreads();
    if (s_abort && tid == 0) {
        // a wait gave up: let the copies already issued land (bounded) before
        // the shared memory is released
        const int n_iss = s_issued;
        for (int k = n_iss - nst < 0 ? 0 : n_iss - nst; k < n_iss; k++) {
            const long long t0 = clock64();
            while (!mbar_test(&bar_full[k % nst], (unsigned)(k / nst) & 1u) && clock64() - t0 < WAIT_LIMIT) {
            }
        }
    }
}

int sm_count_cached() {
    static const int n = [] {
        int dev = 0, v = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v;
    }();
    return n;
}

// Cluster size for `pairs` (row, KV head) pairs: the smallest power of two
// that gives about two CTAs per SM, at most 8, with head_dim / C a multiple
// of 4 floats (the V box's inner extent) and the PV threads within the eight
// consumer warps; SLM_CLUSTER_C (1, 2, 4, 8) overrides it for measurements
// (read at each launch, so a captured graph keeps the value of its capture).
int cl_cluster_size(long long pairs, int hd, int kvm) {
    const char *e = getenv("SLM_CLUSTER_C");
    const int ev = e ? atoi(e) : 0;
    const int env = ev == 1 || ev == 2 || ev == 4 || ev == 8 ? ev : 0;
    int C = 1;
    if (env) {
        C = env;
    } else {
        while (C < CL_MAX && pairs * C < 2LL * sm_count_cached()) C *= 2;
    }
    while (C > 1 && (hd / C) % 4 != 0) C /= 2;
    while (C < CL_MAX && kvm * (hd / C) > 2 * CL_WARPS * 32) C *= 2;  // two chains per thread at most
    return C;
}

}  // namespace

bool attn_decode_cluster_ok(const AttnArgs &a) {
    const int kvm = a.num_heads / a.num_kv_heads;
    if (a.rows <= 0 || a.prefill_run > 0 || a.write_probs || a.shard_n > 1) return false;
    if ((a.head_dim != 64 && a.head_dim != 128) || kvm < 1 || kvm > 4) return false;
    if (a.num_heads != kvm * a.num_kv_heads) return false;
    return cl_shape(kvm, a.head_dim, a.max_len, 0).smem - 1024 <= CL_SCORES_MAX;
}

int attn_decode_cluster_size(const AttnArgs &a) {
    if (!attn_decode_cluster_ok(a)) return 0;
    return cl_cluster_size((long long)a.rows * a.num_kv_heads, a.head_dim, a.num_heads / a.num_kv_heads);
}

namespace {

// Ring depth: the shared memory an SM has, shared by the CTAs it holds when
// the grid is spread evenly, in whole stages (2 to CL_MAX_STAGES; above 8 a
// multiple of 8 so that a stage always returns to the same K warp).
ClShape cl_plan(const AttnArgs &a, int C, bool pm) {
    const int kvm = a.num_heads / a.num_kv_heads, hd = a.head_dim;
    const long long ctas = (long long)a.rows * a.num_kv_heads * C;
    const long long per_sm = (ctas + sm_count_cached() - 1) / sm_count_cached();
    const size_t budget = CL_SMEM_SM / (size_t)(per_sm < 1 ? 1 : per_sm);
    const size_t pf = pm ? cl_prod_floats(kvm, hd, C) : 0;
    const size_t fixed = cl_shape(kvm, hd, a.max_len, 0, pf).smem, sb = cl_stage_bytes(hd);
    long long nst = budget > fixed ? (long long)((budget - fixed) / sb) : 0;
    nst = nst < 2 ? 2 : nst > CL_MAX_STAGES ? CL_MAX_STAGES : nst;
    while (nst > 2 && fixed + (size_t)nst * sb > CL_SMEM_CTA) nst--;
    if (nst > CL_WARPS) nst = nst / CL_WARPS * CL_WARPS;
    return cl_shape(kvm, hd, a.max_len, (int)nst, pf);
}

// Products mode: SLM_CLUSTER_PM = 0 / 1 forces it; by default from the
// batches that put at most two CTAs on an SM (the PV is then bound by the
// length of the chains), when one thread per chain leaves a products warp
// and the buffers leave room for three ring stages.
bool cl_pm(const AttnArgs &a, int C) {
    const int kvm = a.num_heads / a.num_kv_heads, hd = a.head_dim;
    if (kvm * (hd / C) > (CL_WARPS - 1) * 32) return false;
    const char *e = getenv("SLM_CLUSTER_PM");
    bool want;
    if (e && (e[0] == '0' || e[0] == '1')) {
        want = e[0] == '1';
    } else {
        const long long ctas = (long long)a.rows * a.num_kv_heads * C;
        want = ctas <= 2LL * sm_count_cached();
    }
    if (!want) return false;
    // three ring stages within this CTA's share of the SM (the grid in one wave)
    const long long ctas = (long long)a.rows * a.num_kv_heads * C;
    const long long per_sm = (ctas + sm_count_cached() - 1) / sm_count_cached();
    const size_t share = CL_SMEM_SM / (size_t)(per_sm < 1 ? 1 : per_sm);
    const size_t need = cl_shape(kvm, hd, a.max_len, 3, cl_prod_floats(kvm, hd, C)).smem;
    return need <= CL_SMEM_CTA && need <= share;
}

int cl_env_nd() {
    const char *e = getenv("SLM_CLUSTER_ND");
    return e && atoi(e) == 2 ? 2 : 1;
}
// heads per PV thread: SLM_CLUSTER_NH = 1 or "all" (kv_mul); unset: every
// head from 2 CTAs per SM up (the PV is then bound by shared-memory
// wavefronts), one head per thread below (bound by the length of the chains)
int cl_nh(const AttnArgs &a, int C) {
    const char *e = getenv("SLM_CLUSTER_NH");
    if (e && e[0] == '1') return 1;
    if (e && e[0] == 'a') return a.num_heads / a.num_kv_heads;
    const long long ctas = (long long)a.rows * a.num_kv_heads * C;
    return ctas >= 2LL * sm_count_cached() ? a.num_heads / a.num_kv_heads : 1;
}

// PV thread shapes: (ND, NH) = (1, 1) a thread per (head, dim); (2, 1) per
// (head, dim pair); (1, KVM) per dim running every head of the group (V
// loaded once for all heads: fewer shared-memory wavefronts per position)
template <int KVM, int HD>
void cl_go(const AttnArgs &a, const ClShape &f, int C, int nd, int nh, bool pm, const CUtensorMap &kmap,
           const CUtensorMap &vmap, cudaStream_t s) {
    const dim3 grid((unsigned)C, (unsigned)a.num_kv_heads, (unsigned)a.rows), block(CL_THREADS);
    if (pm)
        launch_kernel_cluster(attn_decode_cluster_kernel<KVM, HD, 1, 1, true>, grid, block, f.smem, s, a.pdl,
                              (unsigned)C, a, f.lp, f.nst, kmap, vmap);
    else if (nh > 1)
        launch_kernel_cluster(attn_decode_cluster_kernel<KVM, HD, 1, KVM>, grid, block, f.smem, s, a.pdl,
                              (unsigned)C, a, f.lp, f.nst, kmap, vmap);
    else if (nd == 2)
        launch_kernel_cluster(attn_decode_cluster_kernel<KVM, HD, 2, 1>, grid, block, f.smem, s, a.pdl, (unsigned)C,
                              a, f.lp, f.nst, kmap, vmap);
    else
        launch_kernel_cluster(attn_decode_cluster_kernel<KVM, HD, 1, 1>, grid, block, f.smem, s, a.pdl, (unsigned)C,
                              a, f.lp, f.nst, kmap, vmap);
}

template <int KVM>
void cl_go_hd(const AttnArgs &a, const ClShape &f, int C, int nd, int nh, bool pm, const CUtensorMap &kmap,
              const CUtensorMap &vmap, cudaStream_t s) {
    if (a.head_dim == 64)
        cl_go<KVM, 64>(a, f, C, nd, nh, pm, kmap, vmap, s);
    else
        cl_go<KVM, 128>(a, f, C, nd, nh, pm, kmap, vmap, s);
}

template <int KVM>
void cl_set_smem() {
    for (auto fn : {attn_decode_cluster_kernel<KVM, 64, 1, 1>, attn_decode_cluster_kernel<KVM, 64, 2, 1>,
                    attn_decode_cluster_kernel<KVM, 64, 1, KVM>, attn_decode_cluster_kernel<KVM, 128, 1, 1>,
                    attn_decode_cluster_kernel<KVM, 128, 2, 1>, attn_decode_cluster_kernel<KVM, 128, 1, KVM>,
                    attn_decode_cluster_kernel<KVM, 64, 1, 1, true>, attn_decode_cluster_kernel<KVM, 128, 1, 1, true>})
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CL_SMEM_CTA);
}

}  // namespace

bool attn_decode_cluster_preferred(const AttnArgs &a) {
    const int C = attn_decode_cluster_size(a);
    return C > 0 && cl_pm(a, C);
}

void launch_attn_decode_cluster(const AttnArgs &a, const CUtensorMap &kmap32, const CUtensorMap &vmap_c, int C,
                                cudaStream_t s) {
    const int kvm = a.num_heads / a.num_kv_heads;
    const bool pm = cl_pm(a, C);
    const ClShape f = cl_plan(a, C, pm);
    const int nh = pm ? 1 : cl_nh(a, C);
    const int nd = pm ? 1 : nh == 1 && kvm * (a.head_dim / C) > CL_WARPS * 32 ? 2 : cl_env_nd();
    switch (kvm) {
        case 1: cl_go_hd<1>(a, f, C, nd, nh, pm, kmap32, vmap_c, s); break;
        case 2: cl_go_hd<2>(a, f, C, nd, nh, pm, kmap32, vmap_c, s); break;
        case 3: cl_go_hd<3>(a, f, C, nd, nh, pm, kmap32, vmap_c, s); break;
        default: cl_go_hd<4>(a, f, C, nd, nh, pm, kmap32, vmap_c, s); break;
    }
}

void set_attn_decode_cluster_smem() {
    cl_set_smem<1>();
    cl_set_smem<2>();
    cl_set_smem<3>();
    cl_set_smem<4>();
}

}  // namespace slm
