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

constexpr int FD_KEYS = FD_ITEM_KEYS;  // keys per item (= V box positions)
constexpr int FD_CONS = 64;            // consumer threads: one per key of the item
constexpr int FD_THREADS = FD_CONS + 32;
constexpr int FD_STAGES = 3;
constexpr int FD_BAR_CONS = 1;         // named barrier of the consumer warps

struct FdItem {
    int r, g, c, nk;  // row, KV head, chunk, keys in the chunk; r < 0: end
};

template <int KVM, int HD>
struct FdSmem {
    static constexpr size_t k = (size_t)(HD / 32) * FD_KEYS * 128;  // swizzled K boxes
    static constexpr size_t v = (size_t)FD_KEYS * HD * 4;           // [key][dim]
    static constexpr size_t q = (size_t)KVM * HD * 4;
    static constexpr size_t stage = (k + v + q + 1023) / 1024 * 1024;  // K boxes 1024-aligned
    static constexpr size_t e = (size_t)KVM * FD_KEYS * 4;
    static constexpr size_t red = (size_t)KVM * 4 * 4;
    static constexpr size_t total = 1024 + FD_STAGES * stage + e + red;
};

template <int KVM, int HD>
__global__ void __launch_bounds__(FD_THREADS)
    attn_flash_decode_kernel(AttnArgs a, int nchm, const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap) {
    using SM = FdSmem<KVM, HD>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_full[FD_STAGES], bar_empty[FD_STAGES];
    __shared__ FdItem s_item[FD_STAGES];
    __shared__ int s_abort, s_issued;
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    float *s_e = reinterpret_cast<float *>(base + FD_STAGES * SM::stage);  // [KVM][FD_KEYS]
    float *s_red = s_e + KVM * FD_KEYS;                                    // [KVM][2] max, [KVM][2] sum
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long n_items = (long long)a.rows * a.num_kv_heads * nchm;
    constexpr unsigned stage_tx = (unsigned)(SM::k + SM::v + SM::q);
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
    if (warp == FD_CONS / 32 && lane == 0) {
        // every K and V box of this CTA's items into L2 at once (before the
        // wait: L2 is where the QKV kernel's newest rows land)
        for (long long it = blockIdx.x; it < n_items; it += gridDim.x) {
            const int c = (int)(it % nchm);
            const long long u = it / nchm;
            const int g = (int)(u % a.num_kv_heads), r = (int)(u / a.num_kv_heads);
            if (c * FD_KEYS >= row_len(a, r)) continue;
            const int z = (int)((long long)row_slot(a, r) * a.z_slot + a.z_layer);
            for (int b = 0; b < HD / 32; b++) tma_prefetch_3d(&kmap, g * HD + 32 * b, c * FD_KEYS, z);
            tma_prefetch_3d(&vmap, g * HD, c * FD_KEYS, z);
        }
    }
    __syncthreads();
    pdl_wait();  // q and each row's newest K/V come from the QKV kernel
    pdl_release();

    if (warp == FD_CONS / 32) {
        // ---- producer
        if (lane == 0) {
            int n = 0;
            for (long long it = blockIdx.x;; it += gridDim.x) {
                FdItem item{-1, 0, 0, 0};
                if (it < n_items) {
                    const int c = (int)(it % nchm);
                    const long long u = it / nchm;
                    item.g = (int)(u % a.num_kv_heads);
                    item.r = (int)(u / a.num_kv_heads);
                    const int L = row_len(a, item.r);
                    if (c * FD_KEYS >= L) continue;  // past this row's keys
                    item.c = c;
                    item.nk = L - c * FD_KEYS < FD_KEYS ? L - c * FD_KEYS : FD_KEYS;
                }
                const int st = n % FD_STAGES;
                if (n >= FD_STAGES &&
                    !mbar_wait(&bar_empty[st], (unsigned)((n / FD_STAGES) - 1) & 1u, &s_abort, a.err))
                    break;
                s_item[st] = item;
                if (item.r < 0) {
                    mbar_arrive(&bar_full[st]);  // end marker, no bytes
                    s_issued = n + 1;
                    break;
                }
                unsigned char *dst = base + (size_t)st * SM::stage;
                const int z = (int)((long long)row_slot(a, item.r) * a.z_slot + a.z_layer);
                const int t0 = item.c * FD_KEYS;
                mbar_arrive_expect_tx(&bar_full[st], stage_tx);
#pragma unroll
                for (int b = 0; b < HD / 32; b++)
                    tma_load_3d(dst + (size_t)b * FD_KEYS * 128, &kmap, item.g * HD + 32 * b, t0, z, &bar_full[st]);
                tma_load_3d(dst + SM::k, &vmap, item.g * HD, t0, z, &bar_full[st]);
                bulk_copy(dst + SM::k + SM::v, a.q + (size_t)item.r * a.ldq + (size_t)item.g * KVM * HD,
                          (unsigned)SM::q, &bar_full[st]);
                n++;
                s_issued = n;
            }
        }
        __syncwarp();
    } else {
        // ---- consumers
        for (int n = 0;; n++) {
            const int st = n % FD_STAGES;
            if (!mbar_wait(&bar_full[st], (unsigned)(n / FD_STAGES) & 1u, &s_abort, a.err)) break;
            const FdItem item = s_item[st];
            if (item.r < 0) break;
            const unsigned char *s_k = base + (size_t)st * SM::stage;
            const float *s_v = reinterpret_cast<const float *>(s_k + SM::k);
            const float4 *q4 = reinterpret_cast<const float4 *>(s_k + SM::k + SM::v);
            // scores of key tid for the KVM heads
            float s[KVM];
            {
                // four partial sums per head (x, y, z, w lanes of the float4s):
                // 4*KVM independent FMA chains
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
                    s[h] = tid < item.nk ? d * a.scale : -INFINITY;
                }
            }
            // chunk maximum and exp sums (NaN scores propagate as in the exact path)
#pragma unroll
            for (int h = 0; h < KVM; h++) {
                const float wm = warp_max_nan(s[h]);
                if (lane == 0) s_red[h * 2 + warp] = wm;
            }
            named_bar_or(FD_BAR_CONS, FD_CONS, false);
            float m[KVM], l[KVM];
#pragma unroll
            for (int h = 0; h < KVM; h++) {
                m[h] = fmax_nan(s_red[h * 2], s_red[h * 2 + 1]);
                const float e = tid < item.nk ? __expf(s[h] - m[h]) : 0.0f;
                s_e[h * FD_KEYS + tid] = e;
                float sum = e;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                if (lane == 0) s_red[KVM * 2 + h * 2 + warp] = sum;
            }
            named_bar_or(FD_BAR_CONS, FD_CONS, false);
#pragma unroll
            for (int h = 0; h < KVM; h++) l[h] = s_red[KVM * 2 + h * 2] + s_red[KVM * 2 + h * 2 + 1];
            // partial PV of dims tid, tid + 64, ...
            constexpr int DPT = HD / FD_CONS;  // dims per thread
            // two partial sums per output (even and odd keys)
            float o[KVM][DPT], o2[KVM][DPT];
#pragma unroll
            for (int h = 0; h < KVM; h++)
#pragma unroll
                for (int j = 0; j < DPT; j++) o[h][j] = o2[h][j] = 0.0f;
            const int nk4 = item.nk & ~3;
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
            for (int t = nk4; t < item.nk; t++) {
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
            // write the partial, then count the chunk in
            const size_t unit = (size_t)item.r * a.num_kv_heads + item.g;
            float *part = a.fd_part + (unit * a.fd_nch + item.c) * stride;
#pragma unroll
            for (int h = 0; h < KVM; h++)
#pragma unroll
                for (int j = 0; j < DPT; j++) part[h * HD + tid + FD_CONS * j] = o[h][j];
            if (tid < KVM) {
                part[KVM * HD + tid] = m[tid];
                part[KVM * HD + KVM + tid] = l[tid];
            }
            // s_e and s_red are read again only after the next item's first barrier
            named_bar_or(FD_BAR_CONS, FD_CONS, false);
        }
    }
    __syncthreads();
    if (s_abort && tid == 0) {
        // a wait gave up: let the copies already issued land (bounded)
        const int n_iss = s_issued;
        for (int k = n_iss - FD_STAGES < 0 ? 0 : n_iss - FD_STAGES; k < n_iss; k++) {
            const long long t0 = clock64();
            while (!mbar_test(&bar_full[k % FD_STAGES], (unsigned)(k / FD_STAGES) & 1u) &&
                   clock64() - t0 < WAIT_LIMIT) {
            }
        }
    }
}

// Combine of the chunk partials of one (row, KV head): thread (head h, dim d)
//   M = max_c m_c[h],  out = sum_c exp(m_c - M) o_c[h][d] / sum_c exp(m_c - M) l_c[h]
// then the Q8_0 of the KVM*HD output block (one 32-element block per warp).
template <int KVM, int HD>
__global__ void __launch_bounds__(KVM * HD)
    attn_flash_combine_kernel(AttnArgs a) {
    __shared__ float s_out[KVM * HD];
    constexpr size_t stride = (size_t)KVM * (HD + 2);
    const int g = blockIdx.x, r = blockIdx.y;
    const int tid = threadIdx.x, h = tid / HD, warp = tid >> 5, lane = tid & 31;
    const int nch = (row_len(a, r) + FD_KEYS - 1) / FD_KEYS;
    const float *p0 = a.fd_part + ((size_t)r * a.num_kv_heads + g) * a.fd_nch * stride;
    const float *pm = p0 + KVM * HD + h, *pl = pm + KVM;
    pdl_wait();  // the partials come from the chunk kernel
    // one pass over the chunks, eight at a time (their 24 loads in flight
    // together), rescaling the running sums when the maximum moves
    constexpr int CB = 8;
    float M = -INFINITY, num = 0.0f, den = 0.0f;
    for (int c = 0; c < nch; c += CB) {
        float m[CB], l[CB], o[CB];
#pragma unroll
        for (int u = 0; u < CB; u++) {
            const bool in = c + u < nch;
            m[u] = in ? pm[(c + u) * stride] : -INFINITY;
            l[u] = in ? pl[(c + u) * stride] : 0.0f;
            o[u] = in ? p0[(c + u) * stride + tid] : 0.0f;
        }
        float bm = m[0];
#pragma unroll
        for (int u = 1; u < CB; u++) bm = fmax_nan(bm, m[u]);
        const float Mn = fmax_nan(M, bm);
        const float sc = c == 0 ? 0.0f : __expf(M - Mn);
        num *= sc;
        den *= sc;
#pragma unroll
        for (int u = 0; u < CB; u++) {
            const float w = __expf(m[u] - Mn);
            num = __fmaf_rn(w, o[u], num);
            den = __fmaf_rn(w, l[u], den);
        }
        M = Mn;
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

template <int KVM, int HD>
void launch_fd(const AttnArgs &a, const CUtensorMap &kmap, const CUtensorMap &vmap, cudaStream_t s) {
    using SM = FdSmem<KVM, HD>;
    const int nchm = (a.max_len + FD_KEYS - 1) / FD_KEYS;
    const long long items = (long long)a.rows * a.num_kv_heads * nchm;
    const int per_sm = (int)((220 * 1024) / SM::total) > 0 ? (int)((220 * 1024) / SM::total) : 1;
    long long grid = (long long)sm_count_flash() * per_sm;
    if (grid > items) grid = items;
    launch_kernel(attn_flash_decode_kernel<KVM, HD>, dim3((unsigned)grid), dim3(FD_THREADS), SM::total, s, a.pdl,
                  a, nchm, kmap, vmap);
    launch_kernel(attn_flash_combine_kernel<KVM, HD>, dim3((unsigned)a.num_kv_heads, (unsigned)a.rows),
                  dim3(KVM * HD), 0, s, a.pdl, a);
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
