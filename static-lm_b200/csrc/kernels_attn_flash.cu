// kernels_attn_flash.cu -- opt-in split-K flash-decode attention for decode
// rows (one query row per sequence at position pos, keys 0..pos), the
// tolerance-based counterpart of the exact decode path for
// causal_multi_head_attention_jit (src/model/transformer.rs:273-321).
//
// The exact path must run every PV sum as one sequential chain over all keys
// (the reference's order), so a (row, head) costs at least L dependent adds.
// Here the keys are split into chunks of FD_KEYS; one CTA per (chunk, KV
// head, row) computes, for each of the kv_mul query heads of the KV head,
//   s_t = (q . k_t) * scale               (fused multiply-adds)
//   m   = max_t s_t,  e_t = exp(s_t - m),  l = sum_t e_t
//   o   = sum_t e_t * v_t
// over its chunk and writes (o, m, l); the CTA that finishes last for a
// (row, KV head) combines the chunks:
//   M = max_c m_c,  w_c = exp(m_c - M),  out = sum_c w_c o_c / sum_c w_c l_c.
// The result differs from the exact path by rounding only (about 1e-6
// relative); greedy tokens can differ where Q8_0 quantization of the output
// turns such a difference into a different int8 value near a tie.
//
// K arrives as hd/32 swizzled TMA boxes of 32 floats x 128 keys (the decode K
// tensor map), V as two boxes of hd floats x 64 positions (the V tensor map),
// both on one mbarrier.  Chunks before the row's last were written by earlier
// decode steps and are fetched before griddepcontrol.wait; the last chunk
// holds the row written by the QKV kernel this one follows, so it is fetched
// after the wait.  Every wait is bounded.
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

constexpr int FD_KEYS = K_BOX_KEYS;  // keys per CTA: one K box of the tensor map
constexpr int FD_THREADS = 128;  // scores: thread t = key t of the chunk

template <int KVM, int HD>
struct FdSmem {
    static constexpr size_t k = (size_t)(HD / 32) * FD_KEYS * 128;  // swizzled K boxes
    static constexpr size_t v = (size_t)FD_KEYS * HD * 4;           // [key][dim]
    static constexpr size_t q = (size_t)KVM * HD * 4;
    static constexpr size_t e = (size_t)KVM * FD_KEYS * 4;
    static constexpr int groups = FD_THREADS / HD > 0 ? FD_THREADS / HD : 1;
    static constexpr size_t o = (size_t)groups * KVM * HD * 4;
    static constexpr size_t red = (size_t)KVM * 8 * 4 * 2;
    // 1024 bytes of slack: the swizzled K boxes start on a 1024-byte boundary
    static constexpr size_t total = 1024 + k + v + q + e + o + red;
};

template <int KVM, int HD>
__global__ void __launch_bounds__(FD_THREADS)
    attn_flash_decode_kernel(AttnArgs a, const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap) {
    using SM = FdSmem<KVM, HD>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ int s_abort, s_last;
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    unsigned char *s_k = base;
    float *s_v = reinterpret_cast<float *>(base + SM::k);
    float *s_q = reinterpret_cast<float *>(base + SM::k + SM::v);
    float *s_e = s_q + KVM * HD;                 // [KVM][FD_KEYS]
    float *s_o = s_e + KVM * FD_KEYS;            // [groups][KVM][HD]
    float *s_red = s_o + SM::groups * KVM * HD;  // [KVM][4 warps] max, then sum

    const int c = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L = row_len(a, r);
    const int t0 = c * FD_KEYS;
    if (t0 >= L) return;  // CTA-uniform: past this row's keys
    const int nch = (L + FD_KEYS - 1) / FD_KEYS;
    const int nk = L - t0 < FD_KEYS ? L - t0 : FD_KEYS;
    // plane of this row's layer in both tensor maps (K from the K base, V from the V base)
    const int z = (int)((long long)row_slot(a, r) * a.z_slot + a.z_layer);
    constexpr unsigned tile_bytes = (unsigned)(SM::k + SM::v);

    if (tid == 0) {
        mbar_init(&bar, 1);
        s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    auto issue = [&] {
        mbar_arrive_expect_tx(&bar, tile_bytes);
#pragma unroll
        for (int b = 0; b < HD / 32; b++)
            tma_load_3d(s_k + (size_t)b * FD_KEYS * 128, &kmap, g * HD + 32 * b, t0, z, &bar);
#pragma unroll
        for (int b = 0; b < FD_KEYS / V_BOX_POSITIONS; b++)
            tma_load_3d(s_v + (size_t)b * V_BOX_POSITIONS * HD, &vmap, g * HD, t0 + b * V_BOX_POSITIONS, z, &bar);
    };
    if (tid == 0 && c < nch - 1) issue();
    pdl_wait();  // q and the row at pos come from the QKV kernel
    if (tid == 0 && c == nch - 1) issue();
    const float *qg = a.q + (size_t)r * a.ldq + (size_t)g * KVM * HD;
    for (int i = tid; i < KVM * HD; i += FD_THREADS) s_q[i] = qg[i];
    __syncthreads();
    pdl_release();
    if (!mbar_wait(&bar, 0u, &s_abort, a.err)) {
        // gave up: let the copies land (bounded) before the CTA exits; the
        // error flag is set, the output of this row is left as it was
        if (tid == 0) {
            const long long tw = clock64();
            while (!mbar_test(&bar, 0u) && clock64() - tw < WAIT_LIMIT) {
            }
        }
        __syncthreads();
        return;
    }

    // ---- scores of key t0 + tid for the KVM heads
    float s[KVM];
    {
        float acc[KVM];
#pragma unroll
        for (int h = 0; h < KVM; h++) acc[h] = 0.0f;
        const unsigned sw = (unsigned)(tid & 7);
        const float4 *q4 = reinterpret_cast<const float4 *>(s_q);
#pragma unroll
        for (int b = 0; b < HD / 32; b++) {
            const unsigned char *row = s_k + (size_t)b * FD_KEYS * 128 + (size_t)tid * 128;
#pragma unroll
            for (int cc = 0; cc < 8; cc++) {
                const float4 kk = *reinterpret_cast<const float4 *>(row + ((cc ^ sw) << 4));
#pragma unroll
                for (int h = 0; h < KVM; h++) {
                    const float4 qq = q4[h * (HD / 4) + b * 8 + cc];
                    acc[h] = __fmaf_rn(qq.x, kk.x, acc[h]);
                    acc[h] = __fmaf_rn(qq.y, kk.y, acc[h]);
                    acc[h] = __fmaf_rn(qq.z, kk.z, acc[h]);
                    acc[h] = __fmaf_rn(qq.w, kk.w, acc[h]);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < KVM; h++) s[h] = tid < nk ? acc[h] * a.scale : -INFINITY;
    }
    // ---- chunk maximum and exp sums (NaN scores propagate as in the exact path)
    float m[KVM], l[KVM];
#pragma unroll
    for (int h = 0; h < KVM; h++) {
        const float wm = warp_max_nan(s[h]);
        if (lane == 0) s_red[h * 4 + warp] = wm;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < KVM; h++) {
        float mm = s_red[h * 4];
#pragma unroll
        for (int w = 1; w < FD_THREADS / 32; w++) mm = fmax_nan(mm, s_red[h * 4 + w]);
        m[h] = mm;
        const float e = tid < nk ? __expf(s[h] - mm) : 0.0f;
        s_e[h * FD_KEYS + tid] = e;
        float sum = e;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) s_red[KVM * 4 + h * 4 + warp] = sum;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < KVM; h++) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < FD_THREADS / 32; w++) sum += s_red[KVM * 4 + h * 4 + w];
        l[h] = sum;
    }

    // ---- partial PV: thread (dim d, key group grp) over its keys
    {
        constexpr int G = SM::groups;
        constexpr int KPG = FD_KEYS / G;  // keys per group
        for (int idx = tid; idx < G * HD; idx += FD_THREADS) {
            const int d = idx % HD, grp = idx / HD;
            const int k0 = grp * KPG, k1 = (k0 + KPG < nk) ? k0 + KPG : nk;
            float o[KVM];
#pragma unroll
            for (int h = 0; h < KVM; h++) o[h] = 0.0f;
            int t = k0;
            for (; t + 4 <= k1; t += 4) {
                float v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) v[u] = s_v[(size_t)(t + u) * HD + d];
#pragma unroll
                for (int h = 0; h < KVM; h++) {
                    const float4 e4 = *reinterpret_cast<const float4 *>(s_e + h * FD_KEYS + t);
                    o[h] = __fmaf_rn(e4.x, v[0], o[h]);
                    o[h] = __fmaf_rn(e4.y, v[1], o[h]);
                    o[h] = __fmaf_rn(e4.z, v[2], o[h]);
                    o[h] = __fmaf_rn(e4.w, v[3], o[h]);
                }
            }
            for (; t < k1; t++) {
                const float v = s_v[(size_t)t * HD + d];
#pragma unroll
                for (int h = 0; h < KVM; h++) o[h] = __fmaf_rn(s_e[h * FD_KEYS + t], v, o[h]);
            }
#pragma unroll
            for (int h = 0; h < KVM; h++) s_o[(grp * KVM + h) * HD + d] = o[h];
        }
    }
    __syncthreads();

    float *orow = a.out + (size_t)r * a.ldo + (size_t)g * KVM * HD;
    if (nch == 1) {
        // one chunk: the chunk's result is the row's
        for (int i = tid; i < KVM * HD; i += FD_THREADS) {
            const int h = i / HD;
            float o = 0.0f;
#pragma unroll
            for (int grp = 0; grp < SM::groups; grp++) o += s_o[grp * KVM * HD + i];
            const float res = o / l[h];
            s_o[i] = res;  // group 0's slot, read by this thread only
            orow[i] = res;
        }
    } else {
        // write (o, m, l) of this chunk, then count it in; the last CTA of the
        // (row, KV head) combines every chunk
        const size_t unit = (size_t)r * a.num_kv_heads + g;
        const size_t stride = (size_t)KVM * (HD + 2);
        float *part = a.fd_part + (unit * a.fd_nch + c) * stride;
        for (int i = tid; i < KVM * HD; i += FD_THREADS) {
            float o = 0.0f;
#pragma unroll
            for (int grp = 0; grp < SM::groups; grp++) o += s_o[grp * KVM * HD + i];
            part[i] = o;
        }
        if (tid < KVM) {
            part[KVM * HD + tid] = m[tid];
            part[KVM * HD + KVM + tid] = l[tid];
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const int done = atomicAdd(a.fd_cnt + unit, 1);
            s_last = done == nch - 1;
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (tid == 0) a.fd_cnt[unit] = 0;  // ready for the next launch
        const float *p0 = a.fd_part + unit * a.fd_nch * stride;
        for (int i = tid; i < KVM * HD; i += FD_THREADS) {
            const int h = i / HD;
            float M = -INFINITY;
            for (int cc = 0; cc < nch; cc++) M = fmaxf(M, __ldcg(p0 + cc * stride + KVM * HD + h));
            float num = 0.0f, den = 0.0f;
            for (int cc = 0; cc < nch; cc++) {
                const float w = __expf(__ldcg(p0 + cc * stride + KVM * HD + h) - M);
                num = __fmaf_rn(w, __ldcg(p0 + cc * stride + i), num);
                den = __fmaf_rn(w, __ldcg(p0 + cc * stride + KVM * HD + KVM + h), den);
            }
            const float res = num / den;
            s_o[i] = res;
            orow[i] = res;
        }
    }
    // Q8_0 of the output block this (row, KV head) owns, for the Wo GEMV
    if (a.q8_out.qs) {
        __syncthreads();
        const int nbr = a.dim / 32;
        for (int blk = warp; blk < (KVM * HD) / 32; blk += FD_THREADS / 32)
            q8x_store_block(s_o[blk * 32 + lane], a.q8_out, (size_t)r * nbr + (size_t)(g * KVM * HD) / 32 + blk,
                            lane);
    }
}

template <int KVM, int HD>
void launch_fd(const AttnArgs &a, const CUtensorMap &kmap, const CUtensorMap &vmap, cudaStream_t s) {
    const dim3 grid((unsigned)((a.max_len + FD_KEYS - 1) / FD_KEYS), (unsigned)a.num_kv_heads, (unsigned)a.rows);
    launch_kernel(attn_flash_decode_kernel<KVM, HD>, grid, dim3(FD_THREADS), FdSmem<KVM, HD>::total, s, a.pdl, a,
                  kmap, vmap);
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

template <int HD>
void set_fd_smem_hd() {
    cudaFuncSetAttribute(attn_flash_decode_kernel<1, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)FdSmem<1, HD>::total);
    cudaFuncSetAttribute(attn_flash_decode_kernel<2, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)FdSmem<2, HD>::total);
    cudaFuncSetAttribute(attn_flash_decode_kernel<3, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)FdSmem<3, HD>::total);
    cudaFuncSetAttribute(attn_flash_decode_kernel<4, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)FdSmem<4, HD>::total);
    cudaFuncSetAttribute(attn_flash_decode_kernel<6, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)FdSmem<6, HD>::total);
    cudaFuncSetAttribute(attn_flash_decode_kernel<8, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)FdSmem<8, HD>::total);
}

}  // namespace

int flash_decode_chunks(int max_seq) { return (max_seq + FD_KEYS - 1) / FD_KEYS; }

bool flash_decode_ok(const AttnArgs &a) {
    const int kvm = a.num_heads / a.num_kv_heads;
    const bool kvm_ok = kvm == 1 || kvm == 2 || kvm == 3 || kvm == 4 || kvm == 6 || kvm == 8;
    return kvm_ok && (a.head_dim == 64 || a.head_dim == 128) && a.fd_part && a.fd_cnt &&
           a.fd_nch >= flash_decode_chunks(a.max_len) && (a.kv_dim & 3) == 0 && (a.ldq & 3) == 0 &&
           ((uintptr_t)a.k_base & 15) == 0 && ((uintptr_t)a.v_base & 15) == 0 &&
           ((a.num_heads / a.num_kv_heads) * a.head_dim) % 32 == 0 && a.shard_n <= 1;
}

void launch_flash_decode(const AttnArgs &a, const CUtensorMap &kmap, const CUtensorMap &vmap, cudaStream_t s) {
    if (a.rows <= 0) return;
    if (a.head_dim == 64)
        launch_fd_hd<64>(a, kmap, vmap, s);
    else
        launch_fd_hd<128>(a, kmap, vmap, s);
}

void set_flash_decode_smem() {
    set_fd_smem_hd<64>();
    set_fd_smem_hd<128>();
}

}  // namespace slm
