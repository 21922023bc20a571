// kernels_attn_tc.cu -- causal prefill attention on the 5th-generation tensor
// cores (opt-in mode; the default prefill path is the bit-exact one of
// kernels_attn.cu).
//
// Same result definition as causal_multi_head_attention_jit
// (src/model/transformer.rs:273-321): score = (q.k) * scale, softmax with the
// row maximum subtracted (graph.rs:168-179), out = sum_t p_t v_t.  What
// differs is the arithmetic: QK^T and PV run as tcgen05 kind::tf32 MMAs with a
// 3xTF32 split of both operands (hi = x cut to tf32, lo = x - hi; a.b ~ ah.bh
// + ah.bl + al.bh, ~2^-21 relative error per product), accumulated in f32 in
// TMEM; exp is the hardware exp2 (__expf, a few ulp) instead of the
// reference's polynomial; the subtracted maximum is a running one (online
// softmax), and out = (sum_t e_t v_t) * (1/sum) instead of sum_t (e_t/sum)
// v_t.  Results agree with the exact path to about 1e-6 relative, not bit
// for bit.
//
// One CTA of 256 threads per (128/kv_mul query rows of one prompt, KV head):
// MMA row m is query row m/kv_mul of head m%kv_mul of the group, so the group's
// heads share every staged K and V tile.  One pass over the keys of the
// tile's causal range in tiles of 64:
//   S = Q K^T (M=128 rows, N=64 keys, K=head_dim, TMEM, double-buffered so
//   that S of the next tile is computed during this tile's thread work) ->
//   running row maximum m (moved only when a tile exceeds it by more than 8;
//   then O and the lane sums are scaled by exp(m_old - m_new)) -> e =
//   exp(s - m) with the reference's four lane sums -> E written to shared
//   memory as the A operand -> O += E V (N=head_dim) with V^T as the K-major
//   B operand (two V buffers; S and PV complete on separate mbarriers, so PV
//   of one tile runs while the threads read and stage the next).
// Threads i and i+128 own MMA row i = TMEM lane i (warp w reads lanes
// 32*(w%4)..+31), each half of every tile's key columns and output dims.
// All operands are staged by the threads (global -> registers -> hi/lo split ->
// 128-byte swizzled shared memory); MMAs are issued by thread 0 and complete on
// two mbarriers (bounded waits: on a timeout the kernel sets the error flag,
// lets the committed MMAs finish, frees its TMEM and writes nothing).
#include "attn_rows.cuh"
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace slm {

namespace {

constexpr int TC_M = 128;   // MMA rows per CTA (M, TMEM lanes): (query row, head) pairs
constexpr int TC_THREADS = 256;  // two threads per MMA row
constexpr int TC_N = 64;    // keys per tile
constexpr int TC_COLS = 256;  // TMEM columns: two S buffers at 0 and 64, O at 128..128+hd-1

template <int HD>
constexpr size_t tc_smem_bytes() {
    // Q hi/lo [128][HD], K hi/lo [64][HD], two V^T hi/lo [HD][64], E hi/lo [128][64]
    return 2 * sizeof(float) *
               ((size_t)TC_M * HD + (size_t)TC_N * HD + 2 * (size_t)HD * TC_N + (size_t)TC_M * TC_N) +
           1024;
}

// A K-major operand of R rows x KW f32 (KW a multiple of 32) moved by the 256
// threads in 16-byte chunks: load() issues every global load of the thread
// into registers first (one memory latency for the whole tile, and the loads
// can be in flight while other work runs), store() writes the hi and lo
// copies in the 128-byte swizzled layout.  src(r, k) returns the float4 at
// row r, columns k..k+3.
template <int R, int KW>
struct OperandStage {
    static constexpr int CH = R * (KW / 4) / TC_THREADS;  // chunks per thread
    static_assert(CH * TC_THREADS == R * (KW / 4), "tile shape");
    float4 x[CH];
    template <class Src>
    __device__ __forceinline__ void load(Src src, int tid) {
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int e = tid + c * TC_THREADS;
            x[c] = src(e / (KW / 4), (e % (KW / 4)) * 4);
        }
    }
    __device__ __forceinline__ void store(unsigned char *hi, unsigned char *lo, int tid) const {
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int e = tid + c * TC_THREADS;
            const float4 h = make_float4(tf32_hi(x[c].x), tf32_hi(x[c].y), tf32_hi(x[c].z), tf32_hi(x[c].w));
            const unsigned o = sw128_off(e / (KW / 4), (e % (KW / 4)) * 4, R);
            *reinterpret_cast<float4 *>(hi + o) = h;
            *reinterpret_cast<float4 *>(lo + o) = make_float4(__fsub_rn(x[c].x, h.x), __fsub_rn(x[c].y, h.y),
                                                              __fsub_rn(x[c].z, h.z), __fsub_rn(x[c].w, h.w));
        }
    }
};

// 16 consecutive f32 columns of this thread's TMEM lane, waited for.
__device__ __forceinline__ void tc_ld16(unsigned taddr, float (&v)[16]) {
    unsigned r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]);
}

// The three tf32 products of one operand pair over K = KW, M = 128 rows of A
// and RB rows of B, accumulating into d.  The descriptors are the operands'
// base descriptors: a K step moves the 14-bit start-address field (bits 0-13,
// in 16-byte units, never carrying: shared addresses are below 256 KB) by
// the step's byte offset / 16.
template <int KW, int RB>
__device__ __forceinline__ void mma_3xtf32(unsigned d, uint64_t ahi, uint64_t alo, uint64_t bhi, uint64_t blo,
                                           unsigned idesc, bool accumulate) {
    const uint64_t as[3] = {ahi, ahi, alo}, bs[3] = {bhi, blo, bhi};
#pragma unroll
    for (int p = 0; p < 3; p++)
#pragma unroll
        for (int ks = 0; ks < KW / 8; ks++) {
            const unsigned ao = (unsigned)((ks >> 2) * TC_M * 128 + (ks & 3) * 32);
            const unsigned bo = (unsigned)((ks >> 2) * RB * 128 + (ks & 3) * 32);
            tc_mma_tf32(d, as[p] + (ao >> 4), bs[p] + (bo >> 4), idesc, accumulate || p > 0 || ks > 0);
        }
}

// Multiply this thread's half of its TMEM row of O (columns hf*HD/2 ..) by
// alpha: load, scale, store back, wait for the store.  Warp-wide.
template <int HD>
__device__ __forceinline__ void tmem_scale_half(unsigned t_o, int hf, float alpha) {
    constexpr int OC = HD / 2;
    const unsigned ta = t_o + (unsigned)(hf * OC);
    if constexpr (OC == 32) {
        float v[32];
        tc_ld32(ta, v);
        unsigned r[32];
#pragma unroll
        for (int j = 0; j < 32; j++) r[j] = __float_as_uint(__fmul_rn(v[j], alpha));
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
            "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(ta),
            "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
            "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
            "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
            "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
            : "memory");
    } else {
        float v[16];
        tc_ld16(ta, v);
        unsigned r[16];
#pragma unroll
        for (int j = 0; j < 16; j++) r[j] = __float_as_uint(__fmul_rn(v[j], alpha));
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16};\n" ::"r"(ta),
            "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
            "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
            : "memory");
    }
    asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// max with NaN propagation (one instruction; the maximum itself is exact)
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

template <int HD>
__global__ void __launch_bounds__(TC_THREADS) attn_prefill_tc_kernel(AttnArgs a, int run) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_s, bar_p;  // completions of S and of PV MMAs
    __shared__ unsigned s_taddr;
    __shared__ int s_abort;
    __shared__ float s_mx[TC_THREADS];  // the halves' tile maxima
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    unsigned char *q_hi = base;
    unsigned char *q_lo = q_hi + TC_M * HD * 4;
    unsigned char *k_hi = q_lo + TC_M * HD * 4;
    unsigned char *k_lo = k_hi + TC_N * HD * 4;
    unsigned char *v_hi = k_lo + TC_N * HD * 4;         // two buffers: V(kt) at (kt & 1)
    unsigned char *v_lo = v_hi + 2 * HD * TC_N * 4;
    unsigned char *e_hi = v_lo + 2 * HD * TC_N * 4;
    unsigned char *e_lo = e_hi + TC_M * TC_N * 4;

    // MMA row m = (query row m / kvm, head g*kvm + m % kvm): the kvm heads of
    // KV group g share every K and V tile, staged once
    const int nqt = gridDim.x;
    const int qt = nqt - 1 - (int)blockIdx.x;  // longest causal ranges first
    const int g = blockIdx.y, seq = blockIdx.z;
    const int kvm = a.num_heads / a.num_kv_heads, qr = TC_M / kvm;  // query rows per CTA
    const int r0 = seq * run + qt * qr;
    const int nr = run - qt * qr < qr ? run - qt * qr : qr;
    if (!unit_owned(a, r0, g)) return;  // CTA-uniform: another rank's unit
    const int tid = threadIdx.x, warp = tid >> 5;

    if (warp == 0) tc_alloc(&s_taddr, TC_COLS);
    if (tid == 0) {
        mbar_init(&bar_s, 1);
        mbar_init(&bar_p, 1);
        s_abort = 0;
        mbar_fence_init();
    }
    pdl_wait();  // q and the K/V rows of this prompt come from the QKV kernel

    const int p0 = a.pos ? a.pos[r0] : a.pos_const;
    int lmax = p0 + nr;  // keys of the tile's last row
    lmax = lmax < a.max_seq ? lmax : a.max_seq;
    lmax = lmax < a.max_len ? lmax : a.max_len;
    const int ntile = (lmax + TC_N - 1) / TC_N;
    const size_t kv_row0 = row_slot(a, r0) * a.slot_stride + a.layer_off + (size_t)g * HD;
    const float *kb = a.k_base + kv_row0;
    const float *vb = a.v_base + kv_row0;

    // this thread's MMA row = TMEM lane (warp w reads lanes 32*(w%4)..), and
    // its half of every key tile's columns
    const int i = tid & (TC_M - 1), hf = tid / TC_M;
    const int qi = i / kvm, h = g * kvm + i % kvm;  // query row in the tile, head
    int li = p0 + qi + 1;
    li = li < a.max_seq ? li : a.max_seq;
    li = li < a.max_len ? li : a.max_len;
    if (qi >= nr) li = 0;  // also the rows past qr*kvm

    tc_fence_before();  // the TMEM address is read after the barrier below
    {
        OperandStage<TC_M, HD> qs;
        qs.load(
            [&](int r, int k) {
                return r / kvm < nr ? *reinterpret_cast<const float4 *>(a.q + (size_t)(r0 + r / kvm) * a.ldq +
                                                                        (size_t)(g * kvm + r % kvm) * HD + k)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            },
            tid);
        qs.store(q_hi, q_lo, tid);
    }
    __syncthreads();
    tc_fence_after();
    const unsigned taddr = s_taddr;
    const unsigned t_s = taddr + ((unsigned)(warp * 32) << 16);  // this warp's lanes, S buffers
    const unsigned t_o_col = taddr + 2 * TC_N;                   // O columns (MMA destination)
    const unsigned t_o = t_s + 2 * TC_N;                         // O columns, this warp's lanes
    const unsigned idesc_s = umma_idesc_tf32(TC_M, TC_N), idesc_o = umma_idesc_tf32(TC_M, HD);
    const uint64_t dq_hi = umma_desc_sw128(smem_addr(q_hi)), dq_lo = umma_desc_sw128(smem_addr(q_lo));
    const uint64_t dk_hi = umma_desc_sw128(smem_addr(k_hi)), dk_lo = umma_desc_sw128(smem_addr(k_lo));
    const uint64_t dv_hi = umma_desc_sw128(smem_addr(v_hi)), dv_lo = umma_desc_sw128(smem_addr(v_lo));
    const uint64_t dv_step = (uint64_t)((HD * TC_N * 4) >> 4);  // descriptor offset of V buffer 1
    const uint64_t de_hi = umma_desc_sw128(smem_addr(e_hi)), de_lo = umma_desc_sw128(smem_addr(e_lo));
    unsigned n_s = 0, n_p = 0;            // commits issued on bar_s / bar_p
    unsigned w_s = 0, w_p = 0;            // commits waited for
    bool failed = false;

    // K tile kt: rows = keys, K = head_dim; V tile kt as V^T: rows = dims,
    // K = keys (chunk = 4 keys of one dim, gathered from 4 V rows)
    OperandStage<TC_N, HD> ks;
    OperandStage<HD, TC_N> vs;
    auto load_k = [&](int t0) {
        ks.load(
            [&](int t, int k) {
                return t0 + t < lmax ? *reinterpret_cast<const float4 *>(kb + (size_t)(t0 + t) * a.kv_dim + k)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
            },
            tid);
    };
    auto load_v = [&](int t0) {
        vs.load(
            [&](int d, int t) {
                float x[4];
#pragma unroll
                for (int u = 0; u < 4; u++)
                    x[u] = t0 + t + u < lmax ? vb[(size_t)(t0 + t + u) * a.kv_dim + d] : 0.0f;
                return make_float4(x[0], x[1], x[2], x[3]);
            },
            tid);
    };
    // Thread 0 issues MMAs after every thread's shared-memory writes (the
    // barrier orders them, and the TMEM reads before it), then commits them
    // to `done` (bar_s for S, bar_p for PV: a commit covers everything the
    // thread issued before it).  The same barrier tells every thread whether
    // any thread's wait gave up (then nothing is issued and the caller stops).
    bool waits_ok = true;
    auto issue = [&](auto body, uint64_t *done, unsigned &n_done) {
        fence_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!waits_ok)) return false;
        if (tid == 0) {
            tc_fence_after();
            body();
            tc_commit(done);
        }
        n_done++;
        return true;
    };
    // wait for the next commit of `done` (a give-up is acted on at the next
    // issue barrier)
    auto wait_on = [&](uint64_t *done, unsigned &w) {
        waits_ok = mbar_wait(done, w & 1u, &s_abort, a.err) && waits_ok;
        w++;
        tc_fence_after();
    };
    // S(kt) sits in TMEM buffer kt & 1; S(kt+1) is issued before the thread
    // work of tile kt, so the tensor core computes it meanwhile.
    auto issue_s = [&](int kt) {
        mma_3xtf32<HD, TC_N>(taddr + (unsigned)((kt & 1) * TC_N), dq_hi, dq_lo, dk_hi, dk_lo, idesc_s, false);
    };
    // Online softmax: m is the row's running reference maximum; it moves only
    // when a tile's maximum exceeds it by more than RESCALE_AT (the exps then
    // stay below e^RESCALE_AT), and then O (TMEM) and the lane sums are scaled
    // by exp(m_old - m_new).  The halves of a row agree on m through s_mx.
    constexpr float RESCALE_AT = 8.0f;
    float m = -INFINITY;
    float lane_sum[4] = {0.f, 0.f, 0.f, 0.f}, tail = 0.f;
    const int vl = li & ~3;
    load_k(0);
    ks.store(k_hi, k_lo, tid);
    if (ntile > 1) load_k(TC_N);
    load_v(0);
    issue([&] { issue_s(0); }, &bar_s, n_s);
    for (int kt = 0; kt < ntile && !failed; kt++) {
        const int t0 = kt * TC_N, vbuf = kt & 1;
        wait_on(&bar_s, w_s);  // S(kt); PV(kt-1) may still run
        float v[32];
        tc_ld32(t_s + (unsigned)((kt & 1) * TC_N + hf * 32), v);
        // masked scaled scores and their maximum (a tree: max is exact in any order)
        float tm[32];
#pragma unroll
        for (int j = 0; j < 32; j++) {
            v[j] = __fmul_rn(v[j], a.scale);
            tm[j] = t0 + hf * 32 + j < li ? v[j] : -INFINITY;
        }
#pragma unroll
        for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
            for (int j = 0; j < w; j++) tm[j] = max_nan(tm[j], tm[j + w]);
        s_mx[tid] = tm[0];
        if (kt + 1 < ntile) {
            ks.store(k_hi, k_lo, tid);  // K(kt+1); the K stage is free: S(kt) is done
            if (kt + 2 < ntile) load_k(t0 + 2 * TC_N);
        }
        // V(kt) into buffer kt & 1, last read by PV(kt-2), which completed
        // before E(kt-1) was written
        vs.store(v_hi + vbuf * HD * TC_N * 4, v_lo + vbuf * HD * TC_N * 4, tid);
        if (kt + 1 < ntile) load_v(t0 + TC_N);
        if (kt + 1 < ntile && !issue([&] { issue_s(kt + 1); }, &bar_s, n_s)) {
            failed = true;
            break;
        }
        if (kt + 1 == ntile) __syncthreads();  // s_mx complete (no S issue barrier)
        // the row's tile maximum from both halves (written before the barrier)
        const float rm = max_nan(s_mx[i], s_mx[i + TC_M]);
        const bool move = rm > m + RESCALE_AT || (m == -INFINITY && rm > -INFINITY);
        const float m_new = move ? rm : m;
        const float alpha = move ? __expf(__fsub_rn(m, m_new)) : 1.0f;  // 0 when m was -inf
        if (move) {
#pragma unroll
            for (int q = 0; q < 4; q++) lane_sum[q] = __fmul_rn(lane_sum[q], alpha);
            tail = __fmul_rn(tail, alpha);
        }
        m = m_new;
        // the 32 exps (masked afterwards; rows without keys have m = -inf and
        // s - m = +inf there, masked too)
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __expf(__fsub_rn(v[j], m));
        if (kt > 0) wait_on(&bar_p, w_p);  // PV(kt-1): E and O are free
        // O *= alpha for this thread's half of the row, once O holds PV(0..kt-1);
        // warp-wide TMEM access when any lane of the warp moved
        if (kt > 0 && __any_sync(0xffffffffu, move)) tmem_scale_half<HD>(t_o, hf, alpha);
#pragma unroll
        for (int j4 = 0; j4 < 8; j4++) {
            float ev[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int t = t0 + hf * 32 + j4 * 4 + q;
                ev[q] = t < li ? v[j4 * 4 + q] : 0.0f;
                if (t < vl)
                    lane_sum[q] = __fadd_rn(lane_sum[q], ev[q]);
                else
                    tail = __fadd_rn(tail, ev[q]);  // 0 past li
            }
            const float4 hh = make_float4(tf32_hi(ev[0]), tf32_hi(ev[1]), tf32_hi(ev[2]), tf32_hi(ev[3]));
            const unsigned o = sw128_off(i, hf * 32 + j4 * 4, TC_M);
            *reinterpret_cast<float4 *>(e_hi + o) = hh;
            *reinterpret_cast<float4 *>(e_lo + o) = make_float4(__fsub_rn(ev[0], hh.x), __fsub_rn(ev[1], hh.y),
                                                                __fsub_rn(ev[2], hh.z), __fsub_rn(ev[3], hh.w));
        }
        // O += E V(kt), running while the next tile's S is read and staged
        if (!issue([&] { mma_3xtf32<TC_N, HD>(t_o_col, de_hi, de_lo, dv_hi + vbuf * dv_step, dv_lo + vbuf * dv_step,
                                              idesc_o, kt > 0); },
                   &bar_p, n_p)) {
            failed = true;
            break;
        }
    }
    if (!failed) {  // the last PV
        wait_on(&bar_p, w_p);
        failed = __syncthreads_or(!waits_ok) != 0;
    }

    // [5][TC_THREADS] lane sums and tails in the E buffer (free after the last PV)
    float(*s_part)[TC_THREADS] = reinterpret_cast<float(*)[TC_THREADS]>(e_hi);
    if (!failed) {
        // the two halves' lane sums and tails (each half summed its columns in key order)
#pragma unroll
        for (int u = 0; u < 4; u++) s_part[u][tid] = lane_sum[u];
        s_part[4][tid] = tail;
        __syncthreads();
        float l[5];
#pragma unroll
        for (int u = 0; u < 5; u++) l[u] = __fadd_rn(s_part[u][i], s_part[u][i + TC_M]);
        const float sum = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[1]), __fadd_rn(l[2], l[3])), l[4]);
        const float inv = __fdiv_rn(1.0f, sum);
        const bool store = qi < nr && li > 0;
        // half hf writes output columns [hf*HD/2, (hf+1)*HD/2)
        constexpr int OC = HD / 2;
        float *orow = a.out + (size_t)(r0 + (store ? qi : 0)) * a.ldo + (size_t)h * HD + hf * OC;
        float v[OC];
        if constexpr (OC == 32)
            tc_ld32(t_o + (unsigned)(hf * OC), v);  // warp-wide: every lane, stores predicated
        else
            tc_ld16(t_o + (unsigned)(hf * OC), v);
        if (store)
#pragma unroll
            for (int j = 0; j < OC; j += 4)
                *reinterpret_cast<float4 *>(orow + j) = make_float4(__fmul_rn(v[j], inv), __fmul_rn(v[j + 1], inv),
                                                                    __fmul_rn(v[j + 2], inv), __fmul_rn(v[j + 3], inv));
    }
    pdl_release();
    tc_fence_before();
    __syncthreads();
    if (failed && tid == 0) {
        // a wait gave up: let the MMAs already committed finish (bounded)
        // before the TMEM they write is freed
        const long long tw = clock64();
        while (w_s < n_s && clock64() - tw < WAIT_LIMIT)
            if (mbar_test(&bar_s, w_s & 1u)) w_s++;
        while (w_p < n_p && clock64() - tw < WAIT_LIMIT)
            if (mbar_test(&bar_p, w_p & 1u)) w_p++;
    }
    __syncthreads();
    tc_fence_after();
    // The columns are freed even when that drain gave up too.  Keeping them
    // would leave them allocated for good, and a later CTA's tcgen05.alloc on
    // this SM would then wait for ever; freeing them can at worst let an MMA
    // that is still running after the second bounded wait write into columns
    // another CTA has allocated, and the launch has already set the error
    // flag, so the call that owns this launch reports failure either way.
    if (warp == 0) tc_dealloc(taddr, TC_COLS);
}

}  // namespace

bool attn_prefill_tc_ok(const AttnArgs &a) {
    return a.prefill_run > 0 && a.rows % a.prefill_run == 0 && (a.head_dim == 32 || a.head_dim == 64) &&
           a.num_heads / a.num_kv_heads <= 16 &&
           (a.ldq & 3) == 0 && (a.kv_dim & 3) == 0 && (a.ldo & 3) == 0 && ((uintptr_t)a.q & 15) == 0 &&
           ((uintptr_t)a.k_base & 15) == 0 && ((uintptr_t)a.out & 15) == 0 && (a.slot_stride & 3) == 0 &&
           (a.layer_off & 3) == 0;
}

void launch_attn_prefill_tc(const AttnArgs &a, cudaStream_t s) {
    const int kvm = a.num_heads / a.num_kv_heads, qr = TC_M / kvm;
    const int run = a.prefill_run, nqt = (run + qr - 1) / qr;
    const dim3 grid((unsigned)nqt, (unsigned)a.num_kv_heads, (unsigned)(a.rows / run));
    if (a.head_dim == 32)
        launch_kernel(attn_prefill_tc_kernel<32>, grid, dim3(TC_THREADS), tc_smem_bytes<32>(), s, a.pdl, a, run);
    else
        launch_kernel(attn_prefill_tc_kernel<64>, grid, dim3(TC_THREADS), tc_smem_bytes<64>(), s, a.pdl, a, run);
    if (a.q8_out.qs) launch_quantize_q8x(a.out, a.ldo, a.dim, a.q8_out, a.rows, s);
}

void set_attn_prefill_tc_smem() {
    cudaFuncSetAttribute(attn_prefill_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)tc_smem_bytes<32>());
    cudaFuncSetAttribute(attn_prefill_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)tc_smem_bytes<64>());
}

}  // namespace slm
