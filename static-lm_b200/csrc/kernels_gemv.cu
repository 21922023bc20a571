// kernels_gemv.cu -- Q4_0 x Q8_0 GEMV / GEMM with the reference's AVX2
// numerics and fused epilogues.
//
// Numerics (src/quant/kernels.rs:163-212): for each (row r, activation row b)
// eight f32 lane accumulators; lane k of block j holds the exact int sum of
// elements 4k..4k+3 and is accumulated as acc_k = fma(dw_j*da_j, isum_k,
// acc_k) in block order; the result is ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7)).
// The batched form (gemm_q4_0, kernels.rs:308-394) is the same dot per
// (r, b), so a GEMM equals repeated GEMVs bit for bit.
//
// Mapping: one warp per (32-row weight tile, tile of BT activation rows);
// lane = row.  Every lane keeps RPT*BT*8 accumulators in registers while it
// walks the blocks of its row in order (the order is what the numerics fix;
// the parallelism comes from rows x activation rows).  Weights come from the
// repacked 576-byte tiles -- one coalesced 128-bit load per lane and block,
// PF blocks in flight; the four warps of a CTA work on four row tiles of the
// same activation tile, which cp.async stages in shared memory in chunks of
// JC blocks and the warps read as broadcasts.  BT is chosen per launch so that
// (tiles x activation tiles) gives the SMs enough warps to hide latency.
//
// The int dot of a lane is one dp4a of the unsigned weight nibbles against
// the activation bytes, seeded with c_k = 0x4B400000 - 8*sum(a): the result
// is the bit pattern of 12582912 + isum_k, so isum_k as f32 costs one exact
// subtraction instead of an int->float conversion.
#include <cstdlib>

#include "async.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace slm {

namespace {

constexpr int JC = 64;   // activation blocks per shared-memory chunk (multiple of PF)

// One weight block j of RPT tiles (lane = row) against BT activation blocks:
// acc[t][b][k] = fma(dw*da, isum_k, acc[t][b][k]) for the 8 lanes k.
// slot[t] points at the block's 576 bytes; qs/c/d at activation row 0's block,
// rows `astride` blocks apart.
template <int RPT, int BT>
__device__ __forceinline__ void block_dot(float (&acc)[RPT][BT][8], const uint8_t *const (&slot)[RPT],
                                          const int8_t *qs, const int32_t *c, const float *d,
                                          int astride, int lane) {
    unsigned lo[RPT][4], hi[RPT][4];
    float dw[RPT];
#pragma unroll
    for (int t = 0; t < RPT; t++) {
        const uint4 q = *reinterpret_cast<const uint4 *>(slot[t] + lane * 16);
        dw[t] = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(slot[t] + 512 + lane * 2)));
        const unsigned qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            lo[t][k] = qw[k] & 0x0F0F0F0Fu;
            hi[t][k] = (qw[k] >> 4) & 0x0F0F0F0Fu;
        }
    }
#pragma unroll
    for (int b = 0; b < BT; b++) {
        const int4 a0 = reinterpret_cast<const int4 *>(qs + (size_t)b * astride * 32)[0];
        const int4 a1 = reinterpret_cast<const int4 *>(qs + (size_t)b * astride * 32)[1];
        const int4 c0 = reinterpret_cast<const int4 *>(c + (size_t)b * astride * 8)[0];
        const int4 c1 = reinterpret_cast<const int4 *>(c + (size_t)b * astride * 8)[1];
        const float da = d[(size_t)b * astride];
        const int av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const int cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int t = 0; t < RPT; t++) {
            const float dd = __fmul_rn(dw[t], da);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                float f0 = __fsub_rn(__int_as_float(dp4a_us(lo[t][k], av[k], cv[k])), MAGIC_F);
                acc[t][b][k] = __fmaf_rn(dd, f0, acc[t][b][k]);
                float f1 = __fsub_rn(__int_as_float(dp4a_us(hi[t][k], av[4 + k], cv[4 + k])), MAGIC_F);
                acc[t][b][4 + k] = __fmaf_rn(dd, f1, acc[t][b][4 + k]);
            }
        }
    }
}

// The reduction of the 8 lane accumulators and the fused epilogues
// (store / residual / RoPE + KV append / SwiGLU + Q8) for one warp.
template <int RPT, int BT, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs &a, const float (&acc)[RPT][BT][8],
                                              const int (&tile)[RPT], int total_tiles, int b0,
                                              int lane) {
    float y[RPT][BT];
#pragma unroll
    for (int t = 0; t < RPT; t++)
#pragma unroll
        for (int b = 0; b < BT; b++) {
            float s0 = __fadd_rn(acc[t][b][0], acc[t][b][4]);
            float s1 = __fadd_rn(acc[t][b][1], acc[t][b][5]);
            float s2 = __fadd_rn(acc[t][b][2], acc[t][b][6]);
            float s3 = __fadd_rn(acc[t][b][3], acc[t][b][7]);
            y[t][b] = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
        }

    if constexpr (EPI == EPI_SWIGLU_Q8) {
        const int hdim = (total_tiles / 2) * TILE_ROWS;
        const int nb_out = hdim / 32;
        const int hrow = tile[0] * TILE_ROWS + lane;
#pragma unroll
        for (int b = 0; b < BT; b++) {
            const int bb = b0 + b;
            if (bb >= a.batch) break;  // warp-uniform
            float o = swiglu1(y[0][b], y[RPT - 1][b]);
            if (a.out) a.out[(size_t)bb * a.ld_out + hrow] = o;
            q8x_store_block(o, a.q8_out, (size_t)bb * nb_out + tile[0], lane);
        }
    } else {
        const int row = tile[0] * TILE_ROWS + lane;
#pragma unroll
        for (int b = 0; b < BT; b++) {
            const int bb = b0 + b;
            if (bb >= a.batch) break;  // warp-uniform
            const float v = y[0][b];
            if constexpr (EPI == EPI_STORE) {
                if (row < a.rows) a.out[(size_t)bb * a.ld_out + row] = v;
            } else if constexpr (EPI == EPI_RESIDUAL) {
                if (row < a.rows)
                    a.out[(size_t)bb * a.ld_out + row] =
                        __fadd_rn(a.res[(size_t)bb * a.ld_res + row], v);
            } else if constexpr (EPI == EPI_QKV) {
                const QkvArgs &q = a.qkv;
                // RoPE pairs (2j, 2j+1) sit in lanes (2j, 2j+1) of the same tile
                const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
                const int p = q.pos[bb];
                if (p < 0 || p >= q.max_seq) {  // never write outside the cache
                    if (lane == 0 && q.err) atomicExch(q.err, 2);
                    continue;
                }
                if (row < q.dim + q.kv_dim) {
                    const int local = row < q.dim ? row : row - q.dim;
                    const int i = local % q.head_dim;
                    const int jj = i >> 1;
                    const int half = q.head_dim >> 1;
                    const float cc = q.rope_cos[(size_t)p * half + jj];
                    const float ss = q.rope_sin[(size_t)p * half + jj];
                    float r;
                    if ((i & 1) == 0)  // v0*c - v1*s
                        r = __fsub_rn(__fmul_rn(v, cc), __fmul_rn(partner, ss));
                    else  // v0*s + v1*c
                        r = __fadd_rn(__fmul_rn(partner, ss), __fmul_rn(v, cc));
                    if (row < q.dim) {
                        q.q[(size_t)bb * q.ldq + row] = r;
                    } else {
                        float *kb = q.k_base + (size_t)q.slot[bb] * q.slot_stride + q.layer_off;
                        kb[(size_t)p * q.kv_dim + local] = r;
                    }
                } else if (row < q.dim + 2 * q.kv_dim) {
                    const int local = row - q.dim - q.kv_dim;
                    float *vb = q.v_base + (size_t)q.slot[bb] * q.slot_stride + q.layer_off;
                    vb[(size_t)p * q.kv_dim + local] = v;
                }
            }
        }
    }
}

template <int BT, int EPI>
__global__ void __launch_bounds__(128) gemv_kernel(GemvArgs a, int total_tiles, int units) {
    constexpr int RPT = (EPI == EPI_SWIGLU_Q8) ? 2 : 1;
    constexpr int PF = 8;  // weight-ring depth (launch_bt sizes shared memory for 8)
    extern __shared__ __align__(16) unsigned char smem[];
    int8_t *s_qs = (int8_t *)smem;                    // [BT][JC][32]
    int32_t *s_c = (int32_t *)(smem + BT * JC * 32);  // [BT][JC][8]
    float *s_d = (float *)(smem + BT * JC * 64);      // [BT][JC]
    // per-warp rings of weight blocks: [warp][RPT][PF][576 bytes]
    uint8_t *s_w = smem + BT * JC * 68 + (threadIdx.x >> 5) * (RPT * PF * TILE_BYTES);

    const int lane = threadIdx.x & 31;
    const int unit = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const bool live = unit < units;  // warp-uniform; idle warps still help staging
    const int b0 = blockIdx.y * BT;
    const int nb = a.nb;

    int tile[RPT];
    tile[0] = live ? unit : 0;
    if (RPT == 2) tile[RPT - 1] = tile[0] + total_tiles / 2;

    float acc[RPT][BT][8];
#pragma unroll
    for (int t = 0; t < RPT; t++)
#pragma unroll
        for (int b = 0; b < BT; b++)
#pragma unroll
            for (int k = 0; k < 8; k++) acc[t][b][k] = 0.0f;

    // weight blocks j+1..j+PF-1 are in flight (cp.async into this warp's
    // shared-memory ring) while block j is consumed; lane l copies row l's
    // 16 nibble bytes, lanes 0..3 the 64 bytes of scales
    auto fetch = [&](int j) {
        if (j < nb) {
#pragma unroll
            for (int t = 0; t < RPT; t++) {
                const uint8_t *tp = a.w + tile_offset((size_t)tile[t], nb, j);
                uint8_t *slot = s_w + (t * PF + j % PF) * TILE_BYTES;
                cp_async16(slot + lane * 16, tp + lane * 16);
                if (lane < 4) cp_async16(slot + 512 + lane * 16, tp + 512 + lane * 16);
            }
        }
        asm volatile("cp.async.commit_group;\n" ::);
    };
    if (live) {
        for (int u = 0; u < PF - 1; u++) fetch(u);
    }

    for (int jc = 0; jc < nb; jc += JC) {
        const int jn = nb - jc < JC ? nb - jc : JC;
        __syncthreads();  // the previous chunk has been consumed
        // stage the Q8X blocks [jc, jc+jn) of activation rows [b0, b0+BT):
        // 16-byte pieces 0,1 = int8 values, 2,3 = lane constants
        for (int i = threadIdx.x; i < BT * jn * 4; i += blockDim.x) {
            const int b = i / (jn * 4), rem = i - b * (jn * 4);
            const int jl = rem >> 2, part = rem & 3;
            const int bb = b0 + b;
            void *dst = part < 2 ? (void *)(s_qs + (b * JC + jl) * 32 + part * 16)
                                 : (void *)(s_c + (b * JC + jl) * 8 + (part - 2) * 4);
            if (bb < a.batch) {
                const size_t blk = (size_t)bb * nb + jc + jl;
                const void *src = part < 2 ? (const void *)(a.x.qs + blk * 32 + part * 16)
                                           : (const void *)(a.x.c + blk * 8 + (part - 2) * 4);
                cp_async16(dst, src);
            } else {
                const int fill = part < 2 ? 0 : MAGIC_I;
                *reinterpret_cast<int4 *>(dst) = make_int4(fill, fill, fill, fill);
            }
        }
        asm volatile("cp.async.commit_group;\n" ::);
        for (int i = threadIdx.x; i < BT * jn; i += blockDim.x) {
            const int b = i / jn, jl = i - b * jn;
            const int bb = b0 + b;
            s_d[b * JC + jl] = bb < a.batch ? a.x.d[(size_t)bb * nb + jc + jl] : 0.0f;
        }
        asm volatile("cp.async.wait_group 0;\n" ::);
        __syncthreads();
        if (!live) continue;

        for (int jl = 0; jl < jn; jl++) {
            const int j = jc + jl;
            fetch(j + PF - 1);
            asm volatile("cp.async.wait_group %0;\n" ::"n"(PF - 1));
            __syncwarp();
            const uint8_t *slots[RPT];
#pragma unroll
            for (int t = 0; t < RPT; t++) slots[t] = s_w + (t * PF + j % PF) * TILE_BYTES;
            block_dot<RPT, BT>(acc, slots, s_qs + jl * 32, s_c + jl * 8, s_d + jl, JC, lane);
            __syncwarp();  // the slot may be refilled by the next fetch
        }
    }
    asm volatile("cp.async.wait_group 0;\n" ::);
    if (!live) return;
    gemv_epilogue<RPT, BT, EPI>(a, acc, tile, total_tiles, b0, lane);
}

// Staged GEMV: one CTA per (unit = RPT weight tiles, group of NW*BT
// activation rows), NW warps, warp w owning activation rows w*BT..w*BT+BT-1
// of the group.  The unit's whole tiles (nb blocks each, contiguous in the
// repacked layout) go global -> shared as TMA bulk copies and every warp of
// the CTA reuses them, so the kernel pays one memory latency instead of one
// per PF blocks and reads each tile once per row group.  The activation rows
// complete first on their own mbarrier: as Q8X blocks, or with NORM as f32
// rows that each warp turns into RMSNorm(x)*w (graph.rs:141-155: four lane
// chains of x*x, (l0+l1)+(l2+l3), 1/sqrt(mean+eps)) quantized to Q8_0 while
// the weights are still in flight -- which replaces a separate RMSNorm launch
// and its round trip through global memory.  Both waits are bounded.
constexpr size_t STAGED_SMEM_MAX = 200 * 1024;
constexpr int STAGED_MAX_WARPS = 8;

__host__ __device__ inline size_t staged_smem(int rpt, int rows, int nb, bool norm) {
    size_t s = (size_t)rpt * nb * TILE_BYTES + (size_t)rows * nb * 68;
    if (norm) s += sizeof(float) * ((size_t)(rows + 1) * nb * 32 + 2 * STAGED_MAX_WARPS * 4 + 4);
    return s;
}

template <int BT, int EPI, bool NORM>
__global__ void __launch_bounds__(32 * STAGED_MAX_WARPS, BT > 1 ? 2 : 1)
    gemv_staged_kernel(GemvArgs a, int total_tiles) {
    constexpr int RPT = (EPI == EPI_SWIGLU_Q8) ? 2 : 1;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(8) uint64_t bar_rows, bar_w;
    __shared__ int s_abort;
    const int nb = a.nb, n = nb * 32;
    const int nw = blockDim.x >> 5;
    const int grows = nw * BT;  // activation rows of the group
    const int tile_bytes = nb * TILE_BYTES;
    uint8_t *s_w = smem;                                            // [RPT][nb*576]
    int8_t *s_qs = (int8_t *)(smem + (size_t)RPT * tile_bytes);     // [grows][nb][32]
    int32_t *s_c = (int32_t *)(s_qs + (size_t)grows * nb * 32);     // [grows][nb][8]
    float *s_d = (float *)(s_c + (size_t)grows * nb * 8);           // [grows][nb]
    // NORM: [grows][n] rows, [n] weights, [grows] rms; 16-byte aligned for cp.async
    float *s_x = s_d + ((grows * nb + 3) & ~3);
    float *s_nw = s_x + (size_t)grows * n;
    float *s_rms = s_nw + n;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int unit = blockIdx.x;
    const int g0 = blockIdx.y * grows;     // first activation row of the group
    const int b0 = g0 + warp * BT;         // this warp's first row
    int tile[RPT];
    tile[0] = unit;
    if (RPT == 2) tile[RPT - 1] = unit + total_tiles / 2;

    // One thread puts every copy on the TMA engine (bulk copies, no LSU
    // work): the group's activation rows on bar_rows, the unit's weight
    // tiles on bar_w.  Rows past the batch are padding written by the threads.
    if (threadIdx.x == 0) {
        mbar_init(&bar_rows, 1);
        mbar_init(&bar_w, 1);
        s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    const int valid = a.batch - g0 < grows ? a.batch - g0 : grows;
    // constant data first: it may be fetched while the previous kernel runs
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar_w, (unsigned)RPT * (unsigned)tile_bytes);
#pragma unroll
        for (int t = 0; t < RPT; t++)
            bulk_copy(s_w + (size_t)t * tile_bytes, a.w + tile_offset((size_t)tile[t], nb, 0),
                      (unsigned)tile_bytes, &bar_w);
    }
    pdl_wait();  // the activation rows are the previous kernel's output
    if (threadIdx.x == 0) {
        if constexpr (NORM) {
            mbar_arrive_expect_tx(&bar_rows, (unsigned)(valid + 1) * (unsigned)n * 4u);
            for (int rb = 0; rb < valid; rb++)
                bulk_copy(s_x + (size_t)rb * n, a.nx + (size_t)(g0 + rb) * a.ld_nx, (unsigned)n * 4u,
                          &bar_rows);
            bulk_copy(s_nw, a.nw, (unsigned)n * 4u, &bar_rows);
        } else {
            mbar_arrive_expect_tx(&bar_rows, (unsigned)valid * (unsigned)nb * 64u);
            for (int rb = 0; rb < valid; rb++) {
                const size_t blk = (size_t)(g0 + rb) * nb;
                bulk_copy(s_qs + (size_t)rb * nb * 32, a.x.qs + blk * 32, (unsigned)nb * 32u, &bar_rows);
                bulk_copy(s_c + (size_t)rb * nb * 8, a.x.c + blk * 8, (unsigned)nb * 32u, &bar_rows);
            }
        }
    }
    if constexpr (NORM) {
        for (int i = threadIdx.x; i < (grows - valid) * n; i += blockDim.x) s_x[(size_t)valid * n + i] = 0.0f;
    } else {
        for (int i = threadIdx.x; i < (grows - valid) * nb * 8; i += blockDim.x) {
            reinterpret_cast<int *>(s_qs + (size_t)valid * nb * 32)[i] = 0;
            s_c[(size_t)valid * nb * 8 + i] = MAGIC_I;
        }
        for (int i = threadIdx.x; i < grows * nb; i += blockDim.x) {
            const int rb = i / nb, j = i - rb * nb;
            s_d[i] = rb < valid ? a.x.d[(size_t)(g0 + rb) * nb + j] : 0.0f;
        }
    }

    if constexpr (NORM) {
        mbar_wait(&bar_rows, 0, &s_abort, a.err);  // rows and norm weights landed
        __syncthreads();
        // each warp normalizes its own BT rows: lanes 4b..4b+3 run the four
        // chains of row b
        if (!s_abort) {
            float acc = 0.0f;
            const int rb = lane >> 2, l = lane & 3;
            if (rb < BT) {
                // n % 32 == 0: groups of 8 steps, the next group's loads in
                // flight while the current one is added
                const float *xr = s_x + (size_t)(warp * BT + rb) * n + l;
                const int ng = n >> 5;
                float cur[8], nxt[8];
#pragma unroll
                for (int u = 0; u < 8; u++) cur[u] = xr[4 * u];
                for (int gi = 0; gi < ng; gi++) {
                    if (gi + 1 < ng) {
#pragma unroll
                        for (int u = 0; u < 8; u++) nxt[u] = xr[32 * (gi + 1) + 4 * u];
                    }
#pragma unroll
                    for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, __fmul_rn(cur[u], cur[u]));
#pragma unroll
                    for (int u = 0; u < 8; u++) cur[u] = nxt[u];
                }
            }
            const float a1 = __shfl_down_sync(0xffffffffu, acc, 1);
            const float a2 = __shfl_down_sync(0xffffffffu, acc, 2);
            const float a3 = __shfl_down_sync(0xffffffffu, acc, 3);
            if (rb < BT && l == 0) {
                // n % 4 == 0: no tail
                const float sum = __fadd_rn(__fadd_rn(acc, a1), __fadd_rn(a2, a3));
                const float mean = __fmul_rn(sum, a.inv_n);
                s_rms[warp * BT + rb] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
            }
        }
        __syncwarp();
        // x*rms*w and its Q8_0: lane j quantizes block j of this warp's rows
        // on its own (all blocks of a row in parallel)
        Q8X sq;
        sq.qs = s_qs;
        sq.c = s_c;
        sq.d = s_d;
        for (int qi = lane; qi < (s_abort ? 0 : BT * nb); qi += 32) {
            const int rb = qi / nb, j = qi - rb * nb;
            const int row = warp * BT + rb;
            const float *xr = s_x + (size_t)row * n + j * 32;
            const float *wr = s_nw + j * 32;
            const float rms = s_rms[row];
            q8x_store_block_thread(
                [&](int i) { return __fmul_rn(__fmul_rn(xr[i], rms), wr[i]); }, sq,
                (size_t)row * nb + j, lane & 7);
        }
    }
    if constexpr (!NORM) mbar_wait(&bar_rows, 0, &s_abort, a.err);
    mbar_wait(&bar_w, 0, &s_abort, a.err);
    __syncthreads();  // the weight tiles and the Q8X rows are visible to every warp
    if (s_abort) {
        // a wait gave up: let the copies in flight land (bounded) before the
        // shared memory is released, and write nothing
        if (threadIdx.x == 0) {
            const long long tw = clock64();
            while ((!mbar_test(&bar_rows, 0) || !mbar_test(&bar_w, 0)) && clock64() - tw < WAIT_LIMIT) {
            }
        }
        __syncthreads();
        return;
    }
    if (b0 >= a.batch) return;  // warp-uniform: padding rows only

    float acc[RPT][BT][8];
#pragma unroll
    for (int t = 0; t < RPT; t++)
#pragma unroll
        for (int b = 0; b < BT; b++)
#pragma unroll
            for (int k = 0; k < 8; k++) acc[t][b][k] = 0.0f;
    const int8_t *aq = s_qs + (size_t)warp * BT * nb * 32;
    const int32_t *ac = s_c + (size_t)warp * BT * nb * 8;
    const float *ad = s_d + (size_t)warp * BT * nb;
#pragma unroll 2
    for (int j = 0; j < nb; j++) {
        const uint8_t *slots[RPT];
#pragma unroll
        for (int t = 0; t < RPT; t++) slots[t] = s_w + (size_t)t * tile_bytes + (size_t)j * TILE_BYTES;
        block_dot<RPT, BT>(acc, slots, aq + j * 32, ac + j * 8, ad + j, nb, lane);
    }
    pdl_release();  // the successor may start while this epilogue runs
    gemv_epilogue<RPT, BT, EPI>(a, acc, tile, total_tiles, b0, lane);
}

// ---------------------------------------------------------------------------
// Batch-1 GEMV of wide matrices (nb >= SPLIT_MIN_NB blocks per row): one CTA
// per unit (RPT weight tiles), eight warps.  The reference's order fixes only
// the eight chains acc_k = fma(dw*da, isum_k, acc_k) over the blocks of a row;
// the int8 dot sums isum_k and the scale products dw*da of different blocks
// are independent.  So the blocks go in rounds of SPLIT_ROUND / RPT: warps
// 1..7 form a round's dot sums (as the exact f32 values block_dot uses) and
// dw*da from 16-byte weight loads straight from HBM -- the next round's loads
// in flight while they store -- into one of two buffers, and warp 0 runs its
// lane's eight FMA chains through the previous round in block order.  Same
// values, same order: bit-exact.  Every mbarrier wait is bounded.
constexpr int SPLIT_MIN_NB = 64;
constexpr int SPLIT_ROUND = 32;  // blocks per round for one tile
constexpr int SPLIT_PW = 7;      // warps forming the dot sums

// the activation row (68 B a block) and two rounds' dot sums and scales
// (SPLIT_ROUND blocks x 32 rows x 9 floats each, whatever the tiles per unit)
__host__ __device__ inline size_t split_smem(int nb) {
    return (((size_t)nb * 68 + 15) & ~(size_t)15) + 2 * (size_t)SPLIT_ROUND * 32 * 9 * 4 + 16;
}

template <int EPI>
__global__ void __launch_bounds__(256) gemv_split_kernel(GemvArgs a, int total_tiles) {
    constexpr int RPT = (EPI == EPI_SWIGLU_Q8) ? 2 : 1;
    constexpr int R = SPLIT_ROUND / RPT;                   // blocks per round
    constexpr int WB = (R + SPLIT_PW - 1) / SPLIT_PW;      // blocks a forming warp takes per round
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(8) uint64_t bar_full[2], bar_empty[2];
    __shared__ int s_abort;
    const int nb = a.nb;
    int8_t *s_qs = (int8_t *)smem;                       // [nb][32]
    int32_t *s_c = (int32_t *)(smem + (size_t)nb * 32);  // [nb][8]
    float *s_d = (float *)(smem + (size_t)nb * 64);      // [nb]
    // per buffer: [RPT][R][2][32] float4 of the 8 dot sums (lanes' rows 16 B
    // apart for conflict-free 16-byte loads), then [RPT][R][32] dw*da
    float4 *s_f = (float4 *)(smem + (((size_t)nb * 68 + 15) & ~(size_t)15));
    constexpr int F4 = RPT * R * 2 * 32, SS = RPT * R * 32;
    float *s_s = (float *)(s_f + 2 * F4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int tile[RPT];
    tile[0] = blockIdx.x;
    if (RPT == 2) tile[RPT - 1] = blockIdx.x + total_tiles / 2;
    const int nr = (nb + R - 1) / R;  // rounds

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; b++) {
            mbar_init(&bar_full[b], SPLIT_PW * 32);
            mbar_init(&bar_empty[b], 32);
        }
        s_abort = 0;
        mbar_fence_init();
    }
    // a forming warp's weight blocks of a round: nibbles and scale of row `lane`
    uint4 wq[RPT][WB];
    unsigned short ws[RPT][WB];
    auto load_w = [&](int r0) {
#pragma unroll
        for (int u = 0; u < WB; u++) {
            const int jr = (warp - 1) + u * SPLIT_PW, j = r0 + jr;
#pragma unroll
            for (int t = 0; t < RPT; t++) {
                if (jr < R && j < nb) {
                    const uint8_t *tp = a.w + tile_offset((size_t)tile[t], nb, j);
                    wq[t][u] = __ldg(reinterpret_cast<const uint4 *>(tp + lane * 16));
                    ws[t][u] = __ldg(reinterpret_cast<const unsigned short *>(tp + 512 + lane * 2));
                }
            }
        }
    };
    if (warp > 0) load_w(0);  // constant data: in flight while the previous kernel finishes
    pdl_wait();               // the activation row is the previous kernel's output
    for (int i = threadIdx.x; i < nb * 4; i += blockDim.x) {
        const int j = i >> 2, part = i & 3;
        void *dst = part < 2 ? (void *)(s_qs + j * 32 + part * 16) : (void *)(s_c + j * 8 + (part - 2) * 4);
        const void *src = part < 2 ? (const void *)(a.x.qs + (size_t)j * 32 + part * 16)
                                   : (const void *)(a.x.c + (size_t)j * 8 + (part - 2) * 4);
        cp_async16(dst, src);
    }
    cp_async_commit();
    for (int j = threadIdx.x; j < nb; j += blockDim.x) s_d[j] = a.x.d[j];
    cp_async_wait<0>();
    __syncthreads();  // the activation row and the barriers are ready

    float acc[RPT][1][8];
#pragma unroll
    for (int t = 0; t < RPT; t++)
#pragma unroll
        for (int k = 0; k < 8; k++) acc[t][0][k] = 0.0f;
    if (warp > 0) {
        // ---- forming warps
        for (int r = 0; r < nr; r++) {
            const int b = r & 1, r0 = r * R;
            if (r >= 2 && !mbar_wait(&bar_empty[b], (unsigned)((r >> 1) - 1) & 1u, &s_abort, a.err)) break;
            float4 *f = s_f + (size_t)b * F4;
            float *ss = s_s + (size_t)b * SS;
#pragma unroll
            for (int u = 0; u < WB; u++) {
                const int jr = (warp - 1) + u * SPLIT_PW, j = r0 + jr;
                if (jr < R && j < nb) {
                    const int4 a0 = reinterpret_cast<const int4 *>(s_qs + (size_t)j * 32)[0];
                    const int4 a1 = reinterpret_cast<const int4 *>(s_qs + (size_t)j * 32)[1];
                    const int4 c0 = reinterpret_cast<const int4 *>(s_c + (size_t)j * 8)[0];
                    const int4 c1 = reinterpret_cast<const int4 *>(s_c + (size_t)j * 8)[1];
                    const float da = s_d[j];
                    const int av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    const int cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                    for (int t = 0; t < RPT; t++) {
                        const unsigned qw[4] = {wq[t][u].x, wq[t][u].y, wq[t][u].z, wq[t][u].w};
                        float v[8];
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            v[k] = __fsub_rn(__int_as_float(dp4a_us(qw[k] & 0x0F0F0F0Fu, av[k], cv[k])), MAGIC_F);
                            v[4 + k] = __fsub_rn(
                                __int_as_float(dp4a_us((qw[k] >> 4) & 0x0F0F0F0Fu, av[4 + k], cv[4 + k])), MAGIC_F);
                        }
                        const size_t fi = ((size_t)(t * R + jr) * 2) * 32 + lane;
                        f[fi] = make_float4(v[0], v[1], v[2], v[3]);
                        f[fi + 32] = make_float4(v[4], v[5], v[6], v[7]);
                        ss[(size_t)(t * R + jr) * 32 + lane] =
                            __fmul_rn(__half2float(__ushort_as_half(ws[t][u])), da);
                    }
                }
            }
            if (r + 1 < nr) load_w(r0 + R);  // the next round's blocks, in flight from here
            mbar_arrive(&bar_full[b]);
        }
    } else {
        // ---- warp 0: the chains, round after round in block order
        for (int r = 0; r < nr; r++) {
            const int b = r & 1, rn = nb - r * R < R ? nb - r * R : R;
            if (!mbar_wait(&bar_full[b], (unsigned)(r >> 1) & 1u, &s_abort, a.err)) break;
            const float4 *f = s_f + (size_t)b * F4;
            const float *ss = s_s + (size_t)b * SS;
            for (int jr = 0; jr < rn; jr++) {
#pragma unroll
                for (int t = 0; t < RPT; t++) {
                    const size_t fi = ((size_t)(t * R + jr) * 2) * 32 + lane;
                    const float4 x = f[fi], y = f[fi + 32];
                    const float dd = ss[(size_t)(t * R + jr) * 32 + lane];
                    acc[t][0][0] = __fmaf_rn(dd, x.x, acc[t][0][0]);
                    acc[t][0][1] = __fmaf_rn(dd, x.y, acc[t][0][1]);
                    acc[t][0][2] = __fmaf_rn(dd, x.z, acc[t][0][2]);
                    acc[t][0][3] = __fmaf_rn(dd, x.w, acc[t][0][3]);
                    acc[t][0][4] = __fmaf_rn(dd, y.x, acc[t][0][4]);
                    acc[t][0][5] = __fmaf_rn(dd, y.y, acc[t][0][5]);
                    acc[t][0][6] = __fmaf_rn(dd, y.z, acc[t][0][6]);
                    acc[t][0][7] = __fmaf_rn(dd, y.w, acc[t][0][7]);
                }
            }
            mbar_arrive(&bar_empty[b]);
        }
    }
    pdl_release();
    __syncthreads();
    if (warp == 0 && !s_abort) gemv_epilogue<RPT, 1, EPI>(a, acc, tile, total_tiles, 0, lane);
}

// Tensor-core GEMM (opt-in, prefill-sized batches; not bit-exact).  The int8
// part of the product runs on tcgen05 kind::i8: per 32-element block j the
// MMA gives isum[r][b] = sum_e (w_e - 8) * a_e exactly (s32 in TMEM); the CUDA
// cores then form out[b][r] = sum_j (dw_j * da_j) * isum_j in f32, block by
// block.  The reference accumulates eight 4-element lane sums per block in its
// AVX2 order instead, so results differ by f32 rounding (~1e-7 relative).
//
// CTA tile: 128 weight rows (four 32-row tiles; for SwiGLU the gate tiles and
// the matching up tiles, two MMAs) x N activation rows.  Operands go to shared
// memory in groups of TG_KB blocks (128 bytes of K per row = one 128-byte
// swizzle atom): the activations' int8 bytes by cp.async from Q8X, the
// weights expanded from nibbles to int8 (w - 8) by the threads; two stages.
// One thread issues the group's TG_KB*RPT MMAs (each block into its own TMEM
// columns, not accumulated) with a commit per block; eight warps drain them:
// warp w reads TMEM lanes 32*(w%4).. (weight rows) and half w/4 of the N
// columns.  The f32 results end in the GEMV epilogues (lane = weight row).
constexpr int TG_M = 128;
constexpr int TG_KB = 4;
constexpr int TG_THREADS = 256;

template <int RPT>
struct TgShape {
    static constexpr int N = RPT == 1 ? 64 : 32;  // activation rows per CTA (MMA N)
    static constexpr int CPT = N / 2;             // columns per thread
    static constexpr size_t a = (size_t)RPT * TG_M * 128;
    static constexpr size_t b = (size_t)N * 128;
    static constexpr size_t dw = (size_t)RPT * TG_M * TG_KB * 4;
    static constexpr size_t da = (size_t)TG_KB * N * 4;
    static constexpr size_t stage = (a + b + dw + da + 1023) / 1024 * 1024;
    // at least 80 KB, so that two CTAs share an SM: two x 256 TMEM columns
    static constexpr size_t smem = 1024 + 2 * stage > 80 * 1024 ? 1024 + 2 * stage : 80 * 1024;
    static constexpr unsigned tcols = (unsigned)(TG_KB * RPT * N);  // 256
};

// eight signed 4-bit weights (w - 8) per 32-bit word from unsigned nibbles:
// v ^ 8 is w - 8 as a 4-bit two's complement value, widened to 8 bits
__device__ __forceinline__ unsigned nib_to_s8(unsigned v) {
    const unsigned t = v ^ 0x08080808u;
    return t | ((t & 0x08080808u) * 0x1Eu);
}

template <int RPT, int EPI>
__global__ void __launch_bounds__(TG_THREADS) gemm_tc_kernel(GemvArgs a, int total_tiles) {
    using SH = TgShape<RPT>;
    constexpr int N = SH::N, CPT = SH::CPT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar_mma[TG_KB];
    __shared__ unsigned s_tmem;
    __shared__ int s_abort;
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quad = warp & 3, hf = warp >> 2;
    const int mt = blockIdx.x, n0 = blockIdx.y * N;
    const int nb = a.nb, ng = (nb + TG_KB - 1) / TG_KB;
    const int mtiles = RPT == 2 ? total_tiles / 2 : total_tiles;  // row tiles of one matrix
    auto tile_of = [&](int t, int q) { return 4 * mt + q + (t ? total_tiles / 2 : 0); };
    auto sA = [&](int s, int t) { return base + (size_t)s * SH::stage + (size_t)t * TG_M * 128; };
    auto sB = [&](int s) { return base + (size_t)s * SH::stage + SH::a; };
    auto sDW = [&](int s) { return reinterpret_cast<float *>(base + (size_t)s * SH::stage + SH::a + SH::b); };
    auto sDA = [&](int s) {
        return reinterpret_cast<float *>(base + (size_t)s * SH::stage + SH::a + SH::b + SH::dw);
    };

    if (tid == 0) {
        for (int k = 0; k < TG_KB; k++) mbar_init(&bar_mma[k], 1);
        s_abort = 0;
        mbar_fence_init();
    }
    if (warp == 0) tc_alloc(&s_tmem, SH::tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const unsigned tbase = s_tmem;

    // ---- staging of group g into stage s: activations by cp.async, weights
    // loaded into registers first (their latency overlaps the drain) and
    // expanded into shared memory after it
    constexpr int AI = RPT * TG_M * TG_KB / TG_THREADS;  // (matrix, row, block) items per thread
    uint4 wq[AI];
    float wd[AI];
    auto stage_b = [&](int g, int s) {
        const int j0 = g * TG_KB, nbg = nb - j0 < TG_KB ? nb - j0 : TG_KB;
        unsigned char *dst0 = sB(s);
        for (int i = tid; i < N * 8; i += TG_THREADS) {
            const int b = i >> 3, c = i & 7;
            unsigned char *dst = dst0 + b * 128 + ((c ^ (b & 7)) << 4);
            if ((c >> 1) < nbg && n0 + b < a.batch)
                cp_async16(dst, a.x.qs + ((size_t)(n0 + b) * nb + j0) * 32 + c * 16);
            else
                *reinterpret_cast<int4 *>(dst) = make_int4(0, 0, 0, 0);
        }
        cp_async_commit();
        float *da = sDA(s);
        for (int i = tid; i < TG_KB * N; i += TG_THREADS) {
            const int k = i / N, b = i - k * N;
            da[i] = (k < nbg && n0 + b < a.batch) ? a.x.d[(size_t)(n0 + b) * nb + j0 + k] : 0.0f;
        }
    };
    auto load_a = [&](int g) {
        const int j0 = g * TG_KB, nbg = nb - j0 < TG_KB ? nb - j0 : TG_KB;
#pragma unroll
        for (int u = 0; u < AI; u++) {
            const int i = tid + u * TG_THREADS;
            const int t = i / (TG_M * TG_KB), r = (i / TG_KB) % TG_M, k = i % TG_KB;
            const int T = tile_of(t, r >> 5);
            const bool ok = k < nbg && (T - (t ? total_tiles / 2 : 0)) < mtiles;
            if (ok) {
                const uint8_t *src = a.w + tile_offset((size_t)T, (size_t)nb, (size_t)(j0 + k));
                wq[u] = *reinterpret_cast<const uint4 *>(src + (r & 31) * 16);
                wd[u] = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(src + 512 + (r & 31) * 2)));
            } else {
                wq[u] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // w - 8 = 0
                wd[u] = 0.0f;
            }
        }
    };
    auto store_a = [&](int s) {
#pragma unroll
        for (int u = 0; u < AI; u++) {
            const int i = tid + u * TG_THREADS;
            const int t = i / (TG_M * TG_KB), r = (i / TG_KB) % TG_M, k = i % TG_KB;
            const uint4 q = wq[u];
            const uint4 lo = make_uint4(nib_to_s8(q.x & 0x0F0F0F0Fu), nib_to_s8(q.y & 0x0F0F0F0Fu),
                                        nib_to_s8(q.z & 0x0F0F0F0Fu), nib_to_s8(q.w & 0x0F0F0F0Fu));
            const uint4 hi = make_uint4(nib_to_s8((q.x >> 4) & 0x0F0F0F0Fu), nib_to_s8((q.y >> 4) & 0x0F0F0F0Fu),
                                        nib_to_s8((q.z >> 4) & 0x0F0F0F0Fu), nib_to_s8((q.w >> 4) & 0x0F0F0F0Fu));
            unsigned char *row = sA(s, t) + r * 128;
            *reinterpret_cast<uint4 *>(row + (((2 * k) ^ (r & 7)) << 4)) = lo;      // elements 0..15
            *reinterpret_cast<uint4 *>(row + (((2 * k + 1) ^ (r & 7)) << 4)) = hi;  // elements 16..31
            sDW(s)[(t * TG_M + r) * TG_KB + k] = wd[u];
        }
    };
    auto issue = [&](int g, int s) {  // thread 0
        const int j0 = g * TG_KB, nbg = nb - j0 < TG_KB ? nb - j0 : TG_KB;
        constexpr unsigned idesc = umma_idesc_s8(TG_M, N);
        for (int k = 0; k < nbg; k++) {
#pragma unroll
            for (int t = 0; t < RPT; t++)
                tc_mma_s8(tbase + (unsigned)((k * RPT + t) * N), umma_desc_sw128(smem_addr(sA(s, t)) + 32u * k),
                          umma_desc_sw128(smem_addr(sB(s)) + 32u * k), idesc, false);
            tc_commit(&bar_mma[k]);
        }
    };

    float acc[RPT][CPT];
#pragma unroll
    for (int t = 0; t < RPT; t++)
#pragma unroll
        for (int c = 0; c < CPT; c++) acc[t][c] = 0.0f;

    load_a(0);   // constant weights: before the wait
    pdl_wait();  // the activation rows are the previous kernel's output
    stage_b(0, 0);
    store_a(0);
    cp_async_wait<0>();
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
        tc_fence_after();
        issue(0, 0);
    }
    int issued = 1;  // groups whose MMAs are in flight or done
    for (int g = 0; g < ng && !s_abort; g++) {
        const int s = g & 1;
        const bool more = g + 1 < ng;
        if (more) {
            stage_b(g + 1, s ^ 1);
            load_a(g + 1);
        }
        // drain the blocks of group g
        const int nbg = nb - g * TG_KB < TG_KB ? nb - g * TG_KB : TG_KB;
        for (int k = 0; k < nbg; k++) {
            if (!mbar_wait(&bar_mma[k], (unsigned)g & 1u, &s_abort, a.err)) break;
            tc_fence_after();
            const float *da = sDA(s) + k * N + hf * CPT;
#pragma unroll
            for (int t = 0; t < RPT; t++) {
                unsigned raw[CPT];
                const unsigned ta = tbase + ((unsigned)(quad * 32) << 16) + (unsigned)((k * RPT + t) * N + hf * CPT);
                if constexpr (CPT == 32)
                    tc_ld32_u32(ta, raw);
                else
                    tc_ld16_u32(ta, raw);
                const float dw = sDW(s)[(t * TG_M + quad * 32 + lane) * TG_KB + k];
#pragma unroll
                for (int c = 0; c < CPT; c++)
                    acc[t][c] = __fmaf_rn(__fmul_rn(dw, da[c]), (float)(int)raw[c], acc[t][c]);
            }
        }
        if (more) store_a(s ^ 1);
        cp_async_wait<0>();
        fence_async_smem();
        tc_fence_before();
        __syncthreads();  // TMEM columns drained, stage s^1 complete
        if (more && !s_abort && tid == 0) {
            tc_fence_after();
            issue(g + 1, s ^ 1);
        }
        if (more) issued = g + 2;
    }
    const bool failed = s_abort != 0;
    if (failed && tid == 0) {
        // a wait gave up: let the committed MMAs finish (bounded) before the
        // TMEM they write is freed
        const int g = issued - 1;
        const long long tw = clock64();
        for (int k = 0; k < TG_KB; k++)
            while (!mbar_test(&bar_mma[k], (unsigned)g & 1u) && clock64() - tw < WAIT_LIMIT) {
            }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tc_dealloc(tbase, SH::tcols);
    pdl_release();
    if (failed) return;
    // ---- epilogue: column by column through the GEMV epilogue (lane = row)
    if (tile_of(0, quad) >= mtiles) return;  // warp-uniform: rows past the matrix
    int tile[RPT];
#pragma unroll
    for (int t = 0; t < RPT; t++) tile[t] = tile_of(t, quad);
#pragma unroll 1
    for (int c = 0; c < CPT; c++) {
        const int b = n0 + hf * CPT + c;
        if (b >= a.batch) break;  // warp-uniform
        float one[RPT][1][8];
#pragma unroll
        for (int t = 0; t < RPT; t++) {
            one[t][0][0] = acc[t][c];
#pragma unroll
            for (int k = 1; k < 8; k++) one[t][0][k] = 0.0f;
        }
        gemv_epilogue<RPT, 1, EPI>(a, one, tile, total_tiles, b, lane);
    }
}

constexpr int TARGET_WARPS = 148 * 4;

template <int BT, int EPI>
void launch_bt(const GemvArgs &a, int total_tiles, int units, cudaStream_t s) {
    const int nbt = (a.batch + BT - 1) / BT;
    dim3 grid((unsigned)((units + 3) / 4), (unsigned)nbt);
    constexpr int RPT = (EPI == EPI_SWIGLU_Q8) ? 2 : 1;
    const size_t smem = (size_t)BT * JC * 68 + 4 * (size_t)RPT * 8 * TILE_BYTES;
    gemv_kernel<BT, EPI><<<grid, 128, smem, s>>>(a, total_tiles, units);
}

// SLM_GEMV_SPLIT=0: batch-1 GEMVs of wide matrices take the staged kernel
inline bool split_enabled() {
    static const bool on = [] {
        const char *e = getenv("SLM_GEMV_SPLIT");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Warps per staged CTA: the most (up to 8) that still gives every SM a CTA
// (within 5%), so the weight tiles are shared by as many rows as the grid allows.
// No more warps than activation rows: a warp past the batch has no work and
// its rows' shared memory would only cut the CTAs an SM holds.
inline int pick_nw(int units, int batch) {
    int cap = 1;
    while (cap < batch && cap < STAGED_MAX_WARPS) cap <<= 1;
    for (int nw = cap; nw > 1; nw >>= 1)
        if ((long)units * ((batch + nw - 1) / nw) >= 140) return nw;
    return 1;
}

template <int BT, int EPI, bool NORM>
void launch_staged(const GemvArgs &a, int nw, int total_tiles, int units, cudaStream_t s) {
    constexpr int RPT = (EPI == EPI_SWIGLU_Q8) ? 2 : 1;
    const int groups = (a.batch + nw * BT - 1) / (nw * BT);
    dim3 grid((unsigned)units, (unsigned)groups);
    launch_kernel(gemv_staged_kernel<BT, EPI, NORM>, grid, dim3(32 * nw),
                  staged_smem(RPT, nw * BT, a.nb, NORM), s, a.pdl, a, total_tiles);
}

// the widest activation tile (<= 4) that still leaves enough warps
inline int pick_bt(int units, int batch) {
    auto warps = [&](int bt) { return (long)units * ((batch + bt - 1) / bt); };
    if (batch >= 4 && warps(4) >= TARGET_WARPS) return 4;
    if (batch >= 2 && warps(2) >= TARGET_WARPS) return 2;
    return 1;
}

inline int units_of(int rows, int epi) {
    const int total_tiles = (rows + TILE_ROWS - 1) / TILE_ROWS;
    return epi == EPI_SWIGLU_Q8 ? total_tiles / 2 : total_tiles;
}

// Prefill-sized batches (GEMM): every warp keeps GEMM_BT activation rows, so
// each unpacked weight block serves GEMM_BT rows and the CTA's weight tiles
// serve 8*GEMM_BT rows; the RMSNorm runs as its own launch (a fused prologue
// would repeat it in every weight unit's CTA).
constexpr int GEMM_BT = 4;
constexpr int GEMM_MIN_BATCH = 1024;

// warps per GEMM CTA: 8, or 4 when 8 would keep two CTAs off an SM's shared memory
inline int gemm_nw(int rpt, int nb) {
    return staged_smem(rpt, STAGED_MAX_WARPS * GEMM_BT, nb, false) <= 100 * 1024 ? STAGED_MAX_WARPS
                                                                               : STAGED_MAX_WARPS / 2;
}

// SLM_DECODE_GEMM=1: decode batches of 16+ rows take the GEMM shape whatever
// the CTA count (the RMSNorm of QKV and gate/up then runs as its own launch)
inline bool decode_gemm_forced() {
    static const bool on = [] {
        const char *e = getenv("SLM_DECODE_GEMM");
        return e && e[0] == '1';
    }();
    return on;
}

// The GEMM shape also serves decode-sized batches (32+) of matrices with
// many row tiles, such as lm_head, when its CTAs still cover every SM twice:
// four activation rows per warp cut the weight unpacking per row by four and
// the CTA count by four against one row per warp.
constexpr int GEMM_MIN_BATCH_WIDE = 32;
// the tensor-core GEMM (opt-in) from this many activation rows up
constexpr int TC_MIN_BATCH = 128;

inline bool gemm_shape(int rpt, int nb, int batch, int units) {
    const bool fits = staged_smem(rpt, gemm_nw(rpt, nb) * GEMM_BT, nb, false) <= STAGED_SMEM_MAX;
    if (!fits) return false;
    if (batch >= GEMM_MIN_BATCH) return true;
    if (decode_gemm_forced() && batch >= 16) return true;
    const long groups = (batch + gemm_nw(rpt, nb) * GEMM_BT - 1) / (gemm_nw(rpt, nb) * GEMM_BT);
    return batch >= GEMM_MIN_BATCH_WIDE && (long)units * groups >= 2L * 148;
}

template <int EPI>
void launch_tc(const GemvArgs &a, int total_tiles, cudaStream_t s) {
    constexpr int RPT = (EPI == EPI_SWIGLU_Q8) ? 2 : 1;
    using SH = TgShape<RPT>;
    const int mtiles = RPT == 2 ? total_tiles / 2 : total_tiles;
    const dim3 grid((unsigned)((mtiles + 3) / 4), (unsigned)((a.batch + SH::N - 1) / SH::N));
    launch_kernel(gemm_tc_kernel<RPT, EPI>, grid, dim3(TG_THREADS), SH::smem, s, a.pdl, a, total_tiles);
}

template <int EPI>
void launch_epi(const GemvArgs &a, cudaStream_t s) {
    constexpr int RPT = (EPI == EPI_SWIGLU_Q8) ? 2 : 1;
    const int total_tiles = (a.rows + TILE_ROWS - 1) / TILE_ROWS;
    const int units = units_of(a.rows, EPI);
    const bool norm = a.nx != nullptr;
    if (a.tc && !norm && (a.batch >= TC_MIN_BATCH || a.tc_any_batch)) {
        launch_tc<EPI>(a, total_tiles, s);
        return;
    }
    if (!norm && gemm_shape(RPT, a.nb, a.batch, units)) {
        // decode batches: four warps per CTA, for twice the CTAs
        const int nw = a.batch < GEMM_MIN_BATCH ? STAGED_MAX_WARPS / 2 : gemm_nw(RPT, a.nb);
        launch_staged<GEMM_BT, EPI, false>(a, nw, total_tiles, units, s);
        return;
    }
    if (!norm && a.batch == 1 && a.nb >= SPLIT_MIN_NB && split_enabled() &&
        split_smem(a.nb) <= STAGED_SMEM_MAX) {
        // one activation row of a wide matrix: the blocks of a tile over eight warps
        launch_kernel(gemv_split_kernel<EPI>, dim3((unsigned)units), dim3(256), split_smem(a.nb), s, a.pdl, a,
                      total_tiles);
        return;
    }
    const int nw = pick_nw(units, a.batch);
    if (staged_smem(RPT, nw, a.nb, norm) <= STAGED_SMEM_MAX) {
        // one activation row per warp
        if (norm)
            launch_staged<1, EPI, true>(a, nw, total_tiles, units, s);
        else
            launch_staged<1, EPI, false>(a, nw, total_tiles, units, s);
        return;
    }
    // tiles too large to stage whole: the weight-ring kernel (no norm prologue)
    const int bt = pick_bt(units, a.batch);
    if (bt == 4)
        launch_bt<4, EPI>(a, total_tiles, units, s);
    else if (bt == 2)
        launch_bt<2, EPI>(a, total_tiles, units, s);
    else
        launch_bt<1, EPI>(a, total_tiles, units, s);
}

template <int EPI>
void set_limits(int bytes) {
    cudaFuncSetAttribute(gemm_tc_kernel<(EPI == EPI_SWIGLU_Q8) ? 2 : 1, EPI>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)TgShape<(EPI == EPI_SWIGLU_Q8) ? 2 : 1>::smem);
    cudaFuncSetAttribute(gemv_kernel<1, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(gemv_kernel<2, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(gemv_kernel<4, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    const int st = bytes < (int)STAGED_SMEM_MAX ? bytes : (int)STAGED_SMEM_MAX;
    cudaFuncSetAttribute(gemv_staged_kernel<1, EPI, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, st);
    cudaFuncSetAttribute(gemv_staged_kernel<1, EPI, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, st);
    cudaFuncSetAttribute(gemv_staged_kernel<GEMM_BT, EPI, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, st);
    cudaFuncSetAttribute(gemv_split_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, st);
}

}  // namespace

void set_gemv_smem_limit(int bytes) {
    set_limits<EPI_STORE>(bytes);
    set_limits<EPI_RESIDUAL>(bytes);
    set_limits<EPI_QKV>(bytes);
    set_limits<EPI_SWIGLU_Q8>(bytes);
}

bool gemv_fuses_norm(int rows, int nb, int epi, int batch) {
    const int rpt = epi == EPI_SWIGLU_Q8 ? 2 : 1;
    const int units = units_of(rows, epi);
    if (gemm_shape(rpt, nb, batch, units)) return false;  // the GEMM shape takes normalized Q8X rows
    return staged_smem(rpt, pick_nw(units, batch), nb, true) <= STAGED_SMEM_MAX;
}

void launch_gemv(const GemvArgs &a, cudaStream_t s) {
    if (a.batch <= 0 || a.rows <= 0) return;
    switch (a.epi) {
        case EPI_STORE: launch_epi<EPI_STORE>(a, s); break;
        case EPI_RESIDUAL: launch_epi<EPI_RESIDUAL>(a, s); break;
        case EPI_QKV: launch_epi<EPI_QKV>(a, s); break;
        case EPI_SWIGLU_Q8: launch_epi<EPI_SWIGLU_Q8>(a, s); break;
        default: break;
    }
}

}  // namespace slm
