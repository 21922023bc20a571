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
#include "kernels.h"

namespace slm {

namespace {

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gsrc));
}

constexpr int JC = 64;   // activation blocks per shared-memory chunk (multiple of PF)

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
            unsigned lo[RPT][4], hi[RPT][4];
            float dw[RPT];
#pragma unroll
            for (int t = 0; t < RPT; t++) {
                const uint8_t *slot = s_w + (t * PF + j % PF) * TILE_BYTES;
                const uint4 q = *reinterpret_cast<const uint4 *>(slot + lane * 16);
                dw[t] = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(slot + 512 + lane * 2)));
                const unsigned qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    lo[t][k] = qw[k] & 0x0F0F0F0Fu;
                    hi[t][k] = (qw[k] >> 4) & 0x0F0F0F0Fu;
                }
            }
            __syncwarp();  // the slot may be refilled by the next fetch
#pragma unroll
            for (int b = 0; b < BT; b++) {
                const int4 a0 = reinterpret_cast<const int4 *>(s_qs + (b * JC + jl) * 32)[0];
                const int4 a1 = reinterpret_cast<const int4 *>(s_qs + (b * JC + jl) * 32)[1];
                const int4 c0 = reinterpret_cast<const int4 *>(s_c + (b * JC + jl) * 8)[0];
                const int4 c1 = reinterpret_cast<const int4 *>(s_c + (b * JC + jl) * 8)[1];
                const float da = s_d[b * JC + jl];
                const int av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const int cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                for (int t = 0; t < RPT; t++) {
                    const float d = __fmul_rn(dw[t], da);
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        float f0 = __fsub_rn(__int_as_float(dp4a_us(lo[t][k], av[k], cv[k])), MAGIC_F);
                        acc[t][b][k] = __fmaf_rn(d, f0, acc[t][b][k]);
                        float f1 = __fsub_rn(__int_as_float(dp4a_us(hi[t][k], av[4 + k], cv[4 + k])), MAGIC_F);
                        acc[t][b][4 + k] = __fmaf_rn(d, f1, acc[t][b][4 + k]);
                    }
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;\n" ::);
    if (!live) return;

    // ---- epilogue
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
                    const float c = q.rope_cos[(size_t)p * half + jj];
                    const float s = q.rope_sin[(size_t)p * half + jj];
                    float r;
                    if ((i & 1) == 0)  // v0*c - v1*s
                        r = __fsub_rn(__fmul_rn(v, c), __fmul_rn(partner, s));
                    else  // v0*s + v1*c
                        r = __fadd_rn(__fmul_rn(partner, s), __fmul_rn(v, c));
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

constexpr int TARGET_WARPS = 148 * 4;

template <int BT, int EPI>
void launch_bt(const GemvArgs &a, int total_tiles, int units, cudaStream_t s) {
    const int nbt = (a.batch + BT - 1) / BT;
    dim3 grid((unsigned)((units + 3) / 4), (unsigned)nbt);
    constexpr int RPT = (EPI == EPI_SWIGLU_Q8) ? 2 : 1;
    const size_t smem = (size_t)BT * JC * 68 + 4 * (size_t)RPT * 8 * TILE_BYTES;
    gemv_kernel<BT, EPI><<<grid, 128, smem, s>>>(a, total_tiles, units);
}

template <int EPI>
void launch_epi(const GemvArgs &a, cudaStream_t s) {
    const int total_tiles = (a.rows + TILE_ROWS - 1) / TILE_ROWS;
    const int units = EPI == EPI_SWIGLU_Q8 ? total_tiles / 2 : total_tiles;
    // the widest activation tile (<= 4) that still leaves enough warps
    auto warps = [&](int bt) { return (long)units * ((a.batch + bt - 1) / bt); };
    if (a.batch >= 4 && warps(4) >= TARGET_WARPS)
        launch_bt<4, EPI>(a, total_tiles, units, s);
    else if (a.batch >= 2 && warps(2) >= TARGET_WARPS)
        launch_bt<2, EPI>(a, total_tiles, units, s);
    else
        launch_bt<1, EPI>(a, total_tiles, units, s);
}

template <int EPI>
void set_limits(int bytes) {
    cudaFuncSetAttribute(gemv_kernel<1, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(gemv_kernel<2, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(gemv_kernel<4, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace

void set_gemv_smem_limit(int bytes) {
    set_limits<EPI_STORE>(bytes);
    set_limits<EPI_RESIDUAL>(bytes);
    set_limits<EPI_QKV>(bytes);
    set_limits<EPI_SWIGLU_Q8>(bytes);
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
