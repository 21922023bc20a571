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
// Mapping: a warp owns RPT row tiles (32 rows each, one row per lane per
// tile) and BT activation rows, so every lane keeps RPT*BT*8 accumulators in
// registers while it walks the blocks of its rows in order.  Weights come
// from the repacked 576-byte tiles with one coalesced 128-bit load per lane
// and block; the activation rows of the CTA's batch tile are staged in shared
// memory in chunks of JC blocks and read as warp-wide broadcasts.
//
// The int dot of a lane is one dp4a of the unsigned weight nibbles against
// the activation bytes, seeded with c_k = 0x4B400000 - 8*sum(a): the result
// is the bit pattern of 12582912 + isum_k, so isum_k as f32 costs one exact
// subtraction instead of an int->float conversion.
#include "kernels.h"

namespace slm {

namespace {

constexpr int RPT = 2;   // row tiles per warp
constexpr int JC = 64;   // blocks per shared-memory chunk

template <int BT, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    int8_t *s_qs = (int8_t *)smem;                            // [BT][JC][32]
    int32_t *s_c = (int32_t *)(smem + BT * JC * 32);          // [BT][JC][8]
    float *s_d = (float *)(smem + BT * JC * 64);              // [BT][JC]

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int nb = a.nb;
    const int total_tiles = (a.rows + TILE_ROWS - 1) / TILE_ROWS;
    const int b0 = blockIdx.y * BT;

    // which row tiles this warp owns
    const int unit = blockIdx.x * nwarps + warp;
    int tile[RPT];
    if (EPI == EPI_SWIGLU_Q8) {
        const int half_tiles = total_tiles / 2;
        tile[0] = unit < half_tiles ? unit : -1;
        tile[1] = unit < half_tiles ? unit + half_tiles : -1;
    } else {
#pragma unroll
        for (int t = 0; t < RPT; t++) {
            int ti = unit * RPT + t;
            tile[t] = ti < total_tiles ? ti : -1;
        }
    }

    float acc[RPT][BT][8];
#pragma unroll
    for (int t = 0; t < RPT; t++)
#pragma unroll
        for (int b = 0; b < BT; b++)
#pragma unroll
            for (int k = 0; k < 8; k++) acc[t][b][k] = 0.0f;

    for (int jc = 0; jc < nb; jc += JC) {
        const int jn = nb - jc < JC ? nb - jc : JC;
        __syncthreads();
        // stage activations [b0, b0+BT) x blocks [jc, jc+jn)
        for (int i = threadIdx.x; i < BT * jn * 4; i += blockDim.x) {
            int b = i / (jn * 4), rem = i % (jn * 4);
            int jl = rem >> 2, part = rem & 3;  // part 0,1: qs halves; 2,3: c halves
            int bb = b0 + b;
            int4 v = make_int4(0, 0, 0, 0);
            if (bb < a.batch) {
                size_t blk = (size_t)bb * nb + jc + jl;
                if (part < 2)
                    v = reinterpret_cast<const int4 *>(a.x.qs + blk * 32)[part];
                else
                    v = reinterpret_cast<const int4 *>(a.x.c + blk * 8)[part - 2];
            } else if (part >= 2) {
                v = make_int4(MAGIC_I, MAGIC_I, MAGIC_I, MAGIC_I);
            }
            if (part < 2)
                reinterpret_cast<int4 *>(s_qs + (b * JC + jl) * 32)[part] = v;
            else
                reinterpret_cast<int4 *>(s_c + (b * JC + jl) * 8)[part - 2] = v;
        }
        for (int i = threadIdx.x; i < BT * jn; i += blockDim.x) {
            int b = i / jn, jl = i % jn;
            int bb = b0 + b;
            s_d[b * JC + jl] = bb < a.batch ? a.x.d[(size_t)bb * nb + jc + jl] : 0.0f;
        }
        __syncthreads();

#pragma unroll 2
        for (int jl = 0; jl < jn; jl++) {
            const int j = jc + jl;
            unsigned lo[RPT][4], hi[RPT][4];
            float dw[RPT];
#pragma unroll
            for (int t = 0; t < RPT; t++) {
                if (tile[t] >= 0) {
                    const uint8_t *tp = a.w + tile_offset((size_t)tile[t], nb, j);
                    uint4 q = __ldg(reinterpret_cast<const uint4 *>(tp) + lane);
                    unsigned short hb = __ldg(reinterpret_cast<const unsigned short *>(tp + 512) + lane);
                    dw[t] = __half2float(__ushort_as_half(hb));
                    unsigned qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        lo[t][k] = qw[k] & 0x0F0F0F0Fu;
                        hi[t][k] = (qw[k] >> 4) & 0x0F0F0F0Fu;
                    }
                } else {
                    dw[t] = 0.0f;
#pragma unroll
                    for (int k = 0; k < 4; k++) lo[t][k] = hi[t][k] = 0u;
                }
            }
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
        if (tile[0] < 0) return;  // warp-uniform
        const int hdim = (total_tiles / 2) * TILE_ROWS;
        const int nb_out = hdim / 32;
#pragma unroll
        for (int b = 0; b < BT; b++) {
            const int bb = b0 + b;
            if (bb >= a.batch) break;  // warp-uniform
            const int hrow = tile[0] * TILE_ROWS + lane;
            float o = swiglu1(y[0][b], y[1][b]);
            if (a.out) a.out[(size_t)bb * a.ld_out + hrow] = o;
            q8x_store_block(o, a.q8_out, (size_t)bb * nb_out + tile[0], lane);
        }
    } else {
#pragma unroll
    for (int t = 0; t < RPT; t++) {
        if (tile[t] < 0) continue;  // warp-uniform
        const int row = tile[t] * TILE_ROWS + lane;
#pragma unroll
        for (int b = 0; b < BT; b++) {
            const int bb = b0 + b;
            if (bb >= a.batch) break;  // warp-uniform
            const float v = y[t][b];
            if (EPI == EPI_STORE) {
                if (row < a.rows) a.out[(size_t)bb * a.ld_out + row] = v;
            } else if (EPI == EPI_RESIDUAL) {
                if (row < a.rows)
                    a.out[(size_t)bb * a.ld_out + row] =
                        __fadd_rn(a.res[(size_t)bb * a.ld_res + row], v);
            } else if (EPI == EPI_QKV) {
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
}

template <int BT, int EPI>
void launch_bt(const GemvArgs &a, cudaStream_t s) {
    int total_tiles = (a.rows + TILE_ROWS - 1) / TILE_ROWS;
    int units = EPI == EPI_SWIGLU_Q8 ? total_tiles / 2 : (total_tiles + RPT - 1) / RPT;
    int btiles = (a.batch + BT - 1) / BT;
    // enough CTAs to cover the SMs: shrink the CTA when there are few units
    int nw = 4;
    while (nw > 1 && (long)((units + nw - 1) / nw) * btiles < 2 * 148) nw >>= 1;
    dim3 grid((units + nw - 1) / nw, btiles);
    size_t smem = (size_t)BT * JC * 68;
    gemv_kernel<BT, EPI><<<grid, 32 * nw, smem, s>>>(a);
}

template <int EPI>
void launch_epi(const GemvArgs &a, cudaStream_t s) {
    if (a.batch <= 1)
        launch_bt<1, EPI>(a, s);
    else if (a.batch == 2)
        launch_bt<2, EPI>(a, s);
    else
        launch_bt<4, EPI>(a, s);
}

}  // namespace

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
