// kernels.h -- launchers of the sm_100a kernels (internal to libslm_b200).
#pragma once

#include <cuda.h>  // CUtensorMap
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

#include "common.cuh"

namespace slm {

// Launch `kernel` on `s`, with the programmatic-serialization attribute when
// `pdl` (the kernel must then call pdl_wait() before reading its
// predecessor's outputs).
template <typename... KArgs, typename... Args>
inline void launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t s, bool pdl, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
// The same with thread-block clusters of `cluster_x` CTAs along x (grid.x a
// multiple of it).
template <typename... KArgs, typename... Args>
inline void launch_kernel_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                  bool pdl, unsigned cluster_x, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---- vector ops / quantization (kernels_vec.cu)
// RMSNorm of `rows` rows (graph.rs:141-155) fused with Q8_0 quantization of the
// result into Q8X (n must be a multiple of 32 when q8 is requested).
// y (optional) receives the f32 normalized rows.
void launch_rmsnorm_q8(const float *x, size_t ldx, const float *w, int n, float eps,
                       float *y, size_t ldy, Q8X q8, int rows, cudaStream_t s, bool pdl = false);
void set_rmsnorm_smem_limit(int bytes);
// Q8_0 quantization of f32 rows into Q8X (blocks.rs:102-123).
void launch_quantize_q8x(const float *x, size_t ldx, int n, Q8X q8, int rows, cudaStream_t s);
// Q8_0 quantization into the reference's 34-byte BlockQ8_0 layout.
void launch_quantize_q8_ref(const float *x, void *blocks, size_t n, cudaStream_t s);
// Reference BlockQ8_0 blocks -> Q8X (for callers that hand in pre-quantized input).
void launch_q8_ref_to_q8x(const void *blocks, Q8X q8, size_t nblocks, cudaStream_t s);
// x[r] = dequantize(token_embd row tokens[r]) (transformer.rs:768-770).
void launch_embed(const uint8_t *tiles, int nb, const int32_t *tokens, int vocab, float *x,
                  size_t ldx, int rows, int32_t *err, cudaStream_t s);
// out[r] = argmax(logits[r]) with the first maximum winning (transformer.rs:656-667).
void launch_argmax(const float *logits, size_t ld, int n, int32_t *out, int rows,
                   cudaStream_t s);
// Standalone JIT-op equivalents on one vector of `len` elements.
void launch_softmax_vec(const float *x, float *out, size_t len, cudaStream_t s);
void launch_rmsnorm_vec(const float *x, const float *w, float *out, size_t len, float eps,
                        cudaStream_t s);
// The same with 1/n given (a graph built for n elements run on len)
void launch_rmsnorm_vec_inv_n(const float *x, const float *w, float *out, size_t len, float eps,
                              float inv_n, cudaStream_t s);
void launch_swiglu_vec(const float *g, const float *u, float *out, size_t len, cudaStream_t s);
void launch_residual_add_vec(const float *a, const float *b, float *out, size_t len,
                             cudaStream_t s);
void launch_l2norm_vec(const float *x, float *out, size_t len, float eps, cudaStream_t s);
// accum[i] = sum over rows b (in order) of y[b][i] * inv_batch, starting from
// 0 (the embedding mean pool, transformer.rs:928-940).
void launch_mean_pool(const float *y, size_t ldy, int rows, int n, float inv_batch,
                      float *accum, cudaStream_t s);
// Greedy feedback between decode steps: tokens = next, pos += 1.
void launch_advance(int32_t *tokens, int32_t *pos, const int32_t *next, int rows,
                    cudaStream_t s);
void launch_rope_vec(float *vec, size_t len, const float *cos_row, const float *sin_row,
                     int head_dim, cudaStream_t s);
// BlockQ4_0 rows [nrows][nb][18 B] (device, 2-byte aligned) -> rows
// [row0, row0+nrows) of the repacked 576-byte row tiles.
void launch_repack_q4(const void *raw, uint64_t nrows, int nb, uint64_t row0, uint8_t *tiles,
                      cudaStream_t s);
// One CTA waiting, with limit_cycles as its bound, on an mbarrier that
// nothing arrives on: sets *err = 3 when the wait gives up.
void launch_wait_selftest(long long limit_cycles, int32_t *err, cudaStream_t s);

// ---- Q4_0 x Q8_0 GEMV / GEMM (kernels_gemv.cu)
enum Epilogue : int {
    EPI_STORE = 0,      // out[b*ld_out + r] = y
    EPI_RESIDUAL = 1,   // out[b*ld_out + r] = res[b*ld_res + r] + y
    EPI_QKV = 2,        // RoPE(q), RoPE(k) -> K cache, v -> V cache
    EPI_SWIGLU_Q8 = 3,  // rows [0,h) gate, [h,2h) up -> silu(g)*u -> Q8X (+ f32 copy)
};

// K and V of activation row b live at
//   k_base + slot[b]*slot_stride + layer_off + pos[b]*kv_dim   (same for v_base)
// i.e. the reference's position-major LayerKvCache (transformer.rs:323-338)
// repeated per sequence slot and layer.
struct QkvArgs {
    float *q;                // [rows_b][dim]
    size_t ldq;
    float *k_base, *v_base;
    const int32_t *slot;     // [rows_b] sequence slot of each activation row
    const int32_t *pos;      // [rows_b] position of each activation row
    size_t slot_stride;      // floats between consecutive slots
    size_t layer_off;        // floats from a slot's start to this layer's block
    int dim, kv_dim, head_dim, max_seq;
    const float *rope_cos, *rope_sin;  // [max_seq][head_dim/2]
    int32_t *err;            // set to 2 when a position is out of range
};

struct GemvArgs {
    const uint8_t *w;        // repacked tiles
    int rows;                // logical rows (for SWIGLU: 2*h, gate then up)
    int nb;                  // blocks per row (cols/32)
    Q8X x;                   // activations, batch rows of nb blocks
    int batch;
    int epi;
    float *out;              // EPI_STORE / EPI_RESIDUAL / SWIGLU f32 copy (may be null)
    size_t ld_out;
    const float *res;        // EPI_RESIDUAL
    size_t ld_res;
    Q8X q8_out;              // EPI_SWIGLU_Q8 destination (nb_out = h/32 blocks per row)
    QkvArgs qkv;
    // Fused RMSNorm prologue (graph.rs:141-155): when nx is set, the
    // activations are rmsnorm(nx rows, nw, eps) quantized to Q8_0 inside the
    // kernel and `x` is not read.  Only valid when gemv_fuses_norm() is true.
    const float *nx;
    size_t ld_nx;
    const float *nw;
    float eps, inv_n;
    int32_t *err;            // set to 3 when a bounded copy wait gave up (may be null)
    bool pdl;                // launch with programmatic dependent launch (staged path)
    // opt-in: the int8 products on the tcgen05 tensor cores (kind::i8) for
    // batches of 128+ rows without the fused RMSNorm prologue; ~1e-7
    // relative to the exact result instead of bit for bit
    bool tc;
    // with tc: also below 128 rows (a row-sharded slice of a step whose
    // whole batch takes the tensor cores, so that every rank computes its
    // rows with the arithmetic the unsharded step uses)
    bool tc_any_batch;
};
void launch_gemv(const GemvArgs &a, cudaStream_t s);
// Whether launch_gemv stages whole weight tiles for this shape (and can then
// run the RMSNorm prologue); false for tiles too large for shared memory.
bool gemv_fuses_norm(int rows, int nb, int epi, int batch);
// Opt the GEMV kernels into `bytes` of dynamic shared memory (current device).
void set_gemv_smem_limit(int bytes);

// ---- attention (kernels_attn.cu, kernels_attn_flash.cu, kernels_attn_tc.cu)
// Boxes of the KV-cache tensor maps: K = 32 floats x K_BOX_KEYS positions
// (128-byte swizzle), V = head_dim floats x V_BOX_POSITIONS positions.
constexpr int K_BOX_KEYS = 128;
constexpr int V_BOX_POSITIONS = 64;
// the box of the fine V map (softmax + PV forms with 16/32-position stages)
constexpr int V_FINE_POSITIONS = 16;
// keys of one flash-decode work item (one V box)
constexpr int FD_ITEM_KEYS = V_BOX_POSITIONS;

struct AttnArgs {
    const float *q;          // [rows][dim] (RoPE applied)
    size_t ldq;
    const float *k_base, *v_base;
    const int32_t *slot, *pos;  // per-row slot/position; null = slot 0 / pos_const
    int pos_const;
    size_t slot_stride, layer_off;
    int max_seq;             // positions >= max_seq are never read
    float *att;              // [rows][num_heads][att_ld]
    size_t att_ld;
    float *out;              // [rows][dim]
    size_t ldo;
    int rows, dim, num_heads, num_kv_heads, head_dim, kv_dim;
    int max_len;             // upper bound of pos+1 over rows (grid sizing)
    float scale;             // 1/sqrt(head_dim) computed on the host
    Q8X q8_out;              // fused path: also quantize `out` (qs == null: no)
    bool write_probs;        // fused path: also store the probabilities in att
    int32_t *err;            // set to 3 when a bounded wait gave up (may be null)
    // fused path: V plane of row r in the tensor map = slot*z_slot + z_layer
    long long z_slot, z_layer;
    bool pdl;                // fused path: programmatic dependent launch
    // KV-head sharding of a batched prefill (fused path): rows come in runs of
    // rows_per_seq per sequence; (row r, KV head g) is computed here only when
    // unit (r / rows_per_seq) * num_kv_heads + g is congruent to shard_r
    // modulo shard_n.  shard_n <= 1: every unit.
    int shard_n, shard_r, rows_per_seq;
    // prefill (fused path): rows come in runs of prefill_run rows holding
    // consecutive positions of one sequence (0 = no such structure)
    int prefill_run;
    // prefill (optional): maxima of every 32 scores of each (row, head),
    // [rows][num_heads][tmax_ld], tmax_ld >= ceil(max_len/32)
    float *tmax;
    int tmax_ld;
    // prefill (fused path): 1 = attention on the tensor cores (tcgen05, 3xTF32;
    // ~1e-6 relative to the exact path instead of bit-exact)
    int prefill_tc;
    // fused path, softmax + PV: 0 = one CTA per (row, KV head) running its
    // kv_mul heads, a thread per (head, dim pair); 1 = one CTA per (row,
    // query head), a thread per dim; 2 = the same with a thread per dim pair;
    // 3 = one CTA per (row, KV head), a thread per (head, dim); 4, 5 = the
    // same with a thread per dim running every head / per (head, dim pair);
    // 6, 7 = one CTA per (row, KV head, half of head_dim), a thread per (head,
    // dim) / (head, dim pair); 8, 9 = as 1 with 32- / 16-position V stages
    // (a deeper ring in the same shared memory); 10 = one CTA per (row, query
    // head, half of head_dim), a thread per dim.  Same results.
    int pv_per_head;
    // decode (opt-in split-K flash-decode, kernels_attn_flash.cu): partial
    // results [rows][num_kv_heads][fd_nch][kv_mul*(head_dim+2)]
    float *fd_part;
    int fd_nch;
};
// vmap: the V tensor map of encode_v_map, or null for the three-phase path;
// kmap: the K tensor map of encode_k_map, or null (per-row K copies)
void launch_attention(const AttnArgs &a, const CUtensorMap *vmap, const CUtensorMap *kmap,
                      cudaStream_t s);
// Split-K flash-decode (kernels_attn_flash.cu): (row, KV head, 64-key chunk)
// work items walked by a persistent grid, then one combine launch per (row,
// KV head); about 1e-6 relative to the exact path.
bool flash_decode_ok(const AttnArgs &a);
int flash_decode_chunks(int max_seq);
// kernel launches of one flash-decode attention (1, or 2 with the combine)
int flash_decode_launches(const AttnArgs &a);
// kmap64: K tensor map with FD_ITEM_KEYS-key boxes (encode_k_map)
void launch_flash_decode(const AttnArgs &a, const CUtensorMap &kmap64, const CUtensorMap &vmap, cudaStream_t s);
void set_flash_decode_smem();
// Exact decode attention in one launch (kernels_attn_cluster.cu): a
// thread-block cluster of C CTAs per (row, KV head) splits the keys for the
// scores and the head dims for the PV chains; bit-exact with the two-kernel
// path.  attn_decode_cluster_size() gives C for these rows (0: the form does
// not apply -- prefill rows, probabilities asked for, head_dim other than 64
// or 128, kv_mul above 4, or score rows beyond 96 KB).  kmap32: K tensor map
// with CL_BOX_KEYS-key boxes; vmap_c: V tensor map with a box of head_dim / C
// floats x CL_BOX_KEYS * C positions.
constexpr int CL_BOX_KEYS = 32;
bool attn_decode_cluster_ok(const AttnArgs &a);
int attn_decode_cluster_size(const AttnArgs &a);
// Whether the cluster form is the faster exact form for these rows: its
// products PV applies and fits three ring stages within the CTA's share of an
// SM (measured faster than the two-kernel form at 8 rows of config 3, slower
// where a second wave or the per-head form's PV would be needed).
bool attn_decode_cluster_preferred(const AttnArgs &a);
void launch_attn_decode_cluster(const AttnArgs &a, const CUtensorMap &kmap32, const CUtensorMap &vmap_c, int C,
                                cudaStream_t s);
void set_attn_decode_cluster_smem();
// Tensor-core causal prefill (kernels_attn_tc.cu): one launch per layer over
// (128 query rows, query head) tiles, then the Q8_0 of the output when asked.
bool attn_prefill_tc_ok(const AttnArgs &a);
void launch_attn_prefill_tc(const AttnArgs &a, cudaStream_t s);
void set_attn_prefill_tc_smem();
// the three phases of launch_attention, for callers that time them apart
void launch_attn_scores(const AttnArgs &a, cudaStream_t s);
void launch_attn_softmax(const AttnArgs &a, cudaStream_t s);
void launch_attn_pv(const AttnArgs &a, cudaStream_t s);
// Two-kernel path (tiled scores, then softmax + PV per (row, KV head) with V
// tiles through the TMA engine); same results as the three-phase path.
// attention_fused_ok() says whether shapes and alignments allow it
// (head_dim % 4 and <= 224, kv_mul <= 8, 16-byte bases, scores fit in
// shared memory).
bool attention_fused_ok(const AttnArgs &a);
// amap: the tensor map of encode_att_map over the att scratch (null = no
// query-tiled prefill softmax/PV)
// vmap_half: the V planes with a box head_dim / 2 wide (encode_v_map with
// head_dim / 2), or null; used by the split softmax + PV forms (modes 6, 7)
// vmap_fine: the V planes with a V_FINE_POSITIONS-position box, or null; used
// by the per-head forms with 32- and 16-position stages (modes 8, 9)
void launch_attn_fused(const AttnArgs &a, const CUtensorMap &vmap, const CUtensorMap *kmap,
                       const CUtensorMap *amap, cudaStream_t s, const CUtensorMap *vmap_half = nullptr,
                       const CUtensorMap *vmap_fine = nullptr);
// 3-D tensor map over att [rows][heads][att_ld] f32, box = 64 positions x
// kv_mul heads x 16 rows (the prefill probability tiles).
bool encode_att_map(CUtensorMap *map, const float *att, int att_ld, int heads, uint64_t rows,
                    int kv_mul);
// 3-D tensor map over `planes` consecutive [max_seq][kv_dim] f32 planes from
// `base`, box = head_dim floats x box_pos positions x 1 plane.  False when
// the driver entry point is missing or the shape is not expressible (the
// caller then uses the three-phase path).
bool encode_v_map(CUtensorMap *map, const float *base, int kv_dim, int max_seq,
                  uint64_t planes, int head_dim, int box_pos = V_BOX_POSITIONS);
// The same planes for K, box = 32 floats x box_keys positions with the
// 128-byte swizzle (head_dim % 32 == 0 only): K_BOX_KEYS for the exact
// scores kernels, FD_ITEM_KEYS for the flash-decode kernel.
bool encode_k_map(CUtensorMap *map, const float *base, int kv_dim, int max_seq,
                  uint64_t planes, int head_dim, int box_keys = K_BOX_KEYS);
// Opt the attention kernels into `bytes` of dynamic shared memory (current device).
void set_attention_smem_limit(int bytes);

// KV-head-sharded prefill: the attention outputs of this rank's units into a
// contiguous send buffer [unit i][row][kd] (unit u = i*nranks + rank, rows
// u/kvh*n .. +n, dims (u%kvh)*kd .. +kd of x), and the all-gathered buffer
// [rank q][unit i][row][kd] back into x.  kd = kv_mul*head_dim.
void launch_shard_pack(const float *x, size_t ldx, float *send, int units_per_rank, int nranks,
                       int rank, int kvh, int kd, int n, cudaStream_t s);
void launch_shard_unpack(const float *recv, float *x, size_t ldx, int units_per_rank, int nranks,
                         int kvh, int kd, int n, cudaStream_t s);

}  // namespace slm
