/*
 * oracle.h -- CPU restatement of static-lm's per-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a kernels in static-lm_b200/csrc and the timed CPU baseline of
 * bench.py.  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs
 * load it.  The product library (libslm_b200.so) never links, loads or calls
 * anything in this directory.
 *
 * Parity pinning: the reference (Rust + Cranelift) cannot be built in this
 * image (no cargo/rustc).  The restatement is pinned against every known
 * answer its own unit tests hold (vec-dot saturation answers 32512 / 28448 /
 * -128 clamp, kernels.rs:601-650; zero and negative-extreme quantizer blocks,
 * blocks.rs:190-220; quantizer error bounds blocks.rs:153-188; JIT ops vs the
 * libm scalar forms within 1e-5 including tail lengths, engine.rs:226-486;
 * layer vs scalar reference within 1e-4, transformer.rs:999-1208; batched
 * prefill == sequential decode, transformer.rs:1268-1358; token parity of
 * the production engine and the scalar quantized baseline, bench.rs:1273).
 * Bit-level choices that those tests do not pin (AVX2 lane order, Cranelift
 * 4-lane reduction order, the polynomial exp) are restated line by line from
 * the cited source.
 *
 * Numerics modes (orc_mode):
 *   ORC_MODE_X86     the path the reference runs on x86-64 with AVX2+FMA:
 *                    vec_dot_q4_0_q8_0_avx2 (kernels.rs:163-212) and the
 *                    Cranelift-lowered vector ops (lower.rs:212-480).
 *   ORC_MODE_SCALAR  the reference's unfused scalar quantized baseline
 *                    (bench.rs:446-543): scalar vec-dot (kernels.rs:145-161),
 *                    libm expf, sequential sums, scalar attention
 *                    (transformer.rs:214-271).  Its vec-dot numerics equal
 *                    the aarch64 NEON path (kernels.rs:214-249).
 */
#ifndef SLM_ORACLE_H
#define SLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 32

typedef struct {
    uint16_t d;      /* f16 bits */
    uint8_t qs[16];  /* low nibble = elem j, high nibble = elem j+16, offset -8 */
} __attribute__((packed)) orc_block_q4_0;

typedef struct {
    uint16_t d;      /* f16 bits */
    int8_t qs[32];
} __attribute__((packed)) orc_block_q8_0;

enum { ORC_MODE_X86 = 0, ORC_MODE_SCALAR = 1 };

typedef struct {
    int32_t dim;
    int32_t hidden_dim;
    int32_t num_heads;
    int32_t num_kv_heads;
    int32_t max_seq_len;
    float rms_eps;
} orc_config;

typedef struct {
    const float *rms_att_weight;
    const orc_block_q4_0 *wq, *wk, *wv, *wo;
    const float *rms_ffn_weight;
    const orc_block_q4_0 *w_gate, *w_up, *w_down;
} orc_layer_weights;

typedef struct {
    const orc_block_q4_0 *token_embd;
    const orc_layer_weights *layers;
    int32_t num_layers;
    const float *output_norm;
    const orc_block_q4_0 *lm_head;
    int32_t vocab_size;
} orc_model_weights;

/* ---- f16 (half 2.7.1 from_f32 / to_f32: IEEE binary16, round-to-nearest-even) */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);

/* ---- blocks.rs */
void orc_quantize_row_q4_0(const float *src, orc_block_q4_0 *dst, size_t n);
void orc_dequantize_row_q4_0(const orc_block_q4_0 *src, float *dst, size_t n);
void orc_quantize_row_q8_0(const float *src, orc_block_q8_0 *dst, size_t n);
void orc_dequantize_row_q8_0(const orc_block_q8_0 *src, float *dst, size_t n);

/* ---- kernels.rs */
float orc_vec_dot_scalar(const orc_block_q4_0 *w, const orc_block_q8_0 *a, size_t nb);
float orc_vec_dot_x86(const orc_block_q4_0 *w, const orc_block_q8_0 *a, size_t nb);
/* same numerics as orc_vec_dot_x86, with real AVX2 intrinsics when the host has them */
float orc_vec_dot_avx2(const orc_block_q4_0 *w, const orc_block_q8_0 *a, size_t nb);
int orc_host_has_avx2(void);
/* out[b*rows + r] = dot(W[r], xq[b]); threads<=1 runs serially */
void orc_gemm_q4_0(const orc_block_q4_0 *w, const orc_block_q8_0 *xq, float *out,
                   size_t batch, size_t rows, size_t cols, int mode, int threads);
/* gemv_q4_0_arena / gemm_q4_0_arena: quantize `in` into q8 then gemm */
void orc_gemm_q4_0_f32(const orc_block_q4_0 *w, const float *in, orc_block_q8_0 *q8,
                       float *out, size_t batch, size_t rows, size_t cols, int mode,
                       int threads);
/* reference pool policy: max(logical_cpus/2, 1) threads (kernels.rs:71-76) */
int orc_default_pool_threads(void);

/* ---- jit/graph.rs + jit/lower.rs */
float orc_exp_poly(float x);
void orc_softmax(const float *x, float *out, size_t len, int mode);
void orc_rmsnorm(const float *x, const float *w, float *out, size_t len, float eps, int mode);
void orc_swiglu(const float *g, const float *u, float *out, size_t len, int mode);
void orc_residual_add(const float *a, const float *b, float *out, size_t len);
void orc_l2_norm(const float *x, float *out, size_t len, float eps);

/* ---- transformer.rs: RoPE, attention */
void orc_rope_tables(int32_t max_seq, int32_t head_dim, float *cos_out, float *sin_out);
void orc_apply_rope_cached(float *vec, size_t len, const float *cos_row,
                           const float *sin_row, int32_t head_dim);
void orc_apply_rope_in_place(float *vec, size_t len, int32_t pos, int32_t head_dim);
void orc_attention(const float *q, const float *k_cache, const float *v_cache, float *att,
                   float *out, const orc_config *cfg, int32_t pos, int mode);
int32_t orc_sample_argmax(const float *logits, size_t n);

/* ---- transformer.rs: model driver (one sequence per model, like the reference) */
typedef struct orc_model orc_model;
orc_model *orc_model_new(const orc_config *cfg, int32_t num_layers, int32_t vocab_size,
                         int mode, int threads);
void orc_model_free(orc_model *m);
int orc_model_set_weights(orc_model *m, const orc_model_weights *w);
int32_t orc_forward_token(orc_model *m, int32_t token, int32_t pos);
int32_t orc_prefill_tokens(orc_model *m, const int32_t *tokens, int32_t n, int32_t start_pos);
int32_t orc_generate(orc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t *out,
                     int32_t n_out, int32_t eos /* -1 = none */);
void orc_embed_tokens(orc_model *m, const int32_t *tokens, int32_t n, float *out_embedding);
/* layer-level (forward_token_with_kv on layer `layer`, x = model's x buffer) */
void orc_layer_forward_token(orc_model *m, int32_t layer, int32_t pos);
float *orc_model_x(orc_model *m);
float *orc_model_xb(orc_model *m);
float *orc_model_logits(orc_model *m);
float *orc_model_k_cache(orc_model *m, int32_t layer);
float *orc_model_v_cache(orc_model *m, int32_t layer);
float *orc_model_rope_cos(orc_model *m);
float *orc_model_rope_sin(orc_model *m);

/* ---- synthetic inputs */
/* xorshift32 as in main.rs:18-28 / kernels.rs:425-435: (unit*2-1)*scale */
void orc_xorshift_f32(float *out, size_t n, uint32_t seed, float scale);

#ifdef __cplusplus
}
#endif
#endif
