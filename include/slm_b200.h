/*
 * slm_b200.h -- C ABI of the B200 (sm_100a) implementation of static-lm's
 * per-layer hot path: Q8_0 activation quantization, Q4_0 x Q8_0 GEMV/GEMM,
 * RoPE + KV append, causal GQA attention, the JIT vector ops and the model
 * driver that strings them together.
 *
 * Every entry point replaces one interface of the Rust reference
 * (Bluewraith04/static-lm); the comment above each names it as path:line.
 * Results are bit-identical to the reference's x86-64 (AVX2 + FMA, Cranelift
 * SSE) code path on the same inputs.
 *
 * Conventions
 *  - Functions return SLM_OK (0) or a status code; slm_last_error() returns
 *    the message of the calling thread's last failure.  Where the reference
 *    panics (assert!/bounds), these functions return an error instead.
 *  - "_dev" pointers are device pointers on the object's device; other
 *    pointers are host pointers.  `stream` is a cudaStream_t (NULL = the
 *    legacy default stream); operator calls are stream-ordered and return
 *    once enqueued.
 *  - Nothing here allocates device memory after creation of the object that
 *    owns it (arena, qmatrix, model): the zero-allocation contract of the
 *    reference's hot loop (README.md:7-8).
 */
#ifndef SLM_B200_H
#define SLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SLM_OK = 0,
    SLM_ERR_INVALID_ARG = 1,  /* null pointer, zero/odd size, bad enum */
    SLM_ERR_OUT_OF_BOUNDS = 2, /* slice/position/token/sequence out of range */
    SLM_ERR_OVERLAP = 3,      /* slices that must be disjoint overlap */
    SLM_ERR_SHAPE = 4,        /* sizes that do not match (cols % 32, lengths) */
    SLM_ERR_CAPACITY = 5,     /* arena or scratch too small */
    SLM_ERR_CUDA = 6,         /* a CUDA runtime call failed */
    SLM_ERR_DEVICE_INPUT = 7, /* a device-side input check failed (e.g. token id) */
    SLM_ERR_TIMEOUT = 8       /* a communicator set-up or collective did not complete in time */
};

/* Attention arithmetic of prefill (slm_model_set_prefill_mode,
 * slm_causal_attention_rows): bit-exact CUDA-core chains, or tcgen05 tensor
 * cores with a 3xTF32 split. */
#define SLM_PREFILL_EXACT 0
#define SLM_PREFILL_TENSOR_CORES 1
/* slm_causal_attention_rows only: every row attended as a decode row with
 * the split-K flash-decode kernel (see slm_model_set_decode_mode). */
#define SLM_ATTN_FLASH_DECODE 2

/* Attention arithmetic of decode steps (slm_model_set_decode_mode):
 * SLM_DECODE_EXACT reproduces causal_multi_head_attention_jit bit for bit
 * (every PV sum one sequential chain over the keys); SLM_DECODE_FLASH splits
 * the keys into 128-key chunks (split-K flash-decode: per-chunk maximum, exp
 * sums and PV, combined by the last chunk's CTA), about 1e-6 relative to the
 * exact path. */
#define SLM_DECODE_EXACT 0
#define SLM_DECODE_FLASH 1

/* Message of the calling thread's last failed call ("" if none). */
const char *slm_last_error(void);
/* Library version string. */
const char *slm_version(void);

/* TransformerConfig (src/model/transformer.rs:8-16). */
typedef struct {
    uint32_t dim;
    uint32_t hidden_dim;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t max_seq_len;
    float rms_eps;
} slm_config;

/* ------------------------------------------------------------------ arena
 * One pre-allocated device buffer of f32 with 64-byte aligned bump slices:
 * AlignedArena + ArenaSlice (src/memory/arena.rs:10-122), moved to HBM. */
typedef struct slm_arena slm_arena;

/* ArenaSlice (arena.rs:11-14): offset and length in f32 elements. */
typedef struct {
    uint64_t offset;
    uint64_t len;
} slm_slice;

/* AlignedArena::with_capacity (arena.rs:54-75): zeroed device buffer. */
int slm_arena_create(int device, uint64_t capacity, slm_arena **out);
void slm_arena_destroy(slm_arena *arena);
/* AlignedArena::alloc_slice (arena.rs:96-110). */
int slm_arena_alloc_slice(slm_arena *arena, uint64_t len, slm_slice *out);
/* AlignedArena::alloc_q8_scratch (arena.rs:113-120).  Sized for this
 * library's device activation format (68 bytes per 32-element block: the
 * int8 values, eight dot-product lane constants and the scale), which is
 * opaque to callers. */
int slm_arena_alloc_q8_scratch(slm_arena *arena, uint64_t num_blocks, slm_slice *out);
/* AlignedArena::reset (arena.rs:91-93). */
void slm_arena_reset(slm_arena *arena);
/* AlignedArena::capacity / used (arena.rs:79-88), in f32 elements. */
uint64_t slm_arena_capacity(const slm_arena *arena);
uint64_t slm_arena_used(const slm_arena *arena);
/* Device address of a slice (bounds-checked; NULL on error). */
float *slm_arena_device_ptr(slm_arena *arena, slm_slice s);
/* AlignedArena::get_mut(s).copy_from_slice(host) (arena.rs:146-150);
 * synchronous, n must equal s.len. */
int slm_arena_write(slm_arena *arena, slm_slice s, const float *host, uint64_t n);
/* AlignedArena::get(s) copied to the host (arena.rs:140-144); synchronous. */
int slm_arena_read(slm_arena *arena, slm_slice s, float *host, uint64_t n);

/* ------------------------------------------------------------- Q4_0 weights
 * A rows x cols matrix of BlockQ4_0 (src/quant/blocks.rs:11-16, 18 bytes per
 * 32 weights, row-major as GgufFile::tensor_q4_0 returns it,
 * src/memory/loader.rs:496-500) uploaded to the device and repacked into
 * 32-row tiles for coalesced 128-bit loads. */
typedef struct slm_qmatrix slm_qmatrix;
int slm_qmatrix_upload(int device, const void *blocks, uint64_t rows, uint64_t cols,
                       slm_qmatrix **out);
/* Undo the repacking: writes rows*cols/32 BlockQ4_0 (byte-exact round trip). */
int slm_qmatrix_download(const slm_qmatrix *w, void *blocks_out);
void slm_qmatrix_destroy(slm_qmatrix *w);

/* ---------------------------------------------------------------- operators */

/* gemv_q4_0_arena (src/quant/kernels.rs:289-303): quantize `input` (cols
 * floats) to Q8_0 into q8_scratch, then output[r] = dot(W[r], input_q8). */
int slm_gemv_q4_0_arena(slm_arena *arena, const slm_qmatrix *w, slm_slice input,
                        slm_slice q8_scratch, slm_slice output, uint64_t rows, uint64_t cols,
                        void *stream);
/* gemm_q4_0_arena (kernels.rs:398-415): output[b*rows + r] = dot(W[r], q8(inputs[b])). */
int slm_gemm_q4_0_arena(slm_arena *arena, const slm_qmatrix *w, slm_slice inputs,
                        slm_slice q8_scratch, slm_slice output, uint64_t batch, uint64_t rows,
                        uint64_t cols, void *stream);
/* gemm_q4_0 (kernels.rs:308-394) on pre-quantized BlockQ8_0 input
 * (batch*cols/32 blocks of 34 bytes).  scratch_dev must hold
 * slm_gemm_q4_0_scratch_bytes(batch, cols) bytes, 16-byte aligned. */
int slm_gemm_q4_0(const slm_qmatrix *w, const void *inputs_q8_dev, float *output_dev,
                  uint64_t batch, uint64_t rows, uint64_t cols, void *scratch_dev,
                  uint64_t scratch_bytes, void *stream);
uint64_t slm_gemm_q4_0_scratch_bytes(uint64_t batch, uint64_t cols);
/* No reference counterpart (opt-in arithmetic).  slm_gemm_q4_0 with the int8
 * products on the tcgen05 tensor cores (kind::i8) for batch >= 128: per
 * 32-element block the exact int32 sum of (w - 8) * a, then
 * out += (dw * da) * isum in f32 block by block, where the reference adds eight
 * four-element lane sums per block in its AVX2 order.  Results agree with
 * slm_gemm_q4_0 to f32 rounding (~1e-7 relative), not bit for bit; batches
 * below 128 run the exact kernels.  Same arguments as slm_gemm_q4_0. */
int slm_gemm_q4_0_tensor_cores(const slm_qmatrix *w, const void *inputs_q8_dev, float *output_dev,
                               uint64_t batch, uint64_t rows, uint64_t cols, void *scratch_dev,
                               uint64_t scratch_bytes, void *stream);
/* No counterpart in the reference.  The same product as slm_gemm_q4_0_arena
 * (output[b*rows + r] = dot(W[r], q8(inputs[b]))) for callers that must not
 * allocate device memory on this path: a host running under a device-memory
 * budget fixed at start-up, or one that keeps cudaMalloc/cudaFree (which can
 * synchronize the device and stall every stream) off its serving loop.  The
 * Q8_0 activations go to a static buffer of SLM_NOALLOC_SCRATCH_BYTES in
 * the library's device image, so batch*cols/32 blocks of 68 bytes must fit:
 * batch*cols <= 1,973,760; larger sizes return SLM_ERR_CAPACITY.  The first
 * call on a device looks the buffer's address up (cudaGetSymbolAddress), so
 * make that first call before any stream capture.  The address is cached per
 * process and device ordinal for the life of the process: after a
 * cudaDeviceReset (which destroys the context that holds the buffer) this
 * entry point must not be called again in that process.  All calls share the one
 * buffer: calls that overlap on the GPU (different streams, or different
 * host threads without ordering) race on it and must be serialized by the
 * caller.  inputs_dev is [batch][cols] f32, output_dev [batch][rows] f32,
 * both device memory on the weights' device. */
#define SLM_NOALLOC_SCRATCH_BYTES (4u << 20)
int slm_gemm_q4_0_f32_noalloc(const slm_qmatrix *w, const float *inputs_dev, float *output_dev,
                              uint64_t batch, uint64_t rows, uint64_t cols, void *stream);
/* No reference counterpart (the reference has no device waits).  Runs, on
 * `device`, one CTA whose threads wait on an mbarrier that nothing arrives
 * on, through the same bounded wait every TMA pipeline of this library uses,
 * with limit_cycles (1 .. 2e9 SM clock cycles; the kernels use 2e9, about
 * 1 s) as its bound.  The wait gives up, the kernel sets the device error
 * flag and returns, and this call reports it the way the model entry points
 * do: SLM_ERR_DEVICE_INPUT "a device wait timed out".  The context stays
 * usable.  Any other return means the bounded-wait path is broken. */
int slm_selftest_bounded_wait(int device, uint64_t limit_cycles);
/* quantize_row_q8_0 (src/quant/blocks.rs:102-123) into BlockQ8_0 (34 B). */
int slm_quantize_row_q8_0(const float *src_dev, void *dst_blocks_dev, uint64_t n, void *stream);

/* The JIT vector operators.  Same calling convention as JitKernelFn
 * (src/jit/engine.rs:15): a host array of device input pointers, one output,
 * a length; the graph constants (n, eps) that FuseGraph bakes in at compile
 * time are passed explicitly.  out may alias inputs[0]. */
/* FuseGraph::rmsnorm(len, eps) (graph.rs:141-155), inputs = {x, weight}. */
int slm_exec_rmsnorm(const float *const *inputs, float *out, uint64_t len, float eps,
                     void *stream);
/* FuseGraph::softmax (graph.rs:168-179), inputs = {x}. */
int slm_exec_softmax(const float *const *inputs, float *out, uint64_t len, void *stream);
/* FuseGraph::swiglu (graph.rs:131-138), inputs = {gate, up}. */
int slm_exec_swiglu(const float *const *inputs, float *out, uint64_t len, void *stream);
/* FuseGraph::residual_add (graph.rs:158-164), inputs = {a, b}. */
int slm_exec_residual_add(const float *const *inputs, float *out, uint64_t len, void *stream);
/* FuseGraph::l2_norm(eps) (graph.rs:182-193), inputs = {x}. */
int slm_exec_l2_norm(const float *const *inputs, float *out, uint64_t len, float eps,
                     void *stream);

/* JitKernelFn (src/jit/engine.rs:15): the raw entry point of a compiled
 * FuseGraph, (inputs, output, len).  Here inputs is a host array of device
 * pointers and output a device pointer; the function enqueues the operator
 * on the stream bound at compile time and returns (the reference's runs to
 * completion before returning; here results are stream-ordered). */
typedef void (*slm_jit_kernel_fn)(const float *const *inputs, float *output, size_t len);
enum {
    SLM_JIT_RMSNORM = 0,      /* FuseGraph::rmsnorm(n, eps), inputs {x, weight} (graph.rs:141-155) */
    SLM_JIT_SOFTMAX = 1,      /* FuseGraph::softmax(), inputs {x} (graph.rs:168-179) */
    SLM_JIT_SWIGLU = 2,       /* FuseGraph::swiglu(), inputs {gate, up} (graph.rs:131-138) */
    SLM_JIT_RESIDUAL_ADD = 3, /* FuseGraph::residual_add(), inputs {a, b} (graph.rs:158-164) */
    SLM_JIT_L2_NORM = 4       /* FuseGraph::l2_norm(eps), inputs {x} (graph.rs:182-193) */
};
/* JitEngine::compile (engine.rs:66-72): a function pointer with the
 * JitKernelFn calling convention for operator `op`, with the constants its
 * FuseGraph constructor bakes in (n: the element count whose 1/n RMSNorm
 * uses; eps) and the stream (a cudaStream_t, NULL = legacy default) it
 * enqueues on.  The same (op, n, eps, stream) returns the same pointer (the
 * engine's graph cache); up to 64 distinct ones per process, then
 * SLM_ERR_CAPACITY.  The functions stay valid until the process exits.  A
 * launch failure inside one is reported by slm_last_error() on that thread. */
int slm_jit_compile(int op, uint64_t n, float eps, void *stream, slm_jit_kernel_fn *kernel_out);

/* RoPE tables of LayerWorkspace::allocate (transformer.rs:124-133), computed
 * on the host with the C library's powf/sinf/cosf; cos/sin hold
 * max_seq*head_dim/2 floats. */
int slm_rope_tables(uint32_t max_seq, uint32_t head_dim, float *cos_host, float *sin_host);
/* apply_rope_cached (transformer.rs:178-194), in place on the device. */
int slm_apply_rope_cached(float *vec_dev, uint64_t len, const float *cos_row_dev,
                          const float *sin_row_dev, uint32_t head_dim, void *stream);
/* causal_multi_head_attention_jit (transformer.rs:273-321): q [dim],
 * k/v caches [max_seq_len][kv_dim], att [num_heads][max_seq_len] scratch,
 * out [dim]; attends positions 0..=pos. */
int slm_causal_attention(const float *q_dev, const float *k_cache_dev, const float *v_cache_dev,
                         float *att_dev, float *out_dev, const slm_config *cfg, uint32_t pos,
                         void *stream);
/* The attention of n consecutive rows at positions start_pos..start_pos+n-1
 * of one sequence: the per-token loop of forward_batch_with_kv
 * (transformer.rs:563-593) over causal_multi_head_attention_jit.  q [n][dim],
 * k/v caches [max_seq_len][kv_dim] holding positions < start_pos+n,
 * att [n][num_heads][max_seq_len] scratch, out [n][dim].  mode is
 * SLM_PREFILL_EXACT (bit-exact), SLM_PREFILL_TENSOR_CORES (3xTF32 tensor
 * cores, head_dim 32 or 64; other shapes run exact) or SLM_ATTN_FLASH_DECODE
 * (each row through the split-K flash-decode kernel; head_dim 64 or 128,
 * else SLM_ERR_SHAPE).  Synchronizes `stream`. */
int slm_causal_attention_rows(const float *q_dev, const float *k_cache_dev,
                              const float *v_cache_dev, float *att_dev, float *out_dev,
                              const slm_config *cfg, uint32_t n, uint32_t start_pos, int mode,
                              void *stream);
/* sample_argmax (transformer.rs:654-667): first maximum wins. */
int slm_sample_argmax(const float *logits_dev, uint64_t n, int32_t *out_dev, void *stream);

/* ------------------------------------------------------------------- model
 * TransformerModel (transformer.rs:698-949) for up to `max_sequences`
 * independent sequences, each with its own KV cache, in one device arena.
 * Weights are host pointers in the reference's layout (GgufFile::
 * model_weights, loader.rs:525-553), uploaded once at creation. */
typedef struct {
    const float *rms_att_weight;            /* [dim] */
    const void *wq, *wk, *wv, *wo;          /* BlockQ4_0 [rows*cols/32] */
    const float *rms_ffn_weight;            /* [dim] */
    const void *w_gate, *w_up, *w_down;
} slm_layer_weights;

typedef struct {
    const void *token_embd;                 /* [vocab x dim] BlockQ4_0 */
    const slm_layer_weights *layers;
    uint32_t num_layers;
    const float *output_norm;               /* [dim] */
    const void *lm_head;                    /* NULL = tied to token_embd (loader.rs:534-538) */
    uint32_t vocab_size;
} slm_model_weights;

typedef struct slm_model slm_model;

/* TransformerModel::new (transformer.rs:714-743).  max_rows bounds the
 * number of activation rows of one call: prompt tokens of a prefill, or
 * sequences of a batched decode step. */
int slm_model_create(int device, const slm_config *cfg, const slm_model_weights *w,
                     uint32_t max_sequences, uint32_t max_rows, slm_model **out);
void slm_model_destroy(slm_model *m);
/* The stream every model call runs on (a cudaStream_t). */
void *slm_model_stream(slm_model *m);
/* Bytes of device memory the model holds (weights + arena). */
uint64_t slm_model_device_bytes(const slm_model *m);

/* TransformerModel::forward_token (transformer.rs:747-795) on sequence `seq`. */
int slm_model_forward_token(slm_model *m, uint32_t seq, int32_t token, uint32_t pos,
                            int32_t *next_token);
/* TransformerModel::prefill_tokens (transformer.rs:799-854). */
int slm_model_prefill_tokens(slm_model *m, uint32_t seq, const int32_t *tokens, uint32_t n,
                             uint32_t start_pos, int32_t *next_token);
/* Batched prefill of nseq independent prompts of n tokens each at positions
 * 0..n-1 (tokens [nseq][n], sequence slots seqs[nseq]): one forward over the
 * nseq*n rows, the same per-token results as prefill_tokens on each prompt
 * (forward_batch_with_kv, transformer.rs:491-651).  next[i] = greedy next
 * token of prompt i; logits row i = its logits.  After
 * slm_model_attach_shard with nranks > 1, each rank computes the attention
 * of its (sequence, KV head) units only (slm_shard_units) and one NCCL
 * all-gather per layer assembles the outputs before Wo; when nseq*n divides by
 * nranks, Wo and the FFN then run on this rank's nseq*n/nranks rows and a
 * second, in-place all-gather per layer hands every rank all rows again.
 * Every rank holds the full results (and every sequence's KV: the QKV
 * projection runs on all rows).  Requires nseq*num_kv_heads to divide by
 * nranks. */
int slm_model_prefill_batch(slm_model *m, uint32_t nseq, const uint32_t *seqs,
                            const int32_t *tokens, uint32_t n, int32_t *next);
/* Attention arithmetic of prefill forwards (prefill_tokens, prefill_batch):
 * SLM_PREFILL_EXACT (default) reproduces causal_multi_head_attention_jit
 * (transformer.rs:273-321) bit for bit on the CUDA cores;
 * SLM_PREFILL_TENSOR_CORES runs QK^T and PV on the tcgen05 tensor cores with
 * a 3xTF32 split (about 1e-6 relative to the exact path, not bit-exact) and
 * the int8 products of the Wq/Wk/Wv, Wo, gate/up and down projections on
 * tcgen05 kind::i8 (as slm_gemm_q4_0_tensor_cores), for callers that accept
 * the tolerance.  Decode attention has its own mode
 * (slm_model_set_decode_mode).  No reference counterpart (the reference has
 * one CPU path). */
int slm_model_set_prefill_mode(slm_model *m, int mode);
/* Attention arithmetic of decode steps (decode_batch, forward_token,
 * generate, decode_steps_device, embed excluded): SLM_DECODE_EXACT (default,
 * bit-exact) or SLM_DECODE_FLASH (split-K flash-decode, head_dim 64 or 128
 * and kv_mul 1, 2, 3, 4, 6 or 8; other shapes stay exact).  Flash results are
 * within 1e-3 relative / 1e-4 absolute of the exact attention; greedy tokens
 * may differ where Q8_0 rounding of the attention output flips a near-tie.
 * Drops the captured decode graphs.  No reference counterpart (the reference
 * has one CPU path). */
int slm_model_set_decode_mode(slm_model *m, int mode);
/* NCCL unique id (bytes = 128) for slm_model_attach_shard; made on one rank
 * and sent to the others by the host. */
int slm_nccl_unique_id(void *id_out, uint64_t bytes);
/* Join a group of nranks models (one per GPU, collective: every rank calls it
 * with the same id) for KV-head-sharded batched prefill.  NCCL is loaded at
 * run time (libnccl.so.2).  nranks = 1 detaches nothing and needs no id.
 * The communicator is set up non-blocking: if the group is not complete
 * within the model's communicator timeout (a rank never joins), the call
 * aborts it and returns SLM_ERR_TIMEOUT; it may then be called again.  No
 * reference counterpart (the reference is single-process; it aborts on any
 * fault, Cargo.toml:21). */
int slm_model_attach_shard(slm_model *m, const void *id, uint64_t bytes, int nranks, int rank);
/* Bound, in milliseconds (default 120000), on the communicator set-up of
 * slm_model_attach_shard and on every sharded batched prefill's wait for its
 * collectives.  A prefill whose collectives do not complete in time (a rank
 * stopped taking part) aborts the communicator, which ends its waiting NCCL
 * kernels, and returns SLM_ERR_TIMEOUT; later sharded prefills return
 * SLM_ERR_INVALID_ARG until the group is attached again. */
int slm_model_set_comm_timeout(slm_model *m, uint32_t timeout_ms);
/* Units (sequence*num_kv_heads + KV head) that `rank` computes in a sharded
 * batched prefill, in all-gather order (unit i*nranks + rank); returns their
 * count (0 when nseq*num_kv_heads does not divide by nranks). */
uint32_t slm_shard_units(uint32_t nseq, uint32_t num_kv_heads, uint32_t nranks, uint32_t rank,
                         uint32_t *units_out, uint32_t capacity);
/* TransformerModel::generate (transformer.rs:858-892); eos < 0 = none. */
int slm_model_generate(slm_model *m, uint32_t seq, const int32_t *prompt, uint32_t n_prompt,
                       int32_t *out_tokens, uint32_t n_out, int32_t eos, uint32_t *generated);
/* TransformerModel::embed_tokens (transformer.rs:896-948) on sequence
 * `seq`'s KV cache; out_embedding has dim floats. */
int slm_model_embed_tokens(slm_model *m, uint32_t seq, const int32_t *tokens, uint32_t n,
                           float *out_embedding);
/* One decode step of n independent sequences at once: row i runs
 * forward_token(tokens[i], pos[i]) on sequence seqs[i] (host arrays). */
int slm_model_decode_batch(slm_model *m, uint32_t n, const uint32_t *seqs,
                           const int32_t *tokens, const uint32_t *pos, int32_t *next_tokens);
/* `steps` greedy decode steps of n sequences without leaving the device:
 * step s feeds each row's argmax back as its next token at pos+1.
 * seqs/tokens/pos are device arrays of n entries (tokens and pos advance in
 * place); out_dev receives steps*n token ids (step-major).  Enqueued on the
 * model stream; captured in CUDA graphs.  The n sequences must be distinct
 * (with 16 or more rows, two halves of the batch run concurrently). */
int slm_model_decode_steps_device(slm_model *m, uint32_t n, const uint32_t *seqs_dev,
                                  int32_t *tokens_dev, uint32_t *pos_dev, uint32_t steps,
                                  int32_t *out_dev, uint32_t max_pos_hint);

/* KV-cache access (arena.get / get_mut on LayerKvCache, transformer.rs:323-338):
 * rows [row0, row0+nrows) of K (which = 0) or V (which = 1) of one layer of
 * one sequence, nrows*kv_dim floats, synchronous. */
int slm_model_kv_write(slm_model *m, uint32_t seq, uint32_t layer, uint32_t which,
                       uint32_t row0, uint32_t nrows, const float *host);
int slm_model_kv_read(slm_model *m, uint32_t seq, uint32_t layer, uint32_t which,
                      uint32_t row0, uint32_t nrows, float *host);
/* Device-to-device variant of slm_model_kv_write (src_dev holds nrows*kv_dim
 * floats); enqueued on the model stream. */
int slm_model_kv_write_device(slm_model *m, uint32_t seq, uint32_t layer, uint32_t which,
                              uint32_t row0, uint32_t nrows, const float *src_dev);
/* Logits (vocab floats) of row `row` of the last forward/decode call. */
int slm_model_read_logits(slm_model *m, uint32_t row, float *host);
/* Hidden state x (dim floats) of activation row `row` after the last call. */
int slm_model_read_hidden(slm_model *m, uint32_t row, float *host);

/* ---------------------------------------------------------- measurement
 * Phases of one decode step, in launch order within a layer. */
enum {
    SLM_PHASE_EMBED = 0,
    SLM_PHASE_RMSNORM = 1,       /* fused RMSNorm + Q8_0 quantize */
    SLM_PHASE_QKV = 2,           /* Wq/Wk/Wv GEMV + RoPE + KV append */
    SLM_PHASE_ATTN_SCORES = 3,
    SLM_PHASE_ATTN_SOFTMAX = 4,
    SLM_PHASE_ATTN_PV = 5,
    SLM_PHASE_QUANTIZE = 6,      /* Q8_0 quantize of the attention output */
    SLM_PHASE_WO = 7,            /* Wo GEMV + residual */
    SLM_PHASE_GATE_UP = 8,       /* gate/up GEMV + SwiGLU + Q8_0 quantize */
    SLM_PHASE_DOWN = 9,          /* down GEMV + residual */
    SLM_PHASE_LM_HEAD = 10,
    SLM_PHASE_ARGMAX = 11,
    SLM_PHASE_ADVANCE = 12,
    SLM_PHASE_ATTN_FUSED = 13,   /* scores + softmax + PV (+ Q8_0) in one kernel */
    SLM_NUM_PHASES = 14
};
/* Same work as slm_model_decode_steps_device, launched without graphs and
 * with a CUDA event on the model stream at every phase boundary; adds each
 * phase's device time over all steps and layers into phase_ms
 * [SLM_NUM_PHASES] (milliseconds).  Synchronous. */
int slm_model_profile_decode(slm_model *m, uint32_t n, const uint32_t *seqs_dev,
                             int32_t *tokens_dev, uint32_t *pos_dev, uint32_t steps,
                             uint32_t max_pos_hint, float *phase_ms);
/* Kernel launches one decode step of n rows issues (the kernel nodes of its
 * graph, the greedy advance included). */
uint32_t slm_model_launches_per_decode_step(const slm_model *m, uint32_t n);

#ifdef __cplusplus
}
#endif
#endif /* SLM_B200_H */
