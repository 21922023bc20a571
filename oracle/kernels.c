/*
 * kernels.c -- Q4_0 x Q8_0 dot products, GEMV/GEMM and the row-parallel
 * worker pool (TEST INFRASTRUCTURE: parity checker and timed CPU baseline).
 * Restates static-lm src/quant/kernels.rs.
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#include "oracle.h"

/* kernels.rs:145-161 -- per block: exact int sum, then sumf += isum * (dw*da),
 * multiply and add rounded separately.  The NEON path (kernels.rs:214-249)
 * has the same numerics. */
float orc_vec_dot_scalar(const orc_block_q4_0 *w, const orc_block_q8_0 *a, size_t nb) {
    float sumf = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        int sum_i = 0;
        for (int j = 0; j < 16; j++) {
            int v0 = (int)(w[b].qs[j] & 0x0F) - 8;
            int v1 = (int)(w[b].qs[j] >> 4) - 8;
            sum_i += v0 * (int)a[b].qs[j] + v1 * (int)a[b].qs[j + 16];
        }
        float d = orc_f16_to_f32(w[b].d) * orc_f16_to_f32(a[b].d);
        float prod = (float)sum_i * d;
        sumf = sumf + prod;
    }
    return sumf;
}

/* kernels.rs:163-212 (AVX2+FMA), restated lane by lane.
 * Lane k (0..7) holds the exact int sum of elements 4k..4k+3 (elements 0..15
 * are the low nibbles, 16..31 the high nibbles; activations clamped to >= -127,
 * :189-191).  Each lane accumulates acc_k = fma(dw*da, isum_k, acc_k) in block
 * order; the final horizontal sum is ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7))
 * (:203-211). */
float orc_vec_dot_x86(const orc_block_q4_0 *w, const orc_block_q8_0 *a, size_t nb) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t b = 0; b < nb; b++) {
        float d = orc_f16_to_f32(w[b].d) * orc_f16_to_f32(a[b].d);
        int wv[32], av[32];
        for (int j = 0; j < 16; j++) {
            wv[j] = (int)(w[b].qs[j] & 0x0F) - 8;
            wv[j + 16] = (int)(w[b].qs[j] >> 4) - 8;
        }
        for (int j = 0; j < 32; j++) av[j] = a[b].qs[j] < -127 ? -127 : a[b].qs[j];
        for (int k = 0; k < 8; k++) {
            int isum = wv[4 * k] * av[4 * k] + wv[4 * k + 1] * av[4 * k + 1] +
                       wv[4 * k + 2] * av[4 * k + 2] + wv[4 * k + 3] * av[4 * k + 3];
            acc[k] = __builtin_fmaf(d, (float)isum, acc[k]);
        }
    }
    float s0 = acc[0] + acc[4], s1 = acc[1] + acc[5];
    float s2 = acc[2] + acc[6], s3 = acc[3] + acc[7];
    return (s0 + s1) + (s2 + s3);
}

#if defined(__x86_64__)
/* Same numerics as orc_vec_dot_x86, vectorised.  Built from a different
 * instruction sequence than the reference (sign-extend to i16, madd, hadd);
 * the resulting vector holds reference lanes in the order [0,1,4,5,2,3,6,7],
 * which the final reduction undoes. */
__attribute__((target("avx2,fma"))) static float vec_dot_avx2_impl(
    const orc_block_q4_0 *w, const orc_block_q8_0 *a, size_t nb) {
    const __m128i lo_mask = _mm_set1_epi8(0x0F);
    const __m128i eight = _mm_set1_epi8(8);
    const __m256i floor127 = _mm256_set1_epi8(-127);
    __m256 acc = _mm256_setzero_ps();
    for (size_t b = 0; b < nb; b++) {
        float d = orc_f16_to_f32(w[b].d) * orc_f16_to_f32(a[b].d);
        __m128i raw = _mm_loadu_si128((const __m128i *)w[b].qs);
        __m128i wlo = _mm_sub_epi8(_mm_and_si128(raw, lo_mask), eight);
        __m128i whi = _mm_sub_epi8(_mm_and_si128(_mm_srli_epi16(raw, 4), lo_mask), eight);
        __m256i av = _mm256_max_epi8(_mm256_loadu_si256((const __m256i *)a[b].qs), floor127);
        __m256i w16lo = _mm256_cvtepi8_epi16(wlo);
        __m256i w16hi = _mm256_cvtepi8_epi16(whi);
        __m256i a16lo = _mm256_cvtepi8_epi16(_mm256_castsi256_si128(av));
        __m256i a16hi = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(av, 1));
        __m256i plo = _mm256_madd_epi16(w16lo, a16lo);
        __m256i phi = _mm256_madd_epi16(w16hi, a16hi);
        __m256i lanes = _mm256_hadd_epi32(plo, phi);
        acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(lanes), acc);
    }
    float v[8];
    _mm256_storeu_ps(v, acc);
    /* v = reference lanes [0,1,4,5,2,3,6,7] */
    float r0 = v[0], r1 = v[1], r4 = v[2], r5 = v[3], r2 = v[4], r3 = v[5], r6 = v[6], r7 = v[7];
    float s0 = r0 + r4, s1 = r1 + r5, s2 = r2 + r6, s3 = r3 + r7;
    return (s0 + s1) + (s2 + s3);
}
#endif

int orc_host_has_avx2(void) {
#if defined(__x86_64__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
    return 0;
#endif
}

static int g_has_avx2 = -1;

float orc_vec_dot_avx2(const orc_block_q4_0 *w, const orc_block_q8_0 *a, size_t nb) {
#if defined(__x86_64__)
    if (g_has_avx2 < 0) g_has_avx2 = orc_host_has_avx2();
    if (g_has_avx2) return vec_dot_avx2_impl(w, a, nb);
#endif
    return orc_vec_dot_x86(w, a, nb);
}

typedef float (*dot_fn)(const orc_block_q4_0 *, const orc_block_q8_0 *, size_t);

static dot_fn dot_for_mode(int mode) {
    return mode == ORC_MODE_SCALAR ? orc_vec_dot_scalar : orc_vec_dot_avx2;
}

/* ---- worker pool: kernels.rs:12-142.  Workers claim row chunks from an
 * atomic cursor (chunk = max(rows/(workers+1), 16)); the dispatcher works
 * too, then waits for every worker to report done. */

#define POOL_MAX 256
#define SPIN_ITERS 20000

typedef struct {
    const orc_block_q4_0 *w;
    const orc_block_q8_0 *x;
    float *out;
    size_t batch, rows, nb, chunk;
    dot_fn dot;
    atomic_size_t next_row;
    atomic_int done;
    atomic_ulong generation;
    int workers;
    pthread_t tids[POOL_MAX];
    pthread_mutex_t mu;
    pthread_cond_t cv;
    pthread_mutex_t dispatch;
} pool_t;

static pool_t *g_pool = NULL;
static pthread_mutex_t g_pool_init = PTHREAD_MUTEX_INITIALIZER;

static void run_rows(pool_t *p) {
    for (;;) {
        size_t r0 = atomic_fetch_add_explicit(&p->next_row, p->chunk, memory_order_relaxed);
        if (r0 >= p->rows) break;
        size_t r1 = r0 + p->chunk < p->rows ? r0 + p->chunk : p->rows;
        for (size_t r = r0; r < r1; r++) {
            const orc_block_q4_0 *row = p->w + r * p->nb;
            for (size_t b = 0; b < p->batch; b++)
                p->out[b * p->rows + r] = p->dot(row, p->x + b * p->nb, p->nb);
        }
    }
}

static void *worker_main(void *arg) {
    pool_t *p = (pool_t *)arg;
    unsigned long seen = 0;
    for (;;) {
        unsigned long cur = atomic_load_explicit(&p->generation, memory_order_acquire);
        int spins = 0;
        while (cur == seen) {
            if (spins < SPIN_ITERS) {
#if defined(__x86_64__)
                _mm_pause();
#endif
                spins++;
            } else {
                pthread_mutex_lock(&p->mu);
                cur = atomic_load_explicit(&p->generation, memory_order_acquire);
                if (cur == seen) pthread_cond_wait(&p->cv, &p->mu);
                pthread_mutex_unlock(&p->mu);
            }
            cur = atomic_load_explicit(&p->generation, memory_order_acquire);
        }
        seen = cur;
        run_rows(p);
        atomic_fetch_add_explicit(&p->done, 1, memory_order_release);
    }
    return NULL;
}

int orc_default_pool_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    long t = n / 2;
    return (int)(t < 1 ? 1 : t);
}

/* Like init_gemv_pool (kernels.rs:69-142) the pool is created once, on first
 * parallel use, with `threads - 1` workers; later calls reuse it. */
static pool_t *get_pool(int threads) {
    pthread_mutex_lock(&g_pool_init);
    if (g_pool == NULL) {
        pool_t *p = (pool_t *)calloc(1, sizeof(pool_t));
        p->workers = threads - 1 < POOL_MAX ? threads - 1 : POOL_MAX;
        pthread_mutex_init(&p->mu, NULL);
        pthread_cond_init(&p->cv, NULL);
        pthread_mutex_init(&p->dispatch, NULL);
        for (int i = 0; i < p->workers; i++) {
            pthread_create(&p->tids[i], NULL, worker_main, p);
            pthread_detach(p->tids[i]);
        }
        g_pool = p;
    }
    pthread_mutex_unlock(&g_pool_init);
    return g_pool;
}

void orc_gemm_q4_0(const orc_block_q4_0 *w, const orc_block_q8_0 *xq, float *out,
                   size_t batch, size_t rows, size_t cols, int mode, int threads) {
    size_t nb = cols / ORC_QK;
    dot_fn dot = dot_for_mode(mode);
    if (batch == 0 || rows == 0) return;
    /* kernels.rs:337: parallel when blocks*batch >= 2048 and rows >= 64 */
    if (threads > 1 && rows * nb * batch >= 2048 && rows >= 64) {
        pool_t *p = get_pool(threads);
        if (p->workers > 0 && pthread_mutex_trylock(&p->dispatch) == 0) {
            p->w = w;
            p->x = xq;
            p->out = out;
            p->batch = batch;
            p->rows = rows;
            p->nb = nb;
            p->dot = dot;
            size_t chunk = rows / (size_t)(p->workers + 1);
            p->chunk = chunk < 16 ? 16 : chunk;
            atomic_store_explicit(&p->next_row, 0, memory_order_release);
            atomic_store_explicit(&p->done, 0, memory_order_release);
            pthread_mutex_lock(&p->mu);
            atomic_fetch_add_explicit(&p->generation, 1, memory_order_acq_rel);
            pthread_cond_broadcast(&p->cv);
            pthread_mutex_unlock(&p->mu);
            run_rows(p);
            while (atomic_load_explicit(&p->done, memory_order_acquire) < p->workers) sched_yield();
            pthread_mutex_unlock(&p->dispatch);
            return;
        }
    }
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < batch; b++) out[b * rows + r] = dot(w + r * nb, xq + b * nb, nb);
}

/* kernels.rs:289-303 (gemv_q4_0_arena) and :398-415 (gemm_q4_0_arena) */
void orc_gemm_q4_0_f32(const orc_block_q4_0 *w, const float *in, orc_block_q8_0 *q8,
                       float *out, size_t batch, size_t rows, size_t cols, int mode,
                       int threads) {
    orc_quantize_row_q8_0(in, q8, batch * cols);
    orc_gemm_q4_0(w, q8, out, batch, rows, cols, mode, threads);
}
