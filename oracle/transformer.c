/*
 * transformer.c -- RoPE, GQA attention, the layer bodies (decode and batched
 * prefill), the model driver and the embedding path (TEST INFRASTRUCTURE).
 * Restates static-lm src/model/transformer.rs.  Each orc_model is one
 * sequence with its own KV cache, like one TransformerModel + arena.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"


/* transformer.rs:124-133: freq_j = 1/10000^(2j/hd), angle = pos*freq; host libm */
void orc_rope_tables(int32_t max_seq, int32_t head_dim, float *cos_out, float *sin_out) {
    int half = head_dim / 2;
    float hd_f = (float)head_dim;
    for (int pos = 0; pos < max_seq; pos++) {
        float pos_f = (float)pos;
        for (int j = 0; j < half; j++) {
            float freq = 1.0f / powf(10000.0f, (float)(2 * j) / hd_f);
            float ang = pos_f * freq;
            sin_out[(size_t)pos * half + j] = sinf(ang);
            cos_out[(size_t)pos * half + j] = cosf(ang);
        }
    }
}

/* transformer.rs:178-194 */
void orc_apply_rope_cached(float *vec, size_t len, const float *cos_row,
                           const float *sin_row, int32_t head_dim) {
    int half = head_dim / 2;
    for (size_t h0 = 0; h0 + (size_t)head_dim <= len; h0 += (size_t)head_dim) {
        float *hs = vec + h0;
        for (int j = 0; j < half; j++) {
            float c = cos_row[j], s = sin_row[j];
            float v0 = hs[2 * j], v1 = hs[2 * j + 1];
            hs[2 * j] = v0 * c - v1 * s;
            hs[2 * j + 1] = v0 * s + v1 * c;
        }
    }
}

/* transformer.rs:196-212 (test/baseline form, computes the angles inline) */
void orc_apply_rope_in_place(float *vec, size_t len, int32_t pos, int32_t head_dim) {
    float pos_f = (float)pos, hd_f = (float)head_dim;
    for (size_t h0 = 0; h0 + (size_t)head_dim <= len; h0 += (size_t)head_dim) {
        float *hs = vec + h0;
        for (int i = 0; i < head_dim; i += 2) {
            float freq = 1.0f / powf(10000.0f, (float)i / hd_f);
            float ang = pos_f * freq;
            float s = sinf(ang), c = cosf(ang);
            float v0 = hs[i], v1 = hs[i + 1];
            hs[i] = v0 * c - v1 * s;
            hs[i + 1] = v0 * s + v1 * c;
        }
    }
}

/* ORC_MODE_X86: causal_multi_head_attention_jit (transformer.rs:273-321);
 * ORC_MODE_SCALAR: causal_multi_head_attention (transformer.rs:214-271).
 * att is [num_heads x max_seq_len]; out is zeroed first. */
void orc_attention(const float *q, const float *k_cache, const float *v_cache, float *att,
                   float *out, const orc_config *cfg, int32_t pos, int mode) {
    int hd = cfg->dim / cfg->num_heads;
    int kv_dim = hd * cfg->num_kv_heads;
    int kv_mul = cfg->num_heads / cfg->num_kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    int seq_len = pos + 1;
    memset(out, 0, sizeof(float) * (size_t)cfg->dim);
    for (int h = 0; h < cfg->num_heads; h++) {
        const float *qh = q + (size_t)h * hd;
        size_t kvo = (size_t)(h / kv_mul) * hd;
        float *att_h = att + (size_t)h * cfg->max_seq_len;
        for (int t = 0; t < seq_len; t++) {
            const float *kt = k_cache + (size_t)t * kv_dim + kvo;
            float dot = 0.0f;
            for (int i = 0; i < hd; i++) dot = dot + qh[i] * kt[i];
            att_h[t] = dot * scale;
        }
        orc_softmax(att_h, att_h, (size_t)seq_len, mode);
        float *oh = out + (size_t)h * hd;
        for (int t = 0; t < seq_len; t++) {
            const float *vt = v_cache + (size_t)t * kv_dim + kvo;
            float p = att_h[t];
            for (int i = 0; i < hd; i++) oh[i] = oh[i] + p * vt[i];
        }
    }
}

/* transformer.rs:654-667: strict `>`, first maximum wins */
int32_t orc_sample_argmax(const float *logits, size_t n) {
    size_t best = 0;
    float bv = logits[0];
    for (size_t i = 1; i < n; i++)
        if (logits[i] > bv) {
            bv = logits[i];
            best = i;
        }
    return (int32_t)best;
}

/* ---------------- model ---------------- */

struct orc_model {
    orc_config cfg;
    int n_layers, vocab, mode, threads;
    orc_model_weights w;
    /* LayerWorkspace (transformer.rs:80-136) */
    float *x, *x_mid, *xb, *xb2, *q, *att, *hb, *hb2, *hb_act, *rope_cos, *rope_sin;
    orc_block_q8_0 *q8;
    /* BatchWorkspace (transformer.rs:156-175), max_batch = max_seq_len */
    float *xB, *x_midB, *xbB, *xb2B, *qB, *hbB, *hb2B, *hb_actB;
    orc_block_q8_0 *q8B;
    /* LayerKvCache per layer (transformer.rs:323-338) */
    float **k, **v;
    float *logits, *embed_accum, *embed_norm;
};

static float *fz(size_t n) { return (float *)calloc(n ? n : 1, sizeof(float)); }

orc_model *orc_model_new(const orc_config *cfg, int32_t num_layers, int32_t vocab_size,
                         int mode, int threads) {
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    m->cfg = *cfg;
    m->n_layers = num_layers;
    m->vocab = vocab_size;
    m->mode = mode;
    m->threads = threads;
    int d = cfg->dim, h = cfg->hidden_dim, S = cfg->max_seq_len;
    int hd = d / cfg->num_heads, kvd = hd * cfg->num_kv_heads;
    int maxk = d > h ? d : h;
    m->x = fz(d);
    m->x_mid = fz(d);
    m->xb = fz(d);
    m->xb2 = fz(d);
    m->q = fz(d);
    m->att = fz((size_t)cfg->num_heads * S);
    m->hb = fz(h);
    m->hb2 = fz(h);
    m->hb_act = fz(h);
    m->q8 = (orc_block_q8_0 *)calloc((size_t)maxk / ORC_QK + 1, sizeof(orc_block_q8_0));
    m->rope_cos = fz((size_t)S * (hd / 2));
    m->rope_sin = fz((size_t)S * (hd / 2));
    orc_rope_tables(S, hd, m->rope_cos, m->rope_sin);
    m->xB = fz((size_t)S * d);
    m->x_midB = fz((size_t)S * d);
    m->xbB = fz((size_t)S * d);
    m->xb2B = fz((size_t)S * d);
    m->qB = fz((size_t)S * d);
    m->hbB = fz((size_t)S * h);
    m->hb2B = fz((size_t)S * h);
    m->hb_actB = fz((size_t)S * h);
    m->q8B = (orc_block_q8_0 *)calloc((size_t)S * maxk / ORC_QK + 1, sizeof(orc_block_q8_0));
    m->k = (float **)calloc((size_t)num_layers, sizeof(float *));
    m->v = (float **)calloc((size_t)num_layers, sizeof(float *));
    for (int l = 0; l < num_layers; l++) {
        m->k[l] = fz((size_t)S * kvd);
        m->v[l] = fz((size_t)S * kvd);
    }
    m->logits = fz((size_t)vocab_size);
    m->embed_accum = fz(d);
    m->embed_norm = fz(d);
    return m;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    float *bufs[] = {m->x, m->x_mid, m->xb, m->xb2, m->q, m->att, m->hb, m->hb2, m->hb_act,
                     m->rope_cos, m->rope_sin, m->xB, m->x_midB, m->xbB, m->xb2B, m->qB,
                     m->hbB, m->hb2B, m->hb_actB, m->logits, m->embed_accum, m->embed_norm};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++) free(bufs[i]);
    free(m->q8);
    free(m->q8B);
    for (int l = 0; l < m->n_layers; l++) {
        free(m->k[l]);
        free(m->v[l]);
    }
    free(m->k);
    free(m->v);
    free(m);
}

int orc_model_set_weights(orc_model *m, const orc_model_weights *w) {
    if (w->num_layers != m->n_layers || w->vocab_size != m->vocab) return -1;
    m->w = *w;
    return 0;
}

float *orc_model_x(orc_model *m) { return m->x; }
float *orc_model_xb(orc_model *m) { return m->xb; }
float *orc_model_logits(orc_model *m) { return m->logits; }
float *orc_model_k_cache(orc_model *m, int32_t l) { return m->k[l]; }
float *orc_model_v_cache(orc_model *m, int32_t l) { return m->v[l]; }
float *orc_model_rope_cos(orc_model *m) { return m->rope_cos; }
float *orc_model_rope_sin(orc_model *m) { return m->rope_sin; }

static void gemv(orc_model *m, const orc_block_q4_0 *w, const float *in, float *out, int rows,
                 int cols, int batch, orc_block_q8_0 *q8) {
    orc_gemm_q4_0_f32(w, in, q8, out, (size_t)batch, (size_t)rows, (size_t)cols, m->mode,
                      m->threads);
}

/* TransformerLayer::forward_token_with_kv, transformer.rs:391-487 */
void orc_layer_forward_token(orc_model *m, int32_t l, int32_t pos) {
    const orc_config *c = &m->cfg;
    const orc_layer_weights *lw = &m->w.layers[l];
    int d = c->dim, h = c->hidden_dim, hd = d / c->num_heads, kvd = hd * c->num_kv_heads;
    int half = hd / 2;
    float *kpos = m->k[l] + (size_t)pos * kvd;
    float *vpos = m->v[l] + (size_t)pos * kvd;
    orc_rmsnorm(m->x, lw->rms_att_weight, m->xb, (size_t)d, c->rms_eps, m->mode);
    gemv(m, lw->wq, m->xb, m->q, d, d, 1, m->q8);
    gemv(m, lw->wk, m->xb, kpos, kvd, d, 1, m->q8);
    gemv(m, lw->wv, m->xb, vpos, kvd, d, 1, m->q8);
    const float *cr = m->rope_cos + (size_t)pos * half, *sr = m->rope_sin + (size_t)pos * half;
    orc_apply_rope_cached(m->q, (size_t)d, cr, sr, hd);
    orc_apply_rope_cached(kpos, (size_t)kvd, cr, sr, hd);
    orc_attention(m->q, m->k[l], m->v[l], m->att, m->xb, c, pos, m->mode);
    gemv(m, lw->wo, m->xb, m->xb2, d, d, 1, m->q8);
    orc_residual_add(m->x, m->xb2, m->x_mid, (size_t)d);
    orc_rmsnorm(m->x_mid, lw->rms_ffn_weight, m->xb, (size_t)d, c->rms_eps, m->mode);
    gemv(m, lw->w_gate, m->xb, m->hb, h, d, 1, m->q8);
    gemv(m, lw->w_up, m->xb, m->hb2, h, d, 1, m->q8);
    orc_swiglu(m->hb, m->hb2, m->hb_act, (size_t)h, m->mode);
    gemv(m, lw->w_down, m->hb_act, m->xb, d, h, 1, m->q8);
    orc_residual_add(m->x_mid, m->xb, m->x, (size_t)d);
}

/* TransformerLayer::forward_batch_with_kv, transformer.rs:491-651 */
static void layer_forward_batch(orc_model *m, int l, int start_pos, int B) {
    const orc_config *c = &m->cfg;
    const orc_layer_weights *lw = &m->w.layers[l];
    int d = c->dim, h = c->hidden_dim, hd = d / c->num_heads, kvd = hd * c->num_kv_heads;
    int half = hd / 2;
    for (int b = 0; b < B; b++)
        orc_rmsnorm(m->xB + (size_t)b * d, lw->rms_att_weight, m->xbB + (size_t)b * d,
                    (size_t)d, c->rms_eps, m->mode);
    float *kb = m->k[l] + (size_t)start_pos * kvd, *vb = m->v[l] + (size_t)start_pos * kvd;
    gemv(m, lw->wq, m->xbB, m->qB, d, d, B, m->q8B);
    gemv(m, lw->wk, m->xbB, kb, kvd, d, B, m->q8B);
    gemv(m, lw->wv, m->xbB, vb, kvd, d, B, m->q8B);
    for (int b = 0; b < B; b++) {
        int pos = start_pos + b;
        float *qp = m->qB + (size_t)b * d;
        float *kp = m->k[l] + (size_t)pos * kvd;
        const float *cr = m->rope_cos + (size_t)pos * half;
        const float *sr = m->rope_sin + (size_t)pos * half;
        orc_apply_rope_cached(qp, (size_t)d, cr, sr, hd);
        orc_apply_rope_cached(kp, (size_t)kvd, cr, sr, hd);
        orc_attention(qp, m->k[l], m->v[l], m->att, m->xbB + (size_t)b * d, c, pos, m->mode);
    }
    gemv(m, lw->wo, m->xbB, m->xb2B, d, d, B, m->q8B);
    orc_residual_add(m->xB, m->xb2B, m->x_midB, (size_t)B * d);
    for (int b = 0; b < B; b++)
        orc_rmsnorm(m->x_midB + (size_t)b * d, lw->rms_ffn_weight, m->xbB + (size_t)b * d,
                    (size_t)d, c->rms_eps, m->mode);
    gemv(m, lw->w_gate, m->xbB, m->hbB, h, d, B, m->q8B);
    gemv(m, lw->w_up, m->xbB, m->hb2B, h, d, B, m->q8B);
    orc_swiglu(m->hbB, m->hb2B, m->hb_actB, (size_t)B * h, m->mode);
    gemv(m, lw->w_down, m->hb_actB, m->xbB, d, h, B, m->q8B);
    orc_residual_add(m->x_midB, m->xbB, m->xB, (size_t)B * d);
}

/* TransformerModel::forward_token, transformer.rs:747-795 */
int32_t orc_forward_token(orc_model *m, int32_t token, int32_t pos) {
    int d = m->cfg.dim, nb = d / ORC_QK;
    if (token < 0 || token >= m->vocab || pos < 0 || pos >= m->cfg.max_seq_len) return -1;
    orc_dequantize_row_q4_0(m->w.token_embd + (size_t)token * nb, m->x, (size_t)d);
    for (int l = 0; l < m->n_layers; l++) orc_layer_forward_token(m, l, pos);
    orc_rmsnorm(m->x, m->w.output_norm, m->xb, (size_t)d, m->cfg.rms_eps, m->mode);
    gemv(m, m->w.lm_head, m->xb, m->logits, m->vocab, d, 1, m->q8);
    return orc_sample_argmax(m->logits, (size_t)m->vocab);
}

/* TransformerModel::prefill_tokens, transformer.rs:799-854 */
int32_t orc_prefill_tokens(orc_model *m, const int32_t *tokens, int32_t n, int32_t start_pos) {
    int d = m->cfg.dim, nb = d / ORC_QK;
    if (n <= 0 || n > m->cfg.max_seq_len || start_pos + n > m->cfg.max_seq_len) return -1;
    for (int b = 0; b < n; b++) {
        if (tokens[b] < 0 || tokens[b] >= m->vocab) return -1;
        orc_dequantize_row_q4_0(m->w.token_embd + (size_t)tokens[b] * nb, m->xB + (size_t)b * d,
                                (size_t)d);
    }
    for (int l = 0; l < m->n_layers; l++) layer_forward_batch(m, l, start_pos, n);
    orc_rmsnorm(m->xB + (size_t)(n - 1) * d, m->w.output_norm, m->xb, (size_t)d,
                m->cfg.rms_eps, m->mode);
    gemv(m, m->w.lm_head, m->xb, m->logits, m->vocab, d, 1, m->q8);
    return orc_sample_argmax(m->logits, (size_t)m->vocab);
}

/* TransformerModel::generate, transformer.rs:858-892 */
int32_t orc_generate(orc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t *out,
                     int32_t n_out, int32_t eos) {
    if (n_out <= 0 || n_prompt <= 0) return 0;
    int32_t next = orc_prefill_tokens(m, prompt, n_prompt, 0);
    if (next < 0) return -1;
    out[0] = next;
    int32_t gen = 1;
    if (eos >= 0 && next == eos) return gen;
    int32_t pos = n_prompt;
    while (gen < n_out && pos < m->cfg.max_seq_len) {
        next = orc_forward_token(m, next, pos);
        out[gen++] = next;
        pos++;
        if (eos >= 0 && next == eos) break;
    }
    return gen;
}

/* TransformerModel::embed_tokens, transformer.rs:896-948 */
void orc_embed_tokens(orc_model *m, const int32_t *tokens, int32_t n, float *out_embedding) {
    int d = m->cfg.dim, nb = d / ORC_QK;
    for (int b = 0; b < n; b++)
        orc_dequantize_row_q4_0(m->w.token_embd + (size_t)tokens[b] * nb, m->xB + (size_t)b * d,
                                (size_t)d);
    for (int l = 0; l < m->n_layers; l++) layer_forward_batch(m, l, 0, n);
    for (int i = 0; i < d; i++) m->embed_accum[i] = 0.0f;
    float inv_batch = 1.0f / (float)n;
    for (int b = 0; b < n; b++) {
        orc_rmsnorm(m->xB + (size_t)b * d, m->w.output_norm, m->xb, (size_t)d, m->cfg.rms_eps,
                    m->mode);
        for (int i = 0; i < d; i++) m->embed_accum[i] = m->embed_accum[i] + m->xb[i] * inv_batch;
    }
    orc_l2_norm(m->embed_accum, m->embed_norm, (size_t)d, m->cfg.rms_eps);
    memcpy(out_embedding, m->embed_norm, sizeof(float) * (size_t)d);
}
