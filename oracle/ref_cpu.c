/*
 * ref_cpu.c -- CPU restatement of the MoGemma Mojo engine (TEST INFRASTRUCTURE).
 *
 * Oracle only: called by tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg.  Each function cites the reference file:line it restates
 * (paths inside the cofin/mogemma project).  Compiled with -ffp-contract=off
 * so every product and sum is rounded separately, as the Mojo source writes them.
 */
#include "ref_cpu.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;

void ref_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int ref_get_threads(void) { return g_threads; }

/* SIMD[nelts].reduce_add(): restated as a halving tree (lane i += lane i+n/2). */
static float reduce_add(float *v, int n) {
    while (n > 1) {
        n >>= 1;
        for (int j = 0; j < n; ++j) v[j] = v[j] + v[j + n];
    }
    return v[0];
}

/* ops.mojo:5-30 geglu: 0.5 * g * (1 + erf(g / sqrt(2))) * up, Float32 sqrt_2 constant. */
void ref_geglu(float *out, const float *gate, const float *up, int64_t size, int nelts) {
    const float sqrt_2 = (float)1.4142135623730951;
    for (int64_t i = 0; i < size; ++i) {
        float g = gate[i];
        float gelu_gate = 0.5f * g * (1.0f + erff(g / sqrt_2));
        out[i] = gelu_gate * up[i];
    }
    (void)nelts; /* element-wise: chunking does not change results */
}

/* ops.mojo:33-66 rope_rotate: half-split rotation [x1 c - x2 s, x2 c + x1 s]. */
void ref_rope_rotate(float *vec, const float *c, const float *s, int64_t head_dim, int nelts) {
    int64_t half = head_dim / 2;
    for (int64_t i = 0; i < half; ++i) {
        float x1 = vec[i], x2 = vec[i + half];
        vec[i] = x1 * c[i] - x2 * s[i];
        vec[i + half] = x2 * c[i] + x1 * s[i];
    }
    (void)nelts;
}

/* ops.mojo:69-95 vec_mat_mul: per output row, a scalar fp32 accumulator that
 * receives each nelts-wide chunk's reduce_add, then a scalar tail. */
void ref_vec_mat_mul(float *out, const float *x, const float *w, int64_t in_dim, int64_t out_dim, int nelts) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && out_dim >= 64)
#endif
    for (int64_t o = 0; o < out_dim; ++o) {
        const float *wr = w + o * in_dim;
        float acc = 0.0f;
        int64_t i = 0;
        float p[64];
        for (; i <= in_dim - nelts; i += nelts) {
            for (int j = 0; j < nelts; ++j) p[j] = x[i + j] * wr[i + j];
            acc += reduce_add(p, nelts);
        }
        for (; i < in_dim; ++i) acc += x[i] * wr[i];
        out[o] = acc;
    }
}

/* ops.mojo:98-136 rms_norm: x * (1/sqrt(mean(x^2)+eps)) * (1 + w). */
void ref_rms_norm(float *out, const float *x, const float *w, int64_t size, float eps, int nelts) {
    float sum_sq = 0.0f;
    int64_t i = 0;
    float p[64];
    for (; i <= size - nelts; i += nelts) {
        for (int j = 0; j < nelts; ++j) p[j] = x[i + j] * x[i + j];
        sum_sq += reduce_add(p, nelts);
    }
    for (; i < size; ++i) sum_sq += x[i] * x[i];
    float mean_sq = sum_sq / (float)size;
    float inv_rms = 1.0f / sqrtf(mean_sq + eps);
    for (i = 0; i < size; ++i) out[i] = x[i] * inv_rms * (1.0f + w[i]);
}

/* ops.mojo:139-182 softmax: max seeded at -1e9, exp(v - max), chunked sum, * (1/sum). */
void ref_softmax(float *vec, int64_t size, int nelts) {
    float max_val = -1e9f;
    for (int64_t i = 0; i < size; ++i)
        if (vec[i] > max_val) max_val = vec[i];
    float sum_exp = 0.0f;
    int64_t i = 0;
    float p[64];
    for (; i <= size - nelts; i += nelts) {
        for (int j = 0; j < nelts; ++j) {
            float e = expf(vec[i + j] - max_val);
            p[j] = e;
            vec[i + j] = e;
        }
        sum_exp += reduce_add(p, nelts);
    }
    for (; i < size; ++i) {
        float e = expf(vec[i] - max_val);
        sum_exp += e;
        vec[i] = e;
    }
    float inv_sum = 1.0f / sum_exp;
    for (i = 0; i < size; ++i) vec[i] = vec[i] * inv_sum;
}

/* core.mojo:340-348 RoPE tables: inv_freq = 1/base^(2d/hd), stored at [t*hd + d], d < hd/2. */
void ref_rope_tables(float *cos_t, float *sin_t, int64_t max_seq_len, int64_t head_dim, float base) {
    memset(cos_t, 0, sizeof(float) * (size_t)(max_seq_len * head_dim));
    memset(sin_t, 0, sizeof(float) * (size_t)(max_seq_len * head_dim));
    for (int64_t t = 0; t < max_seq_len; ++t)
        for (int64_t d = 0; d < head_dim / 2; ++d) {
            float e = (float)(d * 2) / (float)head_dim;
            float inv_freq = 1.0f / powf(base, e);
            float freq = (float)t * inv_freq;
            cos_t[t * head_dim + d] = cosf(freq);
            sin_t[t * head_dim + d] = sinf(freq);
        }
}

/* ------------------------------------------------------------------------- */

struct ref_model {
    const float *embed, *final_norm, *lm_head;
    ref_layer_w *layers;
    int32_t L;
    int64_t h, hq, hkv, hd, inter, vocab, max_seq;
    int32_t mode, window, global_every;
    float *cos_local, *sin_local, *cos_global, *sin_global;
    float *k_cache, *v_cache;
    float *scratch;
    int64_t scratch_len;
    int64_t pos;
};

static int layer_is_global(const ref_model *m, int l) {
    if (m->mode == 0) return 1;
    return ((l + 1) % m->global_every) == 0;
}

/* layers.mojo:16-97 forward_attention, scratch frame kept byte-for-byte:
 * q @0, k @q_size, v @q_size+kv_size, attn_out @q_size+2kv_size,
 * scores @attn_out + Hq*hd. `lo` is the first attended position (0 in ref mode). */
static void forward_attention(const ref_model *m, float *out, const float *x, const ref_layer_w *w, int64_t pos,
                              int64_t lo, const float *fc, const float *fs, float *kc, float *vc, float *scratch) {
    const int64_t hd = m->hd, q_size = m->hq * hd, kv_size = m->hkv * hd, H = m->h;
    float *q = scratch, *k = scratch + q_size, *v = scratch + q_size + kv_size;
    ref_vec_mat_mul(q, x, w->q_proj, H, q_size, 16);
    ref_vec_mat_mul(k, x, w->k_proj, H, kv_size, 16);
    ref_vec_mat_mul(v, x, w->v_proj, H, kv_size, 16);
    if (w->q_norm)
        for (int64_t h = 0; h < m->hq; ++h) ref_rms_norm(q + h * hd, q + h * hd, w->q_norm, hd, 1e-6f, 16);
    if (w->k_norm)
        for (int64_t h = 0; h < m->hkv; ++h) ref_rms_norm(k + h * hd, k + h * hd, w->k_norm, hd, 1e-6f, 16);
    for (int64_t h = 0; h < m->hq; ++h) ref_rope_rotate(q + h * hd, fc, fs, hd, 16);
    for (int64_t h = 0; h < m->hkv; ++h) ref_rope_rotate(k + h * hd, fc, fs, hd, 16);
    int64_t kv_off = pos * kv_size;
    for (int64_t i = 0; i < kv_size; ++i) {
        kc[kv_off + i] = k[i];
        vc[kv_off + i] = v[i];
    }
    int64_t heads_per_kv = m->hq / m->hkv;
    float scale = 1.0f / sqrtf((float)hd);
    float *attn_out = scratch + q_size + 2 * kv_size;
    for (int64_t h = 0; h < m->hq; ++h) {
        int64_t kvh = h / heads_per_kv;
        const float *qh = q + h * hd;
        float *scores = attn_out + m->hq * hd;
        int64_t n = pos + 1 - lo;
        for (int64_t t = lo; t <= pos; ++t) {
            const float *kh = kc + t * kv_size + kvh * hd;
            float score = 0.0f;
            for (int64_t d = 0; d < hd; ++d) score += qh[d] * kh[d];
            scores[t - lo] = score * scale;
        }
        ref_softmax(scores, n, 16);
        float *oh = attn_out + h * hd;
        for (int64_t d = 0; d < hd; ++d) oh[d] = 0.0f;
        for (int64_t t = lo; t <= pos; ++t) {
            const float *vh = vc + t * kv_size + kvh * hd;
            float prob = scores[t - lo];
            for (int64_t d = 0; d < hd; ++d) oh[d] = oh[d] + prob * vh[d];
        }
    }
    ref_vec_mat_mul(out, attn_out, w->o_proj, q_size, H, 16);
}

/* layers.mojo:101-118 forward_mlp: gate @0, up @I, geglu @2I in scratch. */
static void forward_mlp(const ref_model *m, float *out, const float *x, const ref_layer_w *w, float *scratch) {
    const int64_t I = m->inter, H = m->h;
    float *g = scratch, *u = scratch + I, *a = scratch + 2 * I;
    ref_vec_mat_mul(g, x, w->gate_proj, H, I, 16);
    ref_vec_mat_mul(u, x, w->up_proj, H, I, 16);
    ref_geglu(a, g, u, I, 16);
    ref_vec_mat_mul(out, a, w->down_proj, I, H, 16);
}

/* layers.mojo:174-220 forward_layer with its scratch offsets (0..7h, attn @2h, mlp @6h). */
static void forward_layer(const ref_model *m, int l, float *out, const float *x, int64_t pos, float *scratch) {
    const int64_t H = m->h;
    const ref_layer_w *w = &m->layers[l];
    int glob = layer_is_global(m, l);
    const float *fc = (glob ? m->cos_global : m->cos_local) + pos * m->hd;
    const float *fs = (glob ? m->sin_global : m->sin_local) + pos * m->hd;
    int64_t lo = 0;
    if (!glob && pos - m->window + 1 > 0) lo = pos - m->window + 1;
    float *kc = m->k_cache + (int64_t)l * m->max_seq * m->hkv * m->hd;
    float *vc = m->v_cache + (int64_t)l * m->max_seq * m->hkv * m->hd;
    float *norm_x = scratch, *attn_out = scratch + H, *attn_scratch = scratch + 2 * H;
    ref_rms_norm(norm_x, x, w->input_layernorm, H, 1e-6f, 16);
    forward_attention(m, attn_out, norm_x, w, pos, lo, fc, fs, kc, vc, attn_scratch);
    float *post_attn = scratch + 2 * H;
    ref_rms_norm(post_attn, attn_out, w->post_attention_layernorm, H, 1e-6f, 16);
    float *resid = scratch + 3 * H;
    for (int64_t i = 0; i < H; ++i) resid[i] = x[i] + post_attn[i];
    float *norm_resid = scratch + 4 * H;
    ref_rms_norm(norm_resid, resid, w->pre_feedforward_layernorm, H, 1e-6f, 16);
    float *mlp_out = scratch + 5 * H, *mlp_scratch = scratch + 6 * H;
    forward_mlp(m, mlp_out, norm_resid, w, mlp_scratch);
    float *post_mlp = scratch + 7 * H;
    ref_rms_norm(post_mlp, mlp_out, w->post_feedforward_layernorm, H, 1e-6f, 16);
    for (int64_t i = 0; i < H; ++i) out[i] = resid[i] + post_mlp[i];
}

ref_model *ref_model_create(const float *embed, const float *final_norm, const float *lm_head,
                            const ref_layer_w *layers, int32_t num_layers, int64_t hidden, int64_t num_heads,
                            int64_t num_kv_heads, int64_t head_dim, int64_t intermediate, int64_t vocab,
                            int64_t max_seq_len, int32_t mode, int32_t sliding_window, int32_t global_every,
                            float theta_local, float theta_global) {
    ref_model *m = (ref_model *)calloc(1, sizeof(ref_model));
    if (!m) return NULL;
    m->embed = embed;
    m->final_norm = final_norm;
    m->lm_head = lm_head;
    m->L = num_layers;
    m->layers = (ref_layer_w *)malloc(sizeof(ref_layer_w) * (size_t)num_layers);
    memcpy(m->layers, layers, sizeof(ref_layer_w) * (size_t)num_layers);
    m->h = hidden;
    m->hq = num_heads;
    m->hkv = num_kv_heads;
    m->hd = head_dim;
    m->inter = intermediate;
    m->vocab = vocab;
    m->max_seq = max_seq_len;
    m->mode = mode;
    m->window = sliding_window > 0 ? sliding_window : (int32_t)max_seq_len;
    m->global_every = global_every > 0 ? global_every : 1;
    size_t tab = (size_t)(max_seq_len * head_dim);
    m->cos_local = (float *)malloc(sizeof(float) * tab);
    m->sin_local = (float *)malloc(sizeof(float) * tab);
    m->cos_global = (float *)malloc(sizeof(float) * tab);
    m->sin_global = (float *)malloc(sizeof(float) * tab);
    /* ref mode: one table with base 10000 (core.mojo:341). */
    float tl = mode == 0 ? 10000.0f : theta_local, tg = mode == 0 ? 10000.0f : theta_global;
    ref_rope_tables(m->cos_local, m->sin_local, max_seq_len, head_dim, tl);
    ref_rope_tables(m->cos_global, m->sin_global, max_seq_len, head_dim, tg);
    size_t kv = (size_t)num_layers * (size_t)max_seq_len * (size_t)num_kv_heads * (size_t)head_dim;
    m->k_cache = (float *)calloc(kv, sizeof(float));
    m->v_cache = (float *)calloc(kv, sizeof(float));
    /* step_mojo allocates hidden*160, generate_embeddings hidden*180 (core.mojo:404,508);
     * the attention score frame needs room for max_seq_len positions on tiny models. */
    int64_t need = 2 * hidden + 2 * hidden + 2 * num_heads * head_dim + 2 * num_kv_heads * head_dim + max_seq_len + 64;
    int64_t n = hidden * 180;
    int64_t need_mlp = 2 * hidden + 6 * hidden + 3 * intermediate + 64;
    if (need > n) n = need;
    if (need_mlp > n) n = need_mlp;
    if (12 * hidden + hidden + 64 > n) n = 13 * hidden + 64;
    m->scratch_len = n;
    m->scratch = (float *)calloc((size_t)n, sizeof(float));
    m->pos = 0;
    return m;
}

void ref_model_destroy(ref_model *m) {
    if (!m) return;
    free(m->layers);
    free(m->cos_local);
    free(m->sin_local);
    free(m->cos_global);
    free(m->sin_global);
    free(m->k_cache);
    free(m->v_cache);
    free(m->scratch);
    free(m);
}

int64_t ref_model_pos(const ref_model *m) { return m->pos; }
void ref_model_set_pos(ref_model *m, int64_t pos) { m->pos = pos; }
const float *ref_model_k_cache(const ref_model *m) { return m->k_cache; }
const float *ref_model_v_cache(const ref_model *m) { return m->v_cache; }

/* layers.mojo:224-288 forward_step (states @0 and @h, layer scratch @2h). */
static int forward_step(ref_model *m, int32_t token_id, float *logits) {
    if (m->pos >= m->max_seq) return -1; /* core.mojo:380-381 */
    const int64_t H = m->h;
    float *scratch = m->scratch;
    memset(scratch, 0, sizeof(float) * (size_t)m->scratch_len);
    float *cur = scratch, *next = scratch + H, *layer_scratch = scratch + 2 * H;
    float emb_scale = sqrtf((float)H);
    const float *src = m->embed + (int64_t)token_id * H; /* model.mojo:62-68 */
    for (int64_t i = 0; i < H; ++i) cur[i] = src[i] * emb_scale;
    for (int l = 0; l < m->L; ++l) {
        forward_layer(m, l, next, cur, m->pos, layer_scratch);
        for (int64_t i = 0; i < H; ++i) cur[i] = next[i];
    }
    ref_rms_norm(next, cur, m->final_norm, H, 1e-6f, 16);
    if (logits) ref_vec_mat_mul(logits, next, m->lm_head, H, m->vocab, 16);
    m->pos += 1; /* core.mojo:459 */
    return 0;
}

int ref_step(ref_model *m, int32_t token_id, float *logits_out) { return forward_step(m, token_id, logits_out); }
int ref_step_no_logits(ref_model *m, int32_t token_id) { return forward_step(m, token_id, NULL); }

/* layers.mojo:292-370 forward_sequence.  With ref_compat the mean-pool
 * accumulator sits at layer_scratch + 10h exactly as in the reference
 * (layers.mojo:315) and so shares memory with the MLP frame at 6h. */
void ref_embed_sequence(ref_model *m, const int32_t *ids, int64_t seq_len, float *out, int ref_compat) {
    const int64_t H = m->h;
    float *scratch = m->scratch;
    memset(scratch, 0, sizeof(float) * (size_t)m->scratch_len);
    float *cur = scratch, *next = scratch + H, *layer_scratch = scratch + 2 * H;
    float *acc_own = NULL;
    float *emb_acc;
    if (ref_compat) {
        emb_acc = layer_scratch + 10 * H;
    } else {
        acc_own = (float *)calloc((size_t)H, sizeof(float));
        emb_acc = acc_own;
    }
    for (int64_t i = 0; i < H; ++i) emb_acc[i] = 0.0f;
    float emb_scale = sqrtf((float)H);
    for (int64_t t = 0; t < seq_len; ++t) {
        const float *src = m->embed + (int64_t)ids[t] * H;
        for (int64_t i = 0; i < H; ++i) cur[i] = src[i] * emb_scale;
        for (int l = 0; l < m->L; ++l) {
            forward_layer(m, l, next, cur, t, layer_scratch);
            for (int64_t i = 0; i < H; ++i) cur[i] = next[i];
        }
        ref_rms_norm(next, cur, m->final_norm, H, 1e-6f, 16);
        for (int64_t i = 0; i < H; ++i) emb_acc[i] = emb_acc[i] + next[i];
    }
    float scale = 1.0f / (float)seq_len;
    for (int64_t i = 0; i < H; ++i) out[i] = emb_acc[i] * scale;
    free(acc_own);
}

/* Raw wrappers: a throw-away single-layer model view over caller buffers. */
static void raw_view(ref_model *v, const ref_layer_w *w, int64_t hidden, int64_t nh, int64_t nkv, int64_t hd,
                     int64_t inter, float *kc, float *vc) {
    memset(v, 0, sizeof(*v));
    v->layers = (ref_layer_w *)w;
    v->L = 1;
    v->h = hidden;
    v->hq = nh;
    v->hkv = nkv;
    v->hd = hd;
    v->inter = inter;
    v->max_seq = 1 << 30;
    v->mode = 0;
    v->window = 1 << 30;
    v->global_every = 1;
    v->k_cache = kc;
    v->v_cache = vc;
}

void ref_forward_attention_raw(float *out, const float *x, const ref_layer_w *w, int64_t pos, int64_t hidden,
                               int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, const float *cos_t,
                               const float *sin_t, float *k_cache, float *v_cache, float *scratch) {
    ref_model v;
    raw_view(&v, w, hidden, num_heads, num_kv_heads, head_dim, 0, k_cache, v_cache);
    forward_attention(&v, out, x, w, pos, 0, cos_t, sin_t, k_cache, v_cache, scratch);
}

void ref_forward_mlp_raw(float *out, const float *x, const ref_layer_w *w, int64_t hidden, int64_t intermediate,
                         float *scratch) {
    ref_model v;
    raw_view(&v, w, hidden, 1, 1, 1, intermediate, NULL, NULL);
    forward_mlp(&v, out, x, w, scratch);
}

void ref_forward_layer_raw(float *out, const float *x, const ref_layer_w *w, int64_t pos, int64_t hidden,
                           int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, int64_t intermediate,
                           const float *cos_t, const float *sin_t, float *k_cache, float *v_cache, float *scratch) {
    ref_model v;
    raw_view(&v, w, hidden, num_heads, num_kv_heads, head_dim, intermediate, k_cache, v_cache);
    /* forward_layer indexes the tables at pos*hd; callers pass tables already offset. */
    v.cos_global = (float *)cos_t - pos * head_dim;
    v.sin_global = (float *)sin_t - pos * head_dim;
    forward_layer(&v, 0, out, x, pos, scratch);
}

/* Bidirectional encoder over one sequence (an EmbeddingGemma-style extension;
 * the reference's generate_embeddings is causal, layers.mojo:292-370).  Each
 * layer is forward_layer's arithmetic (layers.mojo:174-220) with every token
 * attending to every token of the sequence (local layers in gemma3 mode: the
 * symmetric window |t - s| < window).  Then the mean of the final-normed
 * states, the dense head (d0 [d0_out][h], d1 [h][d0_out], both optional
 * together) and L2 normalisation.  Works in freshly allocated buffers. */
int ref_encode_sequence(ref_model *m, const int32_t *ids, int64_t n, const float *d0, int64_t d0_out,
                        const float *d1, float *out) {
    const int64_t H = m->h, hd = m->hd, qs = m->hq * hd, ks = m->hkv * hd, I = m->inter;
    if (n <= 0 || n > m->max_seq) return -1;
    float *x = (float *)calloc((size_t)(n * H), sizeof(float));
    float *q = (float *)calloc((size_t)(n * qs), sizeof(float));
    float *k = (float *)calloc((size_t)(n * ks), sizeof(float));
    float *v = (float *)calloc((size_t)(n * ks), sizeof(float));
    float *att = (float *)calloc((size_t)(n * qs), sizeof(float));
    float *sc = (float *)calloc((size_t)n, sizeof(float));
    float *t1 = (float *)calloc((size_t)(H > qs ? H : qs), sizeof(float));
    /* layer frame: o, post-attn, residual, normed residual, mlp out (5H), gate, up, geglu (3I); head: 2H + d0_out */
    float *t2 = (float *)calloc((size_t)(5 * H + 3 * I + 2 * H + d0_out), sizeof(float));
    const float scale = 1.0f / sqrtf((float)hd);
    for (int64_t t = 0; t < n; ++t)
        for (int64_t i = 0; i < H; ++i) x[t * H + i] = m->embed[(int64_t)ids[t] * H + i] * sqrtf((float)H);
    for (int l = 0; l < m->L; ++l) {
        const ref_layer_w *w = &m->layers[l];
        const int glob = layer_is_global(m, l);
        const float *ct = glob ? m->cos_global : m->cos_local, *st = glob ? m->sin_global : m->sin_local;
        for (int64_t t = 0; t < n; ++t) {
            ref_rms_norm(t1, x + t * H, w->input_layernorm, H, 1e-6f, 16);
            ref_vec_mat_mul(q + t * qs, t1, w->q_proj, H, qs, 16);
            ref_vec_mat_mul(k + t * ks, t1, w->k_proj, H, ks, 16);
            ref_vec_mat_mul(v + t * ks, t1, w->v_proj, H, ks, 16);
            for (int64_t h = 0; h < m->hq; ++h) {
                if (w->q_norm) ref_rms_norm(q + t * qs + h * hd, q + t * qs + h * hd, w->q_norm, hd, 1e-6f, 16);
                ref_rope_rotate(q + t * qs + h * hd, ct + t * hd, st + t * hd, hd, 16);
            }
            for (int64_t h = 0; h < m->hkv; ++h) {
                if (w->k_norm) ref_rms_norm(k + t * ks + h * hd, k + t * ks + h * hd, w->k_norm, hd, 1e-6f, 16);
                ref_rope_rotate(k + t * ks + h * hd, ct + t * hd, st + t * hd, hd, 16);
            }
        }
        for (int64_t t = 0; t < n; ++t) {
            int64_t lo = 0, hi = n - 1;
            if (!glob && m->mode == 1) {
                if (t - m->window + 1 > lo) lo = t - m->window + 1;
                if (t + m->window - 1 < hi) hi = t + m->window - 1;
            }
            for (int64_t h = 0; h < m->hq; ++h) {
                const int64_t kvh = h / (m->hq / m->hkv);
                for (int64_t s = lo; s <= hi; ++s) {
                    float a = 0.0f;
                    for (int64_t d = 0; d < hd; ++d) a += q[t * qs + h * hd + d] * k[s * ks + kvh * hd + d];
                    sc[s - lo] = a * scale;
                }
                ref_softmax(sc, hi - lo + 1, 16);
                float *o = att + t * qs + h * hd;
                for (int64_t d = 0; d < hd; ++d) o[d] = 0.0f;
                for (int64_t s = lo; s <= hi; ++s)
                    for (int64_t d = 0; d < hd; ++d) o[d] = o[d] + sc[s - lo] * v[s * ks + kvh * hd + d];
            }
        }
        for (int64_t t = 0; t < n; ++t) {
            float *ao = t2, *pa = t2 + H, *res = t2 + 2 * H, *nr = t2 + 3 * H, *mo = t2 + 4 * H;
            ref_vec_mat_mul(ao, att + t * qs, w->o_proj, qs, H, 16);
            ref_rms_norm(pa, ao, w->post_attention_layernorm, H, 1e-6f, 16);
            for (int64_t i = 0; i < H; ++i) res[i] = x[t * H + i] + pa[i];
            ref_rms_norm(nr, res, w->pre_feedforward_layernorm, H, 1e-6f, 16);
            float *g = mo + H, *u = g + I, *a = u + I;
            ref_vec_mat_mul(g, nr, w->gate_proj, H, I, 16);
            ref_vec_mat_mul(u, nr, w->up_proj, H, I, 16);
            ref_geglu(a, g, u, I, 16);
            ref_vec_mat_mul(mo, a, w->down_proj, I, H, 16);
            ref_rms_norm(pa, mo, w->post_feedforward_layernorm, H, 1e-6f, 16);
            for (int64_t i = 0; i < H; ++i) x[t * H + i] = res[i] + pa[i];
        }
    }
    float *pool = t2;
    for (int64_t i = 0; i < H; ++i) pool[i] = 0.0f;
    for (int64_t t = 0; t < n; ++t) {
        ref_rms_norm(t1, x + t * H, m->final_norm, H, 1e-6f, 16);
        for (int64_t i = 0; i < H; ++i) pool[i] += t1[i];
    }
    for (int64_t i = 0; i < H; ++i) pool[i] /= (float)n;
    const float *y = pool;
    if (d0 && d1) {
        float *h1 = t2 + H, *h2 = t2 + H + d0_out;
        ref_vec_mat_mul(h1, pool, d0, H, d0_out, 16);
        ref_vec_mat_mul(h2, h1, d1, d0_out, H, 16);
        y = h2;
    }
    double ss = 0.0;
    for (int64_t i = 0; i < H; ++i) ss += (double)y[i] * y[i];
    const float inv = (float)(1.0 / sqrt(ss > 1e-24 ? ss : 1e-24));
    for (int64_t i = 0; i < H; ++i) out[i] = y[i] * inv;
    free(x); free(q); free(k); free(v); free(att); free(sc); free(t1); free(t2);
    return 0;
}

