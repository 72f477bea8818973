/*
 * ref_nano.c -- CPU restatement of the MoGemma Gemma 3n ("nano") decode path
 * (TEST INFRASTRUCTURE: the oracle for this path; only tests/ call it).
 *
 * Each function cites the reference lines it follows (paths inside the
 * cofin/mogemma project).  The shared primitives -- vec_mat_mul with its
 * 16-wide reduce_add chunks, softmax, rope_rotate, geglu -- are ref_cpu.c's.
 * The nano norms are scalar loops, as the reference writes them.  Compiled with
 * -ffp-contract=off like ref_cpu.c.  Scratch buffers are separate arrays: the
 * reference's scratch frames do not overlap while their values are live, so
 * this changes no result.
 */
#include "ref_nano.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "ref_cpu.h"

#define NELTS 16

/* layers.mojo:373-386 _rms_norm_nano_weighted: x * (1 / sqrt(mean(x^2) + eps)) * w (in place allowed). */
static void rms_weighted(float *out, const float *x, const float *w, int64_t n, float eps) {
    float sum_sq = 0.0f;
    for (int64_t i = 0; i < n; ++i) sum_sq += x[i] * x[i];
    float inv_rms = 1.0f / sqrtf(sum_sq / (float)n + eps);
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] * inv_rms * w[i];
}

/* layers.mojo:389-401 _rms_norm_nano_unit. */
static void rms_unit(float *out, const float *x, int64_t n, float eps) {
    float sum_sq = 0.0f;
    for (int64_t i = 0; i < n; ++i) sum_sq += x[i] * x[i];
    float inv_rms = 1.0f / sqrtf(sum_sq / (float)n + eps);
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] * inv_rms;
}

/* layers.mojo:622-631 _vector_magnitude: sqrt(mean(v^2) + 1e-6). */
static float magnitude(const float *v, int64_t n) {
    float sum_sq = 0.0f;
    for (int64_t i = 0; i < n; ++i) sum_sq += v[i] * v[i];
    return sqrtf(sum_sq / (float)n + 1e-6f);
}

void ref_nano_activation_sparsity(float *gate, int64_t size, float sparsity) {
    if (sparsity <= 0.0f) return;
    const float z_score = (float)1.6448536269514722; /* N(0,1)^-1(0.95), the reference's constant */
    float sum = 0.0f;
    for (int64_t i = 0; i < size; ++i) sum += gate[i];
    float mean = sum / (float)size;
    float var_sum = 0.0f;
    for (int64_t i = 0; i < size; ++i) {
        float d = gate[i] - mean;
        var_sum += d * d;
    }
    float sd = sqrtf(var_sum / (float)size);
    float cutoff = mean + sd * z_score;
    for (int64_t i = 0; i < size; ++i) {
        float v = gate[i] - cutoff;
        gate[i] = v < 0.0f ? 0.0f : v;
    }
}

/* layers.mojo:150-171 forward_mlp_nano: the first 10 layers sparsify the gate before GeGLU. */
static void mlp_nano(float *out, const float *x, const ref_nano_layer_w *w, int64_t hidden, int64_t inter,
                     int32_t layer_idx, float *scratch) {
    float *g = scratch, *u = scratch + inter, *a = scratch + 2 * inter;
    ref_vec_mat_mul(g, x, w->gate_proj, hidden, inter, NELTS);
    if (layer_idx < 10) ref_nano_activation_sparsity(g, inter, 0.95f);
    ref_vec_mat_mul(u, x, w->up_proj, hidden, inter, NELTS);
    ref_geglu(a, g, u, inter, NELTS);
    ref_vec_mat_mul(out, a, w->down_proj, inter, hidden, NELTS);
}

/* layers.mojo:404-477 forward_attention_nano: weighted RMSNorm on q and k heads, unit RMSNorm on v
 * heads, RoPE on q and k, scaling 1.0, every cached position 0..pos attended.  Scratch frame:
 * q @0, k @q_size, v @q_size + kv_size, attn_out @q_size + 2 kv_size, scores after attn_out. */
static void attention_nano(float *out, const float *x, const ref_nano_layer_w *w, int64_t pos, int64_t hidden,
                           int64_t hq, int64_t hkv, int64_t hd, const float *fc, const float *fs, float *kc,
                           float *vc, int32_t write_kv, float *scratch) {
    const int64_t q_size = hq * hd, kv_size = hkv * hd;
    float *q = scratch, *k = scratch + q_size, *v = scratch + q_size + kv_size;
    ref_vec_mat_mul(q, x, w->q_proj, hidden, q_size, NELTS);
    for (int64_t h = 0; h < hq; ++h) rms_weighted(q + h * hd, q + h * hd, w->q_norm, hd, 1e-6f);
    for (int64_t h = 0; h < hq; ++h) ref_rope_rotate(q + h * hd, fc, fs, hd, NELTS);
    if (write_kv) {
        ref_vec_mat_mul(k, x, w->k_proj, hidden, kv_size, NELTS);
        ref_vec_mat_mul(v, x, w->v_proj, hidden, kv_size, NELTS);
        for (int64_t h = 0; h < hkv; ++h) {
            rms_weighted(k + h * hd, k + h * hd, w->k_norm, hd, 1e-6f);
            rms_unit(v + h * hd, v + h * hd, hd, 1e-6f);
            ref_rope_rotate(k + h * hd, fc, fs, hd, NELTS);
        }
        const int64_t off = pos * kv_size;
        for (int64_t i = 0; i < kv_size; ++i) {
            kc[off + i] = k[i];
            vc[off + i] = v[i];
        }
    }
    const int64_t per_kv = hq / hkv;
    float *attn_out = scratch + q_size + 2 * kv_size;
    float *scores = attn_out + hq * hd;
    for (int64_t h = 0; h < hq; ++h) {
        const int64_t kvh = h / per_kv;
        const float *qh = q + h * hd;
        for (int64_t t = 0; t <= pos; ++t) {
            const float *kh = kc + t * kv_size + kvh * hd;
            float score = 0.0f;
            for (int64_t d = 0; d < hd; ++d) score += qh[d] * kh[d];
            scores[t] = score;
        }
        ref_softmax(scores, pos + 1, NELTS);
        float *oh = attn_out + h * hd;
        for (int64_t d = 0; d < hd; ++d) oh[d] = 0.0f;
        for (int64_t t = 0; t <= pos; ++t) {
            const float *vh = vc + t * kv_size + kvh * hd;
            const float prob = scores[t];
            for (int64_t d = 0; d < hd; ++d) oh[d] = oh[d] + prob * vh[d];
        }
    }
    ref_vec_mat_mul(out, attn_out, w->o_proj, q_size, hidden, NELTS);
}

void ref_nano_per_layer_mapping(float *out, const float *active, const float *per_layer_input, const float *gate,
                                const float *projection, const float *norm, int64_t hidden, int64_t pld) {
    float *g = (float *)malloc(sizeof(float) * (size_t)pld);
    float *p = (float *)malloc(sizeof(float) * (size_t)hidden);
    const float sqrt_2 = (float)1.4142135623730951;
    ref_vec_mat_mul(g, active, gate, hidden, pld, NELTS);
    for (int64_t i = 0; i < pld; ++i) {
        const float x = g[i];
        const float gelu_x = 0.5f * x * (1.0f + erff(x / sqrt_2));
        g[i] = gelu_x * per_layer_input[i];
    }
    ref_vec_mat_mul(p, g, projection, pld, hidden, NELTS);
    rms_weighted(out, p, norm, hidden, 1e-6f);
    free(g);
    free(p);
}

void ref_nano_laurel(float *out, const float *x, const float *down, const float *up, const float *norm, int64_t hidden,
                     int64_t rank) {
    float *d = (float *)malloc(sizeof(float) * (size_t)rank);
    float *u = (float *)malloc(sizeof(float) * (size_t)hidden * 2);
    float *nu = u + hidden;
    ref_vec_mat_mul(d, x, down, hidden, rank, NELTS);
    ref_vec_mat_mul(u, d, up, rank, hidden, NELTS);
    rms_weighted(nu, u, norm, hidden, 1e-6f);
    for (int64_t i = 0; i < hidden; ++i) out[i] = x[i] + nu[i];
    free(d);
    free(u);
}

/* layers.mojo:525-542 _compute_router_modalities: tanh(router . (norm_w(active) / hidden)). */
static void router_modalities(float *modalities, const float *active, const ref_nano_layer_w *w, int64_t hidden,
                              int32_t nm) {
    float *r = (float *)malloc(sizeof(float) * (size_t)hidden);
    rms_weighted(r, active, w->router_norm, hidden, 1e-6f);
    const float scale = 1.0f / (float)hidden;
    for (int64_t i = 0; i < hidden; ++i) r[i] = r[i] * scale;
    ref_vec_mat_mul(modalities, r, w->router, hidden, nm, NELTS);
    for (int32_t m = 0; m < nm; ++m) modalities[m] = tanhf(modalities[m]);
    free(r);
}

void ref_nano_altup_predict(float *out, const float *streams, const ref_nano_layer_w *w, int64_t hidden, int32_t nm) {
    float modalities[64], coef[64 * 64];
    router_modalities(modalities, streams, w, hidden, nm); /* the active stream is stream 0 */
    /* prediction_coefs[router][out][in] (the JAX einsum layout) */
    for (int32_t in_m = 0; in_m < nm; ++in_m)
        for (int32_t out_m = 0; out_m < nm; ++out_m) {
            float c = 0.0f;
            for (int32_t rm = 0; rm < nm; ++rm)
                c += w->prediction_coefs[(int64_t)rm * nm * nm + (int64_t)out_m * nm + in_m] * modalities[rm];
            coef[in_m * nm + out_m] = c;
        }
    for (int32_t out_m = 0; out_m < nm; ++out_m)
        for (int64_t d = 0; d < hidden; ++d) {
            float pred = streams[(int64_t)out_m * hidden + d];
            for (int32_t in_m = 0; in_m < nm; ++in_m) pred += streams[(int64_t)in_m * hidden + d] * coef[in_m * nm + out_m];
            out[(int64_t)out_m * hidden + d] = pred;
        }
}

void ref_nano_altup_correct(float *out, const float *predictions, const float *activated, const ref_nano_layer_w *w,
                            int64_t hidden, int32_t nm) {
    float modalities[64], corr[64];
    router_modalities(modalities, activated, w, hidden, nm);
    /* correction_coefs[router][out] */
    for (int32_t out_m = 0; out_m < nm; ++out_m) {
        float c = 1.0f;
        for (int32_t rm = 0; rm < nm; ++rm) c += w->correction_coefs[(int64_t)rm * nm + out_m] * modalities[rm];
        corr[out_m] = c;
    }
    for (int64_t d = 0; d < hidden; ++d) {
        const float innovation = activated[d] - predictions[d];
        for (int32_t out_m = 0; out_m < nm; ++out_m) {
            const int64_t idx = (int64_t)out_m * hidden + d;
            out[idx] = predictions[idx] + innovation * corr[out_m];
        }
    }
}

void ref_nano_layer(float *out_streams, const float *in_streams, const ref_nano_layer_w *w, int32_t layer_idx,
                    const float *per_layer_input, int64_t pos, int64_t hidden, int64_t hq, int64_t hkv, int64_t hd,
                    int64_t inter, int64_t pld, const float *cos_t, const float *sin_t, float *kc, float *vc,
                    int32_t nm, int32_t write_kv) {
    const int64_t H = hidden;
    const int64_t nh = (int64_t)nm * H;
    float *buf = (float *)malloc(sizeof(float) * (size_t)(2 * nh + 12 * H));
    float *pred = buf, *corrected = buf + nh;
    float *active_norm = buf + 2 * nh, *laurel = active_norm + H, *attn = laurel + H, *attn_norm = attn + H;
    float *attn_laurel = attn_norm + H, *ffw_in = attn_laurel + H, *ffw = ffw_in + H, *ffw_norm = ffw + H;
    float *activated = ffw_norm + H, *first = activated + H, *delta = first + H;
    const int64_t q_size = hq * hd, kv_size = hkv * hd;
    float *att_scratch = (float *)malloc(sizeof(float) * (size_t)(2 * q_size + 2 * kv_size + pos + 1));
    float *mlp_scratch = (float *)malloc(sizeof(float) * (size_t)(3 * inter));

    ref_nano_altup_predict(pred, in_streams, w, H, nm);
    const float *active = pred; /* stream 0 runs attention and MLP */
    rms_weighted(active_norm, active, w->input_layernorm, H, 1e-6f);
    ref_nano_laurel(laurel, active_norm, w->laurel_down, w->laurel_up, w->laurel_norm, H, w->laurel_rank);
    attention_nano(attn, active_norm, w, pos, H, hq, hkv, hd, cos_t, sin_t, kc, vc, write_kv, att_scratch);
    rms_weighted(attn_norm, attn, w->post_attention_layernorm, H, 1e-6f);
    const float inv_sqrt2 = (float)0.7071067811865475;
    for (int64_t i = 0; i < H; ++i) attn_laurel[i] = (active[i] + attn_norm[i] + laurel[i]) * inv_sqrt2;
    rms_weighted(ffw_in, attn_laurel, w->pre_feedforward_layernorm, H, 1e-6f);
    mlp_nano(ffw, ffw_in, w, H, inter, layer_idx, mlp_scratch);
    rms_weighted(ffw_norm, ffw, w->post_feedforward_layernorm, H, 1e-6f);
    for (int64_t i = 0; i < H; ++i) activated[i] = attn_laurel[i] + ffw_norm[i];
    ref_nano_altup_correct(corrected, pred, activated, w, H, nm);
    for (int64_t i = 0; i < H; ++i) first[i] = corrected[i] * w->output_scale[i];
    ref_nano_per_layer_mapping(delta, first, per_layer_input, w->plm_gate, w->plm_projection, w->plm_norm, H, pld);
    for (int64_t i = 0; i < H; ++i) out_streams[i] = corrected[i];
    for (int32_t m = 1; m < nm; ++m)
        for (int64_t i = 0; i < H; ++i) out_streams[(int64_t)m * H + i] = corrected[(int64_t)m * H + i] + delta[i];
    free(att_scratch);
    free(mlp_scratch);
    free(buf);
}

/* ------------------------------------------------------------------------- */

struct ref_nano_model {
    const float *embed, *final_norm, *lm_head, *ple, *ple_proj, *ple_norm;
    const float *altup_proj[16], *altup_unembed[16];
    ref_nano_layer_w *layers;
    int32_t L, nm;
    int64_t h, hq, hkv, hd, inter, vocab, pld, table_layers, max_seq;
    int64_t kv_share_start;
    float *cos_t, *sin_t, *k_cache, *v_cache;
    int64_t pos;
};

/* core.mojo:250-259 _tensor_is_effectively_zero (a NULL tensor counts as zero). */
static int effectively_zero(const float *t, int64_t n) {
    if (!t) return 1;
    for (int64_t i = 0; i < n; ++i)
        if (t[i] > 1e-8f || t[i] < -1e-8f) return 0;
    return 1;
}

ref_nano_model *ref_nano_create(const float *embed, const float *final_norm, const float *lm_head,
                                const float *per_layer_embed, const float *per_layer_projection,
                                const float *per_layer_norm, const float *const *altup_projections,
                                const float *const *altup_unembeds, const ref_nano_layer_w *layers, int32_t num_layers,
                                int64_t hidden, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                int64_t intermediate, int64_t vocab, int64_t pld, int64_t table_layers, int32_t nm,
                                int64_t max_seq_len) {
    if (nm < 1 || nm > 16 || num_layers < 1) return NULL;
    ref_nano_model *m = (ref_nano_model *)calloc(1, sizeof(ref_nano_model));
    m->embed = embed;
    m->final_norm = final_norm;
    m->lm_head = lm_head;
    m->ple = per_layer_embed;
    m->ple_proj = per_layer_projection;
    m->ple_norm = per_layer_norm;
    for (int32_t i = 0; i + 1 < nm; ++i) {
        m->altup_proj[i] = altup_projections[i];
        m->altup_unembed[i] = altup_unembeds[i];
    }
    m->layers = (ref_nano_layer_w *)malloc(sizeof(ref_nano_layer_w) * (size_t)num_layers);
    memcpy(m->layers, layers, sizeof(ref_nano_layer_w) * (size_t)num_layers);
    m->L = num_layers;
    m->nm = nm;
    m->h = hidden;
    m->hq = num_heads;
    m->hkv = num_kv_heads;
    m->hd = head_dim;
    m->inter = intermediate;
    m->vocab = vocab;
    m->pld = pld;
    m->table_layers = table_layers;
    m->max_seq = max_seq_len;
    /* core.mojo:261-273 _detect_nano_kv_share_start: the first layer with zero k and v after a
     * layer that had them */
    m->kv_share_start = num_layers;
    int seen_non_zero = 0;
    const int64_t kv_n = num_kv_heads * head_dim * hidden;
    for (int32_t i = 0; i < num_layers; ++i) {
        const int z = effectively_zero(layers[i].k_proj, kv_n) && effectively_zero(layers[i].v_proj, kv_n);
        if (!z) {
            seen_non_zero = 1;
            continue;
        }
        if (seen_non_zero) {
            m->kv_share_start = i;
            break;
        }
    }
    /* core.mojo:338-348: one RoPE table, base 10000 */
    m->cos_t = (float *)malloc(sizeof(float) * (size_t)(max_seq_len * head_dim));
    m->sin_t = (float *)malloc(sizeof(float) * (size_t)(max_seq_len * head_dim));
    ref_rope_tables(m->cos_t, m->sin_t, max_seq_len, head_dim, 10000.0f);
    const size_t cache = (size_t)num_layers * (size_t)max_seq_len * (size_t)(num_kv_heads * head_dim);
    m->k_cache = (float *)calloc(cache, sizeof(float));
    m->v_cache = (float *)calloc(cache, sizeof(float));
    m->pos = 0;
    return m;
}

void ref_nano_destroy(ref_nano_model *m) {
    if (!m) return;
    free(m->layers);
    free(m->cos_t);
    free(m->sin_t);
    free(m->k_cache);
    free(m->v_cache);
    free(m);
}

int64_t ref_nano_kv_share_start(const ref_nano_model *m) { return m->kv_share_start; }
int64_t ref_nano_pos(const ref_nano_model *m) { return m->pos; }
void ref_nano_set_pos(ref_nano_model *m, int64_t pos) { m->pos = pos; }
const float *ref_nano_k_cache(const ref_nano_model *m) { return m->k_cache; }

/* layers.mojo:633-657 _prepare_altup_streams: stream 0 = base, streams 1.. = projections of the
 * base, each scaled to the base's magnitude. */
static void prepare_streams(const ref_nano_model *m, float *streams, const float *base) {
    const int64_t H = m->h;
    float *proj = (float *)malloc(sizeof(float) * (size_t)H);
    memmove(streams, base, sizeof(float) * (size_t)H);
    const float target = magnitude(streams, H);
    for (int32_t i = 0; i + 1 < m->nm; ++i) {
        ref_vec_mat_mul(proj, streams, m->altup_proj[i], H, H, NELTS);
        float pm = magnitude(proj, H);
        if (pm < 1e-6f) pm = 1e-6f;
        const float scale = target / pm;
        for (int64_t d = 0; d < H; ++d) streams[(int64_t)(i + 1) * H + d] = proj[d] * scale;
    }
    free(proj);
}

/* layers.mojo:660-693 _build_token_per_layer_inputs: per layer l, norm_w(base . W[:, l, :] / sqrt(h))
 * plus the token's row of the per-layer table * sqrt(pld), times 1/sqrt(2). */
static void per_layer_inputs(const ref_nano_model *m, float *out, const float *base, int32_t token) {
    const int64_t H = m->h, P = m->pld, T = m->table_layers;
    float *proj = (float *)malloc(sizeof(float) * (size_t)P * 2);
    float *pn = proj + P;
    const float projection_scale = 1.0f / sqrtf((float)H);
    const float input_scale = (float)0.7071067811865475;
    const float embed_scale = sqrtf((float)P);
    for (int32_t l = 0; l < m->L; ++l) {
        for (int64_t p = 0; p < P; ++p) {
            float acc = 0.0f;
            for (int64_t d = 0; d < H; ++d) acc += base[d] * m->ple_proj[d * T * P + (int64_t)l * P + p];
            proj[p] = acc * projection_scale;
        }
        rms_weighted(pn, proj, m->ple_norm, P, 1e-6f);
        const float *eb = m->ple + (int64_t)token * T * P + (int64_t)l * P;
        float *ob = out + (int64_t)l * P;
        for (int64_t p = 0; p < P; ++p) {
            const float te = eb[p] * embed_scale;
            ob[p] = (pn[p] + te) * input_scale;
        }
    }
    free(proj);
}

/* layers.mojo:696-725 _collapse_altup_streams: base + unembedded streams scaled to the base's
 * magnitude, averaged over the streams. */
static void collapse_streams(const ref_nano_model *m, float *out, const float *streams) {
    const int64_t H = m->h;
    float *tmp = (float *)malloc(sizeof(float) * (size_t)H * 2);
    float *acc = tmp + H;
    const float target = magnitude(streams, H);
    for (int64_t d = 0; d < H; ++d) acc[d] = streams[d];
    for (int32_t k = 1; k < m->nm; ++k) {
        ref_vec_mat_mul(tmp, streams + (int64_t)k * H, m->altup_unembed[k - 1], H, H, NELTS);
        float nmag = magnitude(tmp, H);
        if (nmag < 1e-6f) nmag = 1e-6f;
        const float scale = target / nmag;
        for (int64_t d = 0; d < H; ++d) acc[d] = acc[d] + tmp[d] * scale;
    }
    const float inv = 1.0f / (float)m->nm;
    for (int64_t d = 0; d < H; ++d) out[d] = acc[d] * inv;
    free(tmp);
}

/* layers.mojo:842-956 _forward_nano_token_hidden: embedding * sqrt(h), AltUp streams, per-layer
 * inputs, the layers (layers from kv_share_start on read the cache of the last earlier layer of
 * their attention kind -- every 5th layer full attention, the rest sliding -- and write none),
 * collapse, final weighted norm. */
static void token_hidden(ref_nano_model *m, float *out, int32_t token, int64_t pos) {
    const int64_t H = m->h, nh = (int64_t)m->nm * H;
    float *cur = (float *)malloc(sizeof(float) * (size_t)(2 * nh));
    float *next = cur + nh;
    float *pli = (float *)malloc(sizeof(float) * (size_t)(m->L * m->pld));
    const float *e = m->embed + (int64_t)token * H;
    const float emb_scale = sqrtf((float)H);
    for (int64_t i = 0; i < H; ++i) cur[i] = e[i] * emb_scale;
    prepare_streams(m, cur, cur);
    per_layer_inputs(m, pli, cur, token);
    const int64_t kss = m->kv_share_start;
    int64_t last_full = kss - 1;
    while (last_full >= 0 && ((last_full + 1) % 5) != 0) --last_full;
    int64_t last_sliding = kss - 1;
    while (last_sliding >= 0 && ((last_sliding + 1) % 5) == 0) --last_sliding;
    const int64_t layer_kv = m->max_seq * m->hkv * m->hd;
    for (int32_t l = 0; l < m->L; ++l) {
        int64_t kv_l = l;
        int32_t write_kv = 1;
        if (kss < m->L && l >= kss) {
            write_kv = 0;
            if (((l + 1) % 5) == 0 && last_full >= 0)
                kv_l = last_full;
            else if (last_sliding >= 0)
                kv_l = last_sliding;
            else
                kv_l = kss - 1;
        }
        ref_nano_layer(next, cur, &m->layers[l], l, pli + (int64_t)l * m->pld, pos, H, m->hq, m->hkv, m->hd, m->inter,
                       m->pld, m->cos_t + pos * m->hd, m->sin_t + pos * m->hd, m->k_cache + kv_l * layer_kv,
                       m->v_cache + kv_l * layer_kv, m->nm, write_kv);
        memcpy(cur, next, sizeof(float) * (size_t)nh);
    }
    collapse_streams(m, out, cur);
    rms_weighted(out, out, m->final_norm, H, 1e-6f);
    free(pli);
    free(cur);
}

int ref_nano_step(ref_nano_model *m, int32_t token_id, float *logits) {
    if (m->pos >= m->max_seq) return -1; /* core.mojo:380-381 "Sequence length exceeded" */
    float *hid = (float *)malloc(sizeof(float) * (size_t)m->h);
    token_hidden(m, hid, token_id, m->pos);
    if (logits) ref_vec_mat_mul(logits, hid, m->lm_head, m->h, m->vocab, NELTS); /* layers.mojo:1004 */
    free(hid);
    m->pos += 1;
    return 0;
}

void ref_nano_embed_sequence(ref_nano_model *m, const int32_t *ids, int64_t n, float *out) {
    const int64_t H = m->h;
    float *acc = (float *)calloc((size_t)H * 2, sizeof(float));
    float *th = acc + H;
    for (int64_t t = 0; t < n; ++t) {
        token_hidden(m, th, ids[t], t);
        for (int64_t i = 0; i < H; ++i) acc[i] = acc[i] + th[i];
    }
    const float scale = 1.0f / (float)n;
    for (int64_t i = 0; i < H; ++i) out[i] = acc[i] * scale;
    free(acc);
}
