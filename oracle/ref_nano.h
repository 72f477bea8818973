/*
 * ref_nano.h -- CPU restatement of the MoGemma Gemma 3n ("nano") decode path
 * (TEST INFRASTRUCTURE: the oracle for this path, used by tests/ only).
 *
 * Restates src/mo/mogemma/layers.mojo:121-171 and 373-1063 and the nano parts
 * of src/mo/mogemma/core.mojo (111-272, 296-312, 410-430).
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One Gemma 3n layer's tensors (row-major [out][in] like the reference's
 * TensorInfo(ptr, shape_0 = out, shape_1 = in)). */
typedef struct ref_nano_layer_w {
    const float *input_layernorm, *post_attention_layernorm, *pre_feedforward_layernorm, *post_feedforward_layernorm;
    const float *q_proj, *k_proj, *v_proj, *o_proj, *gate_proj, *up_proj, *down_proj, *q_norm, *k_norm;
    /* AltUp: router [nm][h], router_norm [h], prediction_coefs [nm][nm][nm], correction_coefs [nm][nm],
     * output_scale [h] */
    const float *router, *router_norm, *prediction_coefs, *correction_coefs, *output_scale;
    /* Laurel: down [rank][h], up [h][rank], norm [h] */
    const float *laurel_down, *laurel_up, *laurel_norm;
    int64_t laurel_rank;
    /* per-layer mapping: gate [pld][h], projection [h][pld], norm [h] */
    const float *plm_gate, *plm_projection, *plm_norm;
} ref_nano_layer_w;

typedef struct ref_nano_model ref_nano_model;

/* layers.mojo:505-522 forward_laurel: out = x + norm_w(up(down(x))). */
void ref_nano_laurel(float *out, const float *x, const float *down, const float *up, const float *norm, int64_t hidden,
                     int64_t rank);
/* layers.mojo:480-502 forward_per_layer_mapping. */
void ref_nano_per_layer_mapping(float *out, const float *active, const float *per_layer_input, const float *gate,
                                const float *projection, const float *norm, int64_t hidden, int64_t pld);
/* layers.mojo:545-581 forward_altup_predict (streams [nm][h] -> predictions [nm][h]). */
void ref_nano_altup_predict(float *out, const float *streams, const ref_nano_layer_w *w, int64_t hidden, int32_t nm);
/* layers.mojo:584-619 forward_altup_correct. */
void ref_nano_altup_correct(float *out, const float *predictions, const float *activated, const ref_nano_layer_w *w,
                            int64_t hidden, int32_t nm);
/* layers.mojo:121-147 _apply_nano_activation_sparsity (in place). */
void ref_nano_activation_sparsity(float *gate, int64_t size, float sparsity);
/* layers.mojo:728-839 forward_nano_layer: one layer over the nm streams. cos/sin point at this
 * position's table row; kc/vc at this layer's (or the shared layer's) cache [max_seq][hkv][hd]. */
void ref_nano_layer(float *out_streams, const float *in_streams, const ref_nano_layer_w *w, int32_t layer_idx,
                    const float *per_layer_input, int64_t pos, int64_t hidden, int64_t hq, int64_t hkv, int64_t hd,
                    int64_t inter, int64_t pld, const float *cos_t, const float *sin_t, float *kc, float *vc,
                    int32_t nm, int32_t write_kv);

/* The model (core.mojo:296-312 dims, 326-348 caches and RoPE tables, 261-273 kv_share_start).
 * altup_projections / altup_unembeds: nm - 1 matrices [h][h] each.  per_layer_embed
 * [vocab][table_layers][pld], per_layer_projection [h][table_layers][pld]. */
ref_nano_model *ref_nano_create(const float *embed, const float *final_norm, const float *lm_head,
                                const float *per_layer_embed, const float *per_layer_projection,
                                const float *per_layer_norm, const float *const *altup_projections,
                                const float *const *altup_unembeds, const ref_nano_layer_w *layers, int32_t num_layers,
                                int64_t hidden, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                int64_t intermediate, int64_t vocab, int64_t pld, int64_t table_layers, int32_t nm,
                                int64_t max_seq_len);
void ref_nano_destroy(ref_nano_model *m);
int64_t ref_nano_kv_share_start(const ref_nano_model *m);
int64_t ref_nano_pos(const ref_nano_model *m);
void ref_nano_set_pos(ref_nano_model *m, int64_t pos);
const float *ref_nano_k_cache(const ref_nano_model *m);
/* core.mojo:366-461 step for arch "nano": forward_nano_step (layers.mojo:959-1004) at the model's
 * position, logits [vocab] (NULL: skip the lm_head), position += 1.  Returns -1 past max_seq_len. */
int ref_nano_step(ref_nano_model *m, int32_t token_id, float *logits);
/* layers.mojo:1007-1063 forward_nano_sequence: mean of the final hidden states over tokens 0..n-1. */
void ref_nano_embed_sequence(ref_nano_model *m, const int32_t *ids, int64_t n, float *out);

#ifdef __cplusplus
}
#endif
