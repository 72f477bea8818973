// nano.cu -- the Gemma 3n ("nano") decode engine behind the C ABI (mg_nano_*).
//
// The reference dispatches on the checkpoint (core.mojo:26-31: an AltUp router
// means arch "nano") and runs forward_nano_step (layers.mojo:959-1004) per
// token.  Here the whole step is one CUDA graph of the kernels in
// nano_kernels.cuh, captured at creation (one graph with the lm_head, one
// without for prefill and embeddings) and replayed per token with the token
// and position in device memory.  Weights stay fp32 in the reference's
// row-major layout.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/mogemma_b200.h"
#include "nano_kernels.cuh"

namespace mg {
mg_status report_error(mg_status st, const char *msg);
}

namespace {

using namespace mg::nano;

struct NanoLayer {
    const float *in_ln, *post_attn_ln, *pre_ff_ln, *post_ff_ln;
    const float *q, *k, *v, *o, *gate, *up, *down, *q_norm, *k_norm;
    const float *router, *router_norm, *pc, *cc, *out_scale;
    const float *laurel_down, *laurel_up, *laurel_norm;
    const float *plm_gate, *plm_proj, *plm_norm;
    int kv_layer;  // cache this layer attends to
    bool write_kv;
};

}  // namespace

struct mg_nano {
    int dev = 0;
    cudaStream_t stream = nullptr;
    int L = 0, H = 0, hq = 0, hkv = 0, hd = 0, I = 0, V = 0, P = 0, T = 0, nm = 0, rank = 0, cap = 0;
    int kv_share_start = 0;
    std::vector<void *> allocs;
    std::vector<NanoLayer> layers;
    const float *embed = nullptr, *final_norm = nullptr, *lm_head = nullptr;
    const float *ple = nullptr, *ple_proj = nullptr, *ple_norm = nullptr;
    std::vector<const float *> altup_proj, altup_unembed;
    float *cos_t = nullptr, *sin_t = nullptr;
    std::vector<float *> kc, vc;
    // activations
    float *streams, *pred, *corrected, *proj, *u, *active_norm, *laurel_d, *laurel_u, *laurel, *q, *k, *v, *att,
        *attn, *attn_norm, *al, *ffin, *gate, *upb, *act, *ff, *activated, *first, *plm_g, *plm_p, *delta, *hidden,
        *ple_projected, *pli, *logits, *emb_acc;
    int32_t *d_tok = nullptr, *d_pos = nullptr;
    int32_t *h_stage = nullptr;  // pinned [tok, pos]
    cudaGraphExec_t g_logits = nullptr, g_hidden = nullptr;
    int pos = 0;
};

namespace {

mg_status fail(mg_status st, const std::string &msg) { return mg::report_error(st, msg.c_str()); }

#define NCU(call)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            return fail(e_ == cudaErrorMemoryAllocation ? MG_ERR_OOM : MG_ERR_CUDA,                 \
                        std::string(#call) + " failed: " + cudaGetErrorString(e_));                 \
    } while (0)

// Device buffer; `zero` clears it on the model's stream (which does not order with the
// synchronous copies of the upload path, so buffers that are uploaded are not cleared).
template <typename T>
mg_status dalloc(mg_nano *m, T **p, size_t count, bool zero = true) {
    void *v = nullptr;
    NCU(cudaMalloc(&v, std::max<size_t>(count * sizeof(T), 16)));
    m->allocs.push_back(v);
    if (zero) NCU(cudaMemsetAsync(v, 0, std::max<size_t>(count * sizeof(T), 16), m->stream));
    *p = static_cast<T *>(v);
    return MG_OK;
}

struct Host {
    const mg_tensor_desc *d;
    int64_t numel() const {
        int64_t n = 1;
        for (int i = 0; i < d->ndim; ++i) n *= d->shape[i];
        return n;
    }
};

// Uploads a tensor as fp32 (bf16 sources are widened exactly).
mg_status upload(mg_nano *m, const mg_tensor_desc *t, const float **out) {
    const int64_t n = Host{t}.numel();
    float *dst = nullptr;
    mg_status s = dalloc(m, &dst, static_cast<size_t>(n), false);
    if (s != MG_OK) return s;
    if (t->dtype == MG_F32) {
        NCU(cudaMemcpy(dst, t->data, sizeof(float) * n, cudaMemcpyHostToDevice));
    } else if (t->dtype == MG_BF16) {
        std::vector<float> tmp(static_cast<size_t>(n));
        const uint16_t *src = static_cast<const uint16_t *>(t->data);
        for (int64_t i = 0; i < n; ++i) {
            const uint32_t b = static_cast<uint32_t>(src[i]) << 16;
            std::memcpy(&tmp[static_cast<size_t>(i)], &b, 4);
        }
        NCU(cudaMemcpy(dst, tmp.data(), sizeof(float) * n, cudaMemcpyHostToDevice));
    } else {
        return fail(MG_ERR_INVALID, std::string("tensor ") + t->name + ": dtype must be F32 or BF16");
    }
    *out = dst;
    return MG_OK;
}

// core.mojo:250-259: a tensor whose every value is within 1e-8 of zero (or absent).
bool effectively_zero(const mg_tensor_desc *t) {
    if (!t || !t->data) return true;
    const int64_t n = Host{t}.numel();
    for (int64_t i = 0; i < n; ++i) {
        float v;
        if (t->dtype == MG_F32) {
            v = static_cast<const float *>(t->data)[i];
        } else {
            const uint32_t b = static_cast<uint32_t>(static_cast<const uint16_t *>(t->data)[i]) << 16;
            std::memcpy(&v, &b, 4);
        }
        if (v > 1e-8f || v < -1e-8f) return false;
    }
    return true;
}

void gemv(mg_nano *m, float *out, const float *x, const float *W, int in, int out_dim, float scale = 1.0f) {
    k_gemv<<<(out_dim + kWarpsPerGemv - 1) / kWarpsPerGemv, kWarpsPerGemv * 32, 0, m->stream>>>(out, x, W, in,
                                                                                               out_dim, scale);
}
int grid_for(int n) { return std::min((n + 255) / 256, 1184); }

// The kernels of one token (forward_nano_step, layers.mojo:959-1004), issued on m->stream.
void issue_step(mg_nano *m, bool with_logits) {
    cudaStream_t s = m->stream;
    const int H = m->H, nm = m->nm, P = m->P;
    float *s0 = m->streams;
    k_embed<<<grid_for(H), 256, 0, s>>>(s0, m->embed, m->d_tok, H, std::sqrt(static_cast<float>(H)));
    for (int i = 0; i + 1 < nm; ++i) gemv(m, m->proj + static_cast<int64_t>(i) * H, s0, m->altup_proj[i], H, H);
    if (nm > 1) k_match_magnitude<<<nm - 1, kBlock, 0, s>>>(m->streams, m->proj, H);
    k_ple_project<<<(m->L * P + 255) / 256, 256, 0, s>>>(m->ple_projected, s0, m->ple_proj, H, m->T, P, m->L,
                                                         1.0f / std::sqrt(static_cast<float>(H)));
    k_ple_finish<<<m->L, kBlock, 0, s>>>(m->pli, m->ple_projected, m->ple_norm, m->ple, m->d_tok, m->T, P);
    const int qs = m->hq * m->hd, kvs = m->hkv * m->hd;
    for (int l = 0; l < m->L; ++l) {
        const NanoLayer &w = m->layers[l];
        k_altup_predict<<<1, kBlock, 0, s>>>(m->pred, m->streams, w.router, w.router_norm, w.pc, H, nm);
        const float *active = m->pred;  // stream 0 runs attention and the MLP
        k_rms<<<1, kBlock, 0, s>>>(m->active_norm, active, w.in_ln, nullptr, H);
        gemv(m, m->laurel_d, m->active_norm, w.laurel_down, H, m->rank);
        gemv(m, m->laurel_u, m->laurel_d, w.laurel_up, m->rank, H);
        k_rms<<<1, kBlock, 0, s>>>(m->laurel, m->laurel_u, w.laurel_norm, m->active_norm, H);
        gemv(m, m->q, m->active_norm, w.q, H, qs);
        if (w.write_kv) {
            gemv(m, m->k, m->active_norm, w.k, H, kvs);
            gemv(m, m->v, m->active_norm, w.v, H, kvs);
        }
        k_qkv_heads<<<m->hq + (w.write_kv ? m->hkv : 0), kBlock, 0, s>>>(m->q, m->k, m->v, w.q_norm, w.k_norm,
                                                                         m->cos_t, m->sin_t, m->d_pos, m->hq, m->hkv,
                                                                         m->hd, m->kc[l], m->vc[l]);
        k_attention<<<m->hq, kBlock, sizeof(float) * m->cap, s>>>(m->att, m->q, m->kc[w.kv_layer], m->vc[w.kv_layer],
                                                                  m->d_pos, m->hq, m->hkv, m->hd);
        gemv(m, m->attn, m->att, w.o, qs, H);
        k_rms<<<1, kBlock, 0, s>>>(m->attn_norm, m->attn, w.post_attn_ln, nullptr, H);
        k_combine3<<<grid_for(H), 256, 0, s>>>(m->al, active, m->attn_norm, m->laurel, H);
        k_rms<<<1, kBlock, 0, s>>>(m->ffin, m->al, w.pre_ff_ln, nullptr, H);
        gemv(m, m->gate, m->ffin, w.gate, H, m->I);
        if (l < 10) k_sparsity<<<1, kBlock, 0, s>>>(m->gate, m->I);  // layers.mojo:166-168
        gemv(m, m->upb, m->ffin, w.up, H, m->I);
        k_gelu_mul<<<grid_for(m->I), 256, 0, s>>>(m->act, m->gate, m->upb, m->I);
        gemv(m, m->ff, m->act, w.down, m->I, H);
        k_rms<<<1, kBlock, 0, s>>>(m->activated, m->ff, w.post_ff_ln, m->al, H);
        k_altup_correct<<<1, kBlock, 0, s>>>(m->corrected, m->first, m->pred, m->activated, w.router, w.router_norm,
                                             w.cc, w.out_scale, H, nm);
        gemv(m, m->plm_g, m->first, w.plm_gate, H, P);
        k_gelu_mul<<<grid_for(P), 256, 0, s>>>(m->plm_g, m->plm_g, m->pli + static_cast<int64_t>(l) * P, P);
        gemv(m, m->plm_p, m->plm_g, w.plm_proj, P, H);
        k_rms<<<1, kBlock, 0, s>>>(m->delta, m->plm_p, w.plm_norm, nullptr, H);
        k_streams_next<<<grid_for(nm * H), 256, 0, s>>>(m->streams, m->corrected, m->delta, H, nm);
    }
    for (int k = 1; k < nm; ++k)
        gemv(m, m->u + static_cast<int64_t>(k - 1) * H, m->streams + static_cast<int64_t>(k) * H, m->altup_unembed[k - 1],
             H, H);
    k_collapse<<<1, kBlock, 0, s>>>(m->hidden, m->streams, m->u, m->final_norm, H, nm);
    if (with_logits) gemv(m, m->logits, m->hidden, m->lm_head, H, m->V);
}

mg_status capture(mg_nano *m, bool with_logits, cudaGraphExec_t *exec) {
    cudaGraph_t g = nullptr;
    NCU(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    issue_step(m, with_logits);
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (e != cudaSuccess) return fail(MG_ERR_CUDA, std::string("graph capture failed: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(MG_ERR_CUDA, std::string("graph instantiation failed: ") + cudaGetErrorString(e));
    return MG_OK;
}

void destroy(mg_nano *m) {
    if (!m) return;
    cudaSetDevice(m->dev);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->g_logits) cudaGraphExecDestroy(m->g_logits);
    if (m->g_hidden) cudaGraphExecDestroy(m->g_hidden);
    for (void *p : m->allocs) cudaFree(p);
    if (m->h_stage) cudaFreeHost(m->h_stage);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

mg_status create(const mg_tensor_desc *descs, int32_t n, int32_t device, int32_t capacity, mg_nano *m) {
    std::unordered_map<std::string, const mg_tensor_desc *> by;
    for (int32_t i = 0; i < n; ++i)
        if (descs[i].name) by[descs[i].name] = &descs[i];
    auto get = [&](const std::string &k) -> const mg_tensor_desc * {
        auto it = by.find(k);
        return it == by.end() ? nullptr : it->second;
    };
    if (!get("model.layers.0.altup.router.weight"))
        return fail(MG_ERR_INVALID, "not a Gemma 3n checkpoint (no model.layers.0.altup.router.weight)");
    while (get("model.layers." + std::to_string(m->L) + ".input_layernorm.weight")) ++m->L;
    if (m->L == 0) return fail(MG_ERR_INVALID, "Invalid Nano model weights: no layers found in metadata");
    const std::string p0 = "model.layers.0.";
    const mg_tensor_desc *E = get("model.embed_tokens.weight"), *LM = get("lm_head.weight"),
                         *PLE = get("model.per_layer_embed.weight");
    const mg_tensor_desc *QN = get(p0 + "self_attn.q_norm.weight"), *KP = get(p0 + "self_attn.k_proj.weight"),
                         *QP = get(p0 + "self_attn.q_proj.weight"), *GP = get(p0 + "mlp.gate_proj.weight"),
                         *PG = get(p0 + "per_layer_map.gate.weight"), *RT = get(p0 + "altup.router.weight"),
                         *LD = get(p0 + "laurel.down_proj.weight");
    for (const mg_tensor_desc *t : {E, LM, PLE, KP, QP, GP, PG, RT, LD})
        if (!t) return fail(MG_ERR_INVALID, "Gemma 3n checkpoint misses a required tensor");
    // dims as init_model_mojo infers them (core.mojo:296-312)
    m->hd = QN ? static_cast<int>(QN->shape[0]) : 256;
    m->H = static_cast<int>(E->shape[1]);
    m->hkv = static_cast<int>(KP->shape[0] / m->hd);
    m->hq = static_cast<int>(QP->shape[0] / m->hd);
    m->I = static_cast<int>(GP->shape[0]);
    m->V = static_cast<int>(LM->shape[0]);
    m->P = static_cast<int>(PG->shape[0]);
    m->nm = static_cast<int>(RT->shape[0]);
    m->rank = static_cast<int>(LD->shape[0]);
    m->T = PLE->ndim >= 3 ? static_cast<int>(PLE->shape[1]) : 0;
    m->cap = capacity;
    if (m->P <= 0) return fail(MG_ERR_INVALID, "Invalid Nano model weights: per_layer_map gate dim must be > 0");
    if (m->T < m->L || PLE->ndim != 3)
        return fail(MG_ERR_INVALID, "per_layer_embed must be [vocab, layers >= num_layers, per_layer_dim]");
    if (m->nm < 1 || m->nm > kMaxModalities) return fail(MG_ERR_UNSUPPORTED, "AltUp modalities outside [1, 8]");
    if (m->hd % 2 || m->hkv < 1 || m->hq % m->hkv) return fail(MG_ERR_INVALID, "inconsistent head shapes");
    if (capacity < 1 || static_cast<size_t>(capacity) * sizeof(float) > 200 * 1024)
        return fail(MG_ERR_INVALID, "capacity must be in [1, 51200] positions");
    m->dev = device;
    NCU(cudaSetDevice(device));
    NCU(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    if (static_cast<size_t>(capacity) * sizeof(float) > 48 * 1024)
        NCU(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(float) * capacity)));
    auto up = [&](const std::string &k, const float **dst, bool required = true) -> mg_status {
        const mg_tensor_desc *t = get(k);
        if (!t) {
            if (!required) return MG_OK;
            return fail(MG_ERR_INVALID, "missing tensor " + k);
        }
        return upload(m, t, dst);
    };
#define NTRY(x)                       \
    do {                              \
        mg_status s_ = (x);           \
        if (s_ != MG_OK) return s_;   \
    } while (0)
    NTRY(up("model.embed_tokens.weight", &m->embed));
    NTRY(up("model.norm.weight", &m->final_norm));
    if (get("lm_head.weight")->data == get("model.embed_tokens.weight")->data)
        m->lm_head = m->embed;  // tied
    else
        NTRY(up("lm_head.weight", &m->lm_head));
    NTRY(up("model.per_layer_embed.weight", &m->ple));
    NTRY(up("model.per_layer_embed.projection.weight", &m->ple_proj));
    NTRY(up("model.per_layer_embed.norm.weight", &m->ple_norm));
    m->altup_proj.resize(m->nm > 1 ? m->nm - 1 : 0);
    m->altup_unembed.resize(m->altup_proj.size());
    for (size_t i = 0; i < m->altup_proj.size(); ++i) {
        NTRY(up("model.altup.projection." + std::to_string(i) + ".weight", &m->altup_proj[i]));
        NTRY(up("model.altup.unembed." + std::to_string(i) + ".weight", &m->altup_unembed[i]));
    }
    // core.mojo:261-273: KV sharing starts at the first zero-k/v layer after one that had k/v
    m->kv_share_start = m->L;
    bool seen = false;
    for (int l = 0; l < m->L; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        const bool z = effectively_zero(get(p + "self_attn.k_proj.weight")) &&
                       effectively_zero(get(p + "self_attn.v_proj.weight"));
        if (!z) {
            seen = true;
            continue;
        }
        if (seen) {
            m->kv_share_start = l;
            break;
        }
    }
    // layers.mojo:889-905: the cache each layer reads
    const int kss = m->kv_share_start;
    int last_full = kss - 1;
    while (last_full >= 0 && ((last_full + 1) % 5) != 0) --last_full;
    int last_sliding = kss - 1;
    while (last_sliding >= 0 && ((last_sliding + 1) % 5) == 0) --last_sliding;
    m->layers.resize(m->L);
    for (int l = 0; l < m->L; ++l) {
        NanoLayer &w = m->layers[l];
        const std::string p = "model.layers." + std::to_string(l) + ".";
        NTRY(up(p + "input_layernorm.weight", &w.in_ln));
        NTRY(up(p + "post_attention_layernorm.weight", &w.post_attn_ln));
        NTRY(up(p + "pre_feedforward_layernorm.weight", &w.pre_ff_ln));
        NTRY(up(p + "post_feedforward_layernorm.weight", &w.post_ff_ln));
        NTRY(up(p + "self_attn.q_proj.weight", &w.q));
        NTRY(up(p + "self_attn.k_proj.weight", &w.k));
        NTRY(up(p + "self_attn.v_proj.weight", &w.v));
        NTRY(up(p + "self_attn.o_proj.weight", &w.o));
        NTRY(up(p + "mlp.gate_proj.weight", &w.gate));
        NTRY(up(p + "mlp.up_proj.weight", &w.up));
        NTRY(up(p + "mlp.down_proj.weight", &w.down));
        NTRY(up(p + "self_attn.q_norm.weight", &w.q_norm));
        NTRY(up(p + "self_attn.k_norm.weight", &w.k_norm));
        NTRY(up(p + "altup.router.weight", &w.router));
        NTRY(up(p + "altup.router_norm.weight", &w.router_norm));
        NTRY(up(p + "altup.prediction_coefs", &w.pc));
        NTRY(up(p + "altup.correction_coefs", &w.cc));
        NTRY(up(p + "altup.output_scale", &w.out_scale));
        NTRY(up(p + "laurel.down_proj.weight", &w.laurel_down));
        NTRY(up(p + "laurel.up_proj.weight", &w.laurel_up));
        NTRY(up(p + "laurel.norm.weight", &w.laurel_norm));
        NTRY(up(p + "per_layer_map.gate.weight", &w.plm_gate));
        NTRY(up(p + "per_layer_map.projection.weight", &w.plm_proj));
        NTRY(up(p + "per_layer_map.norm.weight", &w.plm_norm));
        w.write_kv = true;
        w.kv_layer = l;
        if (kss < m->L && l >= kss) {
            w.write_kv = false;
            if (((l + 1) % 5) == 0 && last_full >= 0)
                w.kv_layer = last_full;
            else if (last_sliding >= 0)
                w.kv_layer = last_sliding;
            else
                w.kv_layer = kss - 1;
        }
    }
    // RoPE tables (core.mojo:338-348): base 10000, cos/sin at [t * hd + d] for d < hd / 2
    {
        std::vector<float> c(static_cast<size_t>(capacity) * m->hd, 0.f), sn(c.size(), 0.f);
        for (int t = 0; t < capacity; ++t)
            for (int d = 0; d < m->hd / 2; ++d) {
                const float e = static_cast<float>(d * 2) / static_cast<float>(m->hd);
                const float inv = 1.0f / powf(10000.0f, e);
                const float f = static_cast<float>(t) * inv;
                c[static_cast<size_t>(t) * m->hd + d] = cosf(f);
                sn[static_cast<size_t>(t) * m->hd + d] = sinf(f);
            }
        NTRY(dalloc(m, &m->cos_t, c.size(), false));
        NTRY(dalloc(m, &m->sin_t, sn.size(), false));
        NCU(cudaMemcpy(m->cos_t, c.data(), sizeof(float) * c.size(), cudaMemcpyHostToDevice));
        NCU(cudaMemcpy(m->sin_t, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice));
    }
    m->kc.assign(m->L, nullptr);
    m->vc.assign(m->L, nullptr);
    const size_t per_layer = static_cast<size_t>(capacity) * m->hkv * m->hd;
    for (int l = 0; l < m->L; ++l) {
        NTRY(dalloc(m, &m->kc[l], per_layer));
        NTRY(dalloc(m, &m->vc[l], per_layer));
    }
    const size_t H = m->H, nh = static_cast<size_t>(m->nm) * H;
    NTRY(dalloc(m, &m->streams, nh));
    NTRY(dalloc(m, &m->pred, nh));
    NTRY(dalloc(m, &m->corrected, nh));
    NTRY(dalloc(m, &m->proj, nh));
    NTRY(dalloc(m, &m->u, nh));
    for (float **b : {&m->active_norm, &m->laurel_u, &m->laurel, &m->attn, &m->attn_norm, &m->al, &m->ffin, &m->ff,
                      &m->activated, &m->first, &m->plm_p, &m->delta, &m->hidden, &m->emb_acc})
        NTRY(dalloc(m, b, H));
    NTRY(dalloc(m, &m->laurel_d, static_cast<size_t>(m->rank)));
    NTRY(dalloc(m, &m->q, static_cast<size_t>(m->hq) * m->hd));
    NTRY(dalloc(m, &m->att, static_cast<size_t>(m->hq) * m->hd));
    NTRY(dalloc(m, &m->k, static_cast<size_t>(m->hkv) * m->hd));
    NTRY(dalloc(m, &m->v, static_cast<size_t>(m->hkv) * m->hd));
    NTRY(dalloc(m, &m->gate, static_cast<size_t>(m->I)));
    NTRY(dalloc(m, &m->upb, static_cast<size_t>(m->I)));
    NTRY(dalloc(m, &m->act, static_cast<size_t>(m->I)));
    NTRY(dalloc(m, &m->plm_g, static_cast<size_t>(m->P)));
    NTRY(dalloc(m, &m->ple_projected, static_cast<size_t>(m->L) * m->P));
    NTRY(dalloc(m, &m->pli, static_cast<size_t>(m->L) * m->P));
    NTRY(dalloc(m, &m->logits, static_cast<size_t>(m->V)));
    NTRY(dalloc(m, &m->d_tok, 1));
    NTRY(dalloc(m, &m->d_pos, 1));
    NCU(cudaMallocHost(&m->h_stage, 2 * sizeof(int32_t)));
    NCU(cudaStreamSynchronize(m->stream));
    NTRY(capture(m, true, &m->g_logits));
    NTRY(capture(m, false, &m->g_hidden));
#undef NTRY
    return MG_OK;
}

// One token at the model's position through the graph; logits_host (nullable) gets [vocab].
mg_status run_token(mg_nano *m, int32_t token, bool logits, float *logits_host) {
    if (m->pos >= m->cap) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
    if (token < 0 || token >= m->V) return fail(MG_ERR_INVALID, "token id " + std::to_string(token) + " outside the vocabulary");
    m->h_stage[0] = token;
    m->h_stage[1] = m->pos;
    NCU(cudaMemcpyAsync(m->d_tok, m->h_stage, sizeof(int32_t), cudaMemcpyHostToDevice, m->stream));
    NCU(cudaMemcpyAsync(m->d_pos, m->h_stage + 1, sizeof(int32_t), cudaMemcpyHostToDevice, m->stream));
    NCU(cudaGraphLaunch(logits ? m->g_logits : m->g_hidden, m->stream));
    if (logits_host)
        NCU(cudaMemcpyAsync(logits_host, m->logits, sizeof(float) * m->V, cudaMemcpyDeviceToHost, m->stream));
    // the staging words are rewritten by the next token only after this one's copies ran
    NCU(cudaStreamSynchronize(m->stream));
    m->pos += 1;
    return MG_OK;
}

}  // namespace

extern "C" mg_status mg_nano_create(const mg_tensor_desc *descs, int32_t n, int32_t device, int32_t capacity,
                                    mg_nano **out) {
    if (!descs || !out || n <= 0) return fail(MG_ERR_INVALID, "null argument");
    *out = nullptr;
    mg_nano *m = new mg_nano();
    mg_status st = create(descs, n, device, capacity, m);
    if (st != MG_OK) {
        destroy(m);
        return st;
    }
    *out = m;
    return MG_OK;
}

extern "C" mg_status mg_nano_destroy(mg_nano *m) {
    destroy(m);
    return MG_OK;
}

extern "C" mg_status mg_nano_info_get(const mg_nano *m, mg_nano_info *info) {
    if (!m || !info) return fail(MG_ERR_INVALID, "null argument");
    info->num_layers = m->L;
    info->num_heads = m->hq;
    info->num_kv_heads = m->hkv;
    info->head_dim = m->hd;
    info->hidden_size = m->H;
    info->intermediate_size = m->I;
    info->vocab_size = m->V;
    info->per_layer_dim = m->P;
    info->modalities = m->nm;
    info->laurel_rank = m->rank;
    info->kv_share_start = m->kv_share_start;
    info->max_seq_len = m->cap;
    return MG_OK;
}

extern "C" mg_status mg_nano_set_pos(mg_nano *m, int32_t pos) {
    if (!m) return fail(MG_ERR_INVALID, "null model");
    if (pos < 0 || pos > m->cap) return fail(MG_ERR_INVALID, "position outside [0, capacity]");
    m->pos = pos;
    return MG_OK;
}

extern "C" mg_status mg_nano_get_pos(const mg_nano *m, int32_t *pos) {
    if (!m || !pos) return fail(MG_ERR_INVALID, "null argument");
    *pos = m->pos;
    return MG_OK;
}

extern "C" mg_status mg_nano_step(mg_nano *m, int32_t token_id, float *logits_host) {
    if (!m) return fail(MG_ERR_INVALID, "null model");
    NCU(cudaSetDevice(m->dev));
    return run_token(m, token_id, logits_host != nullptr, logits_host);
}

extern "C" mg_status mg_nano_prefill(mg_nano *m, const int32_t *ids, int32_t n) {
    if (!m || (!ids && n > 0)) return fail(MG_ERR_INVALID, "null argument");
    NCU(cudaSetDevice(m->dev));
    if (m->pos + n > m->cap) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
    for (int32_t i = 0; i < n; ++i) {
        const mg_status st = run_token(m, ids[i], false, nullptr);
        if (st != MG_OK) return st;
    }
    return MG_OK;
}

extern "C" mg_status mg_nano_embed(mg_nano *m, const int32_t *ids, int32_t n, float *out_host) {
    if (!m || !ids || !out_host) return fail(MG_ERR_INVALID, "null argument");
    if (n <= 0) return fail(MG_ERR_INVALID, "inputs must contain at least one token");
    if (n > m->cap) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
    NCU(cudaSetDevice(m->dev));
    const int saved = m->pos;
    m->pos = 0;
    NCU(cudaMemsetAsync(m->emb_acc, 0, sizeof(float) * m->H, m->stream));
    for (int32_t t = 0; t < n; ++t) {
        mg_status st = run_token(m, ids[t], false, nullptr);
        if (st != MG_OK) {
            m->pos = saved;
            return st;
        }
        k_accumulate<<<grid_for(m->H), 256, 0, m->stream>>>(m->emb_acc, m->hidden, m->H);
    }
    std::vector<float> acc(static_cast<size_t>(m->H));
    NCU(cudaMemcpyAsync(acc.data(), m->emb_acc, sizeof(float) * m->H, cudaMemcpyDeviceToHost, m->stream));
    NCU(cudaStreamSynchronize(m->stream));
    const float scale = 1.0f / static_cast<float>(n);  // layers.mojo:1060-1063
    for (int i = 0; i < m->H; ++i) out_host[i] = acc[static_cast<size_t>(i)] * scale;
    m->pos = saved;
    return MG_OK;
}
