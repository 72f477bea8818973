// engine.cu -- host side of libmogemma_cuda: the C ABI declared in
// include/mogemma_b200.h (model creation, weight upload, decode launches,
// prefill, embeddings, sampling, inspection).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/mogemma_b200.h"
#include "common.cuh"
#include "decode.cuh"

namespace mg {
size_t decode_smem_bytes(int S, int xs_floats, int L);
template <typename WT>
size_t decode_static_smem();
template <typename WT>
cudaError_t decode_prepare(size_t dynamic_smem);
template <typename WT>
int decode_occupancy(size_t smem);
template <typename WT>
cudaError_t decode_launch(const DecodeParams &p, int grid, size_t smem, cudaStream_t stream, bool cooperative);
size_t sample_rows_smem();
cudaError_t sample_rows_launch(const float *logits, int64_t ld, int rows, int V, double temperature, int top_k,
                               double top_p, const double *uniforms, uint64_t seed, uint64_t offset, int32_t *out,
                               int32_t *tok, cudaStream_t stream);
cudaError_t convert_rows_launch(const void *src, int src_dtype, int64_t rows, int64_t cols, void *dst, int dst_dtype,
                                int64_t dst_ld, cudaStream_t stream);
cudaError_t synth_fill_launch(float *dst, int64_t rows, int64_t cols, int64_t row0, int64_t col0, int64_t full_cols,
                              uint64_t key, float std, cudaStream_t stream);
cudaError_t gemm_bf16_tc(const void *A, int64_t lda, const void *B, int64_t ldb, float *C, int64_t ldc, int M, int N,
                         int K, uint32_t *err, cudaStream_t stream, float *ws, size_t ws_floats);
cudaError_t pf_advance(int32_t *pos, int n, cudaStream_t s);
cudaError_t pf_embed(const void *E, int wdtype_bf16, int64_t ld, const int32_t *tok, int N, int H, float scale,
                     float *x, cudaStream_t s);
cudaError_t pf_resnorm(const float *base, const float *add, const float *w_add, const float *w_next, float *res,
                       __nv_bfloat16 *xn, int N, int H, int Kp, float inv_h, cudaStream_t s);
cudaError_t pf_qk_rope_kv(float *qkv, int qkv_ld, int N, int Hq, int Hkv, int hd, int hdp, const float *q_norm,
                          const float *k_norm, const float *cos_t, const float *sin_t, const int32_t *row,
                          const int32_t *pos, float *kc, float *vc, int64_t kv_row_stride, int64_t kv_head_stride,
                          float inv_hd, __nv_bfloat16 *qb, __nv_bfloat16 *kb, __nv_bfloat16 *vt, int64_t vt_ld,
                          cudaStream_t s);
bool attn_tc_supported(int hd);
cudaError_t attn_tc(const __nv_bfloat16 *qb, const __nv_bfloat16 *kb, const __nv_bfloat16 *vt, int64_t vt_ld, int N,
                    int Hq, int Hkv, int hd, const int4 *tiles, int ntiles, int window, int bidir, float scale,
                    __nv_bfloat16 *out, int64_t out_ld, uint32_t *err, cudaStream_t s);
cudaError_t pf_attention(const float *qkv, int qkv_ld, int N, int Hq, int Hkv, int hd, int hdp, const float *kc,
                         const float *vc, const int32_t *row, const int32_t *pos, const int32_t *last,
                         int64_t kv_row_stride, int64_t kv_head_stride, int window, int is_global, float scale,
                         __nv_bfloat16 *out, int out_ld, int max_ctx, float *ws, size_t ws_floats, cudaStream_t s);
cudaError_t pf_encoder_head(const float *x, int H, int N, const int32_t *start, const int32_t *len,
                            const float *final_norm, float inv_h, float *row_inv, const float *d0, int d0_out,
                            const float *d1, float *pool, float *mid, float *out, int B, cudaStream_t s);
cudaError_t pf_geglu(const float *gu, int I, int gu_ld, __nv_bfloat16 *act, int Ip, int N, int il, cudaStream_t s);
cudaError_t gemm_bf16_tc_geglu(const void *A, int64_t lda, const void *B, int64_t ldb, __nv_bfloat16 *act,
                               int64_t ld_act, int M, int N2, int K, uint32_t *err, cudaStream_t stream);
cudaError_t tile_rows_launch(const void *src, int src_dtype, int64_t rows, int64_t cols, int64_t row_off, void *dst,
                             int dst_dtype, int Kp, int rps, int mult, int kc, int nseg, int part,
                             cudaStream_t stream);
}  // namespace mg

using namespace mg;

// ---------------------------------------------------------------- errors
static thread_local std::string g_err;

static mg_status fail(mg_status st, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return st;
}

#define CU(call)                                                                                       \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess)                                                                         \
            return fail(e_ == cudaErrorMemoryAllocation ? MG_ERR_OOM : MG_ERR_CUDA, "%s failed: %s (%s:%d)", \
                        #call, cudaGetErrorString(e_), __FILE__, __LINE__);                            \
    } while (0)

#define TRY(expr)                      \
    do {                               \
        mg_status s_ = (expr);         \
        if (s_ != MG_OK) return s_;    \
    } while (0)

extern "C" const char *mg_last_error(void) { return g_err.c_str(); }
extern "C" int32_t mg_abi_version(void) { return MG_ABI_VERSION; }

// Error reporting for entry points defined in other translation units.
namespace mg {
mg_status report_error(mg_status st, const char *msg) { return fail(st, "%s", msg); }
}  // namespace mg

// ---------------------------------------------------------------- model
struct mg_model {
    int dev = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    int mode = 0, wdtype = MG_F32, decode_path = 0;
    int L = 0, H = 0, Hq = 0, Hkv = 0, hd = 0, I = 0, V = 0, cap = 8192, Bmax = 1;
    int Hp = 0, Ap = 0, Ip = 0, hdp = 0, qkv_rows = 0, A = 0;
    int window = 0, global_every = 1;
    float theta_l = 10000.f, theta_g = 10000.f;
    uint64_t seed = 0, rng_offset = 0;
    int num_sms = 0, G = 0, S = 0, xs_floats = 0, max_ch = 0;
    size_t smem = 0;
    int64_t weight_bytes = 0;

    std::vector<void *> allocs;
    std::vector<LayerPtrs> h_layers;
    LayerPtrs *d_layers = nullptr;
    void *lm_head = nullptr, *embed = nullptr;
    int64_t embed_ld = 0;
    float *final_norm = nullptr;
    float *cos_l = nullptr, *sin_l = nullptr, *cos_g = nullptr, *sin_g = nullptr;
    float *kc = nullptr, *vc = nullptr;
    int64_t kv_layer_stride = 0, kv_row_stride = 0, kv_head_stride = 0;
    // decode activations as tagged words (value + tag of the forward and layer that wrote them)
    uint64_t *h = nullptr, *r = nullptr, *qkv = nullptr, *o_raw = nullptr, *mlp_raw = nullptr;
    uint64_t *split_tag = nullptr;  // exchange words of split row groups [kSplitKinds][G] (tagged block)
    float *split_part = nullptr;    // their partial row sums [kSplitKinds][G][2][kSplitVals]
    bool gemv_split = true;         // MOGEMMA_B200_SPLIT=0: whole row groups per CTA only
    int split_mask = 0;             // phase kinds (bit PH_*) whose row groups are split (split_kinds)
    size_t tagged_words = 0;   // h .. mlp_raw, allocated as one block
    float *act = nullptr, *attn_part = nullptr;
    uint32_t epoch = 0;        // forwards run so far (tags of the next one use epoch + 1)
    float *logits = nullptr, *emb_acc = nullptr;
    uint64_t *cand_key = nullptr;
    int32_t *tok = nullptr, *pos = nullptr, *ids = nullptr, *nvalid = nullptr, *out_tokens = nullptr;
    int64_t ids_cap = 0, out_cap = 0;
    double *uniforms = nullptr;
    uint32_t *sync = nullptr, *err = nullptr;
    size_t sync_words = 0;
    std::vector<int32_t> h_pos;
    int32_t *pinned = nullptr;  // pinned staging for small transfers
    uint64_t *trace = nullptr;  // decode timeline (mg_trace_enable)
    bool trace_on = false;
    uint64_t wait_ns = 0;       // decode-kernel wait budget (0: the default 2 s); mg_set_debug
    int stall_phase = -1;       // test hook: phase whose outputs one CTA withholds; mg_set_debug
    bool no_att_split = false;  // MOGEMMA_B200_ATT_SPLIT=0: attention items per kv head group always
    int max_inflight = 2;       // outstanding bulk copies per CTA (MOGEMMA_B200_INFLIGHT)
    int pf_tiles = 0;           // L2 prefetch distance in tiles (MOGEMMA_B200_PREFETCH)
    int att_chunks = kMaxChunks;  // most split-KV chunks per (row, attention unit) (MOGEMMA_B200_ATT_CHUNKS)

    // tensor parallelism: Hq, Hkv, A, I, V above are this rank's shard; *_g the model's
    int tp = 1, tp_rank = 0;
    int Hq_g = 0, Hkv_g = 0, I_g = 0, V_g = 0, v0 = 0;
    char *xbuf = nullptr;                  // exchange buffer (IPC-shared with the other ranks)
    size_t x_cnt = 0, x_o = 0, x_d = 0, x_cand = 0, x_logits = 0;
    char *xpeer[kMaxTp] = {};              // every rank's exchange buffer (own at tp_rank)
    std::vector<void *> ipc_open;          // peer mappings to close
    bool tp_connected = false;
    uint64_t x_ep = 0, lm_ep = 0;          // exchanges of earlier forwards (same on every rank)
    float *logits_full = nullptr;          // [Bmax][V_g] gathered logits (tp > 1)

    // batched prefill (prefill_path 1): bf16 row-major projection weights for
    // the tensor-core GEMMs and a workspace for pf_cap packed tokens
    int prefill_path = 0;
    struct PfLayer {
        __nv_bfloat16 *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
    };
    std::vector<PfLayer> pf;
    bool gu_il = false;               // PfLayer::gu rows in alternating 128-row gate / up blocks
    __nv_bfloat16 *pf_act = nullptr;  // [cap][Ip] GeGLU output of the fused gate/up GEMM
    int pf_cap = 0, pf_kx = 0, pf_cx = 0;
    float *pf_x = nullptr, *pf_r = nullptr, *pf_c = nullptr;
    __nv_bfloat16 *pf_xn = nullptr;
    int32_t *pf_tok = nullptr, *pf_row = nullptr, *pf_pos = nullptr;
    __nv_bfloat16 *pf_lm = nullptr;  // bf16 lm_head [V][Hp] for batched decode steps
    int32_t *pf_last = nullptr;      // encoder: last key position of each packed token
    // tensor-core attention operands (bf16): Q [N][Hq*hd], K [N][Hkv*hd], V^T [Hkv*hd][pf_vt_ld]
    __nv_bfloat16 *pf_qb = nullptr, *pf_kb = nullptr, *pf_vt = nullptr;
    int64_t pf_vt_ld = 0;
    float *pf_ws = nullptr;     // split-K partial products of small GEMM grids
    size_t pf_ws_floats = 0;
    int32_t *row_ident = nullptr;  // [nrows] = 0, 1, ...: the rows of a batched decode step
    int4 *att_tiles = nullptr;  // {start, len, q0, 0} per 128-query tile
    int att_tiles_cap = 0;
    // encoder head (embed_head.dense0 [d][H], embed_head.dense1 [H][d]; optional)
    float *d0 = nullptr, *d1 = nullptr;
    int d0_out = 0;
    float *enc_pool = nullptr, *enc_mid = nullptr, *enc_out = nullptr;
    int32_t *enc_start = nullptr, *enc_len = nullptr;

    // rows: Bmax in the KV cache; Bdec the most the persistent decode kernel
    // stages (shared memory); steps with more rows take the batched path
    int Bdec = 1, nrows = kMaxRows;
    // per launch row count b (1..Bdec): its activation stage, ring stages and
    // dynamic shared memory -- fewer rows leave room for a deeper ring
    int S_rows[kMaxRows + 1] = {}, xs_rows[kMaxRows + 1] = {};
    size_t smem_rows[kMaxRows + 1] = {};
};

static int split_kinds(const mg_model *m);

template <typename T>
static mg_status dalloc(mg_model *m, T **p, size_t count, bool zero = true) {
    void *v = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess)
        return fail(e == cudaErrorMemoryAllocation ? MG_ERR_OOM : MG_ERR_CUDA, "cudaMalloc(%zu bytes) failed: %s",
                    bytes, cudaGetErrorString(e));
    m->allocs.push_back(v);
    if (zero) {
        e = cudaMemsetAsync(v, 0, bytes, m->stream);
        if (e != cudaSuccess) return fail(MG_ERR_CUDA, "cudaMemset failed: %s", cudaGetErrorString(e));
    }
    *p = static_cast<T *>(v);
    return MG_OK;
}

static int64_t pad128(int64_t x) { return (x + 127) / 128 * 128; }
static size_t dsize(int dt) { return dt == MG_BF16 || dt == MG_F16 ? 2 : 4; }

// RoPE tables, same float32 formula as the reference (core.mojo:340-348), laid
// out [position][head_dim / 2].
static void rope_table(std::vector<float> &c, std::vector<float> &s, int cap, int hd, float base) {
    const int half = hd / 2;
    c.assign(static_cast<size_t>(cap) * half, 0.f);
    s.assign(static_cast<size_t>(cap) * half, 0.f);
    for (int t = 0; t < cap; ++t)
        for (int d = 0; d < half; ++d) {
            const float e = static_cast<float>(d * 2) / static_cast<float>(hd);
            const float inv_freq = 1.0f / powf(base, e);
            const float freq = static_cast<float>(t) * inv_freq;
            c[static_cast<size_t>(t) * half + d] = cosf(freq);
            s[static_cast<size_t>(t) * half + d] = sinf(freq);
        }
}

struct Desc {
    const void *data = nullptr;
    std::vector<int64_t> shape;
    int dtype = MG_F32;
    int64_t ld = 0;  // host row stride in elements (0: the tensor's own width)
    // device-generated tensor (data == nullptr, mg_options.synthetic_std > 0):
    // generator key, std, and the view's first row / column in the full tensor
    bool synthetic = false;
    uint64_t key = 0;
    float std = 0.f;
    int64_t row0 = 0, col0 = 0;
};

// Rows [row0, ...) of a [rows, cols] tensor, and columns [col0, ...) (a strided
// view: rows keep the tensor's stride).  A tensor-parallel rank uploads its
// shard through these.
static Desc rows_view(const Desc &d, int64_t row0) {
    Desc v = d;
    if (d.synthetic) {
        v.row0 += row0;
        return v;
    }
    const int64_t w = d.ld ? d.ld : (d.shape.size() > 1 ? d.shape[1] : 1);
    v.data = static_cast<const char *>(d.data) + row0 * w * static_cast<int64_t>(dsize(d.dtype));
    return v;
}
static Desc cols_view(const Desc &d, int64_t col0) {
    Desc v = d;
    v.ld = d.ld ? d.ld : d.shape[1];
    if (d.synthetic) {
        v.col0 += col0;
        return v;
    }
    v.data = static_cast<const char *>(d.data) + col0 * static_cast<int64_t>(dsize(d.dtype));
    return v;
}

// Host rows [r0, r0 + nr) of d (width cols) into contiguous staging memory
// (generated there for a synthetic tensor).
static cudaError_t stage_rows(mg_model *m, const Desc &d, int64_t r0, int64_t nr, int64_t cols, void *staging) {
    if (d.synthetic) {
        const int64_t full = d.shape.size() > 1 ? d.shape[1] : (d.shape.empty() ? 1 : d.shape[0]);
        return synth_fill_launch(static_cast<float *>(staging), nr, cols, d.row0 + r0, d.col0, full, d.key, d.std,
                                 m->stream);
    }
    const size_t es = dsize(d.dtype);
    const int64_t w = d.ld ? d.ld : cols;
    const char *src = static_cast<const char *>(d.data) + r0 * w * static_cast<int64_t>(es);
    if (w == cols) return cudaMemcpyAsync(staging, src, nr * cols * es, cudaMemcpyHostToDevice, m->stream);
    return cudaMemcpy2DAsync(staging, cols * es, src, w * es, cols * es, nr, cudaMemcpyHostToDevice, m->stream);
}

static const Desc *find(const std::map<std::string, Desc> &d, const std::string &name) {
    auto it = d.find(name);
    return it == d.end() ? nullptr : &it->second;
}

// Upload a [rows, cols] host tensor into dst (device, row stride dst_ld,
// element type m->wdtype or f32), converting and zero-padding columns.
static mg_status upload_matrix(mg_model *m, const Desc &d, int64_t rows, int64_t cols, void *dst, int dst_dtype,
                               int64_t dst_ld, void *staging, size_t staging_bytes) {
    if (d.dtype != MG_F32 && d.dtype != MG_BF16)
        return fail(MG_ERR_INVALID, "unsupported weight dtype %d (expected F32 or BF16)", d.dtype);
    const size_t row_bytes = static_cast<size_t>(cols) * dsize(d.dtype);
    const int64_t rows_per = std::max<int64_t>(1, static_cast<int64_t>(staging_bytes / std::max<size_t>(row_bytes, 1)));
    for (int64_t r0 = 0; r0 < rows; r0 += rows_per) {
        const int64_t nr = std::min(rows_per, rows - r0);
        CU(stage_rows(m, d, r0, nr, cols, staging));
        CU(convert_rows_launch(staging, d.dtype, nr, cols, static_cast<char *>(dst) + r0 * dst_ld * dsize(dst_dtype),
                               dst_dtype, dst_ld, m->stream));
    }
    return MG_OK;
}

// Upload rows [0, rows) of a [rows, cols] host tensor as rows
// [row_off, row_off + rows) of a tiled device matrix (see tile_shape); `part`
// selects the gate (0) or up (1) block of gate/up tiles.
static mg_status upload_tiled(mg_model *m, const Desc &d, int64_t rows, int64_t cols, int64_t row_off, void *dst,
                              int dst_dtype, int Kp, const TileShape &sh, int part, void *staging,
                              size_t staging_bytes) {
    if (d.dtype != MG_F32 && d.dtype != MG_BF16)
        return fail(MG_ERR_INVALID, "unsupported weight dtype %d (expected F32 or BF16)", d.dtype);
    const size_t row_bytes = static_cast<size_t>(cols) * dsize(d.dtype);
    const int64_t rows_per = std::max<int64_t>(1, static_cast<int64_t>(staging_bytes / std::max<size_t>(row_bytes, 1)));
    for (int64_t r0 = 0; r0 < rows; r0 += rows_per) {
        const int64_t nr = std::min(rows_per, rows - r0);
        CU(stage_rows(m, d, r0, nr, cols, staging));
        CU(tile_rows_launch(staging, d.dtype, nr, cols, row_off + r0, dst, dst_dtype, Kp, sh.rps, sh.mult, sh.kc,
                            sh.nseg, part, m->stream));
    }
    return MG_OK;
}

static mg_status destroy_impl(mg_model *m) {
    if (!m) return MG_OK;
    cudaSetDevice(m->dev);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (void *p : m->ipc_open) cudaIpcCloseMemHandle(p);
    for (void *p : m->allocs) cudaFree(p);
    if (m->pinned) cudaFreeHost(m->pinned);
    if (m->own_stream && m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return MG_OK;
}

extern "C" mg_status mg_model_destroy(mg_model *m) { return destroy_impl(m); }
extern "C" void *mg_model_stream(const mg_model *m) { return m ? static_cast<void *>(m->stream) : nullptr; }

static mg_status create_impl(const mg_tensor_desc *descs, int32_t n, const mg_options *opt, mg_model *m) {
    std::map<std::string, Desc> d;
    const bool has_syn = opt && opt->struct_size >= static_cast<int32_t>(offsetof(mg_options, synthetic_seed) +
                                                                         sizeof(uint64_t));
    const float syn_std = has_syn ? opt->synthetic_std : 0.f;
    for (int i = 0; i < n; ++i) {
        if (!descs[i].name) return fail(MG_ERR_INVALID, "tensor %d has no name", i);
        Desc x;
        x.data = descs[i].data;
        x.dtype = descs[i].dtype;
        for (int k = 0; k < descs[i].ndim && k < 4; ++k) x.shape.push_back(descs[i].shape[k]);
        if (!x.data) {
            if (!(syn_std > 0.f))
                return fail(MG_ERR_INVALID, "tensor '%s' has no data (synthetic weights need synthetic_std > 0)",
                            descs[i].name);
            std::string keyname = descs[i].name;
            if (keyname == "lm_head.weight") keyname = "model.embed_tokens.weight";  // tied
            uint64_t h = 1469598103934665603ull ^ opt->synthetic_seed;  // FNV-1a of the name
            for (char ch : keyname) h = (h ^ static_cast<unsigned char>(ch)) * 1099511628211ull;
            x.synthetic = true;
            x.key = h;
            x.std = syn_std;
            x.dtype = MG_F32;  // generated as F32 in the staging buffer
        }
        d[descs[i].name] = x;
    }
    m->dev = opt ? opt->device : 0;
    CU(cudaSetDevice(m->dev));
    if (opt && opt->stream) {
        m->stream = static_cast<cudaStream_t>(opt->stream);
    } else {
        CU(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
        m->own_stream = true;
    }
    m->mode = opt ? opt->mode : 0;
    m->wdtype = opt ? opt->weight_dtype : MG_F32;
    if (m->wdtype != MG_F32 && m->wdtype != MG_BF16) return fail(MG_ERR_INVALID, "weight_dtype must be F32 or BF16");
    m->Bmax = opt && opt->max_batch > 0 ? opt->max_batch : 1;
    if (m->Bmax > kMaxBatch) return fail(MG_ERR_UNSUPPORTED, "max_batch %d exceeds %d", m->Bmax, kMaxBatch);
    m->nrows = std::max(m->Bmax, kMaxRows);
    m->cap = opt && opt->capacity > 0 ? opt->capacity : 8192;
    m->seed = opt ? opt->seed : 0;
    m->decode_path = opt ? opt->decode_path : 0;
    m->prefill_path = opt ? opt->prefill_path : 0;
    if (const char *e = getenv("MOGEMMA_B200_PREFILL")) m->prefill_path = atoi(e);
    m->tp = opt && opt->tp_size > 1 ? opt->tp_size : 1;
    m->tp_rank = m->tp > 1 ? opt->tp_rank : 0;
    if (m->tp > kMaxTp || m->tp_rank < 0 || m->tp_rank >= m->tp)
        return fail(MG_ERR_INVALID, "tensor-parallel rank %d of %d outside [0, tp) or tp > %d", m->tp_rank, m->tp,
                    kMaxTp);

    // ---- dimensions (init_model_mojo, core.mojo:316-325)
    const Desc *emb = find(d, "model.embed_tokens.weight");
    const Desc *fnorm = find(d, "model.norm.weight");
    const Desc *lmh = find(d, "lm_head.weight");
    if (!emb || !fnorm || !lmh) return fail(MG_ERR_INVALID, "missing embed_tokens, norm or lm_head weights");
    int L = 0;
    while (find(d, "model.layers." + std::to_string(L) + ".input_layernorm.weight")) ++L;
    if (L == 0) return fail(MG_ERR_INVALID, "Invalid standard model weights: no layers found in metadata");
    if (L > kMaxLayers) return fail(MG_ERR_UNSUPPORTED, "%d layers (at most %d)", L, kMaxLayers);
    auto lw = [&](int l, const char *k) { return find(d, "model.layers." + std::to_string(l) + "." + k); };
    const Desc *qn0 = lw(0, "self_attn.q_norm.weight");
    int hd = (qn0 && !qn0->shape.empty() && qn0->shape[0] > 0) ? static_cast<int>(qn0->shape[0]) : 256;
    const Desc *k0 = lw(0, "self_attn.k_proj.weight");
    const Desc *q0 = lw(0, "self_attn.q_proj.weight");
    const Desc *g0 = lw(0, "mlp.gate_proj.weight");
    if (!k0 || !q0 || !g0 || emb->shape.size() < 2 || lmh->shape.size() < 2)
        return fail(MG_ERR_INVALID, "missing or malformed projection weights in layer 0");
    m->L = L;
    m->hd = hd;
    m->Hkv = static_cast<int>(k0->shape[0] / hd);
    m->Hq = static_cast<int>(q0->shape[0] / hd);
    m->H = static_cast<int>(emb->shape[1]);
    m->I = static_cast<int>(g0->shape[0]);
    m->V = static_cast<int>(lmh->shape[0]);
    if (m->Hkv <= 0 || m->Hq <= 0 || m->Hq % m->Hkv != 0)
        return fail(MG_ERR_INVALID, "head counts Hq=%d Hkv=%d (head_dim %d) are inconsistent", m->Hq, m->Hkv, hd);
    if (hd > kMaxHeadDim || hd % 2 != 0) return fail(MG_ERR_UNSUPPORTED, "head_dim %d unsupported", hd);
    if (m->Hq / m->Hkv > kMaxQPerKv) return fail(MG_ERR_UNSUPPORTED, "more than %d q heads per kv head", kMaxQPerKv);
    m->A = m->Hq * hd;
    m->Hp = static_cast<int>(pad128(m->H));
    m->Ap = static_cast<int>(pad128(m->A));
    m->Ip = static_cast<int>(pad128(m->I));
    m->hdp = (hd + 7) / 8 * 8;
    m->qkv_rows = m->A + 2 * m->Hkv * hd;
    if (m->mode == 1) {
        m->window = opt && opt->sliding_window > 0 ? opt->sliding_window : 512;
        m->global_every = opt && opt->global_every > 0 ? opt->global_every : 6;
        m->theta_l = opt && opt->rope_theta_local > 0 ? opt->rope_theta_local : 10000.f;
        m->theta_g = opt && opt->rope_theta_global > 0 ? opt->rope_theta_global : 1000000.f;
    }
    // ---- shape checks
    auto need = [&](const Desc *x, int64_t r, int64_t c, const std::string &nm) -> mg_status {
        if (!x) return fail(MG_ERR_INVALID, "missing tensor %s", nm.c_str());
        const int64_t r0 = x->shape.size() > 0 ? x->shape[0] : 0;
        const int64_t c0 = x->shape.size() > 1 ? x->shape[1] : (c == 0 ? 0 : -1);
        if (r0 != r || (c != 0 && c0 != c))
            return fail(MG_ERR_INVALID, "tensor %s has shape (%lld, %lld), expected (%lld, %lld)", nm.c_str(),
                        (long long)r0, (long long)c0, (long long)r, (long long)c);
        if (!x->data && !x->synthetic) return fail(MG_ERR_INVALID, "tensor %s has a null data pointer", nm.c_str());
        return MG_OK;
    };
    TRY(need(emb, m->V, m->H, "model.embed_tokens.weight"));
    TRY(need(lmh, m->V, m->H, "lm_head.weight"));
    TRY(need(fnorm, m->H, 0, "model.norm.weight"));
    for (int l = 0; l < L; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        TRY(need(lw(l, "self_attn.q_proj.weight"), m->A, m->H, p + "self_attn.q_proj.weight"));
        TRY(need(lw(l, "self_attn.k_proj.weight"), m->Hkv * hd, m->H, p + "self_attn.k_proj.weight"));
        TRY(need(lw(l, "self_attn.v_proj.weight"), m->Hkv * hd, m->H, p + "self_attn.v_proj.weight"));
        TRY(need(lw(l, "self_attn.o_proj.weight"), m->H, m->A, p + "self_attn.o_proj.weight"));
        TRY(need(lw(l, "mlp.gate_proj.weight"), m->I, m->H, p + "mlp.gate_proj.weight"));
        TRY(need(lw(l, "mlp.up_proj.weight"), m->I, m->H, p + "mlp.up_proj.weight"));
        TRY(need(lw(l, "mlp.down_proj.weight"), m->H, m->I, p + "mlp.down_proj.weight"));
        for (const char *k : {"input_layernorm.weight", "post_attention_layernorm.weight",
                              "pre_feedforward_layernorm.weight", "post_feedforward_layernorm.weight"})
            TRY(need(lw(l, k), m->H, 0, p + k));
        const Desc *qn = lw(l, "self_attn.q_norm.weight"), *kn = lw(l, "self_attn.k_norm.weight");
        if (qn) TRY(need(qn, hd, 0, p + "self_attn.q_norm.weight"));
        if (kn) TRY(need(kn, hd, 0, p + "self_attn.k_norm.weight"));
    }

    // ---- tensor-parallel shard: q heads, the kv heads they use, FFN rows and
    // vocabulary rows of this rank; o_proj and down_proj are split along their
    // input (columns) so their outputs are partial sums exchanged in the kernel
    m->Hq_g = m->Hq;
    m->Hkv_g = m->Hkv;
    m->I_g = m->I;
    m->V_g = m->V;
    int qh0 = 0, kvh0 = 0, i0 = 0;
    if (m->tp > 1) {
        const int T = m->tp, r = m->tp_rank, Gq_g = m->Hq / m->Hkv;
        if (m->Hq % T != 0 || m->I % T != 0 || m->V % T != 0)
            return fail(MG_ERR_UNSUPPORTED, "tp=%d must divide the q heads (%d), intermediate size (%d) and vocabulary (%d)",
                        T, m->Hq, m->I, m->V);
        const int hq_r = m->Hq / T;
        qh0 = r * hq_r;
        if (m->Hkv % T == 0) {
            m->Hkv = m->Hkv / T;
            kvh0 = r * m->Hkv;
        } else if (Gq_g % hq_r == 0) {  // fewer kv heads than ranks: each rank keeps the one its q heads use
            m->Hkv = 1;
            kvh0 = qh0 / Gq_g;
        } else {
            return fail(MG_ERR_UNSUPPORTED, "tp=%d does not split %d q heads over %d kv heads", T, m->Hq, m->Hkv_g);
        }
        m->Hq = hq_r;
        m->I = m->I / T;
        i0 = r * m->I;
        m->V = m->V / T;
        m->v0 = r * m->V;
        m->A = m->Hq * hd;
        m->Ap = static_cast<int>(pad128(m->A));
        m->Ip = static_cast<int>(pad128(m->I));
        m->qkv_rows = m->A + 2 * m->Hkv * hd;
    }

    // ---- launch geometry
    CU(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, m->dev));
    int max_smem = 0;
    CU(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->dev));
    const int Kmax = std::max(m->Hp, std::max(m->Ap, m->Ip));
    const int Gq = m->Hq / m->Hkv;
    // shared activation stage for Bd rows: GEMV inputs; o_proj input +
    // split-KV weights; attention scratch; top-k selection scratch.  The
    // persistent kernel takes the most rows (<= kMaxRows) whose stage leaves at
    // least two ring stages; steps with more rows take the batched path.
    const size_t static_smem =
        (m->wdtype == MG_F32 ? decode_static_smem<float>() : decode_static_smem<__nv_bfloat16>()) + 64;
    auto stage_floats = [&](int Bd) {
        int xs = Bd * Kmax;
        xs = std::max(xs, Bd * (m->Hp + m->H));  // normed input + staged residual rows
        xs = std::max(xs, Bd * (m->Ap + m->Hq * kMaxChunks));
        // attention: q, k, v, scores of two tiles, m/l/alpha, q/k norm weights, RoPE rows,
        // then the P.V reduction block (1024 * Gq floats in the two-tile pass)
        xs = std::max(xs, (Gq + 2) * hd + Gq * 2 * kAttTile + 3 * kMaxQPerKv + 2 * hd + Bd * hd +
                              std::max(kConsumerThreads, 1024) * Gq + 8);
        // selection and draw: SelectSmem, K keys, two double and one int scratch of K, 4 ints
        xs = std::max(xs, static_cast<int>((sizeof(uint32_t) * 264 + sizeof(uint64_t) * 1024 + kMaxTopK * 8 * 3 +
                                            kMaxTopK * 4 + 16) / 4 + 16));
        return (xs + 31) / 32 * 32;
    };
    m->S = 0;
    for (int Bd = std::min(m->Bmax, kMaxRows); Bd >= 1 && m->S == 0; --Bd) {
        m->xs_floats = stage_floats(Bd);
        for (int S = 8; S >= 2; --S)
            if (decode_smem_bytes(S, m->xs_floats, L) + static_smem <= static_cast<size_t>(max_smem)) {
                m->S = S;
                m->Bdec = Bd;
                break;
            }
    }
    if (m->S < 2)
        return fail(MG_ERR_UNSUPPORTED, "activation stage of %d floats leaves no room for the weight ring",
                    m->xs_floats);
    if (m->Bmax > m->Bdec && m->tp > 1)
        return fail(MG_ERR_UNSUPPORTED,
                    "max_batch %d: the persistent decode kernel holds %d rows of this model, and tensor-parallel "
                    "models run one launch of rows",
                    m->Bmax, m->Bdec);
    m->smem = decode_smem_bytes(m->S, m->xs_floats, L);
    for (int b = 1; b <= m->Bdec; ++b) {
        m->xs_rows[b] = stage_floats(b);
        m->S_rows[b] = m->S;
        m->smem_rows[b] = m->smem;
        for (int S = 8; S > m->S; --S)
            if (decode_smem_bytes(S, m->xs_rows[b], L) + static_smem <= static_cast<size_t>(max_smem)) {
                m->S_rows[b] = S;
                break;
            }
        if (m->S_rows[b] == m->S) m->xs_rows[b] = m->xs_floats;  // the full-width layout
        m->smem_rows[b] = decode_smem_bytes(m->S_rows[b], m->xs_rows[b], L);
        m->smem = std::max(m->smem, m->smem_rows[b]);  // the kernel's allowance covers every launch
    }
    if (m->wdtype == MG_F32) {
        CU(decode_prepare<float>(m->smem));
    } else {
        CU(decode_prepare<__nv_bfloat16>(m->smem));
    }
    const int occ = m->wdtype == MG_F32 ? decode_occupancy<float>(m->smem) : decode_occupancy<__nv_bfloat16>(m->smem);
    if (occ < 1) return fail(MG_ERR_UNSUPPORTED, "decode kernel does not fit on an SM (smem %zu)", m->smem);
    m->G = m->num_sms;  // one persistent CTA per SM
    if (const char *e = getenv("MOGEMMA_B200_INFLIGHT")) m->max_inflight = std::max(1, atoi(e));
    if (const char *e = getenv("MOGEMMA_B200_PREFETCH")) m->pf_tiles = std::max(0, atoi(e));
    if (const char *e = getenv("MOGEMMA_B200_ATT_SPLIT")) m->no_att_split = atoi(e) == 0;
    if (const char *e = getenv("MOGEMMA_B200_ATT_CHUNKS")) m->att_chunks = std::min(kMaxChunks, std::max(1, atoi(e)));
    if (const char *e = getenv("MOGEMMA_B200_SPLIT")) m->gemv_split = atoi(e) != 0;
    m->split_mask = split_kinds(m);
    m->max_ch = kMaxChunks;

    // ---- weights
    const int wd = m->wdtype;
    const size_t we = dsize(wd);
    const size_t staging_bytes = 64ull << 20;
    void *staging = nullptr;
    TRY(dalloc(m, reinterpret_cast<char **>(&staging), staging_bytes, false));
    m->h_layers.resize(L);
    m->weight_bytes = 0;
    const TileShape sh_h = tile_shape(m->Hp, static_cast<int>(we), false);   // q/k/v, lm_head
    const TileShape sh_a = tile_shape(m->Ap, static_cast<int>(we), false);   // o_proj
    const TileShape sh_gu = tile_shape(m->Hp, static_cast<int>(we), true);   // gate + up
    const TileShape sh_i = tile_shape(m->Ip, static_cast<int>(we), false);   // down_proj
    for (int l = 0; l < L; ++l) {
        LayerPtrs &lp = m->h_layers[l];
        void *qkv, *o, *gu, *down;
        TRY(dalloc(m, reinterpret_cast<char **>(&qkv), static_cast<size_t>(tiled_elems(sh_h, m->qkv_rows)) * we));
        TRY(dalloc(m, reinterpret_cast<char **>(&o), static_cast<size_t>(tiled_elems(sh_a, m->H)) * we));
        TRY(dalloc(m, reinterpret_cast<char **>(&gu), static_cast<size_t>(tiled_elems(sh_gu, m->I)) * we));
        TRY(dalloc(m, reinterpret_cast<char **>(&down), static_cast<size_t>(tiled_elems(sh_i, m->H)) * we));
        const int64_t kvr = static_cast<int64_t>(m->Hkv) * hd;
        TRY(upload_tiled(m, rows_view(*lw(l, "self_attn.q_proj.weight"), static_cast<int64_t>(qh0) * hd), m->A,
                         m->H, 0, qkv, wd, m->Hp, sh_h, 0, staging, staging_bytes));
        TRY(upload_tiled(m, rows_view(*lw(l, "self_attn.k_proj.weight"), static_cast<int64_t>(kvh0) * hd), kvr,
                         m->H, m->A, qkv, wd, m->Hp, sh_h, 0, staging, staging_bytes));
        TRY(upload_tiled(m, rows_view(*lw(l, "self_attn.v_proj.weight"), static_cast<int64_t>(kvh0) * hd), kvr,
                         m->H, m->A + kvr, qkv, wd, m->Hp, sh_h, 0, staging, staging_bytes));
        TRY(upload_tiled(m, cols_view(*lw(l, "self_attn.o_proj.weight"), static_cast<int64_t>(qh0) * hd), m->H,
                         m->A, 0, o, wd, m->Ap, sh_a, 0, staging, staging_bytes));
        TRY(upload_tiled(m, rows_view(*lw(l, "mlp.gate_proj.weight"), i0), m->I, m->H, 0, gu, wd, m->Hp, sh_gu, 0,
                         staging, staging_bytes));
        TRY(upload_tiled(m, rows_view(*lw(l, "mlp.up_proj.weight"), i0), m->I, m->H, 0, gu, wd, m->Hp, sh_gu, 1,
                         staging, staging_bytes));
        TRY(upload_tiled(m, cols_view(*lw(l, "mlp.down_proj.weight"), i0), m->H, m->I, 0, down, wd, m->Ip, sh_i, 0,
                         staging, staging_bytes));
        void *gate = gu, *up = nullptr;
        m->weight_bytes += static_cast<int64_t>(we) * (static_cast<int64_t>(m->qkv_rows) * m->H +
                                                        static_cast<int64_t>(m->H) * m->A +
                                                        3 * static_cast<int64_t>(m->I) * m->H);
        float *norms[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
        const char *nn[4] = {"input_layernorm.weight", "post_attention_layernorm.weight",
                             "pre_feedforward_layernorm.weight", "post_feedforward_layernorm.weight"};
        for (int k = 0; k < 4; ++k) {
            TRY(dalloc(m, &norms[k], m->H));
            TRY(upload_matrix(m, *lw(l, nn[k]), 1, m->H, norms[k], MG_F32, m->H, staging, staging_bytes));
        }
        const Desc *qn = lw(l, "self_attn.q_norm.weight"), *kn = lw(l, "self_attn.k_norm.weight");
        if (qn) {
            TRY(dalloc(m, &norms[4], hd));
            TRY(upload_matrix(m, *qn, 1, hd, norms[4], MG_F32, hd, staging, staging_bytes));
        }
        if (kn) {
            TRY(dalloc(m, &norms[5], hd));
            TRY(upload_matrix(m, *kn, 1, hd, norms[5], MG_F32, hd, staging, staging_bytes));
        }
        lp.qkv = qkv;
        lp.o = o;
        lp.gate = gate;
        lp.up = up;
        lp.down = down;
        lp.in_ln = norms[0];
        lp.post_attn_ln = norms[1];
        lp.pre_ff_ln = norms[2];
        lp.post_ff_ln = norms[3];
        lp.q_norm = norms[4];
        lp.k_norm = norms[5];
        lp.is_global = (m->mode == 0) ? 1 : (((l + 1) % m->global_every) == 0 ? 1 : 0);
        if (m->prefill_path == 1 && m->tp == 1) {  // row-major bf16 copies for the prefill GEMMs
            mg_model::PfLayer pl;
            TRY(dalloc(m, &pl.qkv, static_cast<size_t>(m->qkv_rows) * m->Hp));
            TRY(dalloc(m, &pl.o, static_cast<size_t>(m->H) * m->Ap));
            TRY(dalloc(m, &pl.gu, static_cast<size_t>(2) * m->I * m->Hp));
            TRY(dalloc(m, &pl.down, static_cast<size_t>(m->H) * m->Ip));
            TRY(upload_matrix(m, *lw(l, "self_attn.q_proj.weight"), m->A, m->H, pl.qkv, MG_BF16, m->Hp, staging,
                              staging_bytes));
            TRY(upload_matrix(m, *lw(l, "self_attn.k_proj.weight"), kvr, m->H, pl.qkv + static_cast<size_t>(m->A) * m->Hp,
                              MG_BF16, m->Hp, staging, staging_bytes));
            TRY(upload_matrix(m, *lw(l, "self_attn.v_proj.weight"), kvr, m->H,
                              pl.qkv + static_cast<size_t>(m->A + kvr) * m->Hp, MG_BF16, m->Hp, staging, staging_bytes));
            TRY(upload_matrix(m, *lw(l, "self_attn.o_proj.weight"), m->H, m->A, pl.o, MG_BF16, m->Ap, staging,
                              staging_bytes));
            m->gu_il = m->I % 128 == 0;
            if (m->gu_il) {  // 128 gate rows, then the same features' 128 up rows, ...
                for (int64_t f0 = 0; f0 < m->I; f0 += 128) {
                    TRY(upload_matrix(m, rows_view(*lw(l, "mlp.gate_proj.weight"), f0), 128, m->H,
                                      pl.gu + static_cast<size_t>(2 * f0) * m->Hp, MG_BF16, m->Hp, staging,
                                      staging_bytes));
                    TRY(upload_matrix(m, rows_view(*lw(l, "mlp.up_proj.weight"), f0), 128, m->H,
                                      pl.gu + static_cast<size_t>(2 * f0 + 128) * m->Hp, MG_BF16, m->Hp, staging,
                                      staging_bytes));
                }
            } else {
                TRY(upload_matrix(m, *lw(l, "mlp.gate_proj.weight"), m->I, m->H, pl.gu, MG_BF16, m->Hp, staging,
                                  staging_bytes));
                TRY(upload_matrix(m, *lw(l, "mlp.up_proj.weight"), m->I, m->H,
                                  pl.gu + static_cast<size_t>(m->I) * m->Hp, MG_BF16, m->Hp, staging, staging_bytes));
            }
            TRY(upload_matrix(m, *lw(l, "mlp.down_proj.weight"), m->H, m->I, pl.down, MG_BF16, m->Ip, staging,
                              staging_bytes));
            m->pf.push_back(pl);
        }
    }
    TRY(dalloc(m, reinterpret_cast<char **>(&m->lm_head), static_cast<size_t>(tiled_elems(sh_h, m->V)) * we));
    TRY(upload_tiled(m, rows_view(*lmh, m->v0), m->V, m->H, 0, m->lm_head, wd, m->Hp, sh_h, 0, staging,
                     staging_bytes));
    m->weight_bytes += static_cast<int64_t>(we) * m->V * m->H;
    if (m->prefill_path == 1 && m->tp == 1) {  // split-K workspace (8 MB) and the row identity
        m->pf_ws_floats = static_cast<size_t>(2) << 20;
        TRY(dalloc(m, &m->pf_ws, m->pf_ws_floats));
        TRY(dalloc(m, &m->row_ident, m->nrows));
        std::vector<int32_t> ident(m->nrows);
        for (int b = 0; b < m->nrows; ++b) ident[b] = b;
        CU(cudaMemcpyAsync(m->row_ident, ident.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice, m->stream));
        CU(cudaStreamSynchronize(m->stream));
    }
    if (m->Bmax > m->Bdec && m->prefill_path == 1) {  // lm_head for batched tensor-core decode steps
        TRY(dalloc(m, &m->pf_lm, static_cast<size_t>(m->V) * m->Hp));
        TRY(upload_matrix(m, *lmh, m->V, m->H, m->pf_lm, MG_BF16, m->Hp, staging, staging_bytes));
    }
    // embedding rows are gathered, so they stay row-major (a separate copy even
    // when lm_head is tied to them, convert.py:129-131)
    TRY(dalloc(m, reinterpret_cast<char **>(&m->embed), static_cast<size_t>(m->V_g) * m->H * we));
    TRY(upload_matrix(m, *emb, m->V_g, m->H, m->embed, wd, m->H, staging, staging_bytes));
    m->embed_ld = m->H;
    {  // optional encoder head (this library's names for an EmbeddingGemma-style dense head)
        const Desc *d0 = find(d, "embed_head.dense0.weight"), *d1 = find(d, "embed_head.dense1.weight");
        if (d0 && d1 && d0->shape.size() == 2 && d1->shape.size() == 2 && d0->shape[1] == m->H &&
            d1->shape[0] == m->H && d1->shape[1] == d0->shape[0]) {
            m->d0_out = static_cast<int>(d0->shape[0]);
            TRY(dalloc(m, &m->d0, static_cast<size_t>(m->d0_out) * m->H));
            TRY(dalloc(m, &m->d1, static_cast<size_t>(m->d0_out) * m->H));
            TRY(upload_matrix(m, *d0, m->d0_out, m->H, m->d0, MG_F32, m->H, staging, staging_bytes));
            TRY(upload_matrix(m, *d1, m->H, m->d0_out, m->d1, MG_F32, m->d0_out, staging, staging_bytes));
        } else if (d0 || d1) {
            return fail(MG_ERR_INVALID, "embed_head.dense0/dense1 must be [d, hidden] and [hidden, d]");
        }
    }
    TRY(dalloc(m, &m->final_norm, m->H));
    TRY(upload_matrix(m, *fnorm, 1, m->H, m->final_norm, MG_F32, m->H, staging, staging_bytes));
    TRY(dalloc(m, &m->d_layers, L));
    CU(cudaMemcpyAsync(m->d_layers, m->h_layers.data(), sizeof(LayerPtrs) * L, cudaMemcpyHostToDevice, m->stream));

    // ---- RoPE tables
    {
        std::vector<float> c, s;
        const size_t n_tab = static_cast<size_t>(m->cap) * (hd / 2);
        TRY(dalloc(m, &m->cos_l, n_tab));
        TRY(dalloc(m, &m->sin_l, n_tab));
        if (m->mode != 0) {
            TRY(dalloc(m, &m->cos_g, n_tab));
            TRY(dalloc(m, &m->sin_g, n_tab));
        }
        // the clears above run on the model's stream, which does not order with these synchronous copies
        CU(cudaStreamSynchronize(m->stream));
        rope_table(c, s, m->cap, hd, m->mode == 0 ? 10000.f : m->theta_l);
        CU(cudaMemcpy(m->cos_l, c.data(), n_tab * 4, cudaMemcpyHostToDevice));
        CU(cudaMemcpy(m->sin_l, s.data(), n_tab * 4, cudaMemcpyHostToDevice));
        if (m->mode == 0) {
            m->cos_g = m->cos_l;
            m->sin_g = m->sin_l;
        } else {
            rope_table(c, s, m->cap, hd, m->theta_g);
            CU(cudaMemcpy(m->cos_g, c.data(), n_tab * 4, cudaMemcpyHostToDevice));
            CU(cudaMemcpy(m->sin_g, s.data(), n_tab * 4, cudaMemcpyHostToDevice));
        }
    }
    // ---- KV cache [L][Bmax][Hkv][cap][hdp]
    m->kv_head_stride = static_cast<int64_t>(m->cap) * m->hdp;
    m->kv_row_stride = m->kv_head_stride * m->Hkv;
    m->kv_layer_stride = m->kv_row_stride * m->Bmax;
    TRY(dalloc(m, &m->kc, static_cast<size_t>(m->kv_layer_stride) * L));
    TRY(dalloc(m, &m->vc, static_cast<size_t>(m->kv_layer_stride) * L));
    // ---- activations
    const int B = m->Bmax;
    {  // one zeroed block (tag 0 is never expected), each part 256-byte aligned
        const size_t sizes[6] = {static_cast<size_t>(B) * m->H, static_cast<size_t>(B) * m->H,
                                 static_cast<size_t>(B) * m->qkv_rows, static_cast<size_t>(B) * m->H,
                                 static_cast<size_t>(B) * m->H, static_cast<size_t>(kSplitKinds) * m->G};
        size_t total = 0;
        for (size_t n : sizes) total += (n + 31) / 32 * 32;
        uint64_t *blk = nullptr;
        TRY(dalloc(m, &blk, total));
        m->tagged_words = total;
        uint64_t **dst[6] = {&m->h, &m->r, &m->qkv, &m->o_raw, &m->mlp_raw, &m->split_tag};
        size_t off = 0;
        for (int k = 0; k < 6; ++k) {
            *dst[k] = blk + off;
            off += (sizes[k] + 31) / 32 * 32;
        }
    }
    TRY(dalloc(m, &m->act, static_cast<size_t>(B) * m->Ip));
    TRY(dalloc(m, &m->split_part, static_cast<size_t>(kSplitKinds) * m->G * 2 * kSplitVals));
    TRY(dalloc(m, &m->attn_part, static_cast<size_t>(B) * m->Hkv * m->max_ch * Gq * (hd + kPartHead)));
    if (m->tp > 1) {
        // exchange buffer: counters, o_proj / down_proj partials [tp][Bmax][H],
        // lm_head candidates [tp][Bmax][G][kMaxTopK], this rank's logits [Bmax][V]
        size_t off = 0;
        auto take = [&](size_t bytes) {
            const size_t o = off;
            off = (off + bytes + 255) / 256 * 256;
            return o;
        };
        const size_t T = static_cast<size_t>(m->tp);
        m->x_cnt = take(4 * sizeof(uint64_t));
        m->x_o = take(T * B * m->H * sizeof(float));
        m->x_d = take(T * B * m->H * sizeof(float));
        m->x_cand = take(T * B * m->G * kMaxTopK * sizeof(uint64_t));
        m->x_logits = take(static_cast<size_t>(B) * m->V * sizeof(float));
        TRY(dalloc(m, &m->xbuf, off));
        m->logits = reinterpret_cast<float *>(m->xbuf + m->x_logits);
        TRY(dalloc(m, &m->logits_full, static_cast<size_t>(B) * m->V_g));
    } else {
        TRY(dalloc(m, &m->logits, static_cast<size_t>(B) * m->V));
    }
    TRY(dalloc(m, &m->emb_acc, static_cast<size_t>(B) * m->H));
    TRY(dalloc(m, &m->cand_key, static_cast<size_t>(B) * m->G * kMaxTopK));
    TRY(dalloc(m, &m->tok, m->nrows));
    TRY(dalloc(m, &m->pos, m->nrows));
    TRY(dalloc(m, &m->uniforms, m->nrows));
    m->sync_words = num_phases(L) + 1;
    TRY(dalloc(m, &m->sync, m->sync_words));
    TRY(dalloc(m, &m->err, 1));
    CU(cudaMallocHost(&m->pinned, 4096));
    m->h_pos.assign(m->nrows, 0);
    CU(cudaStreamSynchronize(m->stream));
    cudaFree(staging);
    m->allocs.erase(std::find(m->allocs.begin(), m->allocs.end(), staging));
    return MG_OK;
}

extern "C" mg_status mg_model_create(const mg_tensor_desc *descs, int32_t n, const mg_options *opt, mg_model **out) {
    if (!out) return fail(MG_ERR_INVALID, "out is null");
    *out = nullptr;
    if (!descs || n <= 0) return fail(MG_ERR_INVALID, "no tensors given");
    mg_model *m = new mg_model();
    mg_status st = create_impl(descs, n, opt, m);
    if (st != MG_OK) {
        std::string keep = g_err;
        destroy_impl(m);
        g_err = keep;
        return st;
    }
    *out = m;
    return MG_OK;
}

extern "C" int32_t mg_rows_per_launch(const mg_model *m) { return m ? m->Bdec : 0; }

extern "C" mg_status mg_model_info_get(const mg_model *m, mg_model_info *info) {
    if (!m || !info) return fail(MG_ERR_INVALID, "null argument");
    info->num_layers = m->L;
    info->num_heads = m->Hq_g;
    info->num_kv_heads = m->Hkv_g;
    info->head_dim = m->hd;
    info->hidden_size = m->H;
    info->intermediate_size = m->I_g;
    info->vocab_size = m->V_g;
    info->max_seq_len = m->cap;
    info->max_batch = m->Bmax;
    info->mode = m->mode;
    info->weight_dtype = m->wdtype;
    info->tp_size = m->tp;
    info->weight_bytes_per_step = m->weight_bytes;
    info->kv_bytes_per_pos = static_cast<int64_t>(2) * m->L * m->Hkv * m->hd * 4;
    info->num_sms = m->num_sms;
    info->persistent_ctas = m->G;
    return MG_OK;
}

// ---------------------------------------------------------------- launches
static DecodeParams base_params(mg_model *m, int B) {
    DecodeParams p;
    memset(&p, 0, sizeof p);
    p.L = m->L;
    p.H = m->H;
    p.Hp = m->Hp;
    p.Hq = m->Hq;
    p.Hkv = m->Hkv;
    p.hd = m->hd;
    p.hdp = m->hdp;
    p.inv_h = 1.0f / static_cast<float>(m->H);
    p.inv_hd = 1.0f / static_cast<float>(m->hd);
    p.att_scale = 1.0f / sqrtf(static_cast<float>(m->hd));
    p.emb_scale = sqrtf(static_cast<float>(m->H));
    p.I = m->I;
    p.Ip = m->Ip;
    p.V = m->V;
    p.A = m->A;
    p.Ap = m->Ap;
    p.qkv_rows = m->qkv_rows;
    p.B = B;
    p.cap = m->cap;
    p.window = m->window;
    p.S = m->S;
    p.max_ch = m->max_ch;
    p.xs_floats = m->xs_floats;
    p.layers = m->d_layers;
    p.lm_head = m->lm_head;
    p.embed = m->embed;
    p.embed_ld = m->embed_ld;
    p.final_norm = m->final_norm;
    p.rope_cos_l = m->cos_l;
    p.rope_sin_l = m->sin_l;
    p.rope_cos_g = m->cos_g;
    p.rope_sin_g = m->sin_g;
    p.kc = m->kc;
    p.vc = m->vc;
    p.kv_layer_stride = m->kv_layer_stride;
    p.kv_row_stride = m->kv_row_stride;
    p.kv_head_stride = m->kv_head_stride;
    p.h = m->h;
    p.r = m->r;
    p.qkv = m->qkv;
    p.o_raw = m->o_raw;
    p.act = m->act;
    p.mlp_raw = m->mlp_raw;
    p.attn_part = m->attn_part;
    p.split_part = m->split_part;
    p.split_tag = m->split_tag;
    p.gemv_split = m->gemv_split ? m->split_mask : 0;
    p.logits = m->logits;
    p.cand_key = m->cand_key;
    p.emb_acc = m->emb_acc;
    p.tok = m->tok;
    p.pos = m->pos;
    p.seed = m->seed;
    p.sync = m->sync;
    p.err = m->err;
    p.max_inflight = m->max_inflight;
    p.wait_ns = m->wait_ns;
    p.stall_phase = m->stall_phase;
    p.pf_tiles = m->pf_tiles;
    p.trace = m->trace_on ? m->trace : nullptr;
    p.n_phases = num_phases(m->L);
    p.ph_begin = 0;
    p.ph_end = p.n_phases;
    p.V_full = m->V_g;
    p.tp = m->tp;
    p.tp_rank = m->tp_rank;
    p.vocab_off = m->v0;
    p.xB = m->Bmax;
    p.xep = m->x_ep;
    p.lm_ep = m->lm_ep;
    for (int r = 0; r < m->tp && m->tp > 1; ++r) p.xpeer[r] = m->xpeer[r];
    p.x_cnt = static_cast<int64_t>(m->x_cnt);
    p.x_o = static_cast<int64_t>(m->x_o);
    p.x_d = static_cast<int64_t>(m->x_d);
    p.x_cand = static_cast<int64_t>(m->x_cand);
    return p;
}

// Positions per split-KV chunk: up to kMaxChunks chunks per (row, kv head) spread over the CTAs, never more
// than kMaxChunks for the longest row of the launch, whole tiles.
// Projection phases whose whole row groups leave some CTAs two or more tiles
// above the even share (Gemma3-4B down_proj: 160 groups of 10 tiles on 148
// CTAs): the kernel splits their (group, segment) tiles evenly instead, two
// CTAs sharing a group where a slot boundary falls inside it (gemv_geom).
// Every slot must hold at least nseg tiles, so a group has two owners at most.
// Only the bf16 kernels carry the split (the large models); the fp32 kernels
// stay without it.
static int split_kinds(const mg_model *m) {
    if (m->wdtype == MG_F32) return 0;
    const int esz = 2;
    const struct {
        int kind, N, Kp;
        bool pair;
    } phases[4] = {{PH_QKV, m->qkv_rows, m->Hp, false},
                   {PH_O, m->H, m->Ap, false},
                   {PH_GU, m->I, m->Hp, true},
                   {PH_D, m->H, m->Ip, false}};
    int mask = 0;
    for (const auto &f : phases) {
        const TileShape ts = tile_shape(f.Kp, esz, f.pair);
        const int64_t G = m->G, groups = (f.N + ts.rps - 1) / ts.rps, U = groups * ts.nseg;
        if (ts.nseg < 2 || U / G < ts.nseg || U * G >= (int64_t{1} << 31)) continue;
        if ((groups + G - 1) / G * ts.nseg - (U + G - 1) / G >= 2) mask |= 1 << f.kind;
    }
    return mask;
}

static int att_chunk(const mg_model *m, int B, int max_ctx, int units) {
    const int target = std::max(1, std::min(m->att_chunks, m->G / std::max(1, B * units)));
    int ch = std::max((max_ctx + target - 1) / target, (max_ctx + kMaxChunks - 1) / kMaxChunks);
    ch = (ch + kAttTile - 1) / kAttTile * kAttTile;
    return std::max(ch, kAttTile);
}

static mg_status run_decode(mg_model *m, DecodeParams &p, int max_ctx) {
    if (m->tp > 1 && !m->tp_connected)
        return fail(MG_ERR_INVALID, "tensor-parallel model used before mg_tp_connect");
    // batch 1 with head dim 256: an attention item per q head (the CTAs are idle otherwise)
    p.att_split = (m->hd == 256 && m->Hq > m->Hkv && p.B == 1 && !m->no_att_split) ? 1 : 0;
    p.att_ch = att_chunk(m, p.B, max_ctx, p.att_split ? m->Hq : m->Hkv);
    // every forward writes its activations with new tags; before the count
    // wraps, the words are cleared so that no old tag can match again
    if (++m->epoch > kMaxEpoch) {
        CU(cudaMemsetAsync(m->h, 0, m->tagged_words * sizeof(uint64_t), m->stream));
        m->epoch = 1;
    }
    p.epoch = m->epoch;
    // the ring depth and stage of this launch's row count
    const int rb = std::min(std::max(p.B, 1), m->Bdec);
    p.S = m->S_rows[rb];
    p.xs_floats = m->xs_rows[rb];
    const size_t smem = m->smem_rows[rb];
    const bool persistent = m->decode_path == 0;
    if (persistent) {
        cudaError_t e = m->wdtype == MG_F32 ? decode_launch<float>(p, m->G, smem, m->stream, true)
                                            : decode_launch<__nv_bfloat16>(p, m->G, smem, m->stream, true);
        if (e != cudaSuccess) return fail(MG_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(e));
    } else {
        for (int ph = 0; ph < p.n_phases; ++ph) {
            DecodeParams q = p;
            q.ph_begin = ph;
            q.ph_end = ph + 1;
            cudaError_t e = m->wdtype == MG_F32 ? decode_launch<float>(q, m->G, smem, m->stream, false)
                                                : decode_launch<__nv_bfloat16>(q, m->G, smem, m->stream, false);
            if (e != cudaSuccess) return fail(MG_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(e));
        }
    }
    // every rank runs the same forwards, so these stay equal across ranks
    m->x_ep += static_cast<uint64_t>(m->L);
    if (p.lm_mode == kLmLogits) m->lm_ep += 1;
    return MG_OK;
}

// tp > 1: every rank's logits slice into logits_full [B][V_g] (after the
// launch, whose last phase waited for all ranks' lm_head).
static mg_status gather_logits(mg_model *m, int batch) {
    const size_t row = static_cast<size_t>(m->V) * sizeof(float);
    for (int r = 0; r < m->tp; ++r)
        for (int b = 0; b < batch; ++b)
            CU(cudaMemcpyAsync(m->logits_full + static_cast<size_t>(b) * m->V_g + static_cast<size_t>(r) * m->V,
                               m->xpeer[r] + m->x_logits + b * row, row, cudaMemcpyDeviceToDevice, m->stream));
    return MG_OK;
}

// Reads and clears the device error word (synchronises the stream).
static mg_status check_device(mg_model *m) {
    cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return fail(MG_ERR_CUDA, "device error: %s", cudaGetErrorString(e));
    uint32_t code = 0;
    CU(cudaMemcpy(&code, m->err, 4, cudaMemcpyDeviceToHost));
    if (code != 0) {
        CU(cudaMemset(m->err, 0, 4));
        CU(cudaMemset(m->sync, 0, m->sync_words * 4));
        const uint32_t kind = code & 0xffff0000u;
        if (kind == kErrBadToken) return fail(MG_ERR_INVALID, "token id out of range in row %u", code & 0xffffu);
        if (kind == kErrBadPos) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
        return fail(MG_ERR_TIMEOUT, "decode kernel gave up waiting (code 0x%08x); results discarded", code);
    }
    return MG_OK;
}

struct SampleCfg {
    int topk = 0;      // fused candidates
    bool fused = false;
    bool general = false;
};

static SampleCfg sample_cfg(const mg_model *m, const mg_sampling *s) {
    SampleCfg c;
    if (!s) return c;
    if (s->temperature <= 0.0) {
        c.topk = 1;
        c.fused = true;
    } else if (s->top_k > 0 && s->top_k < m->V_g && s->top_k <= kMaxTopK) {
        c.topk = s->top_k;
        c.fused = true;
    } else if (m->V_g <= kMaxTopK && m->tp == 1) {
        c.topk = m->V_g;
        c.fused = true;
    } else {
        c.general = true;
    }
    return c;
}

static mg_status validate_rows(mg_model *m, int batch) {
    if (batch <= 0 || batch > m->Bmax) return fail(MG_ERR_INVALID, "batch %d outside [1, %d]", batch, m->Bmax);
    return MG_OK;
}

// Rows [r0, r0 + nb) of the model as one launch of nb rows: the row-indexed
// state (tokens, positions, KV rows, logits rows, drawn tokens, variates, ids)
// is offset; activations and candidate keys are per-launch scratch.  Steps of
// more rows than the persistent kernel holds run one launch per row group, in
// the reference's fp32 arithmetic (models created with prefill_path 0).
static void row_window(const mg_model *m, DecodeParams &p, int r0, int nb) {
    p.B = nb;
    p.row_base = r0;
    p.tok += r0;
    p.pos += r0;
    p.kc += static_cast<int64_t>(r0) * m->kv_row_stride;
    p.vc += static_cast<int64_t>(r0) * m->kv_row_stride;
    if (p.logits) p.logits += static_cast<int64_t>(r0) * m->V;
    if (p.out_tokens) p.out_tokens += r0;
    if (p.uniforms) p.uniforms += r0;
    if (p.ids) p.ids += static_cast<int64_t>(r0) * p.ids_ld;
    if (p.nvalid) p.nvalid += r0;
    if (p.emb_acc) p.emb_acc += static_cast<int64_t>(r0) * m->H;
}

// The decode launches of one step for rows [0, batch): one launch when the
// persistent kernel holds them all, else one per row group.  `p` is a template
// for rows [0, batch) (lm_mode, sampling, out_tokens, uniforms, ids set).
static mg_status run_rows(mg_model *m, const DecodeParams &p, int batch, const std::vector<int> &ctx) {
    // as few launches as the row limit allows, of equal size (16 rows at a limit of 5: four launches of 4
    // rows, each with the deeper ring of 4 rows)
    const int ngroups = (batch + m->Bdec - 1) / m->Bdec;
    const int per = (batch + ngroups - 1) / ngroups;
    for (int r0 = 0; r0 < batch; r0 += per) {
        const int nb = std::min(per, batch - r0);
        DecodeParams q = p;
        if (batch > m->Bdec) row_window(m, q, r0, nb);
        int max_ctx = 0;
        for (int b = r0; b < r0 + nb; ++b) max_ctx = std::max(max_ctx, ctx[b]);
        TRY(run_decode(m, q, max_ctx));
    }
    return MG_OK;
}

static mg_status step_impl(mg_model *m, int batch, float *logits_host, int32_t *sampled_host, const mg_sampling *s,
                           bool check) {
    for (int b = 0; b < batch; ++b)
        if (m->h_pos[b] >= m->cap) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
    const SampleCfg sc = sample_cfg(m, s);
    DecodeParams p = base_params(m, batch);
    const bool need_logits = logits_host != nullptr || sc.general || sc.fused;
    p.lm_mode = need_logits ? kLmLogits : kLmNone;
    p.topk = sc.fused ? sc.topk : 0;
    p.sample = sc.fused ? 1 : 0;
    if (s) {
        p.temperature = s->temperature;
        p.top_p = s->top_p;
        p.top_k_req = s->top_k;
        if (s->uniforms_host) {
            CU(cudaMemcpyAsync(m->uniforms, s->uniforms_host, sizeof(double) * batch, cudaMemcpyHostToDevice,
                               m->stream));
            p.uniforms = m->uniforms;
        }
    }
    p.rng_offset = m->rng_offset;
    p.out_tokens = nullptr;
    std::vector<int> ctx(batch);
    for (int b = 0; b < batch; ++b) ctx[b] = m->h_pos[b] + 1;
    TRY(run_rows(m, p, batch, ctx));
    float *logits = m->logits;
    if (m->tp > 1 && (sc.general || logits_host)) {
        TRY(gather_logits(m, batch));
        logits = m->logits_full;
    }
    if (sc.general) {
        CU(sample_rows_launch(logits, m->V_g, batch, m->V_g, s->temperature, s->top_k, s->top_p, p.uniforms, m->seed,
                              m->rng_offset, nullptr, m->tok, m->stream));
    }
    if (s) m->rng_offset += 1;
    for (int b = 0; b < batch; ++b) m->h_pos[b] += 1;
    if (logits_host)
        CU(cudaMemcpyAsync(logits_host, logits, sizeof(float) * batch * m->V_g, cudaMemcpyDeviceToHost, m->stream));
    if (sampled_host && s) {
        CU(cudaMemcpyAsync(m->pinned, m->tok, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost, m->stream));
    }
    if (check || logits_host || sampled_host) {
        mg_status st = check_device(m);
        if (st != MG_OK) {
            for (int b = 0; b < batch; ++b) m->h_pos[b] -= 1;
            CU(cudaMemcpy(m->pos, m->h_pos.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice));
            return st;
        }
        if (sampled_host && s) memcpy(sampled_host, m->pinned, sizeof(int32_t) * batch);
    }
    return MG_OK;
}

static mg_status step_batched(mg_model *m, int batch, const int32_t *tok_host, const mg_sampling *s,
                              int32_t *out_tokens_dev);

extern "C" mg_status mg_step(mg_model *m, const int32_t *token_ids_host, int32_t batch, float *logits_host,
                             int32_t *sampled_host, const mg_sampling *s) {
    if (!m || !token_ids_host) return fail(MG_ERR_INVALID, "null argument");
    TRY(validate_rows(m, batch));
    CU(cudaSetDevice(m->dev));
    for (int b = 0; b < batch; ++b)
        if (token_ids_host[b] < 0 || token_ids_host[b] >= m->V_g)
            return fail(MG_ERR_INVALID, "token id %d out of range [0, %d)", token_ids_host[b], m->V_g);
    memcpy(m->pinned, token_ids_host, sizeof(int32_t) * batch);
    CU(cudaMemcpyAsync(m->tok, m->pinned, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, m->stream));
    if (batch <= m->Bdec || m->prefill_path != 1) return step_impl(m, batch, logits_host, sampled_host, s, true);
    // more rows than the persistent kernel holds: batched tensor-core step
    for (int b = 0; b < batch; ++b)
        if (m->h_pos[b] >= m->cap) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
    const std::vector<int32_t> pos0 = m->h_pos;
    mg_status st = step_batched(m, batch, nullptr, s, nullptr);
    if (st == MG_OK && logits_host)
        CU(cudaMemcpyAsync(logits_host, m->logits, sizeof(float) * batch * m->V, cudaMemcpyDeviceToHost, m->stream));
    if (st == MG_OK && sampled_host && s)
        CU(cudaMemcpyAsync(m->pinned, m->tok, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost, m->stream));
    if (st == MG_OK) st = check_device(m);
    if (st != MG_OK) {
        m->h_pos = pos0;
        CU(cudaMemcpy(m->pos, m->h_pos.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice));
        return st;
    }
    if (sampled_host && s) memcpy(sampled_host, m->pinned, sizeof(int32_t) * batch);
    return MG_OK;
}

extern "C" mg_status mg_set_tokens(mg_model *m, const int32_t *token_ids_host, int32_t batch) {
    if (!m || !token_ids_host) return fail(MG_ERR_INVALID, "null argument");
    TRY(validate_rows(m, batch));
    CU(cudaSetDevice(m->dev));
    for (int b = 0; b < batch; ++b)
        if (token_ids_host[b] < 0 || token_ids_host[b] >= m->V_g)
            return fail(MG_ERR_INVALID, "token id %d out of range [0, %d)", token_ids_host[b], m->V_g);
    CU(cudaMemcpyAsync(m->tok, token_ids_host, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    return MG_OK;
}

extern "C" mg_status mg_generate(mg_model *m, int32_t n_steps, int32_t batch, const mg_sampling *s,
                                 int32_t *tokens_host) {
    if (!m || !s) return fail(MG_ERR_INVALID, "null argument");
    TRY(validate_rows(m, batch));
    if (n_steps <= 0) return MG_OK;
    CU(cudaSetDevice(m->dev));
    for (int b = 0; b < batch; ++b)
        if (m->h_pos[b] + n_steps > m->cap) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
    const int64_t need = static_cast<int64_t>(n_steps) * batch;
    if (need > m->out_cap) {
        int32_t *buf = nullptr;
        TRY(dalloc(m, &buf, need));
        m->out_tokens = buf;
        m->out_cap = need;
    }
    const SampleCfg sc = sample_cfg(m, s);
    const std::vector<int32_t> pos0 = m->h_pos;
    const bool tc_steps = batch > m->Bdec && m->prefill_path == 1;
    for (int t = 0; t < n_steps && tc_steps; ++t)  // batched tensor-core steps
        TRY(step_batched(m, batch, nullptr, s, m->out_tokens + static_cast<int64_t>(t) * batch));
    for (int t = 0; t < n_steps && !tc_steps; ++t) {  // decode-kernel launches (per row group)
        DecodeParams p = base_params(m, batch);
        p.lm_mode = kLmLogits;
        p.topk = sc.fused ? sc.topk : 0;
        p.sample = sc.fused ? 1 : 0;
        p.temperature = s->temperature;
        p.top_p = s->top_p;
        p.top_k_req = s->top_k;
        p.rng_offset = m->rng_offset;
        p.out_tokens = m->out_tokens + static_cast<int64_t>(t) * batch;
        std::vector<int> ctx(batch);
        for (int b = 0; b < batch; ++b) ctx[b] = m->h_pos[b] + 1;
        TRY(run_rows(m, p, batch, ctx));
        if (sc.general) {
            float *logits = m->logits;
            if (m->tp > 1) {
                TRY(gather_logits(m, batch));
                logits = m->logits_full;
            }
            CU(sample_rows_launch(logits, m->V_g, batch, m->V_g, s->temperature, s->top_k, s->top_p, nullptr, m->seed,
                                  m->rng_offset, p.out_tokens, m->tok, m->stream));
        }
        m->rng_offset += 1;
        for (int b = 0; b < batch; ++b) m->h_pos[b] += 1;
    }
    if (tokens_host)
        CU(cudaMemcpyAsync(tokens_host, m->out_tokens, sizeof(int32_t) * need, cudaMemcpyDeviceToHost, m->stream));
    mg_status st = check_device(m);
    if (st != MG_OK) {
        m->h_pos = pos0;
        CU(cudaMemcpy(m->pos, m->h_pos.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice));
    }
    return st;
}

static mg_status upload_ids(mg_model *m, const int32_t *ids, const int32_t *lens, int batch, int max_len) {
    const int64_t need = static_cast<int64_t>(batch) * max_len;
    if (need > m->ids_cap) {
        int32_t *buf = nullptr;
        TRY(dalloc(m, &buf, need));
        m->ids = buf;
        m->ids_cap = need;
    }
    if (!m->nvalid) TRY(dalloc(m, &m->nvalid, m->nrows));
    for (int b = 0; b < batch; ++b) {
        if (lens[b] < 0 || lens[b] > max_len) return fail(MG_ERR_INVALID, "row %d length %d outside [0, %d]", b, lens[b], max_len);
        for (int t = 0; t < lens[b]; ++t) {
            const int32_t id = ids[static_cast<int64_t>(b) * max_len + t];
            if (id < 0 || id >= m->V_g) return fail(MG_ERR_INVALID, "token id %d out of range [0, %d)", id, m->V_g);
        }
    }
    CU(cudaMemcpyAsync(m->ids, ids, sizeof(int32_t) * need, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(m->nvalid, lens, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, m->stream));
    return MG_OK;
}

// Batched prefill (prefill_path 1): all prompt tokens of all rows per layer,
// projections on the tensor cores (prefill.cu, gemm_tc.cu).
// Workspace for N packed tokens (kept for later calls).
static mg_status pf_reserve(mg_model *m, int N) {
    if (N > m->pf_cap) {  // workspace for N packed tokens (kept for later calls)
        const int cap = std::max(N, 256);
        m->pf_kx = std::max(m->Hp, std::max(m->Ap, m->Ip));
        m->pf_cx = std::max(m->qkv_rows, std::max(m->H, 2 * m->I));
        TRY(dalloc(m, &m->pf_x, static_cast<size_t>(cap) * m->H));
        TRY(dalloc(m, &m->pf_r, static_cast<size_t>(cap) * m->H));
        TRY(dalloc(m, &m->pf_c, static_cast<size_t>(cap) * m->pf_cx));
        TRY(dalloc(m, &m->pf_xn, static_cast<size_t>(cap) * m->pf_kx));
        TRY(dalloc(m, &m->pf_tok, cap));
        TRY(dalloc(m, &m->pf_row, cap));
        TRY(dalloc(m, &m->pf_pos, cap));
        TRY(dalloc(m, &m->pf_last, cap));
        if (m->gu_il) TRY(dalloc(m, &m->pf_act, static_cast<size_t>(cap) * m->Ip));
        if (attn_tc_supported(m->hd)) {
            m->pf_vt_ld = (cap + 7) / 8 * 8;
            TRY(dalloc(m, &m->pf_qb, static_cast<size_t>(cap) * m->Hq * m->hd));
            TRY(dalloc(m, &m->pf_kb, static_cast<size_t>(cap) * m->Hkv * m->hd));
            TRY(dalloc(m, &m->pf_vt, static_cast<size_t>(m->pf_vt_ld) * m->Hkv * m->hd));
            m->att_tiles_cap = cap / 128 + m->Bmax + 1;
            TRY(dalloc(m, &m->att_tiles, m->att_tiles_cap));
        }
        m->pf_cap = cap;
    }
    return MG_OK;
}

// Every layer for the N tokens in pf_tok / pf_row / pf_pos: K/V into the
// cache, and pf_xn = bf16(final-norm of the last layer's output) per token.
// Upload the 128-query tiles of sequences (start, len) for the tensor-core
// attention; returns the tile count (0: this model uses the CUDA-core kernel).
static int upload_att_tiles(mg_model *m, const std::vector<int32_t> &start, const std::vector<int32_t> &len) {
    if (!attn_tc_supported(m->hd) || !m->att_tiles) return 0;
    std::vector<int4> t;
    for (size_t b = 0; b < start.size(); ++b)
        for (int q0 = 0; q0 < len[b]; q0 += 128) t.push_back(make_int4(start[b], len[b], q0, 0));
    if (t.empty() || static_cast<int>(t.size()) > m->att_tiles_cap) return 0;
    if (cudaMemcpyAsync(m->att_tiles, t.data(), sizeof(int4) * t.size(), cudaMemcpyHostToDevice, m->stream) !=
        cudaSuccess)
        return -1;
    return static_cast<int>(t.size());
}

// ntiles > 0: every token's keys are tokens of this batch (sequences from
// position 0), and the attention runs on the tensor cores over those tiles;
// last (encoder) selects the bidirectional mask.  Otherwise the CUDA-core
// kernel reads the KV cache (prompts that continue a cached prefix).
// max_ctx (> 0): an upper bound of the keys per token, which lets the
// CUDA-core attention split the keys of a few tokens over many CTAs.
static mg_status pf_layers(mg_model *m, int N, const int32_t *last = nullptr, int ntiles = 0, int max_ctx = 0) {
    cudaStream_t st = m->stream;
    const float inv_h = 1.0f / static_cast<float>(m->H), inv_hd = 1.0f / static_cast<float>(m->hd);
    const float att_scale = 1.0f / sqrtf(static_cast<float>(m->hd));
    CU(pf_embed(m->embed, m->wdtype == MG_BF16, m->embed_ld, m->pf_tok, N, m->H, sqrtf(static_cast<float>(m->H)),
                m->pf_x, st));
    CU(pf_resnorm(m->pf_x, nullptr, nullptr, m->h_layers[0].in_ln, m->pf_x, m->pf_xn, N, m->H, m->Hp, inv_h, st));
    auto gemm = [&](const __nv_bfloat16 *a, int lda, const __nv_bfloat16 *w, int n_out, int K, float *c,
                    int ldc) -> mg_status {
        CU(gemm_bf16_tc(a, lda, w, K, c, ldc, N, n_out, K, m->err, st, m->pf_ws, m->pf_ws_floats));
        return MG_OK;
    };
    for (int l = 0; l < m->L; ++l) {
        const LayerPtrs &lp = m->h_layers[l];
        const mg_model::PfLayer &w = m->pf[l];
        float *kc = m->kc + static_cast<int64_t>(l) * m->kv_layer_stride;
        float *vc = m->vc + static_cast<int64_t>(l) * m->kv_layer_stride;
        TRY(gemm(m->pf_xn, m->Hp, w.qkv, m->qkv_rows, m->Hp, m->pf_c, m->qkv_rows));
        const bool tc_att = ntiles > 0;
        // an encoder pass on the tensor cores reads no cache: K / V stay out of it
        const bool to_cache = !(tc_att && last);
        CU(pf_qk_rope_kv(m->pf_c, m->qkv_rows, N, m->Hq, m->Hkv, m->hd, m->hdp, lp.q_norm, lp.k_norm,
                         lp.is_global ? m->cos_g : m->cos_l, lp.is_global ? m->sin_g : m->sin_l, m->pf_row, m->pf_pos,
                         to_cache ? kc : nullptr, to_cache ? vc : nullptr, m->kv_row_stride, m->kv_head_stride,
                         inv_hd, tc_att ? m->pf_qb : nullptr,
                         tc_att ? m->pf_kb : nullptr, tc_att ? m->pf_vt : nullptr, m->pf_vt_ld, st));
        if (m->Ap > m->A) CU(cudaMemsetAsync(m->pf_xn, 0, sizeof(__nv_bfloat16) * N * m->Ap, st));
        if (tc_att)
            CU(attn_tc(m->pf_qb, m->pf_kb, m->pf_vt, m->pf_vt_ld, N, m->Hq, m->Hkv, m->hd, m->att_tiles, ntiles,
                       (!lp.is_global && m->window > 0) ? m->window : 0, last ? 1 : 0, att_scale, m->pf_xn, m->Ap,
                       m->err, st));
        else
            CU(pf_attention(m->pf_c, m->qkv_rows, N, m->Hq, m->Hkv, m->hd, m->hdp, kc, vc, m->pf_row, m->pf_pos,
                            last, m->kv_row_stride, m->kv_head_stride, m->window, lp.is_global, att_scale, m->pf_xn,
                            m->Ap, max_ctx, m->pf_ws, m->pf_ws_floats, st));
        TRY(gemm(m->pf_xn, m->Ap, w.o, m->H, m->Ap, m->pf_c, m->H));
        CU(pf_resnorm(m->pf_x, m->pf_c, lp.post_attn_ln, lp.pre_ff_ln, m->pf_r, m->pf_xn, N, m->H, m->Hp, inv_h, st));
        // gate/up + GeGLU: fused into the GEMM epilogue when the grid fills the GPU
        const __nv_bfloat16 *act = m->pf_xn;
        const cudaError_t fe = m->gu_il ? gemm_bf16_tc_geglu(m->pf_xn, m->Hp, w.gu, m->Hp, m->pf_act, m->Ip, N,
                                                             2 * m->I, m->Hp, m->err, st)
                                        : cudaErrorNotSupported;
        if (fe == cudaSuccess) {
            act = m->pf_act;
        } else if (fe == cudaErrorNotSupported) {
            TRY(gemm(m->pf_xn, m->Hp, w.gu, 2 * m->I, m->Hp, m->pf_c, 2 * m->I));
            CU(pf_geglu(m->pf_c, m->I, 2 * m->I, m->pf_xn, m->Ip, N, m->gu_il ? 1 : 0, st));
        } else {
            CU(fe);
        }
        TRY(gemm(act, m->Ip, w.down, m->H, m->Ip, m->pf_c, m->H));
        const float *w_next = l + 1 < m->L ? m->h_layers[l + 1].in_ln : m->final_norm;
        CU(pf_resnorm(m->pf_r, m->pf_c, lp.post_ff_ln, w_next, m->pf_x, m->pf_xn, N, m->H, m->Hp, inv_h, st));
    }
    return MG_OK;
}

static mg_status prefill_batched(mg_model *m, const int32_t *ids, const int32_t *lens, int batch, int max_len) {
    std::vector<int32_t> tok, row, pos, seq_start, seq_len;
    bool fresh = true;  // every row starts at position 0: all keys are in this batch
    for (int b = 0; b < batch; ++b) {
        if (lens[b] > 0) {
            fresh = fresh && m->h_pos[b] == 0;
            seq_start.push_back(static_cast<int32_t>(tok.size()));
            seq_len.push_back(lens[b]);
        }
        for (int t = 0; t < lens[b]; ++t) {
            tok.push_back(ids[static_cast<int64_t>(b) * max_len + t]);
            row.push_back(b);
            pos.push_back(m->h_pos[b] + t);
        }
    }
    const int N = static_cast<int>(tok.size());
    if (N == 0) return MG_OK;
    TRY(pf_reserve(m, N));
    cudaStream_t st = m->stream;
    CU(cudaMemcpyAsync(m->pf_tok, tok.data(), sizeof(int32_t) * N, cudaMemcpyHostToDevice, st));
    CU(cudaMemcpyAsync(m->pf_row, row.data(), sizeof(int32_t) * N, cudaMemcpyHostToDevice, st));
    CU(cudaMemcpyAsync(m->pf_pos, pos.data(), sizeof(int32_t) * N, cudaMemcpyHostToDevice, st));
    const int ntiles = fresh ? upload_att_tiles(m, seq_start, seq_len) : 0;
    if (ntiles < 0) return fail(MG_ERR_CUDA, "tile upload failed");
    return pf_layers(m, N, nullptr, ntiles);
}

// One decode step for rows [0, batch) on the batched path (more rows than the
// persistent kernel holds): the layers for one token per row, the lm_head as a
// tcgen05 GEMM into logits [batch][V], then the token draw of
// _sample_next_token (model.py:103-150) over each row with the general sampler.
// tok_host null: the rows' current tokens on the device (m->tok).
static mg_status step_batched(mg_model *m, int batch, const int32_t *tok_host, const mg_sampling *s,
                              int32_t *out_tokens_dev) {
    TRY(pf_reserve(m, batch));
    cudaStream_t st = m->stream;
    // rows, positions and tokens come from device arrays (no pageable host
    // copy, which could block the host): the step's launches queue ahead
    if (tok_host)
        CU(cudaMemcpyAsync(m->pf_tok, tok_host, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    else
        CU(cudaMemcpyAsync(m->pf_tok, m->tok, sizeof(int32_t) * batch, cudaMemcpyDeviceToDevice, st));
    CU(cudaMemcpyAsync(m->pf_row, m->row_ident, sizeof(int32_t) * batch, cudaMemcpyDeviceToDevice, st));
    CU(cudaMemcpyAsync(m->pf_pos, m->pos, sizeof(int32_t) * batch, cudaMemcpyDeviceToDevice, st));
    int max_ctx = 0;
    for (int b = 0; b < batch; ++b) max_ctx = std::max(max_ctx, m->h_pos[b] + 1);
    TRY(pf_layers(m, batch, nullptr, 0, max_ctx));
    CU(gemm_bf16_tc(m->pf_xn, m->Hp, m->pf_lm, m->Hp, m->logits, m->V, batch, m->V, m->Hp, m->err, st, m->pf_ws,
                    m->pf_ws_floats));
    if (s) {
        const double *u = nullptr;
        if (s->uniforms_host) {
            CU(cudaMemcpyAsync(m->uniforms, s->uniforms_host, sizeof(double) * batch, cudaMemcpyHostToDevice, st));
            u = m->uniforms;
        }
        CU(sample_rows_launch(m->logits, m->V, batch, m->V, s->temperature, s->top_k, s->top_p, u, m->seed,
                              m->rng_offset, out_tokens_dev, m->tok, st));
        m->rng_offset += 1;
    }
    for (int b = 0; b < batch; ++b) m->h_pos[b] += 1;  // host mirror of the device increment
    CU(pf_advance(m->pos, batch, st));
    return MG_OK;
}

extern "C" mg_status mg_prefill(mg_model *m, const int32_t *token_ids_host, const int32_t *lens_host, int32_t batch,
                                int32_t max_len) {
    if (!m || !token_ids_host || !lens_host) return fail(MG_ERR_INVALID, "null argument");
    TRY(validate_rows(m, batch));
    CU(cudaSetDevice(m->dev));
    int longest = 0;
    for (int b = 0; b < batch; ++b) {
        longest = std::max(longest, lens_host[b]);
        if (m->h_pos[b] + lens_host[b] > m->cap) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
    }
    if (longest == 0) return MG_OK;
    TRY(upload_ids(m, token_ids_host, lens_host, batch, max_len));
    std::vector<int32_t> pos0 = m->h_pos;
    if (m->prefill_path == 1 && m->tp == 1) {
        mg_status st = prefill_batched(m, token_ids_host, lens_host, batch, max_len);
        if (st == MG_OK) {
            for (int b = 0; b < batch; ++b) m->h_pos[b] = pos0[b] + lens_host[b];
            CU(cudaMemcpyAsync(m->pos, m->h_pos.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice,
                               m->stream));
            st = check_device(m);
        }
        if (st != MG_OK) {
            m->h_pos = pos0;
            CU(cudaMemcpy(m->pos, m->h_pos.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice));
        }
        return st;
    }
    for (int t = 0; t < longest; ++t) {
        DecodeParams p = base_params(m, batch);
        p.lm_mode = kLmNone;
        p.ids = m->ids;
        p.ids_ld = max_len;
        p.nvalid = m->nvalid;
        p.step_t = t;
        std::vector<int> ctx(batch);
        for (int b = 0; b < batch; ++b) ctx[b] = pos0[b] + std::min(t, lens_host[b]) + 1;
        TRY(run_rows(m, p, batch, ctx));
    }
    // the last fed token becomes the current token of each row
    for (int b = 0; b < batch; ++b) m->h_pos[b] = pos0[b] + lens_host[b];
    mg_status st = check_device(m);
    if (st != MG_OK) {
        m->h_pos = pos0;
        CU(cudaMemcpy(m->pos, m->h_pos.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice));
    }
    return st;
}

extern "C" mg_status mg_encode(mg_model *m, const int32_t *token_ids_host, const int32_t *lens_host, int32_t batch,
                               int32_t max_len, float *out_host) {
    if (!m || !token_ids_host || !lens_host || !out_host) return fail(MG_ERR_INVALID, "null argument");
    if (batch <= 0) return fail(MG_ERR_INVALID, "inputs must contain at least one row");
    if (m->prefill_path != 1 || m->tp > 1)
        return fail(MG_ERR_UNSUPPORTED, "mg_encode needs a model created with prefill_path 1 (and tp_size 1)");
    CU(cudaSetDevice(m->dev));
    for (int b = 0; b < batch; ++b) {
        if (lens_host[b] <= 0 || lens_host[b] > max_len || lens_host[b] > m->cap)
            return fail(MG_ERR_INVALID, "row %d length %d outside [1, min(max_len, capacity)]", b, lens_host[b]);
        for (int t = 0; t < lens_host[b]; ++t) {
            const int32_t id = token_ids_host[static_cast<int64_t>(b) * max_len + t];
            if (id < 0 || id >= m->V_g) return fail(MG_ERR_INVALID, "token id %d out of range [0, %d)", id, m->V_g);
        }
    }
    if (!m->enc_out) {
        TRY(dalloc(m, &m->enc_pool, static_cast<size_t>(m->Bmax) * m->H));
        TRY(dalloc(m, &m->enc_mid, static_cast<size_t>(m->Bmax) * std::max(m->d0_out, 1)));
        TRY(dalloc(m, &m->enc_out, static_cast<size_t>(m->Bmax) * m->H));
        TRY(dalloc(m, &m->enc_start, m->Bmax));
        TRY(dalloc(m, &m->enc_len, m->Bmax));
    }
    cudaStream_t st = m->stream;
    // sequences go through in groups of max_batch rows; their K/V use the
    // model's cache rows at positions 0.. (the decode state is overwritten)
    for (int b0 = 0; b0 < batch; b0 += m->Bmax) {
        const int nb = std::min(m->Bmax, batch - b0);
        std::vector<int32_t> tok, row, pos, last, start(nb), len(nb);
        for (int b = 0; b < nb; ++b) {
            const int n = lens_host[b0 + b];
            start[b] = static_cast<int32_t>(tok.size());
            len[b] = n;
            for (int t = 0; t < n; ++t) {
                tok.push_back(token_ids_host[static_cast<int64_t>(b0 + b) * max_len + t]);
                row.push_back(b);
                pos.push_back(t);
                last.push_back(n - 1);
            }
        }
        const int N = static_cast<int>(tok.size());
        TRY(pf_reserve(m, N));
        CU(cudaMemcpyAsync(m->pf_tok, tok.data(), sizeof(int32_t) * N, cudaMemcpyHostToDevice, st));
        CU(cudaMemcpyAsync(m->pf_row, row.data(), sizeof(int32_t) * N, cudaMemcpyHostToDevice, st));
        CU(cudaMemcpyAsync(m->pf_pos, pos.data(), sizeof(int32_t) * N, cudaMemcpyHostToDevice, st));
        CU(cudaMemcpyAsync(m->pf_last, last.data(), sizeof(int32_t) * N, cudaMemcpyHostToDevice, st));
        CU(cudaMemcpyAsync(m->enc_start, start.data(), sizeof(int32_t) * nb, cudaMemcpyHostToDevice, st));
        CU(cudaMemcpyAsync(m->enc_len, len.data(), sizeof(int32_t) * nb, cudaMemcpyHostToDevice, st));
        const int ntiles = upload_att_tiles(m, start, len);
        if (ntiles < 0) return fail(MG_ERR_CUDA, "tile upload failed");
        TRY(pf_layers(m, N, m->pf_last, ntiles));
        // per-token 1/rms goes into pf_r (free after the last layer)
        CU(pf_encoder_head(m->pf_x, m->H, N, m->enc_start, m->enc_len, m->final_norm, 1.0f / static_cast<float>(m->H),
                           m->pf_r, m->d0, m->d0_out, m->d1, m->enc_pool, m->enc_mid, m->enc_out, nb, st));
        CU(cudaMemcpyAsync(out_host + static_cast<int64_t>(b0) * m->H, m->enc_out, sizeof(float) * nb * m->H,
                           cudaMemcpyDeviceToHost, st));
        CU(cudaStreamSynchronize(st));  // the host vectors above are reused by the next group
    }
    return check_device(m);
}

extern "C" mg_status mg_embed(mg_model *m, const int32_t *token_ids_host, const int32_t *lens_host, int32_t batch,
                              int32_t max_len, float *out_host) {
    if (!m || !token_ids_host || !lens_host || !out_host) return fail(MG_ERR_INVALID, "null argument");
    if (batch <= 0) return fail(MG_ERR_INVALID, "inputs must contain at least one row");
    CU(cudaSetDevice(m->dev));
    for (int b = 0; b < batch; ++b) {
        if (lens_host[b] <= 0) return fail(MG_ERR_INVALID, "inputs must contain at least one token");
        if (lens_host[b] > m->cap) return fail(MG_ERR_SEQ_EXCEEDED, "Sequence length exceeded");
    }
    const std::vector<int32_t> pos_saved = m->h_pos;
    std::vector<float> acc(static_cast<size_t>(m->Bmax) * m->H);
    for (int b0 = 0; b0 < batch; b0 += m->Bdec) {
        const int nb = std::min(m->Bdec, batch - b0);
        int longest = 0;
        for (int b = 0; b < nb; ++b) longest = std::max(longest, lens_host[b0 + b]);
        TRY(upload_ids(m, token_ids_host + static_cast<int64_t>(b0) * max_len, lens_host + b0, nb, max_len));
        CU(cudaMemsetAsync(m->pos, 0, sizeof(int32_t) * m->nrows, m->stream));
        CU(cudaMemsetAsync(m->emb_acc, 0, sizeof(float) * m->Bmax * m->H, m->stream));
        for (int t = 0; t < longest; ++t) {
            DecodeParams p = base_params(m, nb);
            p.lm_mode = kLmEmbed;
            p.ids = m->ids;
            p.ids_ld = max_len;
            p.nvalid = m->nvalid;
            p.step_t = t;
            TRY(run_decode(m, p, t + 1));
        }
        CU(cudaMemcpyAsync(acc.data(), m->emb_acc, sizeof(float) * nb * m->H, cudaMemcpyDeviceToHost, m->stream));
        TRY(check_device(m));
        for (int b = 0; b < nb; ++b) {
            const float scale = 1.0f / static_cast<float>(lens_host[b0 + b]);  // layers.mojo:368-370
            for (int i = 0; i < m->H; ++i)
                out_host[static_cast<int64_t>(b0 + b) * m->H + i] = acc[static_cast<size_t>(b) * m->H + i] * scale;
        }
    }
    m->h_pos = pos_saved;
    CU(cudaMemcpy(m->pos, m->h_pos.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice));
    return MG_OK;
}

extern "C" mg_status mg_set_debug(mg_model *m, uint64_t wait_budget_ns, int32_t stall_phase) {
    if (!m) return fail(MG_ERR_INVALID, "null model");
    if (stall_phase < -1 || stall_phase >= num_phases(m->L))
        return fail(MG_ERR_INVALID, "stall_phase %d outside [-1, %d)", stall_phase, num_phases(m->L));
    m->wait_ns = wait_budget_ns;
    m->stall_phase = stall_phase;
    return MG_OK;
}

extern "C" mg_status mg_set_pos(mg_model *m, int32_t row, int32_t pos) {
    if (!m) return fail(MG_ERR_INVALID, "null model");
    if (row >= m->Bmax || row < -1) return fail(MG_ERR_INVALID, "row %d outside [-1, %d)", row, m->Bmax);
    if (pos < 0 || pos > m->cap) return fail(MG_ERR_INVALID, "pos %d outside [0, %d]", pos, m->cap);
    CU(cudaSetDevice(m->dev));
    for (int b = 0; b < m->nrows; ++b)
        if (row == -1 || row == b) m->h_pos[b] = pos;
    CU(cudaMemcpyAsync(m->pos, m->h_pos.data(), sizeof(int32_t) * m->nrows, cudaMemcpyHostToDevice, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    return MG_OK;
}

extern "C" mg_status mg_get_pos(const mg_model *m, int32_t *pos_host, int32_t n) {
    if (!m || !pos_host) return fail(MG_ERR_INVALID, "null argument");
    for (int i = 0; i < n && i < m->nrows; ++i) pos_host[i] = m->h_pos[i];
    return MG_OK;
}

extern "C" mg_status mg_read_kv(const mg_model *m, int32_t layer, int32_t row, int32_t pos, float *k_host,
                                float *v_host) {
    if (!m || !k_host || !v_host) return fail(MG_ERR_INVALID, "null argument");
    if (layer < 0 || layer >= m->L || row < 0 || row >= m->Bmax || pos < 0 || pos >= m->cap)
        return fail(MG_ERR_INVALID, "layer/row/pos out of range");
    CU(cudaSetDevice(m->dev));
    CU(cudaStreamSynchronize(m->stream));
    for (int h = 0; h < m->Hkv; ++h) {
        const size_t off = static_cast<size_t>(layer) * m->kv_layer_stride + static_cast<size_t>(row) * m->kv_row_stride +
                           static_cast<size_t>(h) * m->kv_head_stride + static_cast<size_t>(pos) * m->hdp;
        CU(cudaMemcpy(k_host + static_cast<size_t>(h) * m->hd, m->kc + off, sizeof(float) * m->hd,
                      cudaMemcpyDeviceToHost));
        CU(cudaMemcpy(v_host + static_cast<size_t>(h) * m->hd, m->vc + off, sizeof(float) * m->hd,
                      cudaMemcpyDeviceToHost));
    }
    return MG_OK;
}

extern "C" mg_status mg_sample(const float *logits_host, int32_t batch, int32_t vocab, const mg_sampling *s,
                               uint64_t seed, uint64_t offset, int32_t *out_host) {
    if (!logits_host || !s || !out_host || batch <= 0 || vocab <= 0) return fail(MG_ERR_INVALID, "bad argument");
    float *dl = nullptr;
    int32_t *dout = nullptr;
    double *du = nullptr;
    const size_t lb = sizeof(float) * static_cast<size_t>(batch) * vocab;
    CU(cudaMalloc(&dl, lb));
    cudaError_t e = cudaMalloc(&dout, sizeof(int32_t) * batch);
    if (e == cudaSuccess && s->uniforms_host) e = cudaMalloc(&du, sizeof(double) * batch);
    if (e == cudaSuccess) e = cudaMemcpy(dl, logits_host, lb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && du) e = cudaMemcpy(du, s->uniforms_host, sizeof(double) * batch, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = sample_rows_launch(dl, vocab, batch, vocab, s->temperature, s->top_k, s->top_p, du, seed, offset, dout,
                               nullptr, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(out_host, dout, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost);
    cudaFree(dl);
    cudaFree(dout);
    if (du) cudaFree(du);
    if (e != cudaSuccess) return fail(MG_ERR_CUDA, "mg_sample: %s", cudaGetErrorString(e));
    return MG_OK;
}

static size_t trace_words(const mg_model *m) {
    return static_cast<size_t>(m->G) * num_phases(m->L) * kTraceSlots + 2 * static_cast<size_t>(m->G);
}

extern "C" mg_status mg_trace_enable(mg_model *m, int32_t on) {
    if (!m) return fail(MG_ERR_INVALID, "null model");
    CU(cudaSetDevice(m->dev));
    if (on && !m->trace) TRY(dalloc(m, &m->trace, trace_words(m)));
    m->trace_on = on != 0;
    return MG_OK;
}

extern "C" mg_status mg_trace_read(mg_model *m, uint64_t *out_host, int64_t capacity, int64_t *n_out) {
    if (!m || !out_host || !n_out) return fail(MG_ERR_INVALID, "null argument");
    if (!m->trace) return fail(MG_ERR_INVALID, "tracing was never enabled");
    const size_t n = std::min(trace_words(m), static_cast<size_t>(capacity));
    CU(cudaSetDevice(m->dev));
    CU(cudaStreamSynchronize(m->stream));
    CU(cudaMemcpy(out_host, m->trace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    *n_out = static_cast<int64_t>(trace_words(m));
    return MG_OK;
}

extern "C" mg_status mg_tp_ipc_handle(const mg_model *m, void *out) {
    if (!m || !out) return fail(MG_ERR_INVALID, "null argument");
    if (m->tp < 2) return fail(MG_ERR_INVALID, "model is not tensor-parallel");
    static_assert(sizeof(cudaIpcMemHandle_t) == MG_TP_HANDLE_BYTES, "IPC handle size");
    CU(cudaSetDevice(m->dev));
    cudaIpcMemHandle_t h;
    CU(cudaIpcGetMemHandle(&h, m->xbuf));
    memcpy(out, &h, sizeof h);
    return MG_OK;
}

extern "C" mg_status mg_tp_connect(mg_model *m, const void *handles, int32_t n) {
    if (!m || !handles) return fail(MG_ERR_INVALID, "null argument");
    if (m->tp < 2) return fail(MG_ERR_INVALID, "model is not tensor-parallel");
    if (n != m->tp) return fail(MG_ERR_INVALID, "%d handles given for tp=%d", n, m->tp);
    if (m->tp_connected) return fail(MG_ERR_INVALID, "already connected");
    CU(cudaSetDevice(m->dev));
    for (int r = 0; r < m->tp; ++r) {
        if (r == m->tp_rank) {
            m->xpeer[r] = m->xbuf;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char *>(handles) + static_cast<size_t>(r) * MG_TP_HANDLE_BYTES, sizeof h);
        void *ptr = nullptr;
        CU(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        m->ipc_open.push_back(ptr);
        m->xpeer[r] = static_cast<char *>(ptr);
    }
    m->tp_connected = true;
    return MG_OK;
}

extern "C" mg_status mg_tp_disconnect(mg_model *m) {
    if (!m) return fail(MG_ERR_INVALID, "null model");
    CU(cudaSetDevice(m->dev));
    if (m->stream) CU(cudaStreamSynchronize(m->stream));
    for (void *p : m->ipc_open) CU(cudaIpcCloseMemHandle(p));
    m->ipc_open.clear();
    for (int r = 0; r < kMaxTp; ++r) m->xpeer[r] = nullptr;
    m->tp_connected = false;
    return MG_OK;
}
