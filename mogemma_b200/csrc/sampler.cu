// sampler.cu -- token draw over full logits rows (general top-k / top-p cases).
//
// The decode kernel fuses greedy and top-k <= 64 draws into its last phase.
// This kernel covers every other setting of _sample_next_token
// (src/py/mogemma/model.py:103-150): one CTA of 1024 threads per row.
//   * K = top_k if 0 < top_k < vocab else vocab.
//   * K <= kMaxTopKSel: the K best keys are selected and sorted, then the
//     shared draw rules run on them (top-p inside).
//   * otherwise: the K-th best key bounds the kept set (radix select on counts);
//     top-p then bounds it further by a radix select on probability mass; the
//     draw inverts the index-ordered CDF with a block scan.
#include "common.cuh"
#include "decode.cuh"
#include "select.cuh"

namespace mg {

constexpr int kSampThreads = 1024;

struct SampSmem {
    SelectSmem sel;
    uint64_t keys[kMaxTopKSel];
    double f[kMaxTopKSel];
    int order[kMaxTopKSel];
    double dsum[kSampThreads / 32];
    double mass[256];
    double dsh[4];
    uint64_t ksh[2];
};

__device__ __forceinline__ void samp_sync() { __syncthreads(); }

__device__ double block_sum_d(double v, SampSmem &sm) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((tid & 31) == 0) sm.dsum[tid >> 5] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < kSampThreads / 32; ++w) t += sm.dsum[w];
    __syncthreads();
    return t;
}

// Smallest key `thr` such that keys >= thr hold exactly K entries (keys distinct).
template <class KeyAt>
__device__ uint64_t kth_key(int n, int K, KeyAt key_at, SampSmem &sm) {
    const int tid = threadIdx.x;
    uint64_t prefix = 0, mask = 0;
    uint32_t kk = static_cast<uint32_t>(K);
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kSampThreads) sm.sel.hist[i] = 0u;
        __syncthreads();
        for (int i0 = 0; i0 < n; i0 += kSampThreads) {  // warp-aggregated (see block_select_topk)
            const int i = i0 + tid;
            uint32_t dig = 256u;
            if (i < n) {
                const uint64_t k = key_at(i);
                if ((k & mask) == prefix) dig = static_cast<uint32_t>((k >> shift) & 255u);
            }
            const uint32_t same = __match_any_sync(0xffffffffu, dig);
            if (dig != 256u && (tid & 31) == __ffs(same) - 1) atomicAdd(&sm.sel.hist[dig], __popc(same));
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t run = 0;
            for (int d = 255; d >= 0; --d) {
                if (run + sm.sel.hist[d] >= kk) {
                    sm.sel.sh[0] = static_cast<uint32_t>(d);
                    sm.sel.sh[1] = run;
                    break;
                }
                run += sm.sel.hist[d];
            }
        }
        __syncthreads();
        kk -= sm.sel.sh[1];
        prefix |= static_cast<uint64_t>(sm.sel.sh[0]) << shift;
        mask |= 0xffull << shift;
        __syncthreads();
    }
    return prefix;  // all 64 bits decided: the K-th largest key itself
}

__global__ void __launch_bounds__(kSampThreads, 1)
    sample_rows_kernel(const float *logits, int64_t ld, int V, double temperature, int top_k, double top_p,
                       const double *uniforms, uint64_t seed, uint64_t offset, int32_t *out, int32_t *tok) {
    extern __shared__ __align__(16) unsigned char raw[];
    SampSmem &sm = *reinterpret_cast<SampSmem *>(raw);
    const int tid = threadIdx.x;
    const int b = blockIdx.x;
    const float *row = logits + static_cast<int64_t>(b) * ld;
    auto key_at = [&](int i) { return topk_key(row[i], static_cast<uint32_t>(i)); };
    auto sync = [] { __syncthreads(); };
    const double u = uniforms ? uniforms[b] : philox_uniform(seed, offset, static_cast<uint32_t>(b));
    int32_t token;
    const int K = (top_k > 0 && top_k < V) ? top_k : V;
    if (temperature <= 0.0 || K <= kMaxTopKSel) {
        const int kk = temperature <= 0.0 ? 1 : K;
        block_select_topk(V, kk, key_at, sm.keys, sm.sel, tid, kSampThreads, sync);
        if (tid == 0) sm.ksh[0] = static_cast<uint64_t>(draw_from_sorted(sm.keys, kk, temperature, top_p, u, sm.f, sm.order));
        __syncthreads();
        token = static_cast<int32_t>(sm.ksh[0]);
    } else {
        // kept set: keys >= thr
        uint64_t thr = 0;
        if (K < V) thr = kth_key(V, K, key_at, sm);
        // max key -> f0
        block_select_topk(V, 1, key_at, sm.keys, sm.sel, tid, kSampThreads, sync);
        const uint64_t kmax = sm.keys[0];
        const double f0 = static_cast<double>(key_value(kmax)) / temperature;
        if (!isfinite(f0)) {
            token = static_cast<int32_t>(key_index(kmax));
        } else {
            auto weight = [&](int i, uint64_t k) -> double {
                if (k < thr) return 0.0;
                const double f = static_cast<double>(row[i]) / temperature;
                return exp(f - f0);
            };
            double local = 0.0;
            for (int i = tid; i < V; i += kSampThreads) local += weight(i, key_at(i));
            const double S = block_sum_d(local, sm);
            if (top_p > 0.0 && top_p < 1.0) {
                // radix select on mass: the first key (descending) at which the
                // cumulative probability exceeds top_p is the new lower bound.
                const double target = top_p;
                uint64_t prefix = 0, mask = 0;
                double above = 0.0;  // normalised mass strictly above the current bucket
                bool found = false;
                for (int shift = 56; shift >= 0; shift -= 8) {
                    for (int i = tid; i < 256; i += kSampThreads) sm.mass[i] = 0.0;
                    __syncthreads();
                    for (int i = tid; i < V; i += kSampThreads) {
                        const uint64_t k = key_at(i);
                        if (k >= thr && (k & mask) == prefix) atomicAdd(&sm.mass[(k >> shift) & 255u], weight(i, k) / S);
                    }
                    __syncthreads();
                    if (tid == 0) {
                        double run = above;
                        int dsel = -1;
                        for (int d = 255; d >= 0; --d) {
                            if (run + sm.mass[d] > target) {
                                dsel = d;
                                break;
                            }
                            run += sm.mass[d];
                        }
                        sm.dsh[0] = run;
                        sm.dsh[1] = static_cast<double>(dsel);
                    }
                    __syncthreads();
                    const int dsel = static_cast<int>(sm.dsh[1]);
                    if (dsel < 0) break;  // cumulative never exceeds top_p: keep everything
                    above = sm.dsh[0];
                    prefix |= static_cast<uint64_t>(dsel) << shift;
                    mask |= 0xffull << shift;
                    found = true;
                    __syncthreads();
                }
                if (found && prefix > thr) thr = prefix;
            }
            // draw: index-ordered CDF over keys >= thr
            constexpr int kChunk = 256;
            const int nchunks = (V + kChunk - 1) / kChunk;
            double total = 0.0;
            {
                double loc = 0.0;
                for (int c = tid; c < nchunks; c += kSampThreads)
                    for (int i = c * kChunk; i < min(V, (c + 1) * kChunk); ++i) loc += weight(i, key_at(i));
                total = block_sum_d(loc, sm);
            }
            // sequential scan over chunks by thread 0 using per-chunk sums (kept small: V/256 chunks)
            if (tid == 0) sm.ksh[1] = 0xffffffffull;
            __syncthreads();
            // chunk sums into a reused buffer (f holds up to kMaxTopKSel doubles; loop in windows)
            double run = 0.0;
            int found_chunk = -1;
            for (int base = 0; base < nchunks && found_chunk < 0; base += kMaxTopKSel) {
                const int nw = min(kMaxTopKSel, nchunks - base);
                for (int c = tid; c < nw; c += kSampThreads) {
                    double s = 0.0;
                    const int cc = base + c;
                    for (int i = cc * kChunk; i < min(V, (cc + 1) * kChunk); ++i) s += weight(i, key_at(i));
                    sm.f[c] = s;
                }
                __syncthreads();
                if (tid == 0) {
                    double r = run;
                    for (int c = 0; c < nw; ++c) {
                        if ((r + sm.f[c]) / total > u) {
                            sm.ksh[1] = static_cast<uint64_t>(base + c);
                            sm.dsh[2] = r;
                            break;
                        }
                        r += sm.f[c];
                    }
                    sm.dsh[3] = r;
                }
                __syncthreads();
                if (sm.ksh[1] != 0xffffffffull) found_chunk = static_cast<int>(sm.ksh[1]);
                run = sm.dsh[3];
                __syncthreads();
            }
            if (tid == 0) {
                int32_t tk = -1;
                if (found_chunk >= 0) {
                    double r = sm.dsh[2];
                    int last_kept = -1;
                    for (int i = found_chunk * kChunk; i < min(V, (found_chunk + 1) * kChunk); ++i) {
                        const double w = weight(i, key_at(i));
                        if (w > 0.0) last_kept = i;
                        r += w;
                        if (w > 0.0 && r / total > u) {
                            tk = i;
                            break;
                        }
                    }
                    if (tk < 0) tk = last_kept;
                }
                if (tk < 0) tk = static_cast<int32_t>(key_index(kmax));
                sm.ksh[0] = static_cast<uint64_t>(tk);
            }
            __syncthreads();
            token = static_cast<int32_t>(sm.ksh[0]);
        }
    }
    if (tid == 0) {
        if (out) out[b] = token;
        if (tok) tok[b] = token;
    }
}

size_t sample_rows_smem() { return sizeof(SampSmem); }

cudaError_t sample_rows_launch(const float *logits, int64_t ld, int rows, int V, double temperature, int top_k,
                               double top_p, const double *uniforms, uint64_t seed, uint64_t offset, int32_t *out,
                               int32_t *tok, cudaStream_t stream) {
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(sample_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(SampSmem)));
        if (e != cudaSuccess) return e;
        attr = true;
    }
    sample_rows_kernel<<<rows, kSampThreads, sizeof(SampSmem), stream>>>(logits, ld, V, temperature, top_k, top_p,
                                                                         uniforms, seed, offset, out, tok);
    return cudaGetLastError();
}

}  // namespace mg
