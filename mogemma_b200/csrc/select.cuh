// select.cuh -- block-wide top-k selection and the token-draw rules.
//
// Keys are 64-bit: the float's order-preserving bits above ~index, so the
// k largest keys are the k largest logits with ties resolved toward the lower
// vocabulary index (numpy argmax picks the first maximum, model.py:111).
// Selection is an MSB-first radix select with 8-bit digits that stops as soon
// as the bucket holding the k-th key is taken whole.
#pragma once

#include "common.cuh"

namespace mg {

// Largest K block_select_topk handles (its sort buffer lives in shared memory).
constexpr int kMaxTopKSel = 1024;

// Lowest possible key: value -inf, index 0xffffffff.  Used as padding.
constexpr uint64_t kKeyNone = 0x007fffff00000000ull;

struct SelectSmem {
    uint32_t hist[256];
    uint32_t sh[8];
    uint64_t tmp[kMaxTopKSel];  // sort buffer
};

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), counter-based RNG.
__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(M0, c[0]), lo0 = M0 * c[0];
        const uint32_t hi1 = __umulhi(M1, c[2]), lo1 = M1 * c[2];
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
        k0 += W0;
        k1 += W1;
    }
}
// Uniform double in [0, 1) with 53 random bits for (seed, offset, row).
__device__ __forceinline__ double philox_uniform(uint64_t seed, uint64_t offset, uint32_t row) {
    uint32_t c[4] = {static_cast<uint32_t>(offset), static_cast<uint32_t>(offset >> 32), row, 0x6d67u};
    philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
    const uint64_t bits = ((static_cast<uint64_t>(c[0]) << 32) | c[1]) >> 11;
    return static_cast<double>(bits) * (1.0 / 9007199254740992.0);
}

// Block-wide select of the K (<= kMaxTopKSel) largest keys among n keys given by
// key_at(i); result sorted descending in out[0..K).  All nthr threads of the
// group call it; sync() is the group barrier.  n < K pads with kKeyNone.
template <class KeyAt, class Sync>
__device__ void block_select_topk(int n, int K, KeyAt key_at, uint64_t *out, SelectSmem &sm, int tid, int nthr,
                                  Sync sync) {
    if (K == 1) {  // argmax: plain max of keys
        uint64_t best = kKeyNone;
        for (int i = tid; i < n; i += nthr) {
            const uint64_t k = key_at(i);
            best = k > best ? k : best;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if ((tid & 31) == 0) sm.tmp[tid >> 5] = best;
        sync();
        if (tid == 0) {
            uint64_t b = sm.tmp[0];
            for (int w = 1; w < nthr / 32; ++w) b = sm.tmp[w] > b ? sm.tmp[w] : b;
            out[0] = b;
        }
        sync();
        return;
    }
    if (n <= K) {
        for (int i = tid; i < K; i += nthr) sm.tmp[i] = i < n ? key_at(i) : kKeyNone;
    } else {
        uint64_t prefix = 0, mask = 0;
        uint32_t kk = static_cast<uint32_t>(K);
        for (int shift = 56; shift >= 0; shift -= 8) {
            for (int i = tid; i < 256; i += nthr) sm.hist[i] = 0u;
            sync();
            // Warp-aggregated histogram: lanes holding the same digit add once.
            // Candidate keys of similar logits share their top digits, and plain
            // per-key atomics on one bin serialise (tens of us for 9,472 keys).
            for (int i0 = 0; i0 < n; i0 += nthr) {  // warp-uniform trip count
                const int i = i0 + tid;
                uint32_t dig = 256u;  // not in the current bucket
                if (i < n) {
                    const uint64_t k = key_at(i);
                    if ((k & mask) == prefix) dig = static_cast<uint32_t>((k >> shift) & 255u);
                }
                const uint32_t same = __match_any_sync(0xffffffffu, dig);
                if (dig != 256u && (tid & 31) == __ffs(same) - 1) atomicAdd(&sm.hist[dig], __popc(same));
            }
            sync();
            if (tid < 32) {
                const int lane = tid;
                uint32_t c[8], local = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c[j] = sm.hist[255 - 8 * lane - j];
                    local += c[j];
                }
                uint32_t incl = local;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += v;
                }
                const uint32_t excl = incl - local;
                if (excl < kk && kk <= incl) {
                    uint32_t run = excl;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (run + c[j] >= kk) {
                            sm.sh[0] = static_cast<uint32_t>(255 - 8 * lane - j);
                            sm.sh[1] = run;
                            sm.sh[2] = c[j];
                            break;
                        }
                        run += c[j];
                    }
                }
            }
            sync();
            const uint32_t d = sm.sh[0], above = sm.sh[1], cnt = sm.sh[2];
            kk -= above;
            prefix |= static_cast<uint64_t>(d) << shift;
            mask |= 0xffull << shift;
            sync();
            if (cnt == kk) break;
        }
        if (tid == 0) sm.sh[3] = 0u;
        sync();
        for (int i0 = 0; i0 < n; i0 += nthr) {  // one slot reservation per warp
            const int i = i0 + tid;
            uint64_t k = 0;
            bool take = false;
            if (i < n) {
                k = key_at(i);
                take = (k & mask) >= prefix;
            }
            const uint32_t ballot = __ballot_sync(0xffffffffu, take);
            uint32_t base = 0;
            if ((tid & 31) == 0 && ballot) base = atomicAdd(&sm.sh[3], static_cast<uint32_t>(__popc(ballot)));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (take) {
                const uint32_t slot = base + static_cast<uint32_t>(__popc(ballot & ((1u << (tid & 31)) - 1u)));
                if (slot < static_cast<uint32_t>(K)) sm.tmp[slot] = k;
            }
        }
    }
    sync();
    // rank sort (keys are distinct, padding keys only repeat among themselves)
    for (int i = tid; i < K; i += nthr) {
        const uint64_t k = sm.tmp[i];
        int rank = 0;
        for (int j = 0; j < K; ++j) {
            const uint64_t o = sm.tmp[j];
            rank += (o > k) || (o == k && j < i);
        }
        out[rank] = k;
    }
    sync();
}

// The draw rules of _sample_next_token (src/py/mogemma/model.py:103-150) on a
// candidate list sorted by key (value desc, index asc) that holds every token
// the top-k filter keeps.  Runs in one thread; n <= kMaxTopKSel.
//   temperature <= 0 -> first argmax; logits / T in float64; top-p keeps the
//   shortest prefix whose cumulative probability exceeds top_p (the overflowing
//   token included); the draw inverts the index-ordered CDF at u like numpy's
//   Generator.choice (cumsum, normalise by the last entry, searchsorted right).
__device__ inline int32_t draw_from_sorted(const uint64_t *keys, int n, double temperature, double top_p, double u,
                                           double *f /*[n] scratch*/, int *order /*[n] scratch*/) {
    const uint32_t first_idx = key_index(keys[0]);
    if (temperature <= 0.0) return static_cast<int32_t>(first_idx);
    int nv = 0;
    while (nv < n && key_index(keys[nv]) != 0xffffffffu) ++nv;
    if (nv == 0) return 0;
    for (int i = 0; i < nv; ++i) f[i] = static_cast<double>(key_value(keys[i])) / temperature;
    const double fmax = f[0];
    if (!isfinite(fmax)) return static_cast<int32_t>(first_idx);  // +inf -> nan probs; all -inf -> no finite
    int keep = nv;
    if (top_p > 0.0 && top_p < 1.0) {
        double s = 0.0;
        int nfin = 0;
        while (nfin < nv && isfinite(f[nfin])) ++nfin;
        for (int i = 0; i < nfin; ++i) s += exp(f[i] - fmax);
        double cum = 0.0;
        for (int i = 0; i < nfin; ++i) {
            cum += exp(f[i] - fmax) / s;
            if (cum > top_p) {
                keep = i + 1;
                break;
            }
        }
    }
    // probabilities of kept tokens, then the CDF in vocabulary-index order
    double s2 = 0.0;
    for (int i = 0; i < keep; ++i) {
        const double e = exp(f[i] - fmax);
        f[i] = e;
        s2 += e;
    }
    for (int i = 0; i < keep; ++i) {
        int r = 0;
        const uint32_t ii = key_index(keys[i]);
        for (int j = 0; j < keep; ++j) r += key_index(keys[j]) < ii;
        order[r] = i;
    }
    double total = 0.0;
    for (int r = 0; r < keep; ++r) total += f[order[r]] / s2;
    double cdf = 0.0;
    for (int r = 0; r < keep; ++r) {
        cdf += f[order[r]] / s2;
        if (cdf / total > u) return static_cast<int32_t>(key_index(keys[order[r]]));
    }
    return static_cast<int32_t>(key_index(keys[order[keep - 1]]));
}

// draw_from_sorted with its per-candidate float64 work spread over a thread
// group: the divisions by the temperature, the exponentials and the index
// ranks (the O(K^2) part) run one candidate per thread; the sums stay in one
// thread, in the order of the serial rules, so every result is bit-identical
// to draw_from_sorted.  All nthr threads call it; the token is valid in tid 0.
// Scratch (shared memory): f, e [n] doubles, order [n] ints, sh [2] ints.
template <class Sync>
__device__ int32_t draw_block(const uint64_t *keys, int n, double temperature, double top_p, double u, double *f,
                              double *e, int *order, int *sh, int tid, int nthr, Sync sync) {
    if (temperature <= 0.0) return static_cast<int32_t>(key_index(keys[0]));
    for (int i = tid; i < n; i += nthr) f[i] = static_cast<double>(key_value(keys[i])) / temperature;
    sync();
    const double fmax = f[0];
    for (int i = tid; i < n; i += nthr) e[i] = exp(f[i] - fmax);
    sync();
    if (tid == 0) {
        int nv = 0;
        while (nv < n && key_index(keys[nv]) != 0xffffffffu) ++nv;
        int keep = nv;
        if (nv > 0 && isfinite(fmax) && top_p > 0.0 && top_p < 1.0) {
            int nfin = 0;
            while (nfin < nv && isfinite(f[nfin])) ++nfin;
            double s = 0.0;
            for (int i = 0; i < nfin; ++i) s += e[i];
            double cum = 0.0;
            for (int i = 0; i < nfin; ++i) {
                cum += e[i] / s;
                if (cum > top_p) {
                    keep = i + 1;
                    break;
                }
            }
        }
        sh[0] = nv;
        sh[1] = keep;
    }
    sync();
    const int nv = sh[0], keep = sh[1];
    if (nv == 0) return 0;
    if (!isfinite(fmax)) return static_cast<int32_t>(key_index(keys[0]));
    for (int i = tid; i < keep; i += nthr) {
        const uint32_t ii = key_index(keys[i]);
        int r = 0;
        for (int j = 0; j < keep; ++j) r += key_index(keys[j]) < ii;
        order[r] = i;
    }
    sync();
    int32_t token = -1;
    if (tid == 0) {
        double s2 = 0.0;
        for (int i = 0; i < keep; ++i) s2 += e[i];
        double total = 0.0;
        for (int r = 0; r < keep; ++r) total += e[order[r]] / s2;
        double cdf = 0.0;
        token = static_cast<int32_t>(key_index(keys[order[keep - 1]]));
        for (int r = 0; r < keep; ++r) {
            cdf += e[order[r]] / s2;
            if (cdf / total > u) {
                token = static_cast<int32_t>(key_index(keys[order[r]]));
                break;
            }
        }
    }
    return token;
}

}  // namespace mg
