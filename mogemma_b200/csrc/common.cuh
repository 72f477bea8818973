// common.cuh -- device helpers shared by the sm_100a kernels of libmogemma_cuda.
//
// PTX wrappers for mbarriers and 1-D bulk async copies (TMA bulk engine),
// gpu-scope acquire/release counters, and bounded waits.  Every spin-wait in
// this library goes through a helper here: it gives up after a time budget,
// records the site in the device error word and returns false, so a kernel can
// fast-forward to its end instead of hanging the GPU.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mg {

// Budget for any device-side wait (nanoseconds of %globaltimer).
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

// Error word values (low 16 bits: site; high bits: kind).
constexpr uint32_t kErrTimeoutCounter = 0x10000u;
constexpr uint32_t kErrTimeoutFull = 0x20000u;
constexpr uint32_t kErrTimeoutEmpty = 0x30000u;
constexpr uint32_t kErrTimeoutDrain = 0x40000u;
constexpr uint32_t kErrBadToken = 0x50000u;
constexpr uint32_t kErrBadPos = 0x60000u;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- global-memory synchronisation (gpu scope) ----
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u32(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// System-scope variants for counters that other GPUs increment over NVLink.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_release_sys_add_u64(uint64_t *p, uint64_t v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void set_error(uint32_t *err, uint32_t code) { atomicCAS(err, 0u, code); }

// ---- tagged activations: a float and the tag of the step/layer that wrote it
// in one 64-bit word, stored and loaded as single-copy-atomic 64-bit accesses.
// A reader polls the words themselves: a word carrying the expected tag holds
// the value, so no counter, fence or release is needed between a phase's
// writers and its readers (one L2 round trip instead of three).
__device__ __forceinline__ uint64_t tg_pack(float v, uint32_t tag) {
    return (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ float tg_val(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }
__device__ __forceinline__ uint32_t tg_tag(uint64_t w) { return static_cast<uint32_t>(w >> 32); }
__device__ __forceinline__ void tg_store(uint64_t *p, float v, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(tg_pack(v, tag)) : "memory");
}
__device__ __forceinline__ uint64_t tg_load(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Two adjacent words (16-byte aligned); each element is its own 64-bit access.
__device__ __forceinline__ void tg_load2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Re-polls the words w[j] (loaded from src(j)) that do not yet carry `tag`
// until all do.  Bounded like every wait here: false after the budget or once
// another thread has recorded an error (then the values are not to be used).
template <int N, typename Src>
__device__ __forceinline__ bool tg_settle(uint64_t (&w)[N], uint32_t tag, Src src, uint32_t *err, uint32_t site,
                                          uint64_t budget = kWaitBudgetNs) {
    auto all = [&]() {
        bool a = true;
#pragma unroll
        for (int j = 0; j < N; ++j) a = a && tg_tag(w[j]) == tag;
        return a;
    };
    if (all()) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (tg_tag(w[j]) != tag) w[j] = tg_load(src(j));
        if (all()) return true;
        if ((n & 7u) == 0u) {
            if (ld_relaxed_u32(err) != 0u) return false;
            if (globaltimer_ns() - t0 > budget) {
                set_error(err, kErrTimeoutCounter | site);
                return false;
            }
        }
    }
}

// Wait until *ctr >= target (acquire).  Returns false on error/timeout.
__device__ __forceinline__ bool wait_counter_geq(const uint32_t *ctr, uint32_t target, uint32_t *err,
                                                 uint32_t site, uint64_t budget = kWaitBudgetNs) {
    if (ld_acquire_u32(ctr) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
        if (ld_acquire_u32(ctr) >= target) return true;
        // the error word and the clock are checked every 8th poll: each check
        // is another dependent round trip between two polls
        if ((n & 7u) == 0u) {
            if (ld_relaxed_u32(err) != 0u) return false;
            if (globaltimer_ns() - t0 > budget) {
                set_error(err, kErrTimeoutCounter | site);
                return false;
            }
        }
    }
}

// Wait until the 64-bit counter *ctr (incremented by this and peer GPUs)
// reaches target (acquire at system scope).  Returns false on error/timeout.
__device__ __forceinline__ bool wait_counter_geq_sys(const uint64_t *ctr, uint64_t target, uint32_t *err,
                                                     uint32_t site, uint64_t budget = kWaitBudgetNs) {
    if (ld_acquire_sys_u64(ctr) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
        if (ld_acquire_sys_u64(ctr) >= target) return true;
        if ((n & 7u) == 0u) {
            if (ld_relaxed_u32(err) != 0u) return false;
            if (globaltimer_ns() - t0 > budget) {
                set_error(err, kErrTimeoutCounter | site);
                return false;
            }
        }
    }
}

// ---- mbarrier ----
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0u;
}
// Same, but the thread may sleep up to `ns` nanoseconds inside the instruction
// until the phase completes: a waiting warp then takes no issue slots from the
// warps that share its SM sub-partition.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0u;
}
// Non-blocking probe of a phase.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0u;
}
constexpr uint32_t kMbarSleepNs = 20000;  // longest sleep per poll; a completed phase wakes the thread
// Bounded wait for the phase with `parity` to complete.  The error word and
// the clock are consulted only every 32 polls, keeping the hot poll local.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code,
                                          uint64_t budget = kWaitBudgetNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
        if (mbar_try_wait_sleep(bar, parity, kMbarSleepNs)) return true;
        if ((n & 31u) == 0u) {
            if (ld_relaxed_u32(err) != 0u) return false;
            if (globaltimer_ns() - t0 > budget) {
                set_error(err, code);
                return false;
            }
        }
    }
}
// Same, ignoring the error word (used to drain copies already in flight).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
    }
    return true;
}

// ---- 1-D bulk async copy global -> shared (TMA bulk engine), completes on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// Prefetch [src, src + bytes) into L2 (no completion tracking).  16-byte aligned, multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Named barrier among the `nthreads` consumer threads (id 1; id 0 is __syncthreads).
__device__ __forceinline__ void consumer_sync(uint32_t nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// The same barrier, returning whether `v` holds in every consumer thread.
__device__ __forceinline__ bool consumer_all(bool v, uint32_t nthreads) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "r"(nthreads)
        : "memory");
    return r != 0u;
}

// Atomic exchange at gpu scope with acquire-release order: the stores that
// happen before it (this CTA's, through a barrier) are visible to whoever
// reads the value it stores, and what the previous writer stored before its
// exchange is visible after it.
__device__ __forceinline__ uint64_t atom_exch_acq_rel(uint64_t *addr, uint64_t v) {
    uint64_t old;
    asm volatile("atom.acq_rel.gpu.global.exch.b64 %0, [%1], %2;" : "=l"(old) : "l"(addr), "l"(v) : "memory");
    return old;
}

// ---- numeric helpers ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// 1 / sqrt(sum * inv_n + 1e-6): the scale of an RMSNorm (ops.mojo:98-136),
// through rsqrt.approx (relative error about 1e-7) rather than the IEEE divide
// and square root, whose sequence sat on the critical path of every norm
// prologue (about 1.6 us each, measured).  The reference's own sum order
// differs from any parallel one, so parity is a tolerance in any case.
__device__ __forceinline__ float rms_inv(float sum, float inv_n) { return rsqrtf(sum * inv_n + 1e-6f); }
constexpr float kInvSqrt2 = 0.70710678118654752f;  // GeGLU: erf(g / sqrt 2) as erf(g * (1 / sqrt 2))

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Orderable key: larger float -> larger key; ties broken toward the lower index.
__device__ __forceinline__ uint64_t topk_key(float f, uint32_t idx) {
    uint32_t u = __float_as_uint(f);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(~idx);
}
__device__ __forceinline__ float key_value(uint64_t k) {
    uint32_t u = static_cast<uint32_t>(k >> 32);
    u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
    return __uint_as_float(u);
}
__device__ __forceinline__ uint32_t key_index(uint64_t k) { return ~static_cast<uint32_t>(k & 0xffffffffu); }

// 4 weights as fp32 from shared memory (fp32: 16 B; bf16: 8 B).
__device__ __forceinline__ float4 lds_w4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 lds_w4(const __nv_bfloat16 *p) {
    const uint2 v = *reinterpret_cast<const uint2 *>(p);
    float4 r;
    r.x = __uint_as_float(v.x << 16);
    r.y = __uint_as_float(v.x & 0xffff0000u);
    r.z = __uint_as_float(v.y << 16);
    r.w = __uint_as_float(v.y & 0xffff0000u);
    return r;
}
__device__ __forceinline__ float ld_w(const float *p) { return *p; }
__device__ __forceinline__ float ld_w(const __nv_bfloat16 *p) { return __bfloat162float(*p); }

}  // namespace mg
