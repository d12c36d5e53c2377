// common.cuh -- shared device helpers for the sm_100a attention kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bml_attn.h"

namespace bml {

// ---------------------------------------------------------------------------
// Bounded waits.  Every spin on an mbarrier or a global counter gives up
// after kWaitNs nanoseconds of %globaltimer (or a limit passed at launch),
// records BML_E_TIMEOUT in the kernel's error word and lets the CTA run to
// its end without waiting again, so that no kernel of this library can hang
// a GPU.
// ---------------------------------------------------------------------------
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s
constexpr uint32_t kErrTimeout = 1u;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of the same condition.  On sm_100a it returns in a few
// cycles when the phase has completed, where try_wait costs tens of cycles
// even then -- which matters to a thread that feeds the tensor core, whose
// instruction queue holds only about one MMA.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar` to complete.  `abort_flag` (shared) is
// set once any wait of the CTA timed out; later waits then return at once.
// Returns false on timeout.  `limit_ns` bounds the wait (kWaitNs unless a
// kernel takes its limit as a launch parameter).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          volatile uint32_t *abort_flag, uint32_t *err,
                                          uint64_t limit_ns = kWaitNs) {
    if (mbar_test_wait(bar, parity)) return true;
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    while (true) {
        if (*abort_flag) return false;
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) {
            *abort_flag = 1u;
            if (err) atomicOr(err, kErrTimeout);
            return false;
        }
    }
}

// Waits (bounded by limit_ns, ignoring any abort flag) for phase `parity`
// of `bar`: used before a CTA leaves, so that no bulk copy it issued is
// still writing its shared memory.
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > limit_ns) return false;
    return true;
}

// Global-memory loads for counters that other CTAs update: acquire (orders
// the caller's later reads after the value) and relaxed (a fresh value from
// L2, no ordering).
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// 1-D bulk copy global -> shared, completing on an mbarrier (TMA unit).
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 evict-first hint: KV is streamed exactly once.
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes,
                                                uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Named barrier over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 2^x on the SFU (ex2.approx, max relative error about 2^-22).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max of three f32 values in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// ---------------------------------------------------------------------------
// 16-byte chunk -> f32 lanes, per storage dtype.
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<float> {
    static constexpr int kPerChunk = 4;
    static constexpr bml_dtype kCode = BML_F32;
    __device__ __forceinline__ static void widen(const uint4 &c, float *out) {
        out[0] = __uint_as_float(c.x);
        out[1] = __uint_as_float(c.y);
        out[2] = __uint_as_float(c.z);
        out[3] = __uint_as_float(c.w);
    }
    // element pairs (2i, 2i+1) as float2, for the packed f32x2 FMA
    __device__ __forceinline__ static void widen2(const uint4 &c, float2 *out) {
        out[0] = make_float2(__uint_as_float(c.x), __uint_as_float(c.y));
        out[1] = make_float2(__uint_as_float(c.z), __uint_as_float(c.w));
    }
};

template <>
struct Elem<__nv_bfloat16> {
    static constexpr int kPerChunk = 8;
    static constexpr bml_dtype kCode = BML_BF16;
    __device__ __forceinline__ static void widen(const uint4 &c, float *out) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    __device__ __forceinline__ static void widen2(const uint4 &c, float2 *out) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    }
};

template <>
struct Elem<__half> {
    static constexpr int kPerChunk = 8;
    static constexpr bml_dtype kCode = BML_F16;
    __device__ __forceinline__ static void widen(const uint4 &c, float *out) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
            float2 f = __half22float2(h);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    }
    __device__ __forceinline__ static void widen2(const uint4 &c, float2 *out) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
    }
};

__device__ __forceinline__ uint4 lds128(const void *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

inline size_t dtype_size(bml_dtype t) { return t == BML_F32 ? 4 : 2; }

}  // namespace bml
