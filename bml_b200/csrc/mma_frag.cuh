// mma_frag.cuh -- warp-level MMA fragment helpers shared by the decode
// kernels (ldmatrix loads, the movmatrix transpose, m16n8k16 MMAs and the
// exact 16-bit splitting of f32 operands).
#pragma once

#include "common.cuh"

namespace bml {

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

template <bool F16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if (F16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

// x -> (hi, lo) 16-bit terms with x = hi + lo to 2^-16 relative; packed
// as hi in the low half, lo in the high half.
template <bool F16>
__device__ __forceinline__ uint32_t split2(float x) {
    if (F16) {
        const __half h = __float2half_rn(x);
        const __half l = __float2half_rn(x - __half2float(h));
        return (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
    }
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    const __nv_bfloat16 l = __float2bfloat16_rn(x - __bfloat162float(h));
    return (uint32_t)__bfloat16_as_ushort(h) | ((uint32_t)__bfloat16_as_ushort(l) << 16);
}

// one 16-bit term of x (term 0: hi, 1: lo)
template <bool F16>
__device__ __forceinline__ uint16_t term16(float x, int term) {
    if (F16) {
        const __half h = __float2half_rn(x);
        return __half_as_ushort(term == 0 ? h : __float2half_rn(x - __half2float(h)));
    }
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    return __bfloat16_as_ushort(term == 0 ? h : __float2bfloat16_rn(x - __bfloat162float(h)));
}

}  // namespace bml
