// kv_cache.cu -- device side of the KV-cache handle and softmax_f32.
//
// Restates on the GPU the per-slot accessors of HashConsedKV
// (crates/compiler/src/kv_cache.rs:82-141 in SugarFreeDoNoSo/bml) and
// softmax_f32 (kv_cache.rs:188-200).  These are small memory-bound
// kernels; the hot path is decode.cu / prefill.cu.
#include <math.h>

#include "kv_ops.cuh"

namespace bml {

namespace {

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Copies n elements src (type S) -> dst (type D) with rounding to nearest.
template <typename S, typename Dt>
__global__ void convert_kernel(const S *__restrict__ src, Dt *__restrict__ dst, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = from_f32<Dt>(to_f32<S>(src[i]));
}

template <typename S>
cudaError_t convert_to(const S *src, void *dst, bml_dtype dst_t, size_t n, cudaStream_t st) {
    const int threads = 256;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads < 4096 ? (n + threads - 1) / threads : 4096);
    if (n == 0) return cudaSuccess;
    switch (dst_t) {
        case BML_F32: convert_kernel<S, float><<<blocks, threads, 0, st>>>(src, (float *)dst, n); break;
        case BML_F16: convert_kernel<S, __half><<<blocks, threads, 0, st>>>(src, (__half *)dst, n); break;
        case BML_BF16:
            convert_kernel<S, __nv_bfloat16><<<blocks, threads, 0, st>>>(src, (__nv_bfloat16 *)dst, n);
            break;
    }
    return cudaGetLastError();
}

// dot_qk (kv_cache.rs:135-141): one warp; f32 products, f32 sums.
template <typename T>
__global__ void dot_kernel(const float *__restrict__ q, const T *__restrict__ k, uint32_t n,
                           float *__restrict__ out) {
    float acc = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += 32) acc += q[i] * to_f32<T>(k[i]);
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (threadIdx.x == 0) *out = acc;
}

// softmax_f32 (kv_cache.rs:188-200), one CTA per row.  f32::max ignores
// NaN, as fmaxf does; when the sum is not positive (all -inf, or a NaN
// anywhere) the row is uniform 1/n, as in the reference.
__global__ void softmax_kernel(const float *__restrict__ x, uint32_t n, float *__restrict__ out) {
    __shared__ float red[32];
    const float *row = x + (size_t)blockIdx.x * n;
    float *orow = out + (size_t)blockIdx.x * n;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;

    float mx = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, row[i]);
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (warp == 0) {
        float v = lane < nw ? red[lane] : -INFINITY;
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    mx = red[0];
    __syncthreads();

    float sum = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(row[i] - mx);
        orow[i] = e;
        sum += e;
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    if (warp == 0) {
        float v = lane < nw ? red[lane] : 0.f;
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    sum = red[0];
    const bool ok = sum > 0.f;
    const float inv_n = 1.0f / (float)n;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) orow[i] = ok ? orow[i] / sum : inv_n;
}

__global__ void diag_exp2_kernel(const float2 *__restrict__ x, uint32_t n2, int method, float2 *__restrict__ out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n2) return;
    const float2 v = x[i];
    out[i] = method == 1 ? exp2_poly2(v) : make_float2(fast_exp2(v.x), fast_exp2(v.y));
}

}  // namespace

cudaError_t diag_exp2(const float *x, uint32_t n, int method, float *out, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const uint32_t n2 = n / 2;
    diag_exp2_kernel<<<(n2 + 255) / 256, 256, 0, st>>>(reinterpret_cast<const float2 *>(x), n2, method,
                                                        reinterpret_cast<float2 *>(out));
    return cudaGetLastError();
}

cudaError_t kv_store_from_f32(const float *src_dev, void *dst_dev, bml_dtype dst_t, size_t n,
                              cudaStream_t st) {
    return convert_to<float>(src_dev, dst_dev, dst_t, n, st);
}

cudaError_t kv_convert(const void *src_dev, bml_dtype src_t, void *dst_dev, bml_dtype dst_t, size_t n,
                       cudaStream_t st) {
    switch (src_t) {
        case BML_F32: return convert_to<float>((const float *)src_dev, dst_dev, dst_t, n, st);
        case BML_F16: return convert_to<__half>((const __half *)src_dev, dst_dev, dst_t, n, st);
        case BML_BF16: return convert_to<__nv_bfloat16>((const __nv_bfloat16 *)src_dev, dst_dev, dst_t, n, st);
    }
    return cudaErrorInvalidValue;
}

cudaError_t kv_dot(const float *q_dev, const void *k_dev, bml_dtype t, uint32_t n, float *out_dev,
                   cudaStream_t st) {
    switch (t) {
        case BML_F32: dot_kernel<float><<<1, 32, 0, st>>>(q_dev, (const float *)k_dev, n, out_dev); break;
        case BML_F16: dot_kernel<__half><<<1, 32, 0, st>>>(q_dev, (const __half *)k_dev, n, out_dev); break;
        case BML_BF16:
            dot_kernel<__nv_bfloat16><<<1, 32, 0, st>>>(q_dev, (const __nv_bfloat16 *)k_dev, n, out_dev);
            break;
    }
    return cudaGetLastError();
}

cudaError_t softmax_rows(const float *x_dev, uint32_t n_rows, uint32_t n, float *out_dev, cudaStream_t st) {
    if (n_rows == 0 || n == 0) return cudaSuccess;
    softmax_kernel<<<n_rows, 256, 0, st>>>(x_dev, n, out_dev);
    return cudaGetLastError();
}

}  // namespace bml
