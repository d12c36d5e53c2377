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

__global__ void diag_exp2_kernel(const float2 *__restrict__ x, uint32_t n2, float2 *__restrict__ out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n2) return;
    const float2 v = x[i];
    out[i] = make_float2(fast_exp2(v.x), fast_exp2(v.y));
}

// RoPE of gguf_compiler.rs:1290-1317 (interleaved pairs (2i, 2i+1) of each
// head, angle = pos * 10000^(-2i/d), rotation in f64) on q (in place) and k,
// then k and v stored into a cache slot -- the projection tail of
// gguf_compiler.rs:984-1006 for one token.  One thread per q pair, k pair
// and v element.  f32 -> f64 -> rotate -> f32 (as the reference's f64
// vectors land in its f32 cache) -> cache dtype.
// RoPE of one interleaved pair (x[2j], x[2j+1]) of a head at position pos:
// angle pos * 10000^(-2j/d), rotated in f64 and rounded to f32 once
// (gguf_compiler.rs:1290-1317 computes in f64 and stores f32).
__device__ __forceinline__ void rope_pair(float xe_f, float xo_f, uint32_t j, uint32_t d, uint32_t pos,
                                          float &re, float &ro) {
    const double xe = (double)xe_f, xo = (double)xo_f;
    const double freq = 1.0 / pow(10000.0, 2.0 * (double)j / (double)d);
    double sn, cs;
    sincos((double)pos * freq, &sn, &cs);
    re = (float)(xe * cs - xo * sn);
    ro = (float)(xe * sn + xo * cs);
}

template <typename Dt>
__global__ void rope_append_kernel(float *__restrict__ q, uint32_t nq2, const float *__restrict__ k,
                                   const float *__restrict__ v, Dt *__restrict__ kd, Dt *__restrict__ vd,
                                   uint32_t nk2, uint32_t nv, uint32_t d, uint32_t pos) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t half = d / 2;
    if (i < nq2 + nk2) {
        const bool is_q = i < nq2;
        const uint32_t pi = is_q ? i : i - nq2;  // pair index
        const uint32_t j = pi % half;            // pair within the head
        const uint32_t e = (pi / half) * d + 2 * j;
        const float *src = is_q ? q : k;
        float re, ro;
        rope_pair(src[e], src[e + 1], j, d, pos, re, ro);
        if (is_q) {
            q[e] = re;
            q[e + 1] = ro;
        } else {
            kd[e] = from_f32<Dt>(re);
            kd[e + 1] = from_f32<Dt>(ro);
        }
    } else if (i < nq2 + nk2 + nv) {
        const uint32_t e = i - nq2 - nk2;
        vd[e] = from_f32<Dt>(v[e]);
    }
}

// Row `len_i` of each sequence i of a batch gets that sequence's new K and V
// (one decode step's appends for a whole batch in one launch).
template <typename S, typename Dt>
__global__ void append_rows_kernel(const __grid_constant__ AppendRows p, const S *__restrict__ k_src,
                                   const S *__restrict__ v_src) {
    const uint32_t s = blockIdx.y;
    const size_t n = p.row;
    Dt *kd = static_cast<Dt *>(p.k[s]) + (size_t)p.len[s] * n;
    Dt *vd = static_cast<Dt *>(p.v[s]) + (size_t)p.len[s] * n;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        kd[i] = from_f32<Dt>(to_f32<S>(k_src[(size_t)s * n + i]));
        vd[i] = from_f32<Dt>(to_f32<S>(v_src[(size_t)s * n + i]));
    }
}

// The batched form of rope_append_kernel: sequence blockIdx.y rotates its q
// rows in place and its k row at position len[s], then stores k and v into
// row len[s] of its cache.
template <typename Dt>
__global__ void rope_append_rows_kernel(const __grid_constant__ AppendRows p, float *__restrict__ q,
                                        const float *__restrict__ k_src, const float *__restrict__ v_src) {
    const uint32_t s = blockIdx.y;
    const uint32_t d = p.head_dim, half = d / 2, pos = p.len[s];
    const uint32_t nq2 = p.n_heads * half, nk2 = p.row / 2, nv = p.row;
    float *qs = q + (size_t)s * p.n_heads * d;
    const float *ks = k_src + (size_t)s * p.row, *vs = v_src + (size_t)s * p.row;
    Dt *kd = static_cast<Dt *>(p.k[s]) + (size_t)pos * p.row;
    Dt *vd = static_cast<Dt *>(p.v[s]) + (size_t)pos * p.row;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nq2 + nk2 + nv; i += gridDim.x * blockDim.x) {
        if (i < nq2 + nk2) {
            const bool is_q = i < nq2;
            const uint32_t pi = is_q ? i : i - nq2;
            const uint32_t j = pi % half, e = (pi / half) * d + 2 * j;
            float re, ro;
            rope_pair(is_q ? qs[e] : ks[e], is_q ? qs[e + 1] : ks[e + 1], j, d, pos, re, ro);
            if (is_q) {
                qs[e] = re;
                qs[e + 1] = ro;
            } else {
                kd[e] = from_f32<Dt>(re);
                kd[e + 1] = from_f32<Dt>(ro);
            }
        } else {
            const uint32_t e = i - nq2 - nk2;
            vd[e] = from_f32<Dt>(vs[e]);
        }
    }
}

template <typename S>
cudaError_t append_rows_to(const AppendRows &p, const void *k, const void *v, bml_dtype dst_t, dim3 grid,
                           cudaStream_t st) {
    switch (dst_t) {
        case BML_F32: append_rows_kernel<S, float><<<grid, 256, 0, st>>>(p, (const S *)k, (const S *)v); break;
        case BML_F16: append_rows_kernel<S, __half><<<grid, 256, 0, st>>>(p, (const S *)k, (const S *)v); break;
        case BML_BF16:
            append_rows_kernel<S, __nv_bfloat16><<<grid, 256, 0, st>>>(p, (const S *)k, (const S *)v);
            break;
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t kv_append_rows(const AppendRows &p, uint32_t n_seqs, const void *k, const void *v, bml_dtype src_t,
                           bml_dtype dst_t, cudaStream_t st) {
    if (n_seqs == 0) return cudaSuccess;
    const dim3 grid((unsigned)((p.row + 255) / 256 < 64 ? (p.row + 255) / 256 : 64), n_seqs);
    switch (src_t) {
        case BML_F32: return append_rows_to<float>(p, k, v, dst_t, grid, st);
        case BML_F16: return append_rows_to<__half>(p, k, v, dst_t, grid, st);
        case BML_BF16: return append_rows_to<__nv_bfloat16>(p, k, v, dst_t, grid, st);
    }
    return cudaErrorInvalidValue;
}

cudaError_t kv_rope_append_rows(const AppendRows &p, uint32_t n_seqs, float *q, const float *k, const float *v,
                                bml_dtype dst_t, cudaStream_t st) {
    if (n_seqs == 0) return cudaSuccess;
    const uint32_t total = p.n_heads * p.head_dim / 2 + p.row / 2 + p.row;
    const dim3 grid((total + 255) / 256 < 32 ? (total + 255) / 256 : 32, n_seqs);
    switch (dst_t) {
        case BML_F32: rope_append_rows_kernel<float><<<grid, 256, 0, st>>>(p, q, k, v); break;
        case BML_F16: rope_append_rows_kernel<__half><<<grid, 256, 0, st>>>(p, q, k, v); break;
        case BML_BF16: rope_append_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p, q, k, v); break;
    }
    return cudaGetLastError();
}

cudaError_t kv_rope_append(float *q, uint32_t n_heads, const float *k, const float *v, void *kd, void *vd,
                           bml_dtype dst_t, uint32_t n_kv, uint32_t d, uint32_t pos, cudaStream_t st) {
    const uint32_t nq2 = n_heads * d / 2, nk2 = n_kv * d / 2, nv = n_kv * d;
    const uint32_t total = nq2 + nk2 + nv;
    const unsigned blocks = (total + 255) / 256;
    switch (dst_t) {
        case BML_F32:
            rope_append_kernel<float><<<blocks, 256, 0, st>>>(q, nq2, k, v, (float *)kd, (float *)vd, nk2, nv, d, pos);
            break;
        case BML_F16:
            rope_append_kernel<__half><<<blocks, 256, 0, st>>>(q, nq2, k, v, (__half *)kd, (__half *)vd, nk2, nv, d, pos);
            break;
        case BML_BF16:
            rope_append_kernel<__nv_bfloat16>
                <<<blocks, 256, 0, st>>>(q, nq2, k, v, (__nv_bfloat16 *)kd, (__nv_bfloat16 *)vd, nk2, nv, d, pos);
            break;
    }
    return cudaGetLastError();
}

cudaError_t diag_exp2(const float *x, uint32_t n, float *out, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const uint32_t n2 = n / 2;
    diag_exp2_kernel<<<(n2 + 255) / 256, 256, 0, st>>>(reinterpret_cast<const float2 *>(x), n2,
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
