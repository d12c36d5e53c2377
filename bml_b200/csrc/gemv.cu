// gemv.cu -- the reference's weight path on the device (sm_100a):
// read_tensor_f32 (GGUF F32 / F16 / Q4_0 / Q8_0 -> f32) and matmul_f64
// (y = x . W over a weight tensor), crates/compiler/src/gguf_compiler.rs:
// 351-470 and :1239-1255 in SugarFreeDoNoSo/bml.
//
// Layout.  The reference keeps a tensor's values in file order and reads
// W[i][j] at flat index i*n_out + j, where (n_in, n_out) = (dims[0],
// dims[1]) -- so row i of W is n_out consecutive values, and a quantized
// block (32 consecutive values) covers 32 consecutive columns of one row
// when n_out is a multiple of 32.
//
// Dequantisation follows the reference bit for bit: f16 scales widen
// exactly, Q4_0 byte i of a block holds elements 2i (low nibble) and 2i+1
// (high nibble), value (q - 8) * scale; Q8_0 value q * scale; blocks that do
// not fit in the data are zero.
//
// GEMV (HBM-bound: every weight byte is read once, ~2 flops per element).
// The quantized tensor is read as stored -- 0.5625 bytes per value for
// Q4_0 instead of the 4 bytes of the reference's dequantised f32 pool.  A
// CTA owns 256 columns (8 blocks of 32) and a range of rows; thread t takes
// block t % 8 and rows r = t / 8 (mod 32) of the range, keeping 32 f32 sums.
// Each term is x[i] * scale (f32, once per block and row) times (q - 8) or
// q, the small integer made exact with the 2^23 magic-number trick (no
// int-to-float conversion unit in the loop).  The 32 row phases are summed
// in f64 in a fixed order, and the row ranges (when a tensor needs several
// CTAs per column range to fill the GPU) go to a workspace in f64 and are
// summed in range order by a second kernel, so results do not vary between
// runs; against the reference's f64 sums they differ by f32 rounding of the
// terms and partial sums (about 1e-7 of sum |x_i W_ij|).
#include "gemv.cuh"

namespace bml {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kColBlocks = 8;                  // 32-column blocks per CTA
constexpr int kCols = kColBlocks * 32;         // columns per CTA
constexpr int kRowPhases = kGemvThreads / kColBlocks;  // 32

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Exact small integers as floats: 2^23 + u has u in its low mantissa bits.
__device__ __forceinline__ float magic_u(uint32_t u) { return __uint_as_float(0x4B000000u | u) - 8388608.0f; }

// ------------------------------------------------------------ dequant
// One thread per 32-value block.
template <int QT>
__global__ void dequant_q_kernel(const uint8_t *__restrict__ data, uint64_t n_blocks_ok, uint64_t n_elems,
                                 float *__restrict__ out) {
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t n_blocks = (n_elems + 31) / 32;
    if (b >= n_blocks) return;
    float v[32];
    if (b < n_blocks_ok) {
        constexpr uint32_t BB = QT == kGgufQ4_0 ? 18u : 34u;
        const uint16_t *blk = reinterpret_cast<const uint16_t *>(data + b * BB);  // 2-byte aligned
        const float scale = f16_bits_to_f32(blk[0]);
        if (QT == kGgufQ4_0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t two = blk[1 + i];  // bytes 2i, 2i+1 of the 16 nibble bytes
#pragma unroll
                for (int k = 0; k < 4; ++k) v[4 * i + k] = (magic_u((two >> (4 * k)) & 15u) - 8.0f) * scale;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t two = blk[1 + i];
#pragma unroll
                for (int k = 0; k < 2; ++k) v[2 * i + k] = (magic_u(((two >> (8 * k)) & 255u) ^ 128u) - 128.0f) * scale;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
    }
    const uint64_t base = b * 32;
    if (base + 32 <= n_elems) {
        float4 *o = reinterpret_cast<float4 *>(out + base);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
        for (int i = 0; i < 32 && base + i < n_elems; ++i) out[base + i] = v[i];
    }
}

__global__ void dequant_f16_kernel(const uint16_t *__restrict__ data, uint64_t n, float *__restrict__ out) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = f16_bits_to_f32(data[i]);
}

// ------------------------------------------------------------ GEMV
// The 32 values of W in row i, columns [32*cb, 32*cb + 32), times xs.
template <int QT>
struct Block32 {
    __device__ __forceinline__ static void fma(const uint8_t *__restrict__ w, uint64_t row, uint64_t n_out,
                                               uint64_t cb, uint64_t n_blocks_ok, double x, float acc[32]) {
        const uint64_t b = row * (n_out / 32) + cb;
        if (b >= n_blocks_ok) return;  // past the data: zeros
        constexpr uint32_t BB = QT == kGgufQ4_0 ? 18u : 34u;
        const uint16_t *blk = reinterpret_cast<const uint16_t *>(w + b * BB);
        const float xs = (float)x * f16_bits_to_f32(__ldg(blk));
        if (QT == kGgufQ4_0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t two = __ldg(blk + 1 + i);
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[4 * i + k] = fmaf(xs, magic_u((two >> (4 * k)) & 15u) - 8.0f,
                                                                  acc[4 * i + k]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t two = __ldg(blk + 1 + i);
#pragma unroll
                for (int k = 0; k < 2; ++k)
                    acc[2 * i + k] = fmaf(xs, magic_u(((two >> (8 * k)) & 255u) ^ 128u) - 128.0f, acc[2 * i + k]);
            }
        }
    }
};

template <>
struct Block32<kGgufF32> {
    __device__ __forceinline__ static void fma(const uint8_t *__restrict__ w, uint64_t row, uint64_t n_out,
                                               uint64_t cb, uint64_t n_vals, double x, float acc[32]) {
        const uint64_t e0 = row * n_out + cb * 32;
        if (e0 >= n_vals) return;
        const float xf = (float)x;
        const float *p = reinterpret_cast<const float *>(w) + e0;
        if (e0 + 32 <= n_vals && (n_out % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 q = __ldg(reinterpret_cast<const float4 *>(p) + i);
                acc[4 * i] = fmaf(xf, q.x, acc[4 * i]);
                acc[4 * i + 1] = fmaf(xf, q.y, acc[4 * i + 1]);
                acc[4 * i + 2] = fmaf(xf, q.z, acc[4 * i + 2]);
                acc[4 * i + 3] = fmaf(xf, q.w, acc[4 * i + 3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (e0 + i < n_vals) acc[i] = fmaf(xf, __ldg(p + i), acc[i]);
        }
    }
};

template <>
struct Block32<kGgufF16> {
    __device__ __forceinline__ static void fma(const uint8_t *__restrict__ w, uint64_t row, uint64_t n_out,
                                               uint64_t cb, uint64_t n_vals, double x, float acc[32]) {
        const uint64_t e0 = row * n_out + cb * 32;
        if (e0 >= n_vals) return;
        const float xf = (float)x;
        const uint16_t *p = reinterpret_cast<const uint16_t *>(w) + e0;
        if (e0 + 32 <= n_vals && (n_out % 8) == 0) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 q = __ldg(reinterpret_cast<const uint4 *>(p) + i);
                const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wd[k]));
                    acc[8 * i + 2 * k] = fmaf(xf, f.x, acc[8 * i + 2 * k]);
                    acc[8 * i + 2 * k + 1] = fmaf(xf, f.y, acc[8 * i + 2 * k + 1]);
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (e0 + i < n_vals) acc[i] = fmaf(xf, f16_bits_to_f32(__ldg(p + i)), acc[i]);
        }
    }
};

// grid (column tiles, row ranges); partial[range][n_out] (or y when there
// is one range).
template <int QT>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const uint8_t *__restrict__ w, uint64_t n_ok,
                                                            uint64_t n_out, uint64_t rows, uint64_t rows_per_range,
                                                            const double *__restrict__ x, double *__restrict__ dst) {
    __shared__ float part[kRowPhases][kCols + 1];
    const int tid = threadIdx.x;
    const int cbl = tid % kColBlocks, rp = tid / kColBlocks;
    const uint64_t cb = (uint64_t)blockIdx.x * kColBlocks + cbl;  // global 32-column block
    const uint64_t n_cb = (n_out + 31) / 32;
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_range;
    const uint64_t r1 = min(r0 + rows_per_range, rows);
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    if (cb < n_cb) {
        for (uint64_t r = r0 + rp; r < r1; r += kRowPhases) Block32<QT>::fma(w, r, n_out, cb, n_ok, __ldg(x + r), acc);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) part[rp][cbl * 32 + i] = acc[i];
    __syncthreads();
    // one column per thread: the 32 row phases in order, in f64
    const uint64_t j = (uint64_t)blockIdx.x * kCols + tid;
    if (j < n_out) {
        double s = 0.0;
#pragma unroll 8
        for (int k = 0; k < kRowPhases; ++k) s += (double)part[k][tid];
        dst[(uint64_t)blockIdx.y * n_out + j] = s;
    }
}

__global__ void gemv_reduce_kernel(const double *__restrict__ partial, uint32_t n_ranges, uint64_t n_out,
                                   double *__restrict__ y) {
    const uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n_out) return;
    double s = 0.0;
    for (uint32_t r = 0; r < n_ranges; ++r) s += partial[(uint64_t)r * n_out + j];
    y[j] = s;
}

}  // namespace

uint64_t gguf_values_read(int gguf_type, uint64_t data_len, uint64_t n_elems) {
    switch (gguf_type) {
        case kGgufF32: return data_len / 4;
        case kGgufF16: return data_len / 2;
        case kGgufQ4_0:
        case kGgufQ8_0: return n_elems;
        default: return 0;
    }
}

uint64_t gguf_blocks_ok(int gguf_type, uint64_t data_len, uint64_t n_elems) {
    const uint64_t bb = gguf_type == kGgufQ4_0 ? 18 : 34;
    const uint64_t whole = n_elems / 32;
    const uint64_t fit = data_len / bb;
    return whole < fit ? whole : fit;
}

cudaError_t read_tensor_f32(const void *data, uint64_t data_len, int gguf_type, uint64_t n_elems, float *out,
                            cudaStream_t st) {
    const uint64_t n = gguf_values_read(gguf_type, data_len, n_elems);
    if (n == 0) return cudaSuccess;
    switch (gguf_type) {
        case kGgufF32: return cudaMemcpyAsync(out, data, n * 4, cudaMemcpyDeviceToDevice, st);
        case kGgufF16: {
            const unsigned blocks = (unsigned)std::min<uint64_t>((n + 255) / 256, 148u * 16u);
            dequant_f16_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint16_t *>(data), n, out);
            return cudaGetLastError();
        }
        case kGgufQ4_0:
        case kGgufQ8_0: {
            const uint64_t ok = gguf_blocks_ok(gguf_type, data_len, n_elems);
            const uint64_t nb = (n_elems + 31) / 32;
            const unsigned blocks = (unsigned)((nb + 255) / 256);
            if (gguf_type == kGgufQ4_0)
                dequant_q_kernel<kGgufQ4_0><<<blocks, 256, 0, st>>>(static_cast<const uint8_t *>(data), ok, n_elems, out);
            else
                dequant_q_kernel<kGgufQ8_0><<<blocks, 256, 0, st>>>(static_cast<const uint8_t *>(data), ok, n_elems, out);
            return cudaGetLastError();
        }
        default: return cudaErrorInvalidValue;
    }
}

GemvPlan gemv_plan(uint64_t n_in, uint64_t n_out, uint64_t x_len, int num_sms) {
    GemvPlan pl;
    pl.rows = x_len < n_in ? x_len : n_in;
    pl.col_tiles = (n_out + kCols - 1) / kCols;
    // enough CTAs for ~2 per SM, at least 128 rows a range, at most 32 ranges
    uint64_t ranges = (2ull * num_sms + pl.col_tiles - 1) / pl.col_tiles;
    const uint64_t by_rows = (pl.rows + 127) / 128;
    if (ranges > by_rows) ranges = by_rows;
    if (ranges > 32) ranges = 32;
    if (ranges < 1) ranges = 1;
    pl.rows_per_range = (pl.rows + ranges - 1) / ranges;
    pl.ranges = pl.rows_per_range ? (uint32_t)((pl.rows + pl.rows_per_range - 1) / pl.rows_per_range) : 1;
    return pl;
}

size_t gemv_workspace_bytes(uint64_t n_out) { return (size_t)32 * n_out * sizeof(double); }

cudaError_t gemv(const void *w, uint64_t data_len, int gguf_type, uint64_t n_in, uint64_t n_out, const double *x,
                 uint64_t x_len, double *y, double *partial, int num_sms, cudaStream_t st) {
    const GemvPlan pl = gemv_plan(n_in, n_out, x_len, num_sms);
    if (pl.rows == 0) return cudaMemsetAsync(y, 0, n_out * sizeof(double), st);
    uint64_t n_ok = 0;
    if (gguf_type == kGgufQ4_0 || gguf_type == kGgufQ8_0) {
        if (n_out % 32 != 0) return cudaErrorNotSupported;
        n_ok = gguf_blocks_ok(gguf_type, data_len, n_in * n_out);
    } else {
        n_ok = gguf_values_read(gguf_type, data_len, 0);
    }
    double *dst = pl.ranges == 1 ? y : partial;
    const dim3 grid((unsigned)pl.col_tiles, pl.ranges);
    const uint8_t *wb = static_cast<const uint8_t *>(w);
    switch (gguf_type) {
        case kGgufF32: gemv_kernel<kGgufF32><<<grid, kGemvThreads, 0, st>>>(wb, n_ok, n_out, pl.rows, pl.rows_per_range, x, dst); break;
        case kGgufF16: gemv_kernel<kGgufF16><<<grid, kGemvThreads, 0, st>>>(wb, n_ok, n_out, pl.rows, pl.rows_per_range, x, dst); break;
        case kGgufQ4_0: gemv_kernel<kGgufQ4_0><<<grid, kGemvThreads, 0, st>>>(wb, n_ok, n_out, pl.rows, pl.rows_per_range, x, dst); break;
        case kGgufQ8_0: gemv_kernel<kGgufQ8_0><<<grid, kGemvThreads, 0, st>>>(wb, n_ok, n_out, pl.rows, pl.rows_per_range, x, dst); break;
        default: return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || pl.ranges == 1) return e;
    gemv_reduce_kernel<<<(unsigned)((n_out + 255) / 256), 256, 0, st>>>(partial, pl.ranges, n_out, y);
    return cudaGetLastError();
}

}  // namespace bml
