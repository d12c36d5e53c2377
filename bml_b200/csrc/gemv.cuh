// gemv.cuh -- launch interface of the weight-path kernels (gemv.cu).
#pragma once

#include "common.cuh"

namespace bml {

// GGUF tensor type ids the reference reads as f32 (crates/parser/src/gguf.rs:36-43).
constexpr int kGgufF32 = 0, kGgufF16 = 1, kGgufQ4_0 = 2, kGgufQ8_0 = 8;

// Values read_tensor_f32 returns for a tensor of n_elems elements whose data
// is data_len bytes (0 for a type it does not read).
uint64_t gguf_values_read(int gguf_type, uint64_t data_len, uint64_t n_elems);
// Whole quantized blocks that decode (the rest of n_elems is zero).
uint64_t gguf_blocks_ok(int gguf_type, uint64_t data_len, uint64_t n_elems);

cudaError_t read_tensor_f32(const void *data, uint64_t data_len, int gguf_type, uint64_t n_elems, float *out,
                            cudaStream_t st);

struct GemvPlan {
    uint64_t rows;            // min(x_len, n_in)
    bool staged;              // 1024-column tiles through a shared-memory ring
    uint64_t col_tiles;       // 256- (or 1024-, staged) column tiles
    uint64_t rows_per_range;
    uint32_t ranges;          // row ranges summed by gemv_reduce_kernel
};
GemvPlan gemv_plan(uint64_t n_in, uint64_t n_out, uint64_t x_len, int num_sms, bool staged);
// The staged kernel applies: n_out % 256 == 0, W 16-byte aligned, and the
// data holds the whole n_in x n_out tensor.
bool gemv_staged_ok(const void *w, uint64_t data_len, int gguf_type, uint64_t n_in, uint64_t n_out);
// Scratch for the row-range partials: at most 160 ranges of n_out doubles.
size_t gemv_workspace_bytes(uint64_t n_out);

// y[j] = sum_i x[i] * W[i*n_out + j] over the tensor's values (see gemv.cu).
// Quantized types need n_out % 32 == 0 (cudaErrorNotSupported otherwise).
// static_weights: W is not written by the kernel launched just before on
// the stream, so the Q4_0 kernel may be launched as its programmatic
// dependent and start loading W while it ends (x and y wait for it).
cudaError_t gemv(const void *w, uint64_t data_len, int gguf_type, uint64_t n_in, uint64_t n_out, const double *x,
                 uint64_t x_len, double *y, double *partial, int num_sms, bool static_weights, cudaStream_t st);

}  // namespace bml
