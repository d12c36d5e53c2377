/*
 * bml_weights.h -- C ABI of the weight path of libbmlattn.so: GGUF tensor
 * dequantisation and the x . W projections, on the device.
 *
 * Reference interface replaced (paths inside the SugarFreeDoNoSo/bml
 * project):
 *   crates/compiler/src/gguf_compiler.rs:351-470  read_tensor_f32 with
 *                                                  f16_to_f32,
 *                                                  dequantize_q4_0,
 *                                                  dequantize_q8_0
 *   crates/compiler/src/gguf_compiler.rs:1239-1255 InferenceCompiler::
 *                                                  matmul_f64 (the Q, K,
 *                                                  V, O and MLP
 *                                                  projections of
 *                                                  forward_layer_cached)
 *
 * Conventions are those of bml_attn.h (status codes, bml_last_error,
 * device pointers, asynchronous on `stream`).  gguf_type is the GGUF tensor
 * type id (crates/parser/src/gguf.rs:36-43); the reference reads F32 (0),
 * F16 (1), Q4_0 (2) and Q8_0 (8) and nothing else, and so does this ABI
 * (others return BML_E_UNSUPPORTED).
 */
#ifndef BML_WEIGHTS_H
#define BML_WEIGHTS_H

#include "bml_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

#define BML_GGUF_F32  0
#define BML_GGUF_F16  1
#define BML_GGUF_Q4_0 2
#define BML_GGUF_Q8_0 8

/* read_tensor_f32 (gguf_compiler.rs:351-369): a tensor's data (data_len
 * bytes at data_dev, 2-byte aligned; 4-byte aligned for F32) to f32 values
 * at out_dev.  F32 / F16 give data_len / 4 or / 2 values; Q4_0 / Q8_0 give
 * n_elems values: whole 32-value blocks that fit in data_len decode
 * bit-exactly as the reference does (Q4_0 byte i holds values 2i and 2i+1
 * in its low and high nibble, (q - 8) * scale; Q8_0 q * scale), the rest
 * are zero.  *n_values (host) receives the count; out_dev must hold it. */
bml_status bml_read_tensor_f32(const void *data_dev, uint64_t data_len,
                               int32_t gguf_type, uint64_t n_elems,
                               float *out_dev, uint64_t *n_values,
                               void *stream);

/* Scratch bytes bml_matmul_f64 needs for an n_out-column tensor. */
bml_status bml_matmul_workspace_size(uint64_t n_out, size_t *bytes);

/* matmul_f64 (gguf_compiler.rs:1239-1255) straight from the stored tensor:
 * y[j] = sum over i < min(x_len, n_in) of x[i] * W[i*n_out + j], where W is
 * the tensor's values as bml_read_tensor_f32 gives them ((n_in, n_out) =
 * (dims[0], dims[1]), the reference's indexing) and values past the data
 * count as zero.  x_dev, y_dev: f64 device vectors (x_len, n_out).
 * Quantized tensors are read in place (no f32 copy) and need n_out % 32 ==
 * 0.  Terms and partial sums are f32 and the combination f64: results are
 * within ~1e-7 of sum |x_i W_ij| of the reference's f64 sums, and
 * identical from run to run.  workspace: bml_matmul_workspace_size bytes,
 * no initial contents needed; calls sharing it must not overlap. */
bml_status bml_matmul_f64(const void *w_dev, uint64_t data_len,
                          int32_t gguf_type, uint64_t n_in, uint64_t n_out,
                          const double *x_dev, uint64_t x_len, double *y_dev,
                          void *workspace, size_t ws_bytes, void *stream);

/* bml_matmul_f64 with the same arguments and the same result bits, for a
 * weight tensor that no kernel writes while calls are queued (weights
 * uploaded once and read by many calls).  The call may start streaming W
 * while the kernel launched just before it on `stream` is still running
 * (CUDA programmatic dependent launch); x_dev is read and y_dev written
 * only after that kernel has ended, so x may be that kernel's output.
 * Back-to-back projections of a decode step overlap one's start with the
 * previous one's end this way.  W must not be written by the kernel
 * launched immediately before the call. */
bml_status bml_matmul_f64_static(const void *w_dev, uint64_t data_len,
                                 int32_t gguf_type, uint64_t n_in,
                                 uint64_t n_out, const double *x_dev,
                                 uint64_t x_len, double *y_dev,
                                 void *workspace, size_t ws_bytes,
                                 void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BML_WEIGHTS_H */
