// kv_ops.cuh -- launch interface of the KV-cache and softmax kernels.
#pragma once

#include "common.cuh"

namespace bml {

cudaError_t kv_store_from_f32(const float *src_dev, void *dst_dev, bml_dtype dst_t, size_t n,
                              cudaStream_t st);
cudaError_t kv_convert(const void *src_dev, bml_dtype src_t, void *dst_dev, bml_dtype dst_t, size_t n,
                       cudaStream_t st);
cudaError_t kv_dot(const float *q_dev, const void *k_dev, bml_dtype t, uint32_t n, float *out_dev,
                   cudaStream_t st);
// Destinations of a batched append: row len[i] of sequence i's K and V
// buffers ([.][n_kv][D] in the cache dtype), row = n_kv * D elements.
constexpr int kMaxAppendSeqs = 256;
struct AppendRows {
    void *k[kMaxAppendSeqs];
    void *v[kMaxAppendSeqs];
    uint32_t len[kMaxAppendSeqs];
    uint32_t row;       // n_kv * head_dim
    uint32_t n_heads;   // q heads (RoPE form only)
    uint32_t head_dim;
};
cudaError_t kv_append_rows(const AppendRows &p, uint32_t n_seqs, const void *k, const void *v, bml_dtype src_t,
                           bml_dtype dst_t, cudaStream_t st);
// Batched RoPE append: q [n_seqs][n_heads][head_dim] f32 rotated in place at
// each sequence's position len[s]; k, v [n_seqs][row] f32.
cudaError_t kv_rope_append_rows(const AppendRows &p, uint32_t n_seqs, float *q, const float *k, const float *v,
                                bml_dtype dst_t, cudaStream_t st);
cudaError_t kv_rope_append(float *q, uint32_t n_heads, const float *k, const float *v, void *kd, void *vd,
                           bml_dtype dst_t, uint32_t n_kv, uint32_t d, uint32_t pos, cudaStream_t st);
cudaError_t diag_exp2(const float *x, uint32_t n, float *out, cudaStream_t st);
cudaError_t softmax_rows(const float *x_dev, uint32_t n_rows, uint32_t n, float *out_dev, cudaStream_t st);

}  // namespace bml
