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
cudaError_t kv_rope_append(float *q, uint32_t n_heads, const float *k, const float *v, void *kd, void *vd,
                           bml_dtype dst_t, uint32_t n_kv, uint32_t d, uint32_t pos, cudaStream_t st);
cudaError_t diag_exp2(const float *x, uint32_t n, int method, float *out, cudaStream_t st);
cudaError_t softmax_rows(const float *x_dev, uint32_t n_rows, uint32_t n, float *out_dev, cudaStream_t st);

}  // namespace bml
