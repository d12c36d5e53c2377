// prefill.cuh -- launch interface of the tcgen05 causal prefill kernel.
#pragma once

#include "common.cuh"

namespace bml {

struct PrefillArgs {
    const void *q;  // [n_seqs][seq_len][n_heads][head_dim] 16-bit
    const void *k;  // [n_seqs][seq_len][n_kv][head_dim]
    const void *v;
    void *out;      // [n_seqs][seq_len][n_heads][head_dim] f32 or 16-bit
    uint32_t n_seqs, seq_len, n_heads, n_kv, head_dim;
    bml_dtype in_dtype, out_dtype;
    float scale;
    bool causal;
    int num_sms;
};

cudaError_t launch_prefill(const PrefillArgs &a, cudaStream_t stream);

}  // namespace bml
