/*
 * bml_diag.h -- test-only entry points of libbmlattn.so.
 *
 * None of these has a counterpart in the reference (SugarFreeDoNoSo/bml),
 * and a product caller has no use for them: they exist so that tests can
 * reach code paths that the product entry points choose by shape alone, or
 * that no valid input reaches (a bounded device wait that gives up).  Same
 * conventions as bml_attn.h.
 */
#ifndef BML_DIAG_H
#define BML_DIAG_H

#include <stddef.h>
#include <stdint.h>

#include "bml_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Kernel choices of bml_diag_decode_batched. */
#define BML_DIAG_DECODE_DEFAULT 0   /* what bml_attn_decode_batched picks */
#define BML_DIAG_DECODE_CUDA_CORE 1 /* the CUDA-core kernel, for any dtype */

/* Behaviour flags of bml_diag_decode_batched. */
#define BML_DIAG_STALL 1u /* the tensor-core kernel's producer fills no
                             stage, so its consumers' first wait runs out */

/* bml_attn_decode_batched with the kernel, the limit of every bounded
 * device wait (nanoseconds; 0 selects the default 2 s) and behaviour flags
 * chosen by the caller.  With BML_DIAG_STALL and a short limit the launch
 * ends by itself once the limit has passed, its output is not valid, and
 * bml_attn_workspace_check on the same workspace returns BML_E_TIMEOUT.
 * Asynchronous. */
bml_status bml_diag_decode_batched(const bml_seq_desc *seqs_host,
                                   uint32_t n_seqs, uint32_t n_heads,
                                   uint32_t n_kv_heads, uint32_t head_dim,
                                   bml_dtype kv_dtype, float scale,
                                   const float *q_dev, float *out_dev,
                                   void *workspace, size_t workspace_bytes,
                                   int kernel, uint64_t wait_ns,
                                   uint32_t flags, void *stream);

/* Evaluates 2^x with the device exponential the attention kernels use
 * (ex2.approx on the SFU), so tests can bound its error against CUDA's
 * exp2f.  n must be even.  Asynchronous. */
bml_status bml_diag_exp2(const float *x_dev, uint32_t n, float *out_dev,
                         void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BML_DIAG_H */
