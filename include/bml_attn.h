/*
 * bml_attn.h -- C ABI of the B200 attention / KV-cache library
 * (libbmlattn.so, built from bml_b200/csrc for sm_100a).
 *
 * This is the drop-in boundary for bml's attention hot path.  Each entry
 * point names the reference interface it replaces (paths inside the
 * SugarFreeDoNoSo/bml project).  The reference surface is
 *   crates/compiler/src/kv_cache.rs:25-200  (HashConsedKV, softmax_f32,
 *                                            re-exported at lib.rs:33)
 *   crates/compiler/src/gguf_compiler.rs:1008-1050
 *                                           (attention block of
 *                                            forward_layer_cached, reached
 *                                            from forward_cached :929-962)
 *
 * Conventions
 *  - Every function returns a bml_status and never aborts.  Arguments are
 *    validated on the host before anything is launched; a rejected call
 *    returns BML_E_INVALID (where the Rust code would panic, or where this
 *    library declines a shape the reference silently mis-indexes) and
 *    leaves all outputs untouched.  bml_last_error() gives the reason
 *    (thread-local, valid until the next call on that thread).
 *  - "dev" pointers are CUDA device pointers, "host" pointers are host
 *    memory.  The caller owns every pointer it passes.  The library owns
 *    only the device buffers behind a bml_kv handle.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *    stream).  Device-pointer entry points are asynchronous on that stream;
 *    entry points taking host buffers synchronise before returning.
 *  - Layouts are row-major.  A KV cache or K/V tensor is
 *    [position][kv_head][head_dim] (kv_cache.rs:17); queries and outputs
 *    are [head][head_dim] per token (gguf_compiler.rs:1017-1024).
 *  - Scores are scaled by `scale`; pass a negative scale for the
 *    reference's 1/sqrt(head_dim) (gguf_compiler.rs:1010).
 *  - n_heads must be a multiple of n_kv_heads; q head h reads kv head
 *    h / (n_heads / n_kv_heads) (gguf_compiler.rs:1011,1016).
 */
#ifndef BML_ATTN_H
#define BML_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t bml_status;
#define BML_OK            0
#define BML_E_INVALID     1 /* bad argument / shape; nothing launched        */
#define BML_E_CUDA        2 /* a CUDA runtime call failed                    */
#define BML_E_NCCL        3 /* reserved for communicator errors              */
#define BML_E_TIMEOUT     4 /* a bounded device-side wait gave up            */
#define BML_E_OOM         5 /* device allocation failed                      */
#define BML_E_UNSUPPORTED 6 /* valid shape the library has no kernel for    */

typedef enum bml_dtype { BML_F32 = 0, BML_F16 = 1, BML_BF16 = 2 } bml_dtype;

#define BML_WHICH_K 0
#define BML_WHICH_V 1

/* ------------------------------------------------------------------------ */
/* Library                                                                  */
/* ------------------------------------------------------------------------ */

/* Reason for the last non-OK status on this thread ("" if none). */
const char *bml_last_error(void);

/* Library version string. */
const char *bml_version(void);

/* ------------------------------------------------------------------------ */
/* KV cache handle  (HashConsedKV, kv_cache.rs:25-181)                       */
/* ------------------------------------------------------------------------ */

typedef struct bml_kv bml_kv;

typedef struct bml_kv_desc {
    uint32_t n_layers;
    uint32_t n_kv_heads;
    uint32_t head_dim;
    uint32_t max_seq_len;
    bml_dtype dtype; /* storage type of K and V; the reference stores f32 */
    int32_t device;  /* CUDA device ordinal                               */
} bml_kv_desc;

/* HashConsedKV::new (kv_cache.rs:53-72): zero-filled per-layer K and V
 * buffers of max_seq_len * n_kv_heads * head_dim elements each. */
bml_status bml_kv_create(const bml_kv_desc *desc, bml_kv **out);

/* Drop of HashConsedKV: frees the device buffers. NULL is accepted. */
bml_status bml_kv_destroy(bml_kv *kv);

/* store_k / store_v (kv_cache.rs:82-101): writes one head vector from host
 * memory into ring slot pos % max_seq_len and counts the store.  len must
 * be >= head_dim (the reference's copy_from_slice panics otherwise); the
 * first head_dim values are stored, converted to the cache dtype.
 * Synchronous. */
bml_status bml_kv_store(bml_kv *kv, int which, uint32_t layer, uint32_t pos,
                        uint32_t kv_head, const float *host_data, size_t len);

/* load_k / load_v (kv_cache.rs:111-124): copies one head vector (widened
 * to f32) into a caller buffer of head_dim floats.  Synchronous. */
bml_status bml_kv_load(const bml_kv *kv, int which, uint32_t layer,
                       uint32_t pos, uint32_t kv_head, float *host_out);

/* dot_qk (kv_cache.rs:135-141): f32 dot of q (host, q_len floats; the
 * shorter length wins) with K[layer][pos % max][kv_head].  Synchronous. */
bml_status bml_kv_dot_qk(const bml_kv *kv, const float *host_q, size_t q_len,
                         uint32_t layer, uint32_t pos, uint32_t kv_head,
                         float *out);

/* k_stats / v_stats (kv_cache.rs:148-155): (stores, stores, 1.0). */
bml_status bml_kv_stats(const bml_kv *kv, int which, uint64_t *unique,
                        uint64_t *total, double *ratio);

/* byte_size (kv_cache.rs:158-161): bytes of all K and V buffers. */
bml_status bml_kv_byte_size(const bml_kv *kv, uint64_t *out);

/* current_pos / advance / advance_by (kv_cache.rs:168-180). */
bml_status bml_kv_current_pos(const bml_kv *kv, uint32_t *out);
bml_status bml_kv_advance(bml_kv *kv);
bml_status bml_kv_advance_by(bml_kv *kv, uint32_t n);

/* Device address of one layer's K or V buffer
 * ([max_seq_len][n_kv_heads][head_dim] in the cache dtype). */
bml_status bml_kv_layer_ptr(const bml_kv *kv, int which, uint32_t layer,
                            void **dev_out);

/* Device-side store of every kv head of one position (the n_kv_heads
 * store_k/store_v calls of gguf_compiler.rs:994-1006 in one launch).
 * k_dev/v_dev: [n_kv_heads][head_dim] in src_dtype, converted to the cache
 * dtype.  Asynchronous on stream. */
bml_status bml_kv_append(bml_kv *kv, uint32_t layer, uint32_t pos,
                         const void *k_dev, const void *v_dev,
                         bml_dtype src_dtype, void *stream);

/* The projection tail of one token in one launch (gguf_compiler.rs:984-1006
 * with apply_rope_inplace, :1290-1317): RoPE -- interleaved pairs
 * (2i, 2i+1) of each head, angle = pos * 10000^(-2i/head_dim), rotated in
 * f64 -- applied to q in place and to k, then k and v stored into the slot
 * of `pos` like bml_kv_append.  q_dev: [n_heads][head_dim] f32 (n_heads a
 * multiple of n_kv_heads); k_dev (before RoPE), v_dev:
 * [n_kv_heads][head_dim] f32.  Asynchronous on stream. */
bml_status bml_kv_append_rope(bml_kv *kv, uint32_t layer, uint32_t pos,
                              float *q_dev, uint32_t n_heads,
                              const float *k_dev, const float *v_dev,
                              void *stream);

/* ------------------------------------------------------------------------ */
/* Decode attention  (gguf_compiler.rs:1008-1050)                           */
/* ------------------------------------------------------------------------ */

/* The attention block of forward_layer_cached for the token at position
 * pos: every q head attends over K/V positions [0, pos] of `layer`
 * (causal), softmax, P.V.  q_dev: [n_heads][head_dim] f32, out_dev:
 * [n_heads][head_dim] f32.  pos must be < max_seq_len (for the reference's
 * ring wrap past max_seq_len, kv_cache.rs:83, use bml_attn_decode_wrap).
 * Uses the handle's own scratch, so calls on one handle must not overlap in
 * time.  Asynchronous. */
bml_status bml_attn_decode(bml_kv *kv, uint32_t layer, uint32_t pos,
                           uint32_t n_heads, float scale, const float *q_dev,
                           float *out_dev, void *stream);

/* bml_attn_decode for any pos, with the reference's behaviour past the end
 * of the ring: its loop (gguf_compiler.rs:1026-1049) runs over positions
 * 0..pos and reads each through slot p % max_seq_len (kv_cache.rs:83), so
 * once pos >= max_seq_len every slot enters the softmax floor(n / M) or
 * floor(n / M) + 1 times (n = pos + 1, M = max_seq_len; the extra visit for
 * slots below n % M).  Computed as attention over the M slots with each
 * slot's weight scaled by its visit count: two KV-split partials merged
 * with the counts.  pos < max_seq_len is bml_attn_decode itself.  Uses the
 * handle's own scratch (allocated on first use), so calls on one handle
 * must not overlap in time.  Asynchronous. */
bml_status bml_attn_decode_wrap(bml_kv *kv, uint32_t layer, uint32_t pos,
                                uint32_t n_heads, float scale,
                                const float *q_dev, float *out_dev,
                                void *stream);

/* One sequence of a batched decode: a contiguous cache
 * [len][n_kv_heads][head_dim] (K and V), whose query token sits at
 * position len-1 and attends over all len positions. */
typedef struct bml_seq_desc {
    const void *k_dev;
    const void *v_dev;
    uint32_t len;
    uint32_t reserved;
} bml_seq_desc;

/* One decode step's appends for a batch of caller-owned caches (the
 * per-request store_k/store_v of gguf_compiler.rs:994-1006, batched; no
 * reference counterpart -- the reference serves one request at a time):
 * writes row seqs[i].len of sequence i ([capacity][n_kv_heads][head_dim]
 * buffers in kv_dtype, writable, room for that row is the caller's) from
 * k_new_dev / v_new_dev [n_seqs][n_kv_heads][head_dim] in src_dtype.  The
 * caller then advances each len.  Asynchronous on stream. */
bml_status bml_kv_append_batched(const bml_seq_desc *seqs_host, uint32_t n_seqs,
                                 uint32_t n_kv_heads, uint32_t head_dim,
                                 bml_dtype kv_dtype, const void *k_new_dev,
                                 const void *v_new_dev, bml_dtype src_dtype,
                                 void *stream);

/* bml_kv_append_batched with the RoPE of bml_kv_append_rope: sequence i's q
 * rows ([n_seqs][n_heads][head_dim] f32, rotated in place) and its new k row
 * are rotated for position seqs[i].len, then k and v ([n_seqs][n_kv_heads]
 * [head_dim] f32) are stored into row seqs[i].len of its caches.  The
 * per-request RoPE + store of gguf_compiler.rs:984-1006 and :1290-1317 for
 * a whole batch in one launch.  Asynchronous on stream. */
bml_status bml_kv_append_rope_batched(const bml_seq_desc *seqs_host,
                                      uint32_t n_seqs, uint32_t n_heads,
                                      uint32_t n_kv_heads, uint32_t head_dim,
                                      bml_dtype kv_dtype, float *q_dev,
                                      const float *k_new_dev,
                                      const float *v_new_dev, void *stream);

/* Scratch bytes recommended for bml_attn_decode_batched / _partial with
 * n_seqs sequences on `device`: room for the partial results of about 8
 * work chunks per SM.  A smaller workspace down to 2 * n_seqs + (SM count)
 * slots still works (the kernels then cut the work into fewer, larger
 * chunks); below that the call returns BML_E_INVALID. */
bml_status bml_attn_decode_workspace_size(uint32_t n_seqs, uint32_t n_heads,
                                          uint32_t head_dim, int32_t device,
                                          size_t *bytes);

/* Batched split-K flash decoding: for every sequence s, the reference
 * attention block over its whole cache (no reference counterpart as a
 * batch: the reference runs one sequence per forward_cached call).
 *   seqs_host : n_seqs descriptors (host memory)
 *   q_dev     : [n_seqs][n_heads][head_dim] f32
 *   out_dev   : [n_seqs][n_heads][head_dim] f32
 *   workspace : device scratch of bml_attn_decode_workspace_size bytes,
 *               zero-filled before its first use; every call leaves it
 *               ready for the next.  Calls sharing a workspace must not
 *               overlap in time.
 * Asynchronous. */
bml_status bml_attn_decode_batched(const bml_seq_desc *seqs_host,
                                   uint32_t n_seqs, uint32_t n_heads,
                                   uint32_t n_kv_heads, uint32_t head_dim,
                                   bml_dtype kv_dtype, float scale,
                                   const float *q_dev, float *out_dev,
                                   void *workspace, size_t workspace_bytes,
                                   void *stream);

/* Allocation-free variant of bml_attn_decode_batched.  It has no
 * counterpart in the reference.  It is for callers that cannot call
 * cudaMalloc: a host runtime that hands all device memory to its own pool
 * allocator at start-up, or a serving loop in which cudaMalloc's implicit
 * device-wide synchronisation would stall other streams.  It takes no
 * workspace; its scratch is a fixed 4 MiB array in device global memory
 * that every GPU loading this library holds until the process exits, and it
 * allocates nothing itself.  A call whose smallest usable scratch -- partial
 * slots for max(2 * n_seqs + (SM count), (8 / n_kv_heads) * n_seqs) results of n_heads rows
 * of head_dim + 2 floats, plus 72.25 KiB of counters -- is above 4 MiB (e.g.
 * 256 sequences of 64 heads at head_dim 128) returns BML_E_INVALID; below
 * that the kernels size their work to the slots the array holds.  The
 * first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the one array, which keeps the last call's contents: each
 * call first clears the schedule counters on `stream`, so calls that
 * overlap in time on the GPU race with each other and must be serialised
 * (one stream, or events between streams).  The array's error word is not
 * cleared by a call: a bounded device wait that gave up stays recorded
 * until bml_attn_noalloc_check reads it.  Results agree with
 * bml_attn_decode_batched's within the decode tolerance.  Asynchronous. */
bml_status bml_attn_decode_batched_noalloc(const bml_seq_desc *seqs_host,
                                           uint32_t n_seqs, uint32_t n_heads,
                                           uint32_t n_kv_heads, uint32_t head_dim,
                                           bml_dtype kv_dtype, float scale,
                                           const float *q_dev, float *out_dev,
                                           void *stream);

/* Reads and clears the error word of the fixed scratch array of
 * bml_attn_decode_batched_noalloc on the current device: BML_E_TIMEOUT if a
 * bounded device wait of an earlier call gave up (that call's output is not
 * valid), else BML_OK.  Like the entry point it serves, it has no
 * counterpart in the reference and allocates nothing.  Synchronises
 * `stream`. */
bml_status bml_attn_noalloc_check(void *stream);

/* KV-split partial: the same computation over each sequence's slice of the
 * cache, returning per (sequence, q head) the running max m (in log2
 * units: max over positions of scale*log2(e)*q.k), the softmax
 * denominator l relative to m, and the normalised partial output
 * o = sum_p 2^(s_p - m) v_p / l.  Partials from disjoint slices of one
 * cache merge exactly with bml_attn_merge_lse.
 *   m_dev, l_dev : [n_seqs][n_heads] f32;  o_dev : [n_seqs][n_heads][head_dim]
 * Asynchronous. */
bml_status bml_attn_decode_partial(const bml_seq_desc *seqs_host,
                                   uint32_t n_seqs, uint32_t n_heads,
                                   uint32_t n_kv_heads, uint32_t head_dim,
                                   bml_dtype kv_dtype, float scale,
                                   const float *q_dev, float *m_dev,
                                   float *l_dev, float *o_dev,
                                   void *workspace, size_t workspace_bytes,
                                   void *stream);

/* Log-sum-exp merge of n_parts partial triples (as written by
 * bml_attn_decode_partial, stacked along a leading part axis):
 *   m_dev, l_dev : [n_parts][n_rows];  o_dev : [n_parts][n_rows][head_dim]
 *   out_dev      : [n_rows][head_dim] f32
 * out = sum_i 2^(m_i-M) l_i o_i / sum_i 2^(m_i-M) l_i with M = max_i m_i,
 * summed in part order.  Asynchronous. */
bml_status bml_attn_merge_lse(const float *m_dev, const float *l_dev,
                              const float *o_dev, uint32_t n_parts,
                              uint32_t n_rows, uint32_t head_dim,
                              float *out_dev, void *stream);

/* The same merge over partials packed one part after another as
 * [m (n_rows) | l (n_rows) | o (n_rows*head_dim)] -- the layout an
 * all-gather of one packed buffer per GPU produces (KV split across GPUs).
 * Asynchronous. */
bml_status bml_attn_merge_lse_packed(const float *parts_dev, uint32_t n_parts,
                                     uint32_t n_rows, uint32_t head_dim,
                                     float *out_dev, void *stream);

/* ------------------------------------------------------------------------ */
/* Causal prefill  (gguf_compiler.rs:946-958 token loop over :1008-1050)     */
/* ------------------------------------------------------------------------ */

/* Attention for every token of n_seqs prompts of seq_len tokens at once:
 * token t of a sequence attends over positions [0, t] of that sequence
 * (causal != 0) or over all positions (causal == 0).  Tensor-core
 * (tcgen05) kernel: q/k/v are 16-bit (in_dtype BML_BF16 or BML_F16),
 * accumulation is f32.
 *   q_dev   : [n_seqs][seq_len][n_heads][head_dim]
 *   k_dev, v_dev : [n_seqs][seq_len][n_kv_heads][head_dim]
 *   out_dev : [n_seqs][seq_len][n_heads][head_dim] in out_dtype
 *             (BML_F32 or in_dtype)
 * head_dim 64 or 128.  Asynchronous. */
bml_status bml_attn_prefill(const void *q_dev, const void *k_dev,
                            const void *v_dev, uint32_t n_seqs,
                            uint32_t seq_len, uint32_t n_heads,
                            uint32_t n_kv_heads, uint32_t head_dim,
                            bml_dtype in_dtype, float scale, int causal,
                            void *out_dev, bml_dtype out_dtype, void *stream);

/* ------------------------------------------------------------------------ */
/* softmax_f32 (kv_cache.rs:188-200)                                        */
/* ------------------------------------------------------------------------ */

/* Row-wise softmax_f32 of n_rows rows of n floats: max-subtracted exp,
 * divided by the row sum, and uniform 1/n where the sum is not positive.
 * n == 0 is valid and does nothing (the reference returns an empty Vec).
 * Asynchronous. */
bml_status bml_softmax_f32(const float *x_dev, uint32_t n_rows, uint32_t n,
                           float *out_dev, void *stream);

/* ------------------------------------------------------------------------ */
/* KV split of one sequence over GPUs                                       */
/* ------------------------------------------------------------------------ */

/* One long sequence whose KV cache is cut into contiguous slices, one per
 * GPU (one process per GPU).  No reference counterpart: the reference runs
 * the whole loop of gguf_compiler.rs:1026-1049 in one thread.  Every rank
 * decodes its slice and, inside the same kernel, exchanges per-(q head, 32
 * dims) partials (max, sum, normalised output) with every other rank over
 * peer memory (CUDA IPC mappings, plain loads and stores) and merges them
 * in rank order with the log-sum-exp rule; every rank ends with the same
 * output.  Set-up: bml_kvsplit_create on each rank, bml_kvsplit_handle ->
 * BML_KVSPLIT_HANDLE_BYTES bytes, gathered from all ranks in rank order
 * (any host channel), bml_kvsplit_open.  All ranks must then call
 * bml_attn_decode_kvsplit the same number of times with the same shape;
 * a rank whose peers do not arrive within 2 s stops waiting and records
 * BML_E_TIMEOUT in the workspace's error word (bml_attn_workspace_check).
 * The calls' exchange epochs are counted on the device (in the exchange
 * buffer, advanced by each launch), so the calls may be captured in a CUDA
 * graph and replayed, on every rank alike. */
typedef struct bml_kvsplit bml_kvsplit;
#define BML_KVSPLIT_HANDLE_BYTES 64

bml_status bml_kvsplit_create(int32_t device, uint32_t rank, uint32_t world,
                              uint32_t n_heads, uint32_t head_dim,
                              bml_kvsplit **out);
bml_status bml_kvsplit_handle(const bml_kvsplit *h, void *handle_out,
                              size_t bytes);
bml_status bml_kvsplit_open(bml_kvsplit *h, const void *handles,
                            size_t bytes);
/* slice_host: this rank's slice of the cache (one descriptor, its own
 * positions only); q_dev [n_heads][head_dim] f32, the same on every rank;
 * out_dev [n_heads][head_dim] f32.  16-bit caches with the decode kernel's
 * shapes.  Asynchronous. */
bml_status bml_attn_decode_kvsplit(bml_kvsplit *h, const bml_seq_desc *slice_host,
                                   uint32_t n_heads, uint32_t n_kv_heads,
                                   uint32_t head_dim, bml_dtype kv_dtype,
                                   float scale, const float *q_dev,
                                   float *out_dev, void *workspace,
                                   size_t workspace_bytes, void *stream);
bml_status bml_kvsplit_destroy(bml_kvsplit *h);

/* ------------------------------------------------------------------------ */
/* Device-side error word                                                   */
/* ------------------------------------------------------------------------ */

/* Reads and clears the error word kernels set in a decode workspace when a
 * bounded wait gives up.  Returns BML_OK or BML_E_TIMEOUT.  Synchronises
 * the stream. */
bml_status bml_attn_workspace_check(void *workspace, size_t workspace_bytes,
                                    void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BML_ATTN_H */
