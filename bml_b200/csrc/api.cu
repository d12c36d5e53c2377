// api.cpp -- host side of the C ABI declared in include/bml_attn.h.
//
// Every entry point validates its arguments on the host before anything is
// launched and reports failures through a status code and a thread-local
// message; nothing here aborts the process.  The reference this replaces
// (crates/compiler/src/kv_cache.rs and the attention block of
// crates/compiler/src/gguf_compiler.rs:1008-1050 in SugarFreeDoNoSo/bml)
// panics on out-of-range indexing; those cases return BML_E_INVALID here.
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/bml_attn.h"
#include "../../include/bml_diag.h"
#include "../../include/bml_weights.h"
#include "decode.cuh"
#include "gemv.cuh"
#include "kv_ops.cuh"
#include "prefill.cuh"

#define BML_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_last_error;

bml_status fail(bml_status code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

bml_status ok() {
    g_last_error.clear();
    return BML_OK;
}

bml_status cuda_fail(cudaError_t e, const char *what) {
    (void)cudaGetLastError();  // clear a sticky launch error of this thread
    if (e == cudaErrorMemoryAllocation) return fail(BML_E_OOM, "%s: %s", what, cudaGetErrorString(e));
    if (e == cudaErrorNotSupported) return fail(BML_E_UNSUPPORTED, "%s: no kernel for this shape", what);
    return fail(BML_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CUDA_TRY(call, what)                              \
    do {                                                  \
        cudaError_t e_ = (call);                          \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

bool valid_dtype(int t) { return t == BML_F32 || t == BML_F16 || t == BML_BF16; }

}  // namespace

// The status helpers for the other host files of the library (gguf.cu).
namespace bml {
bml_status api_fail(bml_status code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}
bml_status api_ok() { return ok(); }
bml_status api_cuda_fail(cudaError_t e, const char *where) { return cuda_fail(e, where); }
}  // namespace bml

namespace {

int num_sms(int device) {
    static std::mutex mu;
    static int cache[64] = {0};
    std::lock_guard<std::mutex> lk(mu);
    if (device < 0 || device >= 64) return 148;
    if (!cache[device]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
            n = 148;
        cache[device] = n;
    }
    return cache[device];
}

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) d = 0;
    return d;
}

// Switches to `dev` for the lifetime of the guard.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
        else prev = -1;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

float resolve_scale(float scale, uint32_t head_dim) {
    // gguf_compiler.rs:1010: 1/sqrt(head_dim) in f64
    return scale < 0.f ? (float)(1.0 / sqrt((double)head_dim)) : scale;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

struct bml_kv {
    bml_kv_desc desc;
    std::vector<void *> k, v;  // per layer device buffers
    uint64_t n_total_k = 0, n_total_v = 0;
    uint32_t current_pos = 0;
    float *staging = nullptr;  // device scratch: head_dim floats + 1
    void *ws = nullptr;        // decode workspace for bml_attn_decode
    size_t ws_bytes = 0;
    float *wrap = nullptr;     // bml_attn_decode_wrap: two q copies + two partials
    size_t wrap_floats = 0;
    size_t layer_elems() const { return (size_t)desc.max_seq_len * desc.n_kv_heads * desc.head_dim; }
    size_t esize() const { return bml::dtype_size(desc.dtype); }
};

// ---------------------------------------------------------------------------
// library
// ---------------------------------------------------------------------------
BML_API const char *bml_last_error(void) { return g_last_error.c_str(); }
BML_API const char *bml_version(void) { return "bml-attn-b200 0.1 (sm_100a)"; }

// ---------------------------------------------------------------------------
// KV cache handle (kv_cache.rs:25-181)
// ---------------------------------------------------------------------------
BML_API bml_status bml_kv_create(const bml_kv_desc *desc, bml_kv **out) {
    if (!desc || !out) return fail(BML_E_INVALID, "bml_kv_create: null argument");
    *out = nullptr;
    if (desc->n_layers == 0 || desc->n_kv_heads == 0 || desc->head_dim == 0 || desc->max_seq_len == 0)
        return fail(BML_E_INVALID, "bml_kv_create: zero dimension");
    if (!valid_dtype(desc->dtype)) return fail(BML_E_INVALID, "bml_kv_create: bad dtype %d", desc->dtype);
    int ndev = 0;
    CUDA_TRY(cudaGetDeviceCount(&ndev), "bml_kv_create");
    if (desc->device < 0 || desc->device >= ndev)
        return fail(BML_E_INVALID, "bml_kv_create: device %d of %d", desc->device, ndev);
    DeviceGuard g(desc->device);
    bml_kv *kv = new bml_kv();
    kv->desc = *desc;
    const size_t bytes = kv->layer_elems() * kv->esize();
    kv->k.assign(desc->n_layers, nullptr);
    kv->v.assign(desc->n_layers, nullptr);
    cudaError_t e = cudaSuccess;
    for (uint32_t l = 0; l < desc->n_layers && e == cudaSuccess; ++l) {
        e = cudaMalloc(&kv->k[l], bytes);
        if (e == cudaSuccess) e = cudaMalloc(&kv->v[l], bytes);
        if (e == cudaSuccess) e = cudaMemset(kv->k[l], 0, bytes);  // vec![0.0; n] (kv_cache.rs:57)
        if (e == cudaSuccess) e = cudaMemset(kv->v[l], 0, bytes);
    }
    if (e == cudaSuccess) e = cudaMalloc(&kv->staging, (desc->head_dim + 4) * sizeof(float));
    if (e != cudaSuccess) {
        bml_kv_destroy(kv);
        return cuda_fail(e, "bml_kv_create");
    }
    *out = kv;
    return ok();
}

BML_API bml_status bml_kv_destroy(bml_kv *kv) {
    if (!kv) return ok();
    DeviceGuard g(kv->desc.device);
    for (void *p : kv->k) if (p) cudaFree(p);
    for (void *p : kv->v) if (p) cudaFree(p);
    if (kv->staging) cudaFree(kv->staging);
    if (kv->ws) cudaFree(kv->ws);
    if (kv->wrap) cudaFree(kv->wrap);
    delete kv;
    return ok();
}

static bml_status check_slot(const bml_kv *kv, int which, uint32_t layer, uint32_t pos, uint32_t kv_head,
                             const char *fn, size_t *elem_off) {
    if (!kv) return fail(BML_E_INVALID, "%s: null handle", fn);
    if (which != BML_WHICH_K && which != BML_WHICH_V) return fail(BML_E_INVALID, "%s: which=%d", fn, which);
    if (layer >= kv->desc.n_layers)
        return fail(BML_E_INVALID, "%s: layer %u >= n_layers %u", fn, layer, kv->desc.n_layers);
    // kv_cache.rs:83-86: ring slot; the slice start..start+d must be in range
    const size_t stride = (size_t)kv->desc.n_kv_heads * kv->desc.head_dim;
    const size_t start = (size_t)(pos % kv->desc.max_seq_len) * stride + (size_t)kv_head * kv->desc.head_dim;
    if (start + kv->desc.head_dim > kv->layer_elems())
        return fail(BML_E_INVALID, "%s: slot out of range (kv_head %u)", fn, kv_head);
    *elem_off = start;
    return BML_OK;
}

BML_API bml_status bml_kv_store(bml_kv *kv, int which, uint32_t layer, uint32_t pos, uint32_t kv_head,
                                const float *host_data, size_t len) {
    size_t off = 0;
    bml_status st = check_slot(kv, which, layer, pos, kv_head, "bml_kv_store", &off);
    if (st != BML_OK) return st;
    if (!host_data) return fail(BML_E_INVALID, "bml_kv_store: null data");
    const uint32_t d = kv->desc.head_dim;
    // kv_cache.rs:87: copy_from_slice of data[..min(d, len)] into d slots
    if (len < d) return fail(BML_E_INVALID, "bml_kv_store: %zu values for head_dim %u", len, d);
    DeviceGuard g(kv->desc.device);
    CUDA_TRY(cudaMemcpy(kv->staging, host_data, d * sizeof(float), cudaMemcpyHostToDevice), "bml_kv_store");
    void *base = which == BML_WHICH_K ? kv->k[layer] : kv->v[layer];
    void *dst = static_cast<char *>(base) + off * kv->esize();
    CUDA_TRY(bml::kv_store_from_f32(kv->staging, dst, kv->desc.dtype, d, 0), "bml_kv_store");
    CUDA_TRY(cudaStreamSynchronize(0), "bml_kv_store");
    if (which == BML_WHICH_K) kv->n_total_k++;
    else kv->n_total_v++;
    return ok();
}

BML_API bml_status bml_kv_load(const bml_kv *kv, int which, uint32_t layer, uint32_t pos, uint32_t kv_head,
                               float *host_out) {
    size_t off = 0;
    bml_status st = check_slot(kv, which, layer, pos, kv_head, "bml_kv_load", &off);
    if (st != BML_OK) return st;
    if (!host_out) return fail(BML_E_INVALID, "bml_kv_load: null output");
    const uint32_t d = kv->desc.head_dim;
    DeviceGuard g(kv->desc.device);
    const void *base = which == BML_WHICH_K ? kv->k[layer] : kv->v[layer];
    const void *src = static_cast<const char *>(base) + off * kv->esize();
    CUDA_TRY(bml::kv_convert(src, kv->desc.dtype, kv->staging, BML_F32, d, 0), "bml_kv_load");
    CUDA_TRY(cudaMemcpy(host_out, kv->staging, d * sizeof(float), cudaMemcpyDeviceToHost), "bml_kv_load");
    return ok();
}

BML_API bml_status bml_kv_dot_qk(const bml_kv *kv, const float *host_q, size_t q_len, uint32_t layer,
                                 uint32_t pos, uint32_t kv_head, float *out) {
    size_t off = 0;
    bml_status st = check_slot(kv, BML_WHICH_K, layer, pos, kv_head, "bml_kv_dot_qk", &off);
    if (st != BML_OK) return st;
    if (!out || (!host_q && q_len)) return fail(BML_E_INVALID, "bml_kv_dot_qk: null argument");
    const uint32_t n = (uint32_t)std::min<size_t>(q_len, kv->desc.head_dim);  // zip: shorter wins
    DeviceGuard g(kv->desc.device);
    if (n) CUDA_TRY(cudaMemcpy(kv->staging, host_q, n * sizeof(float), cudaMemcpyHostToDevice), "bml_kv_dot_qk");
    const void *src = static_cast<const char *>(kv->k[layer]) + off * kv->esize();
    CUDA_TRY(bml::kv_dot(kv->staging, src, kv->desc.dtype, n, kv->staging + kv->desc.head_dim, 0),
             "bml_kv_dot_qk");
    CUDA_TRY(cudaMemcpy(out, kv->staging + kv->desc.head_dim, sizeof(float), cudaMemcpyDeviceToHost),
             "bml_kv_dot_qk");
    return ok();
}

BML_API bml_status bml_kv_stats(const bml_kv *kv, int which, uint64_t *unique, uint64_t *total, double *ratio) {
    if (!kv || !unique || !total || !ratio) return fail(BML_E_INVALID, "bml_kv_stats: null argument");
    if (which != BML_WHICH_K && which != BML_WHICH_V) return fail(BML_E_INVALID, "bml_kv_stats: which");
    const uint64_t t = which == BML_WHICH_K ? kv->n_total_k : kv->n_total_v;
    *unique = t;
    *total = t;
    *ratio = 1.0;
    return ok();
}

BML_API bml_status bml_kv_byte_size(const bml_kv *kv, uint64_t *out) {
    if (!kv || !out) return fail(BML_E_INVALID, "bml_kv_byte_size: null argument");
    *out = (uint64_t)kv->layer_elems() * kv->esize() * kv->desc.n_layers * 2;
    return ok();
}

BML_API bml_status bml_kv_current_pos(const bml_kv *kv, uint32_t *out) {
    if (!kv || !out) return fail(BML_E_INVALID, "bml_kv_current_pos: null argument");
    *out = kv->current_pos;
    return ok();
}

BML_API bml_status bml_kv_advance(bml_kv *kv) {
    if (!kv) return fail(BML_E_INVALID, "bml_kv_advance: null handle");
    kv->current_pos += 1;
    return ok();
}

BML_API bml_status bml_kv_advance_by(bml_kv *kv, uint32_t n) {
    if (!kv) return fail(BML_E_INVALID, "bml_kv_advance_by: null handle");
    kv->current_pos += n;
    return ok();
}

BML_API bml_status bml_kv_layer_ptr(const bml_kv *kv, int which, uint32_t layer, void **dev_out) {
    if (!kv || !dev_out) return fail(BML_E_INVALID, "bml_kv_layer_ptr: null argument");
    if (which != BML_WHICH_K && which != BML_WHICH_V) return fail(BML_E_INVALID, "bml_kv_layer_ptr: which");
    if (layer >= kv->desc.n_layers) return fail(BML_E_INVALID, "bml_kv_layer_ptr: layer %u", layer);
    *dev_out = which == BML_WHICH_K ? kv->k[layer] : kv->v[layer];
    return ok();
}

BML_API bml_status bml_kv_append(bml_kv *kv, uint32_t layer, uint32_t pos, const void *k_dev, const void *v_dev,
                                 bml_dtype src_dtype, void *stream) {
    size_t off = 0;
    bml_status st = check_slot(kv, BML_WHICH_K, layer, pos, 0, "bml_kv_append", &off);
    if (st != BML_OK) return st;
    if (!k_dev || !v_dev) return fail(BML_E_INVALID, "bml_kv_append: null argument");
    if (!valid_dtype(src_dtype)) return fail(BML_E_INVALID, "bml_kv_append: bad dtype");
    const size_t n = (size_t)kv->desc.n_kv_heads * kv->desc.head_dim;
    DeviceGuard g(kv->desc.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char *kd = static_cast<char *>(kv->k[layer]) + off * kv->esize();
    char *vd = static_cast<char *>(kv->v[layer]) + off * kv->esize();
    CUDA_TRY(bml::kv_convert(k_dev, src_dtype, kd, kv->desc.dtype, n, s), "bml_kv_append");
    CUDA_TRY(bml::kv_convert(v_dev, src_dtype, vd, kv->desc.dtype, n, s), "bml_kv_append");
    kv->n_total_k += kv->desc.n_kv_heads;
    kv->n_total_v += kv->desc.n_kv_heads;
    return ok();
}

BML_API bml_status bml_kv_append_rope(bml_kv *kv, uint32_t layer, uint32_t pos, float *q_dev, uint32_t n_heads,
                                      const float *k_dev, const float *v_dev, void *stream) {
    size_t off = 0;
    bml_status st = check_slot(kv, BML_WHICH_K, layer, pos, 0, "bml_kv_append_rope", &off);
    if (st != BML_OK) return st;
    if (!q_dev || !k_dev || !v_dev) return fail(BML_E_INVALID, "bml_kv_append_rope: null argument");
    const uint32_t n_kv = kv->desc.n_kv_heads, d = kv->desc.head_dim;
    if (n_heads == 0 || n_heads % n_kv != 0)
        return fail(BML_E_INVALID, "bml_kv_append_rope: n_heads %u not a multiple of n_kv_heads %u", n_heads, n_kv);
    if (d % 2 != 0) return fail(BML_E_INVALID, "bml_kv_append_rope: head_dim %u is odd", d);
    DeviceGuard g(kv->desc.device);
    char *kd = static_cast<char *>(kv->k[layer]) + off * kv->esize();
    char *vd = static_cast<char *>(kv->v[layer]) + off * kv->esize();
    CUDA_TRY(bml::kv_rope_append(q_dev, n_heads, k_dev, v_dev, kd, vd, kv->desc.dtype, n_kv, d, pos,
                                 static_cast<cudaStream_t>(stream)),
             "bml_kv_append_rope");
    kv->n_total_k += n_kv;
    kv->n_total_v += n_kv;
    return ok();
}

namespace {

// Fills p with the destinations of seqs_host[base, base + ns) of a batched
// append; a null buffer is an error.
bml_status fill_append_rows(bml::AppendRows &p, const bml_seq_desc *seqs_host, uint32_t base, uint32_t ns,
                            const char *fn) {
    for (uint32_t i = 0; i < ns; ++i) {
        const bml_seq_desc &d = seqs_host[base + i];
        if (!d.k_dev || !d.v_dev) return fail(BML_E_INVALID, "%s: sequence %u has a null buffer", fn, base + i);
        p.k[i] = const_cast<void *>(d.k_dev);
        p.v[i] = const_cast<void *>(d.v_dev);
        p.len[i] = d.len;
    }
    return BML_OK;
}

}  // namespace

BML_API bml_status bml_kv_append_batched(const bml_seq_desc *seqs_host, uint32_t n_seqs, uint32_t n_kv_heads,
                                         uint32_t head_dim, bml_dtype kv_dtype, const void *k_new_dev,
                                         const void *v_new_dev, bml_dtype src_dtype, void *stream) {
    const char *fn = "bml_kv_append_batched";
    if (!seqs_host || !k_new_dev || !v_new_dev) return fail(BML_E_INVALID, "%s: null argument", fn);
    if (!valid_dtype(kv_dtype) || !valid_dtype(src_dtype)) return fail(BML_E_INVALID, "%s: bad dtype", fn);
    if (n_kv_heads == 0 || head_dim == 0) return fail(BML_E_INVALID, "%s: zero dimension", fn);
    static thread_local bml::AppendRows p;  // ~5 KB, kept off the stack
    p.row = n_kv_heads * head_dim;
    p.n_heads = 0;
    p.head_dim = head_dim;
    const size_t src_row = (size_t)p.row * bml::dtype_size(src_dtype);
    for (uint32_t base = 0; base < n_seqs; base += bml::kMaxAppendSeqs) {
        const uint32_t ns = std::min<uint32_t>(n_seqs - base, bml::kMaxAppendSeqs);
        if (bml_status st = fill_append_rows(p, seqs_host, base, ns, fn)) return st;
        CUDA_TRY(bml::kv_append_rows(p, ns, static_cast<const char *>(k_new_dev) + base * src_row,
                                     static_cast<const char *>(v_new_dev) + base * src_row, src_dtype, kv_dtype,
                                     static_cast<cudaStream_t>(stream)),
                 fn);
    }
    return ok();
}

BML_API bml_status bml_kv_append_rope_batched(const bml_seq_desc *seqs_host, uint32_t n_seqs, uint32_t n_heads,
                                              uint32_t n_kv_heads, uint32_t head_dim, bml_dtype kv_dtype,
                                              float *q_dev, const float *k_new_dev, const float *v_new_dev,
                                              void *stream) {
    const char *fn = "bml_kv_append_rope_batched";
    if (!seqs_host || !q_dev || !k_new_dev || !v_new_dev) return fail(BML_E_INVALID, "%s: null argument", fn);
    if (!valid_dtype(kv_dtype)) return fail(BML_E_INVALID, "%s: bad dtype", fn);
    if (n_kv_heads == 0 || head_dim == 0 || n_heads == 0) return fail(BML_E_INVALID, "%s: zero dimension", fn);
    if (n_heads % n_kv_heads) return fail(BML_E_INVALID, "%s: n_heads %% n_kv_heads != 0", fn);
    if (head_dim % 2) return fail(BML_E_INVALID, "%s: RoPE needs an even head_dim", fn);
    static thread_local bml::AppendRows p;
    p.row = n_kv_heads * head_dim;
    p.n_heads = n_heads;
    p.head_dim = head_dim;
    for (uint32_t base = 0; base < n_seqs; base += bml::kMaxAppendSeqs) {
        const uint32_t ns = std::min<uint32_t>(n_seqs - base, bml::kMaxAppendSeqs);
        if (bml_status st = fill_append_rows(p, seqs_host, base, ns, fn)) return st;
        CUDA_TRY(bml::kv_rope_append_rows(p, ns, q_dev + (size_t)base * n_heads * head_dim,
                                          k_new_dev + (size_t)base * p.row, v_new_dev + (size_t)base * p.row,
                                          kv_dtype, static_cast<cudaStream_t>(stream)),
                 fn);
    }
    return ok();
}

// ---------------------------------------------------------------------------
// Decode
// ---------------------------------------------------------------------------
namespace {

bml_status check_decode_shape(uint32_t n_heads, uint32_t n_kv, uint32_t head_dim, bml_dtype dt, const char *fn) {
    if (!valid_dtype(dt)) return fail(BML_E_INVALID, "%s: bad kv dtype %d", fn, (int)dt);
    if (n_kv == 0 || n_heads == 0 || head_dim == 0) return fail(BML_E_INVALID, "%s: zero dimension", fn);
    // gguf_compiler.rs:1011 uses n_heads / n_kv; a remainder would make
    // kv_h = h / group run past the last kv head, which is rejected here.
    if (n_heads % n_kv != 0)
        return fail(BML_E_INVALID, "%s: n_heads %u not a multiple of n_kv_heads %u", fn, n_heads, n_kv);
    const uint32_t g = n_heads / n_kv;
    if (!(n_kv == 1 || n_kv == 2 || n_kv == 4 || n_kv == 8))
        return fail(BML_E_UNSUPPORTED, "%s: n_kv_heads %u (supported: 1, 2, 4, 8)", fn, n_kv);
    if (!(g == 1 || g == 2 || g == 4 || g == 8))
        return fail(BML_E_UNSUPPORTED, "%s: %u q heads per kv head (supported: 1, 2, 4, 8)", fn, g);
    if (!(head_dim == 64 || head_dim == 128))
        return fail(BML_E_UNSUPPORTED, "%s: head_dim %u (supported: 64, 128)", fn, head_dim);
    return BML_OK;
}

// Schedule knobs of the claimed-schedule kernel (decode_bulk_kernel).
struct BulkPlan {
    uint32_t claim_tiles = 4;  // tiles per claim
    uint32_t join_min = 4;     // unclaimed tiles per CTA on a sequence worth a join
    uint32_t merge_rows = 8;   // q-head rows per merge item
    uint32_t merge_wpr = 1;    // warps sharing one row in the merge
    uint32_t merge_dsplit = 1; // head-dim slices per merge item
};

// Tiles per claim: four (~5 us of one SM at the HBM rate).  Measured on
// B200: with one tile per claim a claim's atomic, issued one claim ahead, no
// longer hides behind the ring (the Llama-3 batch streams at 6.0 instead of
// 7.3 TB/s); four beat two by 2-12% on the Llama-3 and ragged TinyLlama
// batches, and claiming a sequence's last 4-16 tiles one at a time, to even
// out the end, lost 1-11% to the same atomic latency.  A started sequence is
// joined only while it has at least 4 unclaimed tiles per CTA on it: a join
// costs three dependent round trips (~3 us), about two tiles.
// Merge: a row of a sequence has about nph * (grid / n_seqs + 2) partial
// slots; each warp combines up to 16 of them in one round of loads, so a
// row is shared by up to 8 warps (one long sequence: one row per CTA), and
// where one warp per row suffices and the items would not fit one round of
// the grid, a warp takes two rows.
BulkPlan bulk_plan(uint32_t n_seqs, uint32_t n_heads, uint32_t head_dim, uint32_t nph, uint32_t parts_per_seq,
                   int grid) {
    BulkPlan b;
    const uint32_t nw = bml::decode_bulk_warps(head_dim);  // consumer warps
    const uint32_t per_row = std::min<uint32_t>(parts_per_seq, (uint32_t)grid / n_seqs + 2u) * nph;
    uint32_t wpr = 1;
    while (wpr < nw && per_row > 16u * wpr) wpr *= 2;
    uint32_t rows = nw / wpr;
    if (wpr == 1 && n_heads % (2u * nw) == 0 && (uint64_t)n_seqs * n_heads / nw > (uint64_t)grid) rows = 2u * nw;
    while (rows > 1 && n_heads % rows) rows /= 2;  // small head counts
    if (rows * wpr < nw) wpr = nw / rows;
    b.merge_rows = rows;
    b.merge_wpr = wpr;
    // few rows with many slots each (a long sequence): split the head dims
    // too, so that more CTAs share the merge and each lane keeps all its
    // slots in flight at once
    while (b.merge_dsplit < 4 && wpr == nw && 32u * b.merge_dsplit * 2u <= head_dim &&
           (uint64_t)n_seqs * (n_heads / rows) * b.merge_dsplit * 2u <= (uint64_t)grid)
        b.merge_dsplit *= 2;
    return b;
}

// A KV split over GPUs: this rank, its device-side call counter and every
// rank's exchange buffer (mapped into this process).
struct ExchangeArgs {
    uint32_t world = 1, rank = 0;
    uint32_t *epoch = nullptr;
    float *base[bml::kMaxExchangeRanks] = {};
};

// Shared body of bml_attn_decode_batched / _partial, the test-only variant
// (kernel choice, wait limit and behaviour flags given) and the KV split
// over GPUs (exchange given).
bml_status decode_impl(const bml_seq_desc *seqs, uint32_t n_seqs, uint32_t n_heads, uint32_t n_kv,
                       uint32_t head_dim, bml_dtype dt, float scale, const float *q, float *out, float *pm,
                       float *pl, float *po, void *workspace, size_t ws_bytes, void *stream, int mode,
                       const char *fn, int force_kernel = 0, uint64_t wait_ns = bml::kWaitNs, uint32_t diag = 0,
                       const ExchangeArgs *xa = nullptr) {
    bml_status st = check_decode_shape(n_heads, n_kv, head_dim, dt, fn);
    if (st != BML_OK) return st;
    if (!seqs || n_seqs == 0) return fail(BML_E_INVALID, "%s: no sequences", fn);
    if (!q || !aligned16(q)) return fail(BML_E_INVALID, "%s: q must be a 16-byte aligned device pointer", fn);
    if (mode == bml::kModeFinal && (!out || !aligned16(out)))
        return fail(BML_E_INVALID, "%s: out must be a 16-byte aligned device pointer", fn);
    if (mode == bml::kModePartial && (!pm || !pl || !po || !aligned16(po)))
        return fail(BML_E_INVALID, "%s: null or misaligned partial output", fn);
    if (!aligned16(workspace)) return fail(BML_E_INVALID, "%s: workspace must be 16-byte aligned", fn);
    for (uint32_t s = 0; s < n_seqs; ++s) {
        if (seqs[s].len == 0) return fail(BML_E_INVALID, "%s: sequence %u has no positions", fn, s);
        if (!seqs[s].k_dev || !seqs[s].v_dev || !aligned16(seqs[s].k_dev) || !aligned16(seqs[s].v_dev))
            return fail(BML_E_INVALID, "%s: sequence %u K/V must be 16-byte aligned device pointers", fn, s);
    }
    const int dev = current_device();
    const int sms = num_sms(dev);
    bml::DecodeWorkspace ws;
    if (!bml::decode_workspace_carve(workspace, ws_bytes, n_seqs, n_heads, n_kv, head_dim, sms, &ws))
        return fail(BML_E_INVALID, "%s: workspace of %zu bytes, need %zu", fn, ws_bytes,
                    bml::decode_workspace_min_bytes(n_seqs, n_heads, n_kv, head_dim, sms));

    const float sc = resolve_scale(scale, head_dim);
    const size_t es = bml::dtype_size(dt);
    const uint32_t T = bml::decode_rows_per_tile(dt, head_dim, n_kv);
    const uint32_t group = n_heads / n_kv;
    const bml::DecodeKernel kern =
        force_kernel == BML_DIAG_DECODE_CUDA_CORE ? bml::kKernCuda : bml::decode_select(dt, head_dim, n_kv, group);
    const bool split = xa && xa->world > 1;
    if (split && (kern != bml::kKernBulk || n_seqs != 1 || mode != bml::kModeFinal))
        return fail(BML_E_UNSUPPORTED, "%s: the KV split over GPUs takes one 16-bit sequence", fn);
    static thread_local bml::DecodeParams p;  // ~8 KB, kept off the stack
    for (uint32_t base = 0; base < n_seqs; base += (uint32_t)bml::kMaxSeqsPerLaunch) {
        const uint32_t ns = std::min<uint32_t>(n_seqs - base, (uint32_t)bml::kMaxSeqsPerLaunch);
        memset(&p, 0, offsetof(bml::DecodeParams, seqs));
        p.n_seqs = ns;
        p.n_kv = n_kv;
        p.rows_per_tile = T;  // the schedule below counts tiles with it
        uint64_t total = 0;
        uint32_t slot = 0, max_slots_seq = 0;
        for (uint32_t s = 0; s < ns; ++s) {
            const bml_seq_desc &d = seqs[base + s];
            bml::DecodeSeq &e = p.seqs[s];
            e.k = d.k_dev;
            e.v = d.v_dev;
            e.len = d.len;
            e.tile_begin = (uint32_t)total;
            total += (d.len + T - 1) / T;
        }
        if (total > 0x7fffffffull) return fail(BML_E_INVALID, "%s: batch too large", fn);
        int grid = 0;
        if (kern == bml::kKernBulk) {
            // Claimed schedule: at most one CTA per SM and per tile; parts
            // per sequence as the workspace's slots allow (each CTA visits a
            // sequence at most once, so more than `grid` are never used) and
            // at least the busiest sequence's home CTAs (fewer CTAs if the
            // slots are short).
            grid = (int)std::min<uint64_t>((uint64_t)sms, total);
            const uint32_t nph = bml::decode_bulk_phases(n_kv, head_dim);
            size_t pps = 0;
            while (true) {
                pps = std::min<size_t>({(size_t)grid, ws.max_slots / ((size_t)ns * nph), bml::kMaxPartTiles / ns});
                if (pps >= std::max<uint32_t>(1u, bml::decode_assign_homes(p, (uint32_t)grid)) || grid == 1) break;
                grid = std::max(1, grid * 3 / 4);
            }
            if (pps == 0) return fail(BML_E_INVALID, "%s: internal part overflow", fn);
            const BulkPlan plan = bulk_plan(ns, n_heads, head_dim, nph, (uint32_t)pps, grid);
            p.parts_per_seq = (uint32_t)pps;
            p.claim_tiles = plan.claim_tiles;
            p.join_min = plan.join_min;
            p.merge_rows = plan.merge_rows;
            p.merge_wpr = plan.merge_wpr;
            p.merge_dsplit = plan.merge_dsplit;
            if (split) {  // one merge item per exchange unit: a row x 32 dims
                p.merge_rows = 1;
                p.merge_wpr = bml::decode_bulk_warps(head_dim);
                p.merge_dsplit = head_dim / 32;
                p.x_world = xa->world;
                p.x_rank = xa->rank;
                p.x_epoch = xa->epoch;
                p.x_units = n_heads * (head_dim / 32);
                for (uint32_t r = 0; r < xa->world; ++r) p.x_base[r] = xa->base[r];
            }
            p.sched = ws.sched;
            p.part_tiles = ws.part_tiles;
        } else {
            // Static schedule: contiguous ranges of tpc tiles per CTA.
            const uint32_t tpc = (uint32_t)((total + sms - 1) / sms);
            grid = (int)((total + tpc - 1) / tpc);
            for (uint32_t s = 0; s < ns; ++s) {
                bml::DecodeSeq &e = p.seqs[s];
                const uint32_t nt = (e.len + T - 1) / T;
                e.slot_base = slot;
                e.n_slots = (e.tile_begin + nt - 1) / tpc - e.tile_begin / tpc + 1;
                slot += e.n_slots;
                max_slots_seq = std::max(max_slots_seq, e.n_slots);
            }
            if (slot > ws.max_slots) return fail(BML_E_INVALID, "%s: internal slot overflow", fn);
            p.tiles_per_cta = tpc;
            p.merge_in_kernel = max_slots_seq <= bml::kInKernelMergeMaxSlots ? 1 : 0;
        }
        p.q = q + (size_t)base * n_heads * head_dim;
        p.out = out ? out + (size_t)base * n_heads * head_dim : nullptr;
        p.part_m = pm ? pm + (size_t)base * n_heads : nullptr;
        p.part_l = pl ? pl + (size_t)base * n_heads : nullptr;
        p.part_o = po ? po + (size_t)base * n_heads * head_dim : nullptr;
        p.slot_ml = ws.slot_ml;
        p.slot_o = ws.slot_o;
        p.counters = ws.counters;
        p.err = ws.err;
        p.n_heads = n_heads;
        p.rows_per_tile = T;
        p.total_tiles = (uint32_t)total;
        p.row_bytes = (uint32_t)(n_kv * head_dim * es);
        p.qscale = (float)((double)sc * 1.4426950408889634);
        p.mode = mode;
        p.wait_ns = wait_ns;
        p.diag = diag;
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (kern == bml::kKernBulk) {
            CUDA_TRY(bml::launch_decode_bulk(p, dt, head_dim, group, grid, s), fn);
        } else {
            CUDA_TRY(bml::launch_decode(p, dt, head_dim, group, grid, s), fn);
            if (!p.merge_in_kernel) CUDA_TRY(bml::launch_slot_merge(p, head_dim, s), fn);
        }
    }
    return ok();
}

}  // namespace

BML_API bml_status bml_attn_decode_workspace_size(uint32_t n_seqs, uint32_t n_heads, uint32_t head_dim,
                                                  int32_t device, size_t *bytes) {
    if (!bytes) return fail(BML_E_INVALID, "bml_attn_decode_workspace_size: null output");
    if (n_seqs == 0 || n_heads == 0 || head_dim == 0)
        return fail(BML_E_INVALID, "bml_attn_decode_workspace_size: zero dimension");
    *bytes = bml::decode_workspace_bytes(n_seqs, n_heads, head_dim, num_sms(device));
    return ok();
}

BML_API bml_status bml_attn_decode_batched(const bml_seq_desc *seqs_host, uint32_t n_seqs, uint32_t n_heads,
                                           uint32_t n_kv_heads, uint32_t head_dim, bml_dtype kv_dtype, float scale,
                                           const float *q_dev, float *out_dev, void *workspace,
                                           size_t workspace_bytes, void *stream) {
    return decode_impl(seqs_host, n_seqs, n_heads, n_kv_heads, head_dim, kv_dtype, scale, q_dev, out_dev, nullptr,
                       nullptr, nullptr, workspace, workspace_bytes, stream, bml::kModeFinal,
                       "bml_attn_decode_batched");
}

BML_API bml_status bml_attn_decode_partial(const bml_seq_desc *seqs_host, uint32_t n_seqs, uint32_t n_heads,
                                           uint32_t n_kv_heads, uint32_t head_dim, bml_dtype kv_dtype, float scale,
                                           const float *q_dev, float *m_dev, float *l_dev, float *o_dev,
                                           void *workspace, size_t workspace_bytes, void *stream) {
    return decode_impl(seqs_host, n_seqs, n_heads, n_kv_heads, head_dim, kv_dtype, scale, q_dev, nullptr, m_dev,
                       l_dev, o_dev, workspace, workspace_bytes, stream, bml::kModePartial,
                       "bml_attn_decode_partial");
}

BML_API bml_status bml_attn_decode(bml_kv *kv, uint32_t layer, uint32_t pos, uint32_t n_heads, float scale,
                                   const float *q_dev, float *out_dev, void *stream) {
    if (!kv) return fail(BML_E_INVALID, "bml_attn_decode: null handle");
    if (layer >= kv->desc.n_layers) return fail(BML_E_INVALID, "bml_attn_decode: layer %u", layer);
    if (pos >= kv->desc.max_seq_len)
        return fail(BML_E_INVALID, "bml_attn_decode: pos %u >= max_seq_len %u (the ring wrap is bml_attn_decode_wrap)", pos,
                    kv->desc.max_seq_len);
    bml_status st = check_decode_shape(n_heads, kv->desc.n_kv_heads, kv->desc.head_dim, kv->desc.dtype,
                                       "bml_attn_decode");
    if (st != BML_OK) return st;
    DeviceGuard g(kv->desc.device);
    const size_t need = bml::decode_workspace_bytes(1, n_heads, kv->desc.head_dim, num_sms(kv->desc.device));
    if (kv->ws_bytes < need) {
        if (kv->ws) cudaFree(kv->ws);
        kv->ws = nullptr;
        kv->ws_bytes = 0;
        CUDA_TRY(cudaMalloc(&kv->ws, need), "bml_attn_decode");
        CUDA_TRY(cudaMemset(kv->ws, 0, need), "bml_attn_decode");
        kv->ws_bytes = need;
    }
    bml_seq_desc d{kv->k[layer], kv->v[layer], pos + 1, 0};
    return decode_impl(&d, 1, n_heads, kv->desc.n_kv_heads, kv->desc.head_dim, kv->desc.dtype, scale, q_dev,
                       out_dev, nullptr, nullptr, nullptr, kv->ws, kv->ws_bytes, stream, bml::kModeFinal,
                       "bml_attn_decode");
}

BML_API bml_status bml_attn_decode_wrap(bml_kv *kv, uint32_t layer, uint32_t pos, uint32_t n_heads, float scale,
                                        const float *q_dev, float *out_dev, void *stream) {
    const char *fn = "bml_attn_decode_wrap";
    if (!kv) return fail(BML_E_INVALID, "%s: null handle", fn);
    const uint32_t M = kv->desc.max_seq_len;
    if (pos < M) return bml_attn_decode(kv, layer, pos, n_heads, scale, q_dev, out_dev, stream);
    if (layer >= kv->desc.n_layers) return fail(BML_E_INVALID, "%s: layer %u", fn, layer);
    bml_status st = check_decode_shape(n_heads, kv->desc.n_kv_heads, kv->desc.head_dim, kv->desc.dtype, fn);
    if (st != BML_OK) return st;
    if (!q_dev || !out_dev || !aligned16(q_dev)) return fail(BML_E_INVALID, "%s: q and out must be device pointers", fn);
    DeviceGuard g(kv->desc.device);
    const uint32_t d = kv->desc.head_dim;
    // The loop of gguf_compiler.rs:1026 visits positions 0..pos through
    // slot p % M (kv_cache.rs:83): slot s is visited n/M times, plus once
    // more for s < n % M (n = pos + 1).  Identical scores give identical
    // softmax terms, so the result is attention over the M slots with each
    // slot's weight multiplied by its visit count: two partials (slots
    // below and from n % M) merged with counts c+1 and c.
    const uint64_t n = (uint64_t)pos + 1;
    const uint32_t r = (uint32_t)(n % M);
    const float c = (float)(n / M);
    const size_t need_ws = bml::decode_workspace_bytes(2, n_heads, d, num_sms(kv->desc.device));
    if (kv->ws_bytes < need_ws) {
        if (kv->ws) cudaFree(kv->ws);
        kv->ws = nullptr;
        kv->ws_bytes = 0;
        CUDA_TRY(cudaMalloc(&kv->ws, need_ws), fn);
        CUDA_TRY(cudaMemset(kv->ws, 0, need_ws), fn);
        kv->ws_bytes = need_ws;
    }
    const size_t hd = (size_t)n_heads * d;
    const size_t need_f = 2 * hd + 2 * (2 * n_heads + hd);  // q copies; m, l, o of two parts
    if (kv->wrap_floats < need_f) {
        if (kv->wrap) cudaFree(kv->wrap);
        kv->wrap = nullptr;
        kv->wrap_floats = 0;
        CUDA_TRY(cudaMalloc(&kv->wrap, need_f * sizeof(float)), fn);
        kv->wrap_floats = need_f;
    }
    float *qq = kv->wrap, *pm = qq + 2 * hd, *pl = pm + 2 * n_heads, *po = pl + 2 * n_heads;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t row = (size_t)kv->desc.n_kv_heads * d * kv->esize();
    bml_seq_desc parts[2];
    uint32_t np = 0;
    float counts[2];
    if (r > 0) {
        parts[np] = {kv->k[layer], kv->v[layer], r, 0};
        counts[np++] = c + 1.f;
    }
    parts[np] = {static_cast<const char *>(kv->k[layer]) + r * row, static_cast<const char *>(kv->v[layer]) + r * row,
                 M - r, 0};
    counts[np++] = c;
    for (uint32_t k = 0; k < np; ++k)
        CUDA_TRY(cudaMemcpyAsync(qq + k * hd, q_dev, hd * sizeof(float), cudaMemcpyDeviceToDevice, s), fn);
    st = decode_impl(parts, np, n_heads, kv->desc.n_kv_heads, d, kv->desc.dtype, scale, qq, nullptr, pm, pl, po,
                     kv->ws, kv->ws_bytes, stream, bml::kModePartial, fn);
    if (st != BML_OK) return st;
    CUDA_TRY(bml::launch_merge_counted(pm, pl, po, np, counts, n_heads, d, out_dev, s), fn);
    return ok();
}

BML_API bml_status bml_attn_merge_lse(const float *m_dev, const float *l_dev, const float *o_dev, uint32_t n_parts,
                                      uint32_t n_rows, uint32_t head_dim, float *out_dev, void *stream) {
    if (!m_dev || !l_dev || !o_dev || !out_dev) return fail(BML_E_INVALID, "bml_attn_merge_lse: null argument");
    if (n_parts == 0 || head_dim == 0) return fail(BML_E_INVALID, "bml_attn_merge_lse: zero dimension");
    CUDA_TRY(bml::launch_merge_lse(m_dev, l_dev, o_dev, n_parts, n_rows, head_dim, out_dev,
                                   static_cast<cudaStream_t>(stream)),
             "bml_attn_merge_lse");
    return ok();
}

BML_API bml_status bml_attn_merge_lse_packed(const float *parts_dev, uint32_t n_parts, uint32_t n_rows,
                                             uint32_t head_dim, float *out_dev, void *stream) {
    if (!parts_dev || !out_dev) return fail(BML_E_INVALID, "bml_attn_merge_lse_packed: null argument");
    if (n_parts == 0 || head_dim == 0) return fail(BML_E_INVALID, "bml_attn_merge_lse_packed: zero dimension");
    CUDA_TRY(bml::launch_merge_lse_packed(parts_dev, n_parts, n_rows, head_dim, out_dev,
                                          static_cast<cudaStream_t>(stream)),
             "bml_attn_merge_lse_packed");
    return ok();
}

BML_API bml_status bml_attn_workspace_check(void *workspace, size_t workspace_bytes, void *stream) {
    if (!workspace || workspace_bytes < 256) return fail(BML_E_INVALID, "bml_attn_workspace_check: workspace");
    uint32_t err = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    CUDA_TRY(cudaMemcpyAsync(&err, workspace, sizeof err, cudaMemcpyDeviceToHost, s), "bml_attn_workspace_check");
    CUDA_TRY(cudaStreamSynchronize(s), "bml_attn_workspace_check");
    if (err) {
        const uint32_t zero = 0;
        CUDA_TRY(cudaMemcpyAsync(workspace, &zero, sizeof zero, cudaMemcpyHostToDevice, s),
                 "bml_attn_workspace_check");
        CUDA_TRY(cudaStreamSynchronize(s), "bml_attn_workspace_check");
        return fail(BML_E_TIMEOUT, "a bounded device wait gave up (error word 0x%x)", err);
    }
    return ok();
}

// ---------------------------------------------------------------------------
// Prefill
// ---------------------------------------------------------------------------
BML_API bml_status bml_attn_prefill(const void *q_dev, const void *k_dev, const void *v_dev, uint32_t n_seqs,
                                    uint32_t seq_len, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                    bml_dtype in_dtype, float scale, int causal, void *out_dev,
                                    bml_dtype out_dtype, void *stream) {
    const char *fn = "bml_attn_prefill";
    if (!q_dev || !k_dev || !v_dev || !out_dev) return fail(BML_E_INVALID, "%s: null argument", fn);
    if (!aligned16(q_dev) || !aligned16(k_dev) || !aligned16(v_dev) || !aligned16(out_dev))
        return fail(BML_E_INVALID, "%s: pointers must be 16-byte aligned", fn);
    if (n_seqs == 0 || seq_len == 0 || n_heads == 0 || n_kv_heads == 0)
        return fail(BML_E_INVALID, "%s: zero dimension", fn);
    if (n_heads % n_kv_heads != 0)
        return fail(BML_E_INVALID, "%s: n_heads %u not a multiple of n_kv_heads %u", fn, n_heads, n_kv_heads);
    if (!(in_dtype == BML_BF16 || in_dtype == BML_F16))
        return fail(BML_E_UNSUPPORTED, "%s: inputs must be bf16 or f16", fn);
    if (!(out_dtype == BML_F32 || out_dtype == in_dtype))
        return fail(BML_E_INVALID, "%s: out dtype must be f32 or the input dtype", fn);
    if (!(head_dim == 64 || head_dim == 128))
        return fail(BML_E_UNSUPPORTED, "%s: head_dim %u (supported: 64, 128)", fn, head_dim);
    bml::PrefillArgs a;
    a.q = q_dev;
    a.k = k_dev;
    a.v = v_dev;
    a.out = out_dev;
    a.n_seqs = n_seqs;
    a.seq_len = seq_len;
    a.n_heads = n_heads;
    a.n_kv = n_kv_heads;
    a.head_dim = head_dim;
    a.in_dtype = in_dtype;
    a.out_dtype = out_dtype;
    a.scale = resolve_scale(scale, head_dim);
    a.causal = causal != 0;
    a.num_sms = num_sms(current_device());
    CUDA_TRY(bml::launch_prefill(a, static_cast<cudaStream_t>(stream)), fn);
    return ok();
}

// ---------------------------------------------------------------------------
// Test-only entry points (include/bml_diag.h)
// ---------------------------------------------------------------------------
BML_API bml_status bml_diag_exp2(const float *x_dev, uint32_t n, float *out_dev, void *stream) {
    if (!x_dev || !out_dev || (n & 1u)) return fail(BML_E_INVALID, "bml_diag_exp2: bad argument");
    if (!aligned16(x_dev) || !aligned16(out_dev)) return fail(BML_E_INVALID, "bml_diag_exp2: alignment");
    CUDA_TRY(bml::diag_exp2(x_dev, n, out_dev, static_cast<cudaStream_t>(stream)), "bml_diag_exp2");
    return ok();
}

BML_API bml_status bml_diag_decode_batched(const bml_seq_desc *seqs_host, uint32_t n_seqs, uint32_t n_heads,
                                           uint32_t n_kv_heads, uint32_t head_dim, bml_dtype kv_dtype, float scale,
                                           const float *q_dev, float *out_dev, void *workspace,
                                           size_t workspace_bytes, int kernel, uint64_t wait_ns, uint32_t flags,
                                           void *stream) {
    const char *fn = "bml_diag_decode_batched";
    if (kernel != BML_DIAG_DECODE_DEFAULT && kernel != BML_DIAG_DECODE_CUDA_CORE)
        return fail(BML_E_INVALID, "%s: kernel %d", fn, kernel);
    if (flags & ~BML_DIAG_STALL) return fail(BML_E_INVALID, "%s: flags 0x%x", fn, flags);
    return decode_impl(seqs_host, n_seqs, n_heads, n_kv_heads, head_dim, kv_dtype, scale, q_dev, out_dev, nullptr,
                       nullptr, nullptr, workspace, workspace_bytes, stream, bml::kModeFinal, fn, kernel,
                       wait_ns ? wait_ns : bml::kWaitNs, (flags & BML_DIAG_STALL) ? bml::kDiagStall : 0u);
}

// ---------------------------------------------------------------------------
// softmax_f32 (kv_cache.rs:188-200)
// ---------------------------------------------------------------------------
BML_API bml_status bml_softmax_f32(const float *x_dev, uint32_t n_rows, uint32_t n, float *out_dev, void *stream) {
    if (n == 0 || n_rows == 0) return ok();  // empty in, empty out (kv_cache.rs:189-191)
    if (!x_dev || !out_dev) return fail(BML_E_INVALID, "bml_softmax_f32: null argument");
    CUDA_TRY(bml::softmax_rows(x_dev, n_rows, n, out_dev, static_cast<cudaStream_t>(stream)), "bml_softmax_f32");
    return ok();
}

// ---------------------------------------------------------------------------
// Allocation-free batched decode.
//
// Some callers cannot call cudaMalloc at all: a host runtime that hands all
// device memory to its own pool allocator when it starts, or a serving loop
// in which cudaMalloc's implicit device-wide synchronisation would stall
// the other streams.  For them this entry point takes its split-K scratch
// from a fixed array in device global memory instead of a caller workspace.
// ---------------------------------------------------------------------------
namespace {

// 4 MiB: on a 148-SM B200, enough for 64 sequences x 32 heads x d=128 (the
// 32-sequence Llama-3 decode batch needs 3.0 MB).
constexpr size_t kNoAllocScratchBytes = 4u << 20;

// Every GPU that loads this library holds this array until the process
// exits.  In host code its name is only a stand-in: the device address comes
// from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch array on the current device; looked up once
// per device, with that device current.
bml_status noalloc_scratch(int dev, void **out) {
    if (dev < 0 || dev >= 64) return fail(BML_E_INVALID, "bml_attn_decode_batched_noalloc: device %d", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return cuda_fail(e, "bml_attn_decode_batched_noalloc: cudaGetSymbolAddress");
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return BML_OK;
}

}  // namespace

BML_API bml_status bml_attn_decode_batched_noalloc(const bml_seq_desc *seqs_host, uint32_t n_seqs,
                                                   uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                                   bml_dtype kv_dtype, float scale, const float *q_dev,
                                                   float *out_dev, void *stream) {
    const char *fn = "bml_attn_decode_batched_noalloc";
    bml_status st = check_decode_shape(n_heads, n_kv_heads, head_dim, kv_dtype, fn);
    if (st != BML_OK) return st;
    if (!seqs_host || n_seqs == 0) return fail(BML_E_INVALID, "%s: no sequences", fn);
    const int dev = current_device();
    const size_t need = bml::decode_workspace_min_bytes(n_seqs, n_heads, n_kv_heads, head_dim, num_sms(dev));
    if (need > kNoAllocScratchBytes)
        return fail(BML_E_INVALID, "%s: needs %zu bytes of scratch, above the fixed %zu-byte maximum", fn, need,
                    kNoAllocScratchBytes);
    void *scratch = nullptr;
    st = noalloc_scratch(dev, &scratch);
    if (st != BML_OK) return st;
    // Every call shares the array, which keeps the last call's contents:
    // clear the schedule counters, which must start at zero (each call also
    // leaves them zero).  The error word at offset 0 is left alone, so that
    // a timeout stays recorded until bml_attn_noalloc_check reads it.
    CUDA_TRY(cudaMemsetAsync(static_cast<uint8_t *>(scratch) + 64, 0, bml::decode_workspace_zero_bytes() - 64,
                             static_cast<cudaStream_t>(stream)),
             fn);
    return decode_impl(seqs_host, n_seqs, n_heads, n_kv_heads, head_dim, kv_dtype, scale, q_dev, out_dev, nullptr,
                       nullptr, nullptr, scratch, kNoAllocScratchBytes, stream, bml::kModeFinal, fn);
}

BML_API bml_status bml_attn_noalloc_check(void *stream) {
    void *scratch = nullptr;
    bml_status st = noalloc_scratch(current_device(), &scratch);
    if (st != BML_OK) return st;
    return bml_attn_workspace_check(scratch, kNoAllocScratchBytes, stream);
}

// ---------------------------------------------------------------------------
// KV split of one sequence over GPUs with the exchange in the decode kernel
// ---------------------------------------------------------------------------
struct bml_kvsplit {
    int32_t device = 0;
    uint32_t rank = 0, world = 1, n_heads = 0, head_dim = 0, units = 0;
    float *buf = nullptr;  // this rank's exchange buffer
    size_t bytes = 0;
    float *peer[bml::kMaxExchangeRanks] = {};  // every rank's buffer, mapped here
    bool opened = false;
};

BML_API bml_status bml_kvsplit_create(int32_t device, uint32_t rank, uint32_t world, uint32_t n_heads,
                                      uint32_t head_dim, bml_kvsplit **out) {
    const char *fn = "bml_kvsplit_create";
    if (!out) return fail(BML_E_INVALID, "%s: null output", fn);
    *out = nullptr;
    if (world == 0 || world > (uint32_t)bml::kMaxExchangeRanks || rank >= world)
        return fail(BML_E_INVALID, "%s: rank %u of world %u (at most %d ranks)", fn, rank, world,
                    bml::kMaxExchangeRanks);
    if (n_heads == 0 || n_heads > 256 || !(head_dim == 64 || head_dim == 128))
        return fail(BML_E_UNSUPPORTED, "%s: %u heads of dim %u", fn, n_heads, head_dim);
    DeviceGuard g(device);
    bml_kvsplit *h = new bml_kvsplit();
    h->device = device;
    h->rank = rank;
    h->world = world;
    h->n_heads = n_heads;
    h->head_dim = head_dim;
    h->units = n_heads * (head_dim / 32);
    h->bytes = bml::exchange_bytes(h->units);
    cudaError_t e = cudaMalloc(&h->buf, h->bytes);
    if (e == cudaSuccess) e = cudaMemset(h->buf, 0, h->bytes);  // flags start below every epoch
    if (e != cudaSuccess) {
        if (h->buf) cudaFree(h->buf);
        delete h;
        return cuda_fail(e, fn);
    }
    h->peer[rank] = h->buf;
    *out = h;
    return ok();
}

BML_API bml_status bml_kvsplit_handle(const bml_kvsplit *h, void *handle_out, size_t bytes) {
    if (!h || !handle_out || bytes < BML_KVSPLIT_HANDLE_BYTES)
        return fail(BML_E_INVALID, "bml_kvsplit_handle: null argument or %zu < %d bytes", bytes,
                    BML_KVSPLIT_HANDLE_BYTES);
    DeviceGuard g(h->device);
    cudaIpcMemHandle_t m;
    CUDA_TRY(cudaIpcGetMemHandle(&m, h->buf), "bml_kvsplit_handle");
    memcpy(handle_out, &m, sizeof m);
    return ok();
}

BML_API bml_status bml_kvsplit_open(bml_kvsplit *h, const void *handles, size_t bytes) {
    const char *fn = "bml_kvsplit_open";
    if (!h || !handles) return fail(BML_E_INVALID, "%s: null argument", fn);
    if (h->opened) return fail(BML_E_INVALID, "%s: already open", fn);
    if (bytes != (size_t)h->world * BML_KVSPLIT_HANDLE_BYTES)
        return fail(BML_E_INVALID, "%s: %zu bytes of handles for %u ranks", fn, bytes, h->world);
    DeviceGuard g(h->device);
    for (uint32_t r = 0; r < h->world; ++r) {
        if (r == h->rank) continue;
        cudaIpcMemHandle_t m;
        memcpy(&m, static_cast<const char *>(handles) + (size_t)r * BML_KVSPLIT_HANDLE_BYTES, sizeof m);
        void *ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, m, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (uint32_t q = 0; q < r; ++q)
                if (q != h->rank && h->peer[q]) cudaIpcCloseMemHandle(h->peer[q]);
            return cuda_fail(e, fn);
        }
        h->peer[r] = static_cast<float *>(ptr);
    }
    h->opened = true;
    return ok();
}

BML_API bml_status bml_attn_decode_kvsplit(bml_kvsplit *h, const bml_seq_desc *slice_host, uint32_t n_heads,
                                           uint32_t n_kv_heads, uint32_t head_dim, bml_dtype kv_dtype, float scale,
                                           const float *q_dev, float *out_dev, void *workspace,
                                           size_t workspace_bytes, void *stream) {
    const char *fn = "bml_attn_decode_kvsplit";
    if (!h || !slice_host) return fail(BML_E_INVALID, "%s: null argument", fn);
    if (h->world > 1 && !h->opened) return fail(BML_E_INVALID, "%s: peers not opened", fn);
    if (n_heads != h->n_heads || head_dim != h->head_dim)
        return fail(BML_E_INVALID, "%s: %u heads of dim %u, the handle has %u of dim %u", fn, n_heads, head_dim,
                    h->n_heads, h->head_dim);
    DeviceGuard g(h->device);
    if (h->world == 1)
        return decode_impl(slice_host, 1, n_heads, n_kv_heads, head_dim, kv_dtype, scale, q_dev, out_dev, nullptr,
                           nullptr, nullptr, workspace, workspace_bytes, stream, bml::kModeFinal, fn);
    ExchangeArgs xa;
    xa.world = h->world;
    xa.rank = h->rank;
    // the epoch lives on the device (the kernel advances it), so a call may
    // be captured in a CUDA graph and replayed
    xa.epoch = reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(h->buf) + bml::exchange_epoch_offset(h->units));
    for (uint32_t r = 0; r < h->world; ++r) xa.base[r] = h->peer[r];
    return decode_impl(slice_host, 1, n_heads, n_kv_heads, head_dim, kv_dtype, scale, q_dev, out_dev, nullptr, nullptr,
                       nullptr, workspace, workspace_bytes, stream, bml::kModeFinal, fn, 0, bml::kWaitNs, 0, &xa);
}

BML_API bml_status bml_kvsplit_destroy(bml_kvsplit *h) {
    if (!h) return ok();
    DeviceGuard g(h->device);
    for (uint32_t r = 0; r < h->world; ++r)
        if (r != h->rank && h->peer[r]) cudaIpcCloseMemHandle(h->peer[r]);
    if (h->buf) cudaFree(h->buf);
    delete h;
    return ok();
}

// ---------------------------------------------------------------------------
// Weight path: read_tensor_f32 and matmul_f64 (gguf_compiler.rs:351-470,
// :1239-1255)
// ---------------------------------------------------------------------------
namespace {

bool gguf_type_read(int32_t t) {
    return t == BML_GGUF_F32 || t == BML_GGUF_F16 || t == BML_GGUF_Q4_0 || t == BML_GGUF_Q8_0;
}

bool aligned_to(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

BML_API bml_status bml_read_tensor_f32(const void *data_dev, uint64_t data_len, int32_t gguf_type, uint64_t n_elems,
                                       float *out_dev, uint64_t *n_values, void *stream) {
    const char *fn = "bml_read_tensor_f32";
    if (!gguf_type_read(gguf_type))
        return fail(BML_E_UNSUPPORTED, "%s: GGUF type %d (the reference reads F32, F16, Q4_0, Q8_0)", fn, gguf_type);
    if (!n_values) return fail(BML_E_INVALID, "%s: null n_values", fn);
    const uint64_t n = bml::gguf_values_read(gguf_type, data_len, n_elems);
    if (n && (!data_dev || !out_dev)) return fail(BML_E_INVALID, "%s: null argument", fn);
    if (n && (!aligned_to(data_dev, gguf_type == BML_GGUF_F32 ? 4 : 2) || !aligned_to(out_dev, 16)))
        return fail(BML_E_INVALID, "%s: data must be %d-byte and out 16-byte aligned", fn,
                    gguf_type == BML_GGUF_F32 ? 4 : 2);
    CUDA_TRY(bml::read_tensor_f32(data_dev, data_len, gguf_type, n_elems, out_dev, static_cast<cudaStream_t>(stream)),
             fn);
    *n_values = n;
    return ok();
}

BML_API bml_status bml_matmul_workspace_size(uint64_t n_out, size_t *bytes) {
    if (!bytes) return fail(BML_E_INVALID, "bml_matmul_workspace_size: null output");
    *bytes = bml::gemv_workspace_bytes(n_out);
    return ok();
}

static bml_status matmul_impl(const char *fn, const void *w_dev, uint64_t data_len, int32_t gguf_type, uint64_t n_in,
                              uint64_t n_out, const double *x_dev, uint64_t x_len, double *y_dev, void *workspace,
                              size_t ws_bytes, bool static_weights, void *stream) {
    if (!gguf_type_read(gguf_type))
        return fail(BML_E_UNSUPPORTED, "%s: GGUF type %d (the reference reads F32, F16, Q4_0, Q8_0)", fn, gguf_type);
    if (n_out == 0) return ok();
    if (!y_dev || (x_len && (!w_dev || !x_dev))) return fail(BML_E_INVALID, "%s: null argument", fn);
    if ((gguf_type == BML_GGUF_Q4_0 || gguf_type == BML_GGUF_Q8_0) && n_out % 32 != 0)
        return fail(BML_E_UNSUPPORTED, "%s: quantized tensors need n_out %% 32 == 0 (n_out %llu)", fn,
                    (unsigned long long)n_out);
    const uintptr_t wa = gguf_type == BML_GGUF_F32 ? 16 : gguf_type == BML_GGUF_F16 ? 16 : 2;
    if ((w_dev && !aligned_to(w_dev, wa)) || !aligned_to(y_dev, 8) || (x_dev && !aligned_to(x_dev, 8)))
        return fail(BML_E_INVALID, "%s: W must be %u-byte aligned, x and y 8-byte aligned", fn, (unsigned)wa);
    if (n_in > (1ull << 40) || n_out > (1ull << 40)) return fail(BML_E_INVALID, "%s: dimensions too large", fn);
    const int sms = num_sms(current_device());
    const bml::GemvPlan pl =
        bml::gemv_plan(n_in, n_out, x_len, sms, bml::gemv_staged_ok(w_dev, data_len, gguf_type, n_in, n_out));
    if (pl.ranges > 1 && (!workspace || ws_bytes < (size_t)pl.ranges * n_out * sizeof(double)))
        return fail(BML_E_INVALID, "%s: workspace of %zu bytes, need %zu", fn, ws_bytes,
                    bml::gemv_workspace_bytes(n_out));
    CUDA_TRY(bml::gemv(w_dev, data_len, gguf_type, n_in, n_out, x_dev, x_len, y_dev, static_cast<double *>(workspace),
                       sms, static_weights, static_cast<cudaStream_t>(stream)),
             fn);
    return ok();
}

BML_API bml_status bml_matmul_f64(const void *w_dev, uint64_t data_len, int32_t gguf_type, uint64_t n_in,
                                  uint64_t n_out, const double *x_dev, uint64_t x_len, double *y_dev, void *workspace,
                                  size_t ws_bytes, void *stream) {
    return matmul_impl("bml_matmul_f64", w_dev, data_len, gguf_type, n_in, n_out, x_dev, x_len, y_dev, workspace,
                       ws_bytes, false, stream);
}

BML_API bml_status bml_matmul_f64_static(const void *w_dev, uint64_t data_len, int32_t gguf_type, uint64_t n_in,
                                         uint64_t n_out, const double *x_dev, uint64_t x_len, double *y_dev,
                                         void *workspace, size_t ws_bytes, void *stream) {
    return matmul_impl("bml_matmul_f64_static", w_dev, data_len, gguf_type, n_in, n_out, x_dev, x_len, y_dev,
                       workspace, ws_bytes, true, stream);
}
