/*
 * bml_oracle.c -- CPU restatement of bml's attention / KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library
 * (bml_b200/libbmlattn.so).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * path never calls it and has no CPU fallback.
 *
 * What it restates (paths inside the SugarFreeDoNoSo/bml project):
 *   crates/compiler/src/kv_cache.rs:25-181     HashConsedKV (flat f32 buffers,
 *                                              ring index pos % max_seq_len)
 *   crates/compiler/src/kv_cache.rs:188-200    softmax_f32
 *   crates/compiler/src/gguf_compiler.rs:1008-1050
 *                                              GQA attention of one token
 *   crates/compiler/src/gguf_compiler.rs:946-958
 *                                              prefill = per-token causal loop
 *   crates/compiler/src/gguf_compiler.rs:1290-1317
 *                                              RoPE (theta 10000, interleaved)
 *
 * Numerics follow the Rust types exactly: the Q.K dot is a sequential f32
 * sum of f32 products (Rust never contracts to FMA, so this file must be
 * compiled with -ffp-contract=off and without fast-math), the scale is f64,
 * scores are rounded to f32 for softmax_f32 (expf from libm, which is what
 * Rust's f32::exp calls on Linux), and P.V is accumulated in f64 in
 * position order.
 *
 * Pinning: the KV-cache, softmax and RoPE pieces are checked against every
 * unit test the reference holds for them (kv_cache.rs:211-316,
 * eml.rs:237-266).  The reference has no test and no golden vector for the
 * attention loop itself, and it cannot be built here (Rust toolchain absent),
 * so end-to-end attention parity is unpinned by reference-produced vectors:
 * it rests on this restatement plus analytic known-answer cases.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_K 0
#define ORC_V 1

/* ------------------------------------------------------------------------ */
/* HashConsedKV (kv_cache.rs:25-181)                                          */
/* ------------------------------------------------------------------------ */

typedef struct orc_kv {
    float **k_buffers; /* [n_layers][max_seq_len * stride] */
    float **v_buffers;
    uint32_t n_layers, n_kv_heads, head_dim, max_seq_len;
    size_t stride;     /* n_kv_heads * head_dim (kv_cache.rs:54) */
    uint32_t current_pos;
    uint64_t n_total_k, n_total_v;
} orc_kv;

/* HashConsedKV::new (kv_cache.rs:53-72): zeroed per-layer buffers. */
orc_kv *orc_kv_new(uint32_t n_layers, uint32_t n_kv_heads, uint32_t head_dim,
                   uint32_t max_seq_len) {
    orc_kv *kv = (orc_kv *)calloc(1, sizeof(orc_kv));
    if (!kv) return NULL;
    kv->n_layers = n_layers;
    kv->n_kv_heads = n_kv_heads;
    kv->head_dim = head_dim;
    kv->max_seq_len = max_seq_len;
    kv->stride = (size_t)n_kv_heads * head_dim;
    size_t n = kv->stride * max_seq_len;
    kv->k_buffers = (float **)calloc(n_layers ? n_layers : 1, sizeof(float *));
    kv->v_buffers = (float **)calloc(n_layers ? n_layers : 1, sizeof(float *));
    for (uint32_t l = 0; l < n_layers; ++l) {
        kv->k_buffers[l] = (float *)calloc(n ? n : 1, sizeof(float));
        kv->v_buffers[l] = (float *)calloc(n ? n : 1, sizeof(float));
    }
    return kv;
}

void orc_kv_free(orc_kv *kv) {
    if (!kv) return;
    for (uint32_t l = 0; l < kv->n_layers; ++l) {
        free(kv->k_buffers[l]);
        free(kv->v_buffers[l]);
    }
    free(kv->k_buffers);
    free(kv->v_buffers);
    free(kv);
}

static size_t orc_slot(const orc_kv *kv, uint32_t pos, uint32_t kv_head) {
    size_t pos_idx = (size_t)(pos % kv->max_seq_len);
    return pos_idx * kv->stride + (size_t)kv_head * kv->head_dim;
}

/* store_k / store_v (kv_cache.rs:82-101): copies min(head_dim, len) floats
 * into ring slot pos % max_seq_len and counts the store.  Returns -1 where
 * the Rust code would panic (slice index out of range). */
int orc_kv_store(orc_kv *kv, int which, uint32_t layer, uint32_t pos,
                 uint32_t kv_head, const float *data, size_t len) {
    size_t d = kv->head_dim;
    size_t n = len < d ? len : d;
    if (layer >= kv->n_layers) return -1;
    size_t start = orc_slot(kv, pos, kv_head);
    if (start + d > kv->stride * kv->max_seq_len) return -1;
    /* Rust's copy_from_slice panics unless both sides have equal length:
     * dst is [start..start+d], src is data[..min(d,len)]. */
    if (n != d) return -1;
    float *dst = (which == ORC_K ? kv->k_buffers : kv->v_buffers)[layer] + start;
    memcpy(dst, data, n * sizeof(float));
    if (which == ORC_K) kv->n_total_k++; else kv->n_total_v++;
    return 0;
}

/* load_k / load_v (kv_cache.rs:111-124): owned copy of one head vector. */
int orc_kv_load(const orc_kv *kv, int which, uint32_t layer, uint32_t pos,
                uint32_t kv_head, float *out) {
    if (layer >= kv->n_layers) return -1;
    size_t start = orc_slot(kv, pos, kv_head);
    if (start + kv->head_dim > kv->stride * kv->max_seq_len) return -1;
    const float *src = (which == ORC_K ? kv->k_buffers : kv->v_buffers)[layer] + start;
    memcpy(out, src, kv->head_dim * sizeof(float));
    return 0;
}

/* dot_qk (kv_cache.rs:135-141): zip stops at the shorter slice; sequential
 * f32 sum of f32 products. */
float orc_kv_dot_qk(const orc_kv *kv, const float *q, size_t q_len,
                    uint32_t layer, uint32_t pos, uint32_t kv_head) {
    size_t start = orc_slot(kv, pos, kv_head);
    const float *k = kv->k_buffers[layer] + start;
    size_t n = q_len < kv->head_dim ? q_len : kv->head_dim;
    float acc = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        float prod = q[i] * k[i];
        acc = acc + prod;
    }
    return acc;
}

/* k_stats / v_stats (kv_cache.rs:148-155): no dedup, unique == total. */
void orc_kv_stats(const orc_kv *kv, int which, uint64_t *unique,
                  uint64_t *total, double *ratio) {
    uint64_t t = which == ORC_K ? kv->n_total_k : kv->n_total_v;
    *unique = t;
    *total = t;
    *ratio = 1.0;
}

/* byte_size (kv_cache.rs:158-161). */
uint64_t orc_kv_byte_size(const orc_kv *kv) {
    uint64_t per_layer = (uint64_t)kv->stride * kv->max_seq_len * sizeof(float);
    return per_layer * kv->n_layers * 2;
}

uint32_t orc_kv_current_pos(const orc_kv *kv) { return kv->current_pos; }
void orc_kv_advance(orc_kv *kv) { kv->current_pos += 1; }
void orc_kv_advance_by(orc_kv *kv, uint32_t n) { kv->current_pos += n; }
float *orc_kv_buffer(orc_kv *kv, int which, uint32_t layer) {
    return (which == ORC_K ? kv->k_buffers : kv->v_buffers)[layer];
}

/* ------------------------------------------------------------------------ */
/* softmax_f32 (kv_cache.rs:188-200)                                        */
/* ------------------------------------------------------------------------ */

/* f32::max: if one operand is NaN the other is returned. */
static float rust_f32_max(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

/* Writes n probabilities to out (out may alias s). Returns n. */
size_t orc_softmax_f32(const float *s, size_t n, float *out) {
    if (n == 0) return 0;
    float mx = -INFINITY;
    for (size_t i = 0; i < n; ++i) mx = rust_f32_max(mx, s[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        float e = expf(s[i] - mx);
        out[i] = e;
        sum = sum + e;
    }
    if (sum > 0.0f) {
        for (size_t i = 0; i < n; ++i) out[i] = out[i] / sum;
    } else {
        float u = 1.0f / (float)n;
        for (size_t i = 0; i < n; ++i) out[i] = u;
    }
    return n;
}

/* ------------------------------------------------------------------------ */
/* RoPE (gguf_compiler.rs:1290-1317)                                        */
/* ------------------------------------------------------------------------ */

/* In place on an f64 vector of n_heads*head_dim values at position pos. */
void orc_rope_inplace_f64(double *x, size_t len, size_t pos, size_t head_dim) {
    size_t n_half = head_dim / 2;
    size_t n_heads = len / head_dim;
    for (size_t h = 0; h < n_heads; ++h) {
        for (size_t i = 0; i < n_half; ++i) {
            size_t e = h * head_dim + i * 2, o = e + 1;
            double xe = e < len ? x[e] : 0.0;
            double xo = o < len ? x[o] : 0.0;
            double freq = 1.0 / pow(10000.0, 2.0 * (double)i / (double)head_dim);
            double angle = (double)pos * freq;
            double c = cos(angle), s = sin(angle);
            double re = xe * c - xo * s;
            double ro = xe * s + xo * c;
            if (e < len) x[e] = re;
            if (o < len) x[o] = ro;
        }
    }
}

/* Applies RoPE to rows of f32 vectors [n_rows][row_len] at positions
 * pos0 + r, through f64 exactly as the reference does (f32 -> f64 ->
 * rotate -> stored back as f32). */
void orc_rope_rows_f32(float *x, size_t n_rows, size_t row_len, size_t pos0,
                       size_t head_dim) {
    double *tmp = (double *)malloc(row_len * sizeof(double));
    for (size_t r = 0; r < n_rows; ++r) {
        float *row = x + r * row_len;
        for (size_t i = 0; i < row_len; ++i) tmp[i] = (double)row[i];
        orc_rope_inplace_f64(tmp, row_len, pos0 + r, head_dim);
        for (size_t i = 0; i < row_len; ++i) row[i] = (float)tmp[i];
    }
    free(tmp);
}

/* ------------------------------------------------------------------------ */
/* Attention block (gguf_compiler.rs:1008-1050)                             */
/* ------------------------------------------------------------------------ */

/* 16-bit storage formats widen exactly to f32. */
static float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float orc_bf16_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* dtype codes match bml_dtype in include/bml_attn.h */
#define ORC_F32 0
#define ORC_F16 1
#define ORC_BF16 2

static inline float orc_elem(const void *base, size_t idx, int dtype) {
    if (dtype == ORC_F32) return ((const float *)base)[idx];
    uint16_t u = ((const uint16_t *)base)[idx];
    return dtype == ORC_F16 ? orc_f16_to_f32(u) : orc_bf16_to_f32(u);
}

/*
 * One head of the attention block for the token at absolute position pos:
 * scores over p in [p_lo, pos] (the reference always uses p_lo = 0; a
 * nonzero p_lo is not a reference feature and is only used to build
 * KV-split test cases), softmax_f32, f64 P.V.
 *   q_head : [head_dim] f32
 *   kbuf/vbuf : flat cache [max_seq_len][n_kv][head_dim] in `dtype`, ring
 *               index p % max_seq_len (kv_cache.rs:83)
 *   scores : scratch of pos+1 floats
 *   out    : [head_dim] f64
 */
static void orc_attn_one_head(const float *q_head, const void *kbuf,
                              const void *vbuf, int dtype, uint32_t max_seq_len,
                              uint32_t n_kv, uint32_t head_dim, uint32_t kv_h,
                              uint32_t pos, double scale, float *scores,
                              double *out) {
    size_t stride = (size_t)n_kv * head_dim;
    uint32_t n = pos + 1;
    /* :1026-1034 */
    for (uint32_t p = 0; p <= pos; ++p) {
        size_t base = (size_t)(p % max_seq_len) * stride + (size_t)kv_h * head_dim;
        float dot = 0.0f;
        for (uint32_t i = 0; i < head_dim; ++i) {
            float prod = q_head[i] * orc_elem(kbuf, base + i, dtype);
            dot = dot + prod;
        }
        double sc = (double)dot * scale;
        scores[p] = (float)sc; /* :1038 casts each score to f32 */
    }
    /* :1037-1038 */
    orc_softmax_f32(scores, n, scores);
    /* :1042-1049: for each d, sum over p in f64 */
    for (uint32_t d = 0; d < head_dim; ++d) out[d] = 0.0;
    for (uint32_t p = 0; p <= pos; ++p) {
        size_t base = (size_t)(p % max_seq_len) * stride + (size_t)kv_h * head_dim;
        double a = (double)scores[p];
        for (uint32_t d = 0; d < head_dim; ++d) {
            /* the per-d sums are independent and each is still summed in
             * increasing p, so swapping the loop order keeps every f64
             * rounding step of the reference's d-outer loop. */
            out[d] = out[d] + a * (double)orc_elem(vbuf, base + d, dtype);
        }
    }
}

/* Checks the GQA head map of gguf_compiler.rs:991-1016.  Returns the
 * q-heads-per-kv-head group size, or 0 when the shape is rejected. */
static uint32_t orc_group(uint32_t n_heads, uint32_t n_kv) {
    if (n_kv == 0 || n_heads == 0) return 0;
    uint32_t g = n_heads / n_kv;
    if (g == 0 || g * n_kv != n_heads) return 0;
    return g;
}

/*
 * Decode attention of one token at position pos (gguf_compiler.rs:1008-1050)
 * over one sequence's cache.  q: [n_heads][head_dim] f32.  out: [n_heads]
 * [head_dim] f64.  scale < 0 means the reference's 1/sqrt(head_dim) in f64.
 * Returns 0, or -1 for a rejected shape.
 */
int orc_attn_decode(const float *q, const void *kbuf, const void *vbuf,
                    int dtype, uint32_t max_seq_len, uint32_t n_kv,
                    uint32_t head_dim, uint32_t n_heads, uint32_t pos,
                    double scale, double *out, int n_threads) {
    uint32_t g = orc_group(n_heads, n_kv);
    if (!g || head_dim == 0 || max_seq_len == 0) return -1;
    if (scale < 0) scale = 1.0 / sqrt((double)head_dim);
#ifdef _OPENMP
    if (n_threads < 1) n_threads = omp_get_max_threads();
#pragma omp parallel num_threads(n_threads) if (n_threads > 1)
#endif
    {
        float *scores = (float *)malloc(((size_t)pos + 1) * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int h = 0; h < (int)n_heads; ++h) {
            uint32_t kv_h = (uint32_t)h / g;
            orc_attn_one_head(q + (size_t)h * head_dim, kbuf, vbuf, dtype,
                              max_seq_len, n_kv, head_dim, kv_h, pos, scale,
                              scores, out + (size_t)h * head_dim);
        }
        free(scores);
    }
    return 0;
}

/*
 * Batched decode: sequence s has its own contiguous cache of lens[s]
 * positions ([len][n_kv][head_dim]); its query token sits at position
 * lens[s]-1 and attends over all of them.  k_ptrs/v_ptrs are per-sequence
 * base pointers.  q: [n_seqs][n_heads][head_dim]; out likewise in f64.
 * Parallel over (sequence, head) with n_threads (1 = the reference's single
 * thread).
 */
int orc_attn_decode_batched(const float *q, const void *const *k_ptrs,
                            const void *const *v_ptrs, const uint32_t *lens,
                            uint32_t n_seqs, int dtype, uint32_t n_kv,
                            uint32_t head_dim, uint32_t n_heads, double scale,
                            double *out, int n_threads) {
    uint32_t g = orc_group(n_heads, n_kv);
    if (!g || head_dim == 0) return -1;
    for (uint32_t s = 0; s < n_seqs; ++s)
        if (lens[s] == 0) return -1;
    if (scale < 0) scale = 1.0 / sqrt((double)head_dim);
    uint32_t max_len = 0;
    for (uint32_t s = 0; s < n_seqs; ++s) if (lens[s] > max_len) max_len = lens[s];
    long total = (long)n_seqs * n_heads;
#ifdef _OPENMP
    if (n_threads < 1) n_threads = omp_get_max_threads();
#pragma omp parallel num_threads(n_threads) if (n_threads > 1)
#endif
    {
        float *scores = (float *)malloc((size_t)max_len * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (long w = 0; w < total; ++w) {
            uint32_t s = (uint32_t)(w / n_heads), h = (uint32_t)(w % n_heads);
            orc_attn_one_head(q + ((size_t)s * n_heads + h) * head_dim,
                              k_ptrs[s], v_ptrs[s], dtype, lens[s], n_kv,
                              head_dim, h / g, lens[s] - 1, scale, scores,
                              out + ((size_t)s * n_heads + h) * head_dim);
        }
        free(scores);
    }
    return 0;
}

/*
 * Causal prefill = the forward_cached token loop (gguf_compiler.rs:946-958)
 * with start_pos = 0: token t attends over [0, t] of the same sequence.
 * q: [n_seqs][seq_len][n_heads][head_dim] f32 (RoPE already applied),
 * k/v: [n_seqs][seq_len][n_kv][head_dim] in dtype, out: same shape as q in
 * f64.  Only query rows [row_lo, row_hi) are computed (the rest of out is
 * untouched) so that large shapes can be checked on a sample of rows.
 */
int orc_attn_prefill(const float *q, const void *k, const void *v, int dtype,
                     uint32_t n_seqs, uint32_t seq_len, uint32_t n_heads,
                     uint32_t n_kv, uint32_t head_dim, double scale,
                     uint32_t row_lo, uint32_t row_hi, double *out,
                     int n_threads) {
    uint32_t g = orc_group(n_heads, n_kv);
    if (!g || head_dim == 0 || seq_len == 0) return -1;
    if (row_hi > seq_len) row_hi = seq_len;
    if (row_lo >= row_hi) return 0;
    if (scale < 0) scale = 1.0 / sqrt((double)head_dim);
    size_t es = dtype == ORC_F32 ? 4 : 2;
    size_t kv_seq_elems = (size_t)seq_len * n_kv * head_dim;
    long rows = (long)row_hi - row_lo;
    long total = (long)n_seqs * rows * n_heads;
#ifdef _OPENMP
    if (n_threads < 1) n_threads = omp_get_max_threads();
#pragma omp parallel num_threads(n_threads) if (n_threads > 1)
#endif
    {
        float *scores = (float *)malloc((size_t)seq_len * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
        for (long w = 0; w < total; ++w) {
            uint32_t h = (uint32_t)(w % n_heads);
            long rest = w / n_heads;
            uint32_t t = row_lo + (uint32_t)(rest % rows);
            uint32_t s = (uint32_t)(rest / rows);
            const char *ks = (const char *)k + (size_t)s * kv_seq_elems * es;
            const char *vs = (const char *)v + (size_t)s * kv_seq_elems * es;
            size_t qo = (((size_t)s * seq_len + t) * n_heads + h) * head_dim;
            orc_attn_one_head(q + qo, ks, vs, dtype, seq_len, n_kv, head_dim,
                              h / g, t, scale, scores, out + qo);
        }
        free(scores);
    }
    return 0;
}

/*
 * Prefill at query rows chosen by the caller: row r of the result is query
 * position rows[2r + 1] of sequence rows[2r], for q heads [h_lo, h_hi).
 * Each row is the same per-token causal attention as orc_attn_prefill
 * (gguf_compiler.rs:946-958 over :1008-1050), and rows do not depend on one
 * another, so a subset gives exactly the values of the full loop.
 * out: [n_rows][h_hi - h_lo][head_dim] f64.  Parallel over (row, head).
 */
int orc_attn_prefill_rows(const float *q, const void *k, const void *v, int dtype,
                          uint32_t n_seqs, uint32_t seq_len, uint32_t n_heads,
                          uint32_t n_kv, uint32_t head_dim, double scale,
                          const uint32_t *rows, uint32_t n_rows, uint32_t h_lo,
                          uint32_t h_hi, double *out, int n_threads) {
    uint32_t g = orc_group(n_heads, n_kv);
    if (!g || head_dim == 0 || seq_len == 0 || h_lo >= h_hi || h_hi > n_heads) return -1;
    for (uint32_t r = 0; r < n_rows; ++r)
        if (rows[2 * r] >= n_seqs || rows[2 * r + 1] >= seq_len) return -1;
    if (scale < 0) scale = 1.0 / sqrt((double)head_dim);
    size_t es = dtype == ORC_F32 ? 4 : 2;
    size_t kv_seq_elems = (size_t)seq_len * n_kv * head_dim;
    uint32_t nh = h_hi - h_lo;
    long total = (long)n_rows * nh;
#ifdef _OPENMP
    if (n_threads < 1) n_threads = omp_get_max_threads();
#pragma omp parallel num_threads(n_threads) if (n_threads > 1)
#endif
    {
        float *scores = (float *)malloc((size_t)seq_len * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
        for (long w = 0; w < total; ++w) {
            uint32_t r = (uint32_t)(w / nh), h = h_lo + (uint32_t)(w % nh);
            uint32_t s = rows[2 * r], t = rows[2 * r + 1];
            const char *ks = (const char *)k + (size_t)s * kv_seq_elems * es;
            const char *vs = (const char *)v + (size_t)s * kv_seq_elems * es;
            size_t qo = (((size_t)s * seq_len + t) * n_heads + h) * head_dim;
            orc_attn_one_head(q + qo, ks, vs, dtype, seq_len, n_kv, head_dim, h / g, t, scale, scores,
                              out + ((size_t)r * nh + (h - h_lo)) * head_dim);
        }
        free(scores);
    }
    return 0;
}

/*
 * The reference's literal access pattern for one decode token
 * (gguf_compiler.rs:1026-1049): a fresh heap copy for every load_k, and for
 * every load_v inside the head_dim loop, which makes the loop O(H*d*d*L).
 * Numerically identical to orc_attn_decode; it exists only so the CPU
 * baseline can also be timed with the reference's own memory behaviour.
 */
int orc_attn_decode_literal(const float *q, const float *kbuf,
                            const float *vbuf, uint32_t max_seq_len,
                            uint32_t n_kv, uint32_t head_dim, uint32_t n_heads,
                            uint32_t h_lo, uint32_t h_hi, uint32_t pos,
                            double *out) {
    uint32_t g = orc_group(n_heads, n_kv);
    if (!g) return -1;
    double scale = 1.0 / sqrt((double)head_dim);
    size_t stride = (size_t)n_kv * head_dim;
    float *scores = (float *)malloc(((size_t)pos + 1) * sizeof(float));
    for (uint32_t h = h_lo; h < h_hi && h < n_heads; ++h) {
        uint32_t kv_h = h / g;
        const float *qh = q + (size_t)h * head_dim;
        for (uint32_t p = 0; p <= pos; ++p) {
            size_t base = (size_t)(p % max_seq_len) * stride + (size_t)kv_h * head_dim;
            float *kc = (float *)malloc(head_dim * sizeof(float));
            memcpy(kc, kbuf + base, head_dim * sizeof(float));
            float dot = 0.0f;
            for (uint32_t i = 0; i < head_dim; ++i) {
                float prod = qh[i] * kc[i];
                dot = dot + prod;
            }
            free(kc);
            scores[p] = (float)((double)dot * scale);
        }
        orc_softmax_f32(scores, (size_t)pos + 1, scores);
        for (uint32_t d = 0; d < head_dim; ++d) {
            double sum = 0.0;
            for (uint32_t p = 0; p <= pos; ++p) {
                size_t base = (size_t)(p % max_seq_len) * stride + (size_t)kv_h * head_dim;
                float *vc = (float *)malloc(head_dim * sizeof(float));
                memcpy(vc, vbuf + base, head_dim * sizeof(float));
                sum += (double)scores[p] * (double)vc[d];
                free(vc);
            }
            out[(size_t)h * head_dim + d] = sum;
        }
    }
    free(scores);
    return 0;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* Weight path: read_tensor_f32 and matmul_f64                              */
/* (gguf_compiler.rs:351-470, :1239-1255)                                   */
/* ------------------------------------------------------------------------ */

/* f16_to_f32 (gguf_compiler.rs:373-403): sign, 5-bit exponent, 10-bit
 * mantissa; subnormals mant * 2^-24, exponent 31 -> inf / NaN, otherwise
 * (1 + mant/1024) * 2^(exp-15), all exact in f32. */
float orc_gguf_f16_to_f32(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1u, ex = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    float val;
    if (ex == 0) {
        if (mant == 0) return sign ? -0.0f : 0.0f;
        val = (float)mant * ldexpf(1.0f, -24);
    } else if (ex == 0x1F) {
        if (mant == 0) return sign ? -INFINITY : INFINITY;
        return NAN;
    } else {
        val = (1.0f + (float)mant / 1024.0f) * ldexpf(1.0f, (int)ex - 15);
    }
    return sign ? -val : val;
}

/* GGUF tensor types the reference reads as f32 (read_tensor_f32). */
enum { ORC_GGUF_F32 = 0, ORC_GGUF_F16 = 1, ORC_GGUF_Q4_0 = 2, ORC_GGUF_Q8_0 = 8 };

/* read_tensor_f32 (gguf_compiler.rs:351-369) for n_elems elements of a
 * tensor whose data is `data` (data_len bytes).  F32 / F16: one value per
 * 4 / 2 bytes (chunks_exact: a trailing partial chunk is dropped, so the
 * output has data_len / 4 or / 2 values).  Q4_0 (dequantize_q4_0,
 * :405-438): blocks of 18 bytes, an f16 scale then 16 bytes; byte i gives
 * elements 2i (low nibble) and 2i+1 (high nibble), value (q - 8) * scale.
 * Q8_0 (dequantize_q8_0, :440-470): blocks of 34 bytes, an f16 scale then
 * 32 int8, value q * scale.  Quantized types decode n_elems / 32 whole
 * blocks, stop at the first block that does not fit in data_len, and pad
 * with zeros up to n_elems.  Returns the number of values written, or -1
 * for a type the reference does not read. */
int64_t orc_read_tensor_f32(const uint8_t *data, uint64_t data_len, int type, uint64_t n_elems, float *out) {
    if (type == ORC_GGUF_F32) {
        const uint64_t n = data_len / 4;
        for (uint64_t i = 0; i < n; ++i) memcpy(&out[i], data + 4 * i, 4);
        return (int64_t)n;
    }
    if (type == ORC_GGUF_F16) {
        const uint64_t n = data_len / 2;
        for (uint64_t i = 0; i < n; ++i) {
            const uint16_t h = (uint16_t)(data[2 * i] | (data[2 * i + 1] << 8));
            out[i] = orc_gguf_f16_to_f32(h);
        }
        return (int64_t)n;
    }
    if (type != ORC_GGUF_Q4_0 && type != ORC_GGUF_Q8_0) return -1;
    const uint64_t block_bytes = type == ORC_GGUF_Q4_0 ? 18 : 34;
    const uint64_t n_blocks = n_elems / 32;
    uint64_t w = 0;
    for (uint64_t b = 0; b < n_blocks; ++b) {
        const uint64_t off = b * block_bytes;
        if (off + block_bytes > data_len) break;
        const float scale = orc_gguf_f16_to_f32((uint16_t)(data[off] | (data[off + 1] << 8)));
        if (type == ORC_GGUF_Q4_0) {
            for (int i = 0; i < 16; ++i) {
                const uint8_t byte = data[off + 2 + i];
                out[w++] = (float)((int)(byte & 0x0F) - 8) * scale;
                out[w++] = (float)((int)((byte >> 4) & 0x0F) - 8) * scale;
            }
        } else {
            for (int i = 0; i < 32; ++i) out[w++] = (float)(int8_t)data[off + 2 + i] * scale;
        }
    }
    while (w < n_elems) out[w++] = 0.0f;
    return (int64_t)w;
}

/* matmul_f64 (gguf_compiler.rs:1239-1255): y[j] = sum over i < min(x_len,
 * n_in) of x[i] * W[i*n_out + j], with W the tensor's f32 values in file
 * order (w_len of them; terms past the end are skipped, as the reference
 * skips indices past its pool), accumulated in f64 in order of i. */
void orc_matmul_f64(const float *W, uint64_t w_len, uint64_t n_in, uint64_t n_out, const double *x, uint64_t x_len,
                    double *y) {
    const uint64_t rows = x_len < n_in ? x_len : n_in;
    for (uint64_t j = 0; j < n_out; ++j) {
        double dot = 0.0;
        for (uint64_t i = 0; i < rows; ++i) {
            const uint64_t idx = i * n_out + j;
            if (idx < w_len) dot += x[i] * (double)W[idx];
        }
        y[j] = dot;
    }
}
