// bml_attn.hpp -- header-only C++ mirror of bml's Rust attention API over the
// C ABI in bml_attn.h.
//
// It reproduces the surface of crates/compiler/src/kv_cache.rs
// (SugarFreeDoNoSo/bml): HashConsedKV with new / store_k / store_v /
// load_k / load_v / dot_qk / k_stats / v_stats / byte_size / current_pos /
// advance / advance_by, and softmax_f32.  Where the Rust code panics on an
// out-of-range index, these methods throw bml::Panic.  The cache lives on a
// CUDA device; attention() is the attention block of forward_layer_cached
// (crates/compiler/src/gguf_compiler.rs:1008-1050) run on that device.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "bml_attn.h"

namespace bml {

// Raised for BML_E_INVALID: the reference panics in these cases.
struct Panic : std::out_of_range {
    using std::out_of_range::out_of_range;
};

// Raised for every other non-OK status.
struct Error : std::runtime_error {
    bml_status status;
    Error(bml_status s, const std::string &m) : std::runtime_error(m), status(s) {}
};

inline void check(bml_status s, const char *fn) {
    if (s == BML_OK) return;
    std::string msg = std::string(fn) + ": " + bml_last_error();
    if (s == BML_E_INVALID) throw Panic(msg);
    throw Error(s, msg);
}

class HashConsedKV {
  public:
    // HashConsedKV::new (kv_cache.rs:53)
    HashConsedKV(uint32_t n_layers, uint32_t n_kv_heads, uint32_t head_dim, uint32_t max_seq_len,
                 bml_dtype dtype = BML_F32, int device = 0)
        : head_dim_(head_dim) {
        bml_kv_desc d{n_layers, n_kv_heads, head_dim, max_seq_len, dtype, device};
        check(bml_kv_create(&d, &kv_), "HashConsedKV::new");
    }
    ~HashConsedKV() { bml_kv_destroy(kv_); }
    HashConsedKV(const HashConsedKV &) = delete;
    HashConsedKV &operator=(const HashConsedKV &) = delete;

    // store_k / store_v (kv_cache.rs:82-101)
    void store_k(uint32_t layer, uint32_t pos, uint32_t kv_head, const std::vector<float> &data) {
        check(bml_kv_store(kv_, BML_WHICH_K, layer, pos, kv_head, data.data(), data.size()), "store_k");
    }
    void store_v(uint32_t layer, uint32_t pos, uint32_t kv_head, const std::vector<float> &data) {
        check(bml_kv_store(kv_, BML_WHICH_V, layer, pos, kv_head, data.data(), data.size()), "store_v");
    }

    // load_k / load_v (kv_cache.rs:111-124): an owned copy, as in Rust
    std::vector<float> load_k(uint32_t layer, uint32_t pos, uint32_t kv_head) const {
        std::vector<float> out(head_dim_);
        check(bml_kv_load(kv_, BML_WHICH_K, layer, pos, kv_head, out.data()), "load_k");
        return out;
    }
    std::vector<float> load_v(uint32_t layer, uint32_t pos, uint32_t kv_head) const {
        std::vector<float> out(head_dim_);
        check(bml_kv_load(kv_, BML_WHICH_V, layer, pos, kv_head, out.data()), "load_v");
        return out;
    }

    // dot_qk (kv_cache.rs:135-141)
    float dot_qk(const std::vector<float> &q, uint32_t layer, uint32_t pos, uint32_t kv_head) const {
        float out = 0.f;
        check(bml_kv_dot_qk(kv_, q.data(), q.size(), layer, pos, kv_head, &out), "dot_qk");
        return out;
    }

    // k_stats / v_stats (kv_cache.rs:148-155)
    std::tuple<uint64_t, uint64_t, double> k_stats() const { return stats(BML_WHICH_K); }
    std::tuple<uint64_t, uint64_t, double> v_stats() const { return stats(BML_WHICH_V); }

    // byte_size (kv_cache.rs:158-161)
    uint64_t byte_size() const {
        uint64_t b = 0;
        check(bml_kv_byte_size(kv_, &b), "byte_size");
        return b;
    }

    // current_pos / advance / advance_by (kv_cache.rs:168-180)
    uint32_t current_pos() const {
        uint32_t p = 0;
        check(bml_kv_current_pos(kv_, &p), "current_pos");
        return p;
    }
    void advance() { check(bml_kv_advance(kv_), "advance"); }
    void advance_by(uint32_t n) { check(bml_kv_advance_by(kv_, n), "advance_by"); }

    // Attention of one token at `pos` over positions [0, pos] of `layer`
    // (gguf_compiler.rs:1008-1050).  q: n_heads*head_dim host floats; returns
    // n_heads*head_dim floats.  Synchronous convenience wrapper.
    std::vector<float> attention(const std::vector<float> &q, uint32_t layer, uint32_t pos,
                                 float scale = -1.f) {
        const size_t n = q.size();
        float *dq = nullptr, *dout = nullptr;
        if (cudaMalloc(&dq, n * sizeof(float)) != cudaSuccess) throw Error(BML_E_OOM, "attention: cudaMalloc");
        if (cudaMalloc(&dout, n * sizeof(float)) != cudaSuccess) {
            cudaFree(dq);
            throw Error(BML_E_OOM, "attention: cudaMalloc");
        }
        std::vector<float> out(n);
        bml_status st = BML_E_CUDA;
        if (cudaMemcpy(dq, q.data(), n * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess) {
            st = bml_attn_decode(kv_, layer, pos, (uint32_t)(n / head_dim_), scale, dq, dout, nullptr);
            if (st == BML_OK && cudaMemcpy(out.data(), dout, n * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
                st = BML_E_CUDA;
        }
        cudaFree(dq);
        cudaFree(dout);
        check(st, "attention");
        return out;
    }

    bml_kv *raw() const { return kv_; }

  private:
    std::tuple<uint64_t, uint64_t, double> stats(int which) const {
        uint64_t u = 0, t = 0;
        double r = 0;
        check(bml_kv_stats(kv_, which, &u, &t, &r), "stats");
        return {u, t, r};
    }
    bml_kv *kv_ = nullptr;
    uint32_t head_dim_;
};

// softmax_f32 (kv_cache.rs:188-200) on the device, host vectors in and out.
inline std::vector<float> softmax_f32(const std::vector<float> &scores) {
    std::vector<float> out(scores.size());
    if (scores.empty()) return out;
    float *d = nullptr;
    const size_t bytes = scores.size() * sizeof(float);
    if (cudaMalloc(&d, 2 * bytes) != cudaSuccess) throw Error(BML_E_OOM, "softmax_f32: cudaMalloc");
    bml_status st = BML_E_CUDA;
    if (cudaMemcpy(d, scores.data(), bytes, cudaMemcpyHostToDevice) == cudaSuccess) {
        st = bml_softmax_f32(d, 1, (uint32_t)scores.size(), d + scores.size(), nullptr);
        if (st == BML_OK && cudaMemcpy(out.data(), d + scores.size(), bytes, cudaMemcpyDeviceToHost) != cudaSuccess)
            st = BML_E_CUDA;
    }
    cudaFree(d);
    check(st, "softmax_f32");
    return out;
}

}  // namespace bml
