// The reference's kv_cache.rs unit tests (crates/compiler/src/kv_cache.rs:
// 211-316 in SugarFreeDoNoSo/bml), ported one to one onto the C++ mirror of
// the API (include/bml_attn.hpp), running on the GPU through the C ABI.
// Prints one "ok <name>" line per test; exits non-zero on the first failure.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../../include/bml_attn.hpp"

#define ASSERT(c, ...)                                              \
    do {                                                            \
        if (!(c)) {                                                 \
            std::fprintf(stderr, "FAILED %s:%d: ", __func__, __LINE__); \
            std::fprintf(stderr, __VA_ARGS__);                      \
            std::fprintf(stderr, "\n");                             \
            std::exit(1);                                           \
        }                                                           \
    } while (0)

static void store_load_roundtrip() {
    bml::HashConsedKV kv(1, 4, 64, 128);
    std::vector<float> k(64, 0.5f), v(64, -0.3f);
    kv.store_k(0, 0, 0, k);
    kv.store_v(0, 0, 0, v);
    auto lk = kv.load_k(0, 0, 0), lv = kv.load_v(0, 0, 0);
    for (int i = 0; i < 64; ++i) {
        ASSERT(std::fabs(lk[i] - k[i]) < 1e-6f, "K mismatch at %d", i);
        ASSERT(std::fabs(lv[i] - v[i]) < 1e-6f, "V mismatch at %d", i);
    }
}

static void ring_buffer_wrapping() {
    bml::HashConsedKV kv(1, 1, 4, 8);
    kv.store_k(0, 0, 0, {0.1f, 0.2f, 0.3f, 0.4f});
    kv.store_k(0, 8, 0, {0.9f, 0.8f, 0.7f, 0.6f});
    auto loaded = kv.load_k(0, 0, 0);
    ASSERT(std::fabs(loaded[0] - 0.9f) < 1e-6f, "Ring buffer wrap failed");
    ASSERT(std::fabs(loaded[3] - 0.6f) < 1e-6f, "Ring buffer wrap failed");
}

static void dot_qk_exact() {
    bml::HashConsedKV kv(1, 1, 4, 8);
    std::vector<float> k = {0.5f, -0.3f, 0.8f, 0.1f}, q = {0.4f, 0.2f, -0.5f, 0.7f};
    kv.store_k(0, 0, 0, k);
    float dot = kv.dot_qk(q, 0, 0, 0);
    float expected = 0.f;
    for (int i = 0; i < 4; ++i) expected += q[i] * k[i];
    ASSERT(std::fabs(dot - expected) < 1e-5f, "dot=%g, expected=%g", dot, expected);
}

static void multi_layer_multi_head() {
    bml::HashConsedKV kv(2, 4, 64, 128);
    kv.store_k(1, 5, 2, std::vector<float>(64, 0.1f));
    kv.store_v(1, 5, 2, std::vector<float>(64, 0.2f));
    auto lk = kv.load_k(1, 5, 2), lv = kv.load_v(1, 5, 2);
    ASSERT(lk.size() == 64 && lv.size() == 64, "length");
    ASSERT(std::fabs(lk[0] - 0.1f) < 1e-6f, "k value");
    ASSERT(std::fabs(lv[0] - 0.2f) < 1e-6f, "v value");
    ASSERT(std::fabs(kv.load_k(1, 0, 0)[0]) < 1e-6f, "Otras posiciones deben estar en 0");
}

static void stats_no_dedup() {
    bml::HashConsedKV kv(2, 4, 64, 128);
    kv.store_k(0, 0, 0, std::vector<float>(64, 0.1f));
    kv.store_k(0, 1, 0, std::vector<float>(64, 0.1f));
    auto [unique, total, ratio] = kv.k_stats();
    ASSERT(total == 2, "total");
    ASSERT(unique == total, "unique");
    ASSERT(std::fabs(ratio - 1.0) < 1e-6, "ratio");
}

static void softmax_sums_to_one() {
    auto probs = bml::softmax_f32({1.0f, 2.0f, 3.0f, 0.5f});
    float sum = 0.f;
    for (float p : probs) sum += p;
    ASSERT(std::fabs(sum - 1.0f) < 1e-5f, "sum = %g", sum);
    ASSERT(probs[2] > probs[1] && probs[1] > probs[0], "order");
}

static void softmax_empty() { ASSERT(bml::softmax_f32({}).empty(), "empty"); }

// The panics of the Rust code become bml::Panic.
static void out_of_range_panics() {
    bml::HashConsedKV kv(1, 1, 4, 8);
    bool thrown = false;
    try {
        kv.store_k(1, 0, 0, {0.f, 0.f, 0.f, 0.f});
    } catch (const bml::Panic &) {
        thrown = true;
    }
    ASSERT(thrown, "layer out of range must panic");
}

// Attention through the handle: one position returns v exactly.
static void attention_single_position() {
    bml::HashConsedKV kv(1, 2, 64, 16);
    std::vector<float> k(64), v0(64), v1(64);
    for (int i = 0; i < 64; ++i) {
        k[i] = 0.01f * i;
        v0[i] = 1.f + i;
        v1[i] = -1.f - i;
    }
    kv.store_k(0, 0, 0, k);
    kv.store_k(0, 0, 1, k);
    kv.store_v(0, 0, 0, v0);
    kv.store_v(0, 0, 1, v1);
    std::vector<float> q(4 * 64, 0.3f);
    auto out = kv.attention(q, 0, 0);
    for (int h = 0; h < 4; ++h)
        for (int i = 0; i < 64; ++i) {
            const float want = h < 2 ? v0[i] : v1[i];
            ASSERT(std::fabs(out[h * 64 + i] - want) < 1e-6f, "head %d elem %d", h, i);
        }
}

int main() {
#define RUN(t) (t(), std::printf("ok %s\n", #t))
    RUN(store_load_roundtrip);
    RUN(ring_buffer_wrapping);
    RUN(dot_qk_exact);
    RUN(multi_layer_multi_head);
    RUN(stats_no_dedup);
    RUN(softmax_sums_to_one);
    RUN(softmax_empty);
    RUN(out_of_range_panics);
    RUN(attention_single_position);
    return 0;
}
