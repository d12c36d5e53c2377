"""The reference's own unit tests for the path, run against the CPU oracle.

These pin the oracle's restatement to the reference:
  crates/compiler/src/kv_cache.rs:211-316  (HashConsedKV, softmax_f32)
  crates/compiler/src/eml.rs:237-266       (RoPE rotation convention; the
      identical formula is apply_rope_inplace, gguf_compiler.rs:1290-1317)
Each test keeps the reference test's name, inputs and tolerance.
"""
import math

import numpy as np
import pytest

import oracle
from oracle import HashConsedKV, softmax_f32


def test_store_load_roundtrip():  # kv_cache.rs:211-226
    kv = HashConsedKV(1, 4, 64, 128)
    k = [0.5] * 64
    v = [-0.3] * 64
    kv.store_k(0, 0, 0, k)
    kv.store_v(0, 0, 0, v)
    lk, lv = kv.load_k(0, 0, 0), kv.load_v(0, 0, 0)
    for i in range(64):
        assert abs(lk[i] - np.float32(k[i])) < 1e-6, f"K mismatch at {i}"
        assert abs(lv[i] - np.float32(v[i])) < 1e-6, f"V mismatch at {i}"


def test_ring_buffer_wrapping():  # kv_cache.rs:229-241
    kv = HashConsedKV(1, 1, 4, 8)
    kv.store_k(0, 0, 0, [0.1, 0.2, 0.3, 0.4])
    kv.store_k(0, 8, 0, [0.9, 0.8, 0.7, 0.6])  # pos 8 -> slot 0
    loaded = kv.load_k(0, 0, 0)
    assert abs(loaded[0] - 0.9) < 1e-6
    assert abs(loaded[3] - 0.6) < 1e-6


def test_dot_qk_exact():  # kv_cache.rs:244-258
    kv = HashConsedKV(1, 1, 4, 8)
    k = np.array([0.5, -0.3, 0.8, 0.1], np.float32)
    q = np.array([0.4, 0.2, -0.5, 0.7], np.float32)
    kv.store_k(0, 0, 0, k)
    dot = kv.dot_qk(q, 0, 0, 0)
    expected = np.float32(0.0)
    for a, b in zip(q, k):
        expected = np.float32(expected + np.float32(a * b))
    assert abs(dot - expected) < 1e-5


def test_multi_layer_multi_head():  # kv_cache.rs:261-284
    kv = HashConsedKV(2, 4, 64, 128)
    kv.store_k(1, 5, 2, [0.1] * 64)
    kv.store_v(1, 5, 2, [0.2] * 64)
    lk, lv = kv.load_k(1, 5, 2), kv.load_v(1, 5, 2)
    assert len(lk) == 64 and len(lv) == 64
    assert abs(lk[0] - 0.1) < 1e-6
    assert abs(lv[0] - 0.2) < 1e-6
    assert abs(kv.load_k(1, 0, 0)[0]) < 1e-6, "other positions stay 0"


def test_stats_no_dedup():  # kv_cache.rs:287-300
    kv = HashConsedKV(2, 4, 64, 128)
    kv.store_k(0, 0, 0, [0.1] * 64)
    kv.store_k(0, 1, 0, [0.1] * 64)
    unique, total, ratio = kv.k_stats()
    assert total == 2
    assert unique == total
    assert abs(ratio - 1.0) < 1e-6


def test_softmax_sums_to_one():  # kv_cache.rs:303-310
    probs = softmax_f32([1.0, 2.0, 3.0, 0.5])
    s = np.float32(0)
    for p in probs:
        s = np.float32(s + p)
    assert abs(s - 1.0) < 1e-5
    assert probs[2] > probs[1] > probs[0]


def test_softmax_empty():  # kv_cache.rs:313-316
    assert softmax_f32([]).size == 0


# RoPE (eml.rs:237-266 pins the rotation; gguf_compiler.rs:1301-1307 uses it)
def test_rope_constants_shape():  # eml.rs:237-248
    for pos in range(4):
        for i in range(2):
            freq = 1.0 / (10000.0 ** (2.0 * i / 4))
            c, s = math.cos(pos * freq), math.sin(pos * freq)
            assert abs(c * c + s * s - 1.0) < 1e-9
    # and the oracle's rotation preserves each pair's norm
    x = np.array([3.0, 4.0, 1.0, -2.0], np.float64)
    y = oracle.rope_inplace_f64(x.copy(), 3, 4)
    assert abs(np.hypot(y[0], y[1]) - 5.0) < 1e-12
    assert abs(np.hypot(y[2], y[3]) - math.sqrt(5.0)) < 1e-12


def test_rope_apply_identity_at_zero():  # eml.rs:251-257
    x = np.array([3.0, 4.0], np.float64)
    y = oracle.rope_inplace_f64(x.copy(), 0, 2)
    assert abs(y[0] - 3.0) < 1e-12 and abs(y[1] - 4.0) < 1e-12


def test_rope_apply_rotation():  # eml.rs:260-266: angle pi/2 -> (-x_odd, x_even)
    # head_dim 2: freq_0 = 1, so position p rotates by p radians; the
    # reference test's (cos, sin) = (0, 1) is the rotation by pi/2.
    x = np.array([3.0, 4.0], np.float64)
    c, s = 0.0, 1.0
    expect = (3.0 * c - 4.0 * s, 3.0 * s + 4.0 * c)
    assert abs(expect[0] + 4.0) < 1e-12 and abs(expect[1] - 3.0) < 1e-12
    y = oracle.rope_inplace_f64(x.copy(), 1, 2)
    assert abs(y[0] - (3.0 * math.cos(1) - 4.0 * math.sin(1))) < 1e-12
    assert abs(y[1] - (3.0 * math.sin(1) + 4.0 * math.cos(1))) < 1e-12


# Panics of the Rust code surface as errors in the oracle
def test_store_short_slice_panics():  # copy_from_slice length mismatch, kv_cache.rs:87
    kv = HashConsedKV(1, 1, 4, 8)
    with pytest.raises(IndexError):
        kv.store_k(0, 0, 0, [1.0, 2.0])


def test_layer_out_of_range_panics():  # k_buffers[layer] indexing, kv_cache.rs:86
    kv = HashConsedKV(1, 1, 4, 8)
    with pytest.raises(IndexError):
        kv.store_k(1, 0, 0, [0.0] * 4)


def test_byte_size_and_positions():  # kv_cache.rs:158-180
    kv = HashConsedKV(3, 4, 64, 128)
    assert kv.byte_size() == 4 * 64 * 128 * 4 * 3 * 2
    assert kv.current_pos() == 0
    kv.advance()
    kv.advance_by(5)
    assert kv.current_pos() == 6
