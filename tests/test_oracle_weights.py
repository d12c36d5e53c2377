"""The oracle's restatement of the reference's weight path, checked on the
CPU: f16_to_f32 (gguf_compiler.rs:373-403) against IEEE half widening for
every 16-bit pattern, dequantize_q4_0 / dequantize_q8_0 (:405-470) on
hand-computed blocks (including the reference's nibble order and its
truncation / padding rules) and matmul_f64 (:1239-1255) against numpy in
f64.  The reference ships no tests or fixtures for these functions, so the
restatement is pinned by these known answers only."""
import struct

import numpy as np
import pytest

import oracle


def test_f16_to_f32_every_pattern():
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(v)) for v in h], np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))  # signed zeros too


def q4_block(scale_bits, nibbles):
    """An 18-byte Q4_0 block in the reference's element order: element 2i is
    the low nibble of byte i, element 2i+1 the high nibble."""
    assert len(nibbles) == 32
    body = bytes((nibbles[2 * i] & 15) | ((nibbles[2 * i + 1] & 15) << 4) for i in range(16))
    return struct.pack("<H", scale_bits) + body


def test_q4_0_known_block():
    nib = list(range(16)) + list(range(15, -1, -1))
    blk = q4_block(0x3800, nib)  # scale 0.5
    got = oracle.read_tensor_f32(blk, oracle.GGUF_Q4_0, 32)
    want = np.array([(q - 8) * 0.5 for q in nib], np.float32)
    assert np.array_equal(got, want)
    assert got[0] == -4.0 and got[1] == -3.5 and got[15] == 3.5


def test_q8_0_known_block():
    q = [-128, 127, 0, 1, -1] + list(range(27))
    blk = struct.pack("<H", 0x4000) + struct.pack("<32b", *q)  # scale 2.0
    got = oracle.read_tensor_f32(blk, oracle.GGUF_Q8_0, 32)
    assert np.array_equal(got, np.array(q, np.float32) * 2.0)


def test_quantized_truncation_and_padding():
    rng = np.random.default_rng(0)
    blocks = [q4_block(0x3C00, list(rng.integers(0, 16, 32))) for _ in range(3)]
    data = b"".join(blocks)
    full = oracle.read_tensor_f32(data, oracle.GGUF_Q4_0, 96)
    # a cut inside block 2 stops there and pads with zeros
    cut = oracle.read_tensor_f32(data[:18 * 2 + 5], oracle.GGUF_Q4_0, 96)
    assert np.array_equal(cut[:64], full[:64]) and not cut[64:].any() and cut.size == 96
    # n_elems not a multiple of 32: only whole blocks decode, the rest is zero
    part = oracle.read_tensor_f32(data, oracle.GGUF_Q4_0, 80)
    assert np.array_equal(part[:64], full[:64]) and not part[64:].any() and part.size == 80


def test_f32_f16_types_and_unsupported():
    x = np.array([1.5, -2.25, 3e-8], np.float32)
    assert np.array_equal(oracle.read_tensor_f32(x.tobytes(), oracle.GGUF_F32, 3), x)
    h = np.array([1.0, -0.5, 65504.0], np.float16)
    assert np.array_equal(oracle.read_tensor_f32(h.tobytes(), oracle.GGUF_F16, 3), h.astype(np.float32))
    with pytest.raises(ValueError):
        oracle.read_tensor_f32(b"\0" * 64, 12, 64)  # Q4_K: the reference returns None


@pytest.mark.parametrize("n_in,n_out,x_len", [(64, 96, 64), (96, 64, 50), (33, 17, 40)])
def test_matmul_f64_matches_numpy(n_in, n_out, x_len):
    rng = np.random.default_rng(n_in + n_out)
    w = rng.standard_normal(n_in * n_out).astype(np.float32)
    x = rng.standard_normal(x_len)
    got = oracle.matmul_f64(w, n_in, n_out, x)
    r = min(n_in, x_len)
    want = x[:r] @ w.reshape(n_in, n_out)[:r].astype(np.float64)
    assert np.allclose(got, want, rtol=1e-13, atol=1e-13)
