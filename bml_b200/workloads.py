"""Seeded synthetic workloads for the attention path.

The reference publishes no attention benchmark data, so every workload is
synthetic: standard normals from numpy's PCG64 ``default_rng(seed)``, drawn
as float32 and rounded to the storage dtype (round to nearest even).  The
same generator feeds the CPU oracle and the GPU, so both see identical bits.

Shapes (TinyLlama-1.1B: 32 q heads / 4 kv heads, d=64; Llama-3-8B: 32 / 8,
d=128):
  decode_tinyllama    seed 0: q [32,64] f32, K/V [512,4,64] f32, pos 511
  prefill_tinyllama   seed 1: Q [1,512,32,64], K/V [1,512,4,64] f32, RoPE
                      (theta 10000, interleaved pairs) applied to Q and K
  batched_tinyllama   seed 2: 64 sequences, lengths U[128, 4096], K/V
                      [L,4,64] f16, q [64,32,64] f32
  llama3_decode       seed 3: 32 sequences x 8192, K/V bf16, q [32,32,128]
  llama3_prefill      seed 3: Q/K/V [4,8192,{32,8},128] bf16
  longctx_decode      seed 4: one sequence of 131072 positions, K/V bf16
"""
from __future__ import annotations

import numpy as np

HEAD_SHAPES = {"tinyllama": (32, 4, 64), "llama3": (32, 8, 128)}


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def rope_rows(x: np.ndarray, head_dim: int, pos0: int = 0) -> np.ndarray:
    """RoPE of gguf_compiler.rs:1290-1317 on rows [S, n_heads*head_dim]:
    pairs (2i, 2i+1) of each head rotated by pos * 10000^(-2i/head_dim),
    computed in f64 and stored back as f32."""
    S = x.shape[0]
    flat = x.reshape(S, -1).astype(np.float64)
    n_heads = flat.shape[1] // head_dim
    i = np.arange(head_dim // 2, dtype=np.float64)
    freq = 1.0 / np.power(10000.0, 2.0 * i / head_dim)
    pos = (np.arange(S, dtype=np.float64) + pos0)[:, None]
    ang = pos * freq[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    h = flat.reshape(S, n_heads, head_dim // 2, 2)
    xe, xo = h[..., 0], h[..., 1]
    out = np.empty_like(h)
    out[..., 0] = xe * c - xo * s
    out[..., 1] = xe * s + xo * c
    return out.reshape(x.shape).astype(np.float32)


def _normal(rng, shape) -> np.ndarray:
    return rng.standard_normal(shape, dtype=np.float32)


def decode_tinyllama(seed: int = 0, length: int = 512):
    """q [32,64] f32, K/V [length,4,64] f32."""
    H, Hkv, d = HEAD_SHAPES["tinyllama"]
    rng = np.random.default_rng(seed)
    q = _normal(rng, (H, d))
    k = _normal(rng, (length, Hkv, d))
    v = _normal(rng, (length, Hkv, d))
    return q, k, v


def prefill_tinyllama(seed: int = 1, seq_len: int = 512):
    """Q [1,S,32,64], K/V [1,S,4,64] f32 with RoPE applied to Q and K."""
    H, Hkv, d = HEAD_SHAPES["tinyllama"]
    rng = np.random.default_rng(seed)
    q = _normal(rng, (seq_len, H, d))
    k = _normal(rng, (seq_len, Hkv, d))
    v = _normal(rng, (seq_len, Hkv, d))
    q = rope_rows(q, d)
    k = rope_rows(k, d)
    return q[None], k[None], v[None]


def batched_lengths(seed: int = 2, n_seqs: int = 64, lo: int = 128, hi: int = 4096) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, n_seqs)


def batched_tinyllama(seed: int = 2, n_seqs: int = 64, lo: int = 128, hi: int = 4096):
    """Per-sequence f16 K/V [L_i,4,64] with L_i ~ U[lo, hi]; q [n,32,64] f32.
    Draw order: lengths, q, then K and V of each sequence in turn."""
    H, Hkv, d = HEAD_SHAPES["tinyllama"]
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, n_seqs)
    q = _normal(rng, (n_seqs, H, d))
    ks, vs = [], []
    for L in lens:
        ks.append(_normal(rng, (int(L), Hkv, d)).astype(np.float16))
        vs.append(_normal(rng, (int(L), Hkv, d)).astype(np.float16))
    return q, ks, vs


def llama3_decode(seed: int = 3, n_seqs: int = 32, length: int = 8192):
    """q [n,32,128] f32; K/V [n, length, 8, 128] as bf16 bits (uint16)."""
    H, Hkv, d = HEAD_SHAPES["llama3"]
    rng = np.random.default_rng(seed)
    q = _normal(rng, (n_seqs, H, d))
    k = np.empty((n_seqs, length, Hkv, d), np.uint16)
    v = np.empty_like(k)
    for s in range(n_seqs):
        k[s] = f32_to_bf16_bits(_normal(rng, (length, Hkv, d)))
        v[s] = f32_to_bf16_bits(_normal(rng, (length, Hkv, d)))
    return q, k, v


def llama3_prefill(seed: int = 3, n_seqs: int = 4, seq_len: int = 8192):
    """Q [n,S,32,128], K/V [n,S,8,128] as bf16 bits (uint16)."""
    H, Hkv, d = HEAD_SHAPES["llama3"]
    rng = np.random.default_rng(seed)
    q = f32_to_bf16_bits(_normal(rng, (n_seqs, seq_len, H, d)))
    k = f32_to_bf16_bits(_normal(rng, (n_seqs, seq_len, Hkv, d)))
    v = f32_to_bf16_bits(_normal(rng, (n_seqs, seq_len, Hkv, d)))
    return q, k, v


def longctx_decode(seed: int = 4, length: int = 131072):
    """q [32,128] f32; K/V [length, 8, 128] bf16 bits."""
    H, Hkv, d = HEAD_SHAPES["llama3"]
    rng = np.random.default_rng(seed)
    q = _normal(rng, (H, d))
    k = f32_to_bf16_bits(_normal(rng, (length, Hkv, d)))
    v = f32_to_bf16_bits(_normal(rng, (length, Hkv, d)))
    return q, k, v


# Algorithmic work per unit (decode: bytes read/written once; prefill:
# 4*d*H_q FLOPs per causal (query, key) pair).
def decode_bytes(total_positions: int, n_kv: int, d: int, kv_elem_bytes: int, n_seqs: int,
                 n_heads: int) -> int:
    return 2 * total_positions * n_kv * d * kv_elem_bytes + n_seqs * n_heads * d * (4 + 4)


def prefill_flops(n_seqs: int, seq_len: int, n_heads: int, d: int, causal: bool = True) -> int:
    pairs = seq_len * (seq_len + 1) // 2 if causal else seq_len * seq_len
    return 4 * d * n_heads * pairs * n_seqs
