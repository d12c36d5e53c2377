"""Generates tests/golden/golden.npz: oracle outputs on seeded inputs.

Run from the repository root:  python tests/golden/make_golden.py
The inputs are regenerated from their seeds by bml_b200.workloads; the file
stores their SHA-256 so a change of numpy's generator stream is detected
instead of silently comparing against different inputs.
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from bml_b200 import workloads as W  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")

PREFILL_ROWS = np.r_[0:8, 248:256, 504:512]


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def small_batch():
    """Ragged f16 batch, TinyLlama heads: lengths hitting tile edges."""
    rng = np.random.default_rng(7)
    lens = [1, 5, 33, 64, 100, 257]
    q = rng.standard_normal((len(lens), 32, 64), dtype=np.float32)
    ks = [rng.standard_normal((L, 4, 64), dtype=np.float32).astype(np.float16) for L in lens]
    vs = [rng.standard_normal((L, 4, 64), dtype=np.float32).astype(np.float16) for L in lens]
    return q, ks, vs


def softmax_cases():
    return [np.array(c, np.float32) for c in (
        [1.0, 2.0, 3.0, 0.5],
        [0.0],
        [-1e30, 0.0, 1e30],
        [100.0, 100.0, 100.0],
        list(np.linspace(-20, 20, 37)),
    )]


def main():
    d = {}
    q, k, v = W.decode_tinyllama()
    d["decode_tinyllama_sha"] = np.array(sha(q, k, v))
    d["decode_tinyllama"] = oracle.attn_decode(q, k, v)

    q, ks, vs = small_batch()
    d["batch_small_sha"] = np.array(sha(q, *ks, *vs))
    d["batch_small"] = oracle.attn_decode_batched(q, ks, vs, n_threads=1)

    q, k, v = W.prefill_tinyllama()
    d["prefill_tinyllama_sha"] = np.array(sha(q, k, v))
    full = oracle.attn_prefill(q, k, v, n_threads=0)
    d["prefill_tinyllama_rows"] = PREFILL_ROWS
    d["prefill_tinyllama"] = full[0, PREFILL_ROWS].astype(np.float32)

    for i, c in enumerate(softmax_cases()):
        d[f"softmax_in_{i}"] = c
        d[f"softmax_out_{i}"] = oracle.softmax_f32(c)
    np.savez_compressed(OUT, **d)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
