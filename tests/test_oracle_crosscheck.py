"""Cross-checks of the C oracle: against an independent pure-Python
restatement of gguf_compiler.rs:1008-1050, against analytic known answers
that follow from the reference's arithmetic, and against the committed
golden fixtures (tests/golden/make_golden.py)."""
import hashlib
import math
import os

import numpy as np
import pytest

import oracle
from bml_b200 import workloads as W

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


def py_attention(q, k, v, pos):
    """Pure-Python loops with numpy scalar types, written from the Rust:
    f32 sequential dot, f64 scale, scores rounded to f32, softmax_f32,
    f64 P.V in position order."""
    n_heads, d = q.shape
    n_kv = k.shape[1]
    group = n_heads // n_kv
    scale = 1.0 / math.sqrt(d)
    out = np.zeros((n_heads, d), np.float64)
    for h in range(n_heads):
        kvh = h // group
        scores = []
        for p in range(pos + 1):
            dot = np.float32(0.0)
            for i in range(d):
                dot = np.float32(dot + np.float32(q[h, i] * k[p, kvh, i]))
            scores.append(np.float32(float(dot) * scale))
        mx = max(scores)
        exps = [np.float32(math.exp(float(np.float32(s - mx)))) for s in scores]
        tot = np.float32(0.0)
        for e in exps:
            tot = np.float32(tot + e)
        attn = [np.float32(e / tot) for e in exps] if tot > 0 else [np.float32(1.0 / len(scores))] * len(scores)
        for dd in range(d):
            acc = 0.0
            for p in range(pos + 1):
                acc += float(attn[p]) * float(k.dtype.type(v[p, kvh, dd]))
            out[h, dd] = acc
    return out


@pytest.mark.parametrize("n_heads,n_kv,d,L", [(4, 2, 8, 5), (8, 1, 16, 9), (6, 3, 4, 1)])
def test_oracle_matches_python_restatement(n_heads, n_kv, d, L):
    rng = np.random.default_rng(11)
    q = rng.standard_normal((n_heads, d), dtype=np.float32)
    k = rng.standard_normal((L, n_kv, d), dtype=np.float32)
    v = rng.standard_normal((L, n_kv, d), dtype=np.float32)
    for pos in range(L):
        want = py_attention(q, k, v, pos)
        got = oracle.attn_decode(q, k, v, pos=pos)
        # expf in C vs math.exp rounded to f32 may differ by one ulp
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-6)


def test_single_position_returns_v():
    """pos 0: softmax of one score is exactly 1, so out == v[0]."""
    q, k, v = W.decode_tinyllama()
    out = oracle.attn_decode(q, k, v, pos=0)
    group = 32 // 4
    for h in range(32):
        np.testing.assert_array_equal(out[h], v[0, h // group].astype(np.float64))


def test_equal_keys_give_mean_of_values():
    rng = np.random.default_rng(3)
    L, d = 37, 16
    k = np.repeat(rng.standard_normal((1, 2, d), dtype=np.float32), L, axis=0)
    v = rng.standard_normal((L, 2, d), dtype=np.float32)
    q = rng.standard_normal((4, d), dtype=np.float32)
    out = oracle.attn_decode(q, k, v)
    np.testing.assert_allclose(out[0], v[:, 0].astype(np.float64).mean(0), atol=1e-6)
    np.testing.assert_allclose(out[3], v[:, 1].astype(np.float64).mean(0), atol=1e-6)


def test_gqa_head_map():
    """q heads h and h' with h//group == h'//group read the same kv head."""
    rng = np.random.default_rng(4)
    k = rng.standard_normal((20, 4, 8), dtype=np.float32)
    v = rng.standard_normal((20, 4, 8), dtype=np.float32)
    q1 = rng.standard_normal((1, 8), dtype=np.float32)
    q = np.repeat(q1, 16, axis=0)
    out = oracle.attn_decode(q, k, v)
    for h in range(16):
        np.testing.assert_array_equal(out[h], out[(h // 4) * 4])
    assert not np.array_equal(out[0], out[4])


def test_prefill_rows_equal_decode_at_each_position():
    """gguf_compiler.rs:946-955: token t of a prompt sees exactly [0, t]."""
    q, k, v = W.prefill_tinyllama(seq_len=24)
    pre = oracle.attn_prefill(q, k, v)
    for t in (0, 1, 7, 23):
        dec = oracle.attn_decode(q[0, t], k[0], v[0], pos=t)
        np.testing.assert_array_equal(pre[0, t], dec)


def test_batched_equals_single():
    rng = np.random.default_rng(5)
    lens = [3, 17, 1]
    q = rng.standard_normal((3, 8, 16), dtype=np.float32)
    ks = [rng.standard_normal((L, 2, 16), dtype=np.float32) for L in lens]
    vs = [rng.standard_normal((L, 2, 16), dtype=np.float32) for L in lens]
    out = oracle.attn_decode_batched(q, ks, vs, n_threads=2)
    for s in range(3):
        np.testing.assert_array_equal(out[s], oracle.attn_decode(q[s], ks[s], vs[s]))


def test_16bit_storage_widens_exactly():
    rng = np.random.default_rng(6)
    k32 = rng.standard_normal((9, 2, 16), dtype=np.float32)
    v32 = rng.standard_normal((9, 2, 16), dtype=np.float32)
    q = rng.standard_normal((4, 16), dtype=np.float32)
    kh, vh = k32.astype(np.float16), v32.astype(np.float16)
    np.testing.assert_array_equal(oracle.attn_decode(q, kh, vh),
                                  oracle.attn_decode(q, kh.astype(np.float32), vh.astype(np.float32)))
    kb, vb = W.f32_to_bf16_bits(k32), W.f32_to_bf16_bits(v32)
    np.testing.assert_array_equal(
        oracle.attn_decode(q, kb, vb, dtype=oracle.BF16),
        oracle.attn_decode(q, W.bf16_bits_to_f32(kb), W.bf16_bits_to_f32(vb)))


def test_softmax_reference_edges():
    # uniform fallback when the sum is not positive (kv_cache.rs:195-198)
    out = oracle.softmax_f32([-np.inf, -np.inf])
    np.testing.assert_array_equal(out, [0.5, 0.5])
    out = oracle.softmax_f32([1.0, np.nan, 2.0])
    np.testing.assert_array_equal(out, np.full(3, np.float32(1.0) / np.float32(3.0)))


def test_literal_pattern_matches():
    q, k, v = W.decode_tinyllama(length=40)
    a = oracle.attn_decode(q, k, v)
    b = oracle.attn_decode_literal(q, k, v, pos=39, heads=(0, 32))
    np.testing.assert_array_equal(a, b)


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_golden_fixtures():
    g = np.load(GOLDEN)
    q, k, v = W.decode_tinyllama()
    assert _sha(q, k, v) == str(g["decode_tinyllama_sha"]), "input generator drifted"
    np.testing.assert_array_equal(oracle.attn_decode(q, k, v), g["decode_tinyllama"])

    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(GOLDEN), "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    q, ks, vs = mg.small_batch()
    assert _sha(q, *ks, *vs) == str(g["batch_small_sha"])
    np.testing.assert_array_equal(oracle.attn_decode_batched(q, ks, vs), g["batch_small"])

    q, k, v = W.prefill_tinyllama()
    assert _sha(q, k, v) == str(g["prefill_tinyllama_sha"])
    rows = g["prefill_tinyllama_rows"]
    part = oracle.attn_prefill(q, k, v, rows=(int(rows[-8]), int(rows[-1]) + 1))
    np.testing.assert_array_equal(part[0, rows[-8:]].astype(np.float32), g["prefill_tinyllama"][-8:])

    for i in range(5):
        np.testing.assert_array_equal(oracle.softmax_f32(g[f"softmax_in_{i}"]), g[f"softmax_out_{i}"])


def test_batched_lengths_total_143173_positions():
    """The 64 ragged lengths U[128, 4096] (seed 2) add up to 143,173 positions."""
    assert int(W.batched_lengths().sum()) == 143173


def test_prefill_rows_subset_equals_full_loop():
    """attn_prefill_rows (any subset of query rows and heads) gives exactly
    the values of the full per-token loop at those rows."""
    rng = np.random.default_rng(12)
    q = rng.standard_normal((3, 70, 8, 64), dtype=np.float32)
    k = rng.standard_normal((3, 70, 2, 64), dtype=np.float32)
    v = rng.standard_normal((3, 70, 2, 64), dtype=np.float32)
    full = oracle.attn_prefill(q, k, v)
    rows = [(0, 0), (2, 69), (1, 33), (0, 64), (2, 1)]
    got = oracle.attn_prefill_rows(q, k, v, rows, heads=(3, 7))
    np.testing.assert_array_equal(got, np.stack([full[s, t, 3:7] for s, t in rows]))
