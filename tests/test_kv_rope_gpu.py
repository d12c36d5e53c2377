"""GPU parity of bml_kv_append_rope: RoPE of gguf_compiler.rs:1290-1317 on q
and k (f64 rotation), then the store of k and v into the cache slot
(gguf_compiler.rs:984-1006), against the oracle's restatement of the same
steps.  Values leave the rotation as f32 (like the reference's f64 vectors
landing in its f32 cache); tolerance: 2 f32 ulps of |x| for q and f32
caches, one 16-bit rounding for f16/bf16 caches."""
import numpy as np
import pytest
import torch

import oracle
from bml_b200 import workloads as W

pytestmark = pytest.mark.gpu


def f16_round(x, dtype):
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return W.bf16_bits_to_f32(W.f32_to_bf16_bits(x))
    return x


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n_heads,n_kv,d", [(32, 4, 64), (32, 8, 128)])
@pytest.mark.parametrize("pos", [0, 1, 77, 511])
def test_append_rope_matches_oracle(cuda, dtype, n_heads, n_kv, d, pos):
    import bml_b200
    rng = np.random.default_rng(pos * 7 + d + n_kv)
    q = rng.standard_normal((n_heads, d), dtype=np.float32)
    k = rng.standard_normal((n_kv, d), dtype=np.float32)
    v = rng.standard_normal((n_kv, d), dtype=np.float32)
    kv = bml_b200.HashConsedKV(2, n_kv, d, 512, dtype=dtype)
    qd = torch.from_numpy(q.copy()).cuda()
    kv.append_rope(1, pos, qd, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()

    want_q = oracle.rope_rows_f32(q.reshape(1, -1).copy(), d, pos).reshape(n_heads, d)
    want_k = oracle.rope_rows_f32(k.reshape(1, -1).copy(), d, pos).reshape(n_kv, d)
    got_q = qd.cpu().numpy()
    assert np.all(np.abs(got_q - want_q) <= 2.4e-7 * np.abs(want_q) + 1e-30), np.abs(got_q - want_q).max()
    for h in range(n_kv):
        gk, gv = kv.load_k(1, pos, h), kv.load_v(1, pos, h)
        ek, ev = f16_round(want_k[h], dtype), f16_round(v[h], dtype)
        if dtype == "f32":
            assert np.all(np.abs(gk - ek) <= 2.4e-7 * np.abs(ek) + 1e-30)
        else:
            # the f64 rotation may land one f32 ulp away, which can flip a
            # 16-bit rounding: at most one 16-bit ulp
            ulp = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
            assert np.all(np.abs(gk - ek) <= ulp * np.abs(ek) + 1e-30)
        assert np.array_equal(gv, ev)
    # other slots untouched
    assert not np.any(kv.load_k(0, pos, 0)) and not np.any(kv.load_v(1, (pos + 1) % 512, 0))


def test_append_rope_then_attention(cuda):
    """A token stream through append_rope + attention equals the oracle's
    decode over RoPE'd keys."""
    import bml_b200
    rng = np.random.default_rng(3)
    n_heads, n_kv, d, L = 32, 4, 64, 40
    kv = bml_b200.HashConsedKV(1, n_kv, d, 64, dtype="f32")
    ks, vs = [], []
    for p in range(L):
        q = rng.standard_normal((n_heads, d), dtype=np.float32)
        k = rng.standard_normal((n_kv, d), dtype=np.float32)
        v = rng.standard_normal((n_kv, d), dtype=np.float32)
        qd = torch.from_numpy(q.copy()).cuda()
        kv.append_rope(0, p, qd, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
        ks.append(oracle.rope_rows_f32(k.reshape(1, -1).copy(), d, p).reshape(n_kv, d))
        vs.append(v)
        out = kv.attention(qd, 0, p).cpu().numpy()
        want = oracle.attn_decode(qd.cpu().numpy(), np.stack(ks), np.stack(vs))
        assert np.abs(out - want).max() < 1e-4
