"""GPU parity of DecodeBatcher, the continuous-batching caller: requests with
prompts of different lengths join and leave between tokens; every layer of
every token is one batched append (with or without RoPE) and one batched
decode.  Each step is checked against the oracle: the stored K row against
the oracle's RoPE (gguf_compiler.rs:1290-1317) rounded to the cache dtype
(within one 16-bit ulp for f16/bf16 caches, 2 f32 ulps for f32), V exact,
earlier rows untouched, and the attention output against the oracle's
decode (gguf_compiler.rs:1008-1050) over the cache as stored, 1e-4 max-abs."""
import numpy as np
import pytest
import torch

import oracle
from bml_b200 import workloads as W

pytestmark = pytest.mark.gpu

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def to_np(t):
    """A cache tensor as the oracle reads it (bf16 as uint16 bits)."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def as_f32(a, dtype):
    return W.bf16_bits_to_f32(a) if dtype == "bf16" else a.astype(np.float32)


def rounded(x, dtype):
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return W.bf16_bits_to_f32(W.f32_to_bf16_bits(x))
    return x


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("rope", [True, False])
@pytest.mark.parametrize("n_heads,n_kv,d", [(8, 2, 64), (16, 4, 128)])
def test_batcher_matches_oracle(cuda, dtype, rope, n_heads, n_kv, d):
    import bml_b200
    rng = np.random.default_rng(11 + d + n_kv + (dtype == "f16") + 2 * rope)
    n_layers = 2
    tdt = TORCH_DT[dtype]
    code = oracle.BF16 if dtype == "bf16" else None
    b = bml_b200.DecodeBatcher(n_layers, n_heads, n_kv, d, dtype=tdt, rope=rope, max_requests=5)

    def admit(rid, prompt, cap):
        kp = torch.from_numpy(rng.standard_normal((n_layers, prompt, n_kv, d), dtype=np.float32)).cuda().to(tdt)
        vp = torch.from_numpy(rng.standard_normal((n_layers, prompt, n_kv, d), dtype=np.float32)).cuda().to(tdt)
        b.add(rid, cap, kp if prompt else None, vp if prompt else None)

    admit("a", 0, 40)
    admit("b", 17, 40)
    admit("c", 130, 160)
    schedule = {3: ("remove", "b"), 4: ("add", "d", 64, 80), 6: ("add", "e", 1, 20), 8: ("remove", "a")}
    worst = 0.0
    for t in range(12):
        ev = schedule.get(t)
        if ev and ev[0] == "remove":
            b.remove(ev[1])
        elif ev:
            admit(ev[1], ev[2], ev[3])
        n = len(b)
        for layer in range(n_layers):
            before = {r: tuple(to_np(x) for x in b.cache(r, layer)) for r in b.active}
            q = rng.standard_normal((n, n_heads, d), dtype=np.float32)
            k = rng.standard_normal((n, n_kv, d), dtype=np.float32)
            v = rng.standard_normal((n, n_kv, d), dtype=np.float32)
            qd = torch.from_numpy(q.copy()).cuda()
            kd, vd = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
            if not rope and dtype != "f32":
                kd, vd = kd.to(tdt), vd.to(tdt)   # non-RoPE append converts any source dtype
            out = b.step(layer, qd, kd, vd).cpu().numpy()
            q_used = qd.cpu().numpy()
            ks, vs = [], []
            for i, rid in enumerate(b.active):
                L0 = b.length(rid)
                r = b._reqs[rid]
                kc = to_np(r.k[layer, :L0 + 1])
                vc = to_np(r.v[layer, :L0 + 1])
                assert np.array_equal(kc[:L0], before[rid][0]) and np.array_equal(vc[:L0], before[rid][1])
                want_k, want_v = k[i].copy(), v[i]
                if rope:
                    want_k = oracle.rope_rows_f32(want_k.reshape(1, -1), d, L0).reshape(n_kv, d)
                    want_q = oracle.rope_rows_f32(q[i].reshape(1, -1).copy(), d, L0).reshape(n_heads, d)
                    assert np.all(np.abs(q_used[i] - want_q) <= 2.4e-7 * np.abs(want_q) + 1e-30)
                else:
                    assert np.array_equal(q_used[i], q[i])
                got_k = as_f32(kc[L0], dtype)
                ek = rounded(want_k, dtype)
                ulp = {"f32": 2.4e-7, "f16": 2.0 ** -10, "bf16": 2.0 ** -7}[dtype]
                assert np.all(np.abs(got_k - ek) <= ulp * np.abs(ek) + 1e-30)
                assert np.array_equal(as_f32(vc[L0], dtype), rounded(want_v, dtype))
                ks.append(kc)
                vs.append(vc)
            want = oracle.attn_decode_batched(q_used, ks, vs, dtype=code)
            worst = max(worst, float(np.abs(out - want).max()))
        b.advance()
    assert worst < 1e-4, worst
    assert sorted(b.active) == ["c", "d", "e"] and b.length("e") == 1 + 6


def test_batcher_limits(cuda):
    import bml_b200
    b = bml_b200.DecodeBatcher(1, 4, 2, 64, dtype=torch.bfloat16, max_requests=2)
    b.add(0, 2)
    b.add(1, 3)
    with pytest.raises(bml_b200.AtCapacity):
        b.add(2, 4)
    with pytest.raises(KeyError):
        b.add(1, 4)
    q = torch.zeros(2, 4, 64, device="cuda")
    kv = torch.zeros(2, 2, 64, device="cuda")
    for _ in range(2):
        b.step(0, q, kv, kv)
        b.advance()
    with pytest.raises(ValueError, match="full"):
        b.step(0, q, kv, kv)
    b.remove(0)
    out = b.step(0, q[:1], kv[:1], kv[:1])
    assert out.shape == (1, 4, 64) and b.length(1) == 2
    with pytest.raises(ValueError):
        b.step(0, q, kv, kv)   # 2 rows for 1 request
