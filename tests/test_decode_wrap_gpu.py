"""GPU parity of the ring-wrap decode (bml_attn_decode_wrap) against the CPU
oracle, whose loop reads positions 0..pos through slot p % max_seq_len as
gguf_compiler.rs:1026-1049 with kv_cache.rs:83 does.

Tolerance: 1e-4 max-abs, as the other decode parity tests."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-4


def bf16_bits(a):
    """f32 -> bf16 bits, round to nearest even."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_wrap_matches_oracle(cuda, dtype):
    """A full ring of M = 64 slots, read at positions past its end (one
    visit count for every slot, and two counts split at n % M)."""
    from bml_b200 import HashConsedKV
    rng = np.random.default_rng(31)
    M, n_kv, d, H = 64, 4, 64, 32
    k = rng.standard_normal((M, n_kv, d), dtype=np.float32)
    v = rng.standard_normal((M, n_kv, d), dtype=np.float32)
    q = rng.standard_normal((H, d), dtype=np.float32)
    kv = HashConsedKV(1, n_kv, d, M, dtype)
    if dtype == "bf16":
        kb, vb = bf16_bits(k), bf16_bits(v)
        kv.layer_tensor(0, 0).copy_(torch.from_numpy(kb.view(np.int16)).view(torch.bfloat16))
        kv.layer_tensor(1, 0).copy_(torch.from_numpy(vb.view(np.int16)).view(torch.bfloat16))
        ko, vo, code = kb, vb, oracle.BF16
    else:
        kv.layer_tensor(0, 0).copy_(torch.from_numpy(k))
        kv.layer_tensor(1, 0).copy_(torch.from_numpy(v))
        ko, vo, code = k, v, oracle.F32
    qd = torch.from_numpy(q).cuda()
    for pos in (0, 40, M - 1, M, M + 5, 2 * M - 1, 2 * M, 3 * M + 7, 20 * M + 33):
        got = kv.attention(qd, 0, pos, wrap_compat=True).cpu().numpy()
        want = oracle.attn_decode(q, ko, vo, pos=pos, dtype=code)
        assert np.abs(got - want).max() < TOL, pos
    # the plain entry point still refuses a position past the ring
    import bml_b200
    with pytest.raises(bml_b200.BmlInvalid):
        kv.attention(qd, 0, M)


def test_wrap_token_by_token(cuda):
    """Decode past the end of a 24-slot ring as forward_cached does it:
    the new token's K/V overwrite slot pos % M, then attention over 0..pos."""
    from bml_b200 import HashConsedKV
    rng = np.random.default_rng(32)
    M, n_kv, d, H, T = 24, 2, 128, 8, 61
    k = rng.standard_normal((T, n_kv, d), dtype=np.float32)
    v = rng.standard_normal((T, n_kv, d), dtype=np.float32)
    q = rng.standard_normal((T, H, d), dtype=np.float32)
    kv = HashConsedKV(2, n_kv, d, M, "f32")
    kd, vd, qd = (torch.from_numpy(a).cuda() for a in (k, v, q))
    ring_k = np.zeros((M, n_kv, d), np.float32)
    ring_v = np.zeros((M, n_kv, d), np.float32)
    for pos in range(T):
        kv.append(1, pos, kd[pos], vd[pos])
        ring_k[pos % M] = k[pos]
        ring_v[pos % M] = v[pos]
        got = kv.attention(qd[pos], 1, pos, wrap_compat=True).cpu().numpy()
        want = oracle.attn_decode(q[pos], ring_k, ring_v, pos=pos)
        assert np.abs(got - want).max() < TOL, pos
