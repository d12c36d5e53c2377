"""GPU parity of the tcgen05 causal prefill kernel.

Against the CPU oracle (the reference's per-token loop, gguf_compiler.rs:
946-958 over :1008-1050) on identical seeded inputs: bf16 operands with f32
accumulation must stay within 2e-2 max-abs and 1e-2 relative L2.  The
non-causal mode (no reference counterpart) is checked against a plain
PyTorch fp32 attention."""
import numpy as np
import pytest
import torch

import oracle
from bml_b200 import workloads as W

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def to_dev16(a_f32, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a_f32)).cuda().to(dtype)


def bits_to_dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def check(got, want, label=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert np.isfinite(got).all(), f"{label}: non-finite output"
    err = np.abs(got - want).max()
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err < MAX_ABS and rel < REL_L2, f"{label}: max-abs {err:.3e}, rel-L2 {rel:.3e}"
    return err, rel


def test_prefill_tinyllama_full(cuda):
    """S=512, 32/4 heads, d=64, RoPE pre-applied (seed 1); GPU casts to bf16."""
    import bml_b200
    q, k, v = W.prefill_tinyllama()
    got = bml_b200.prefill(to_dev16(q), to_dev16(k), to_dev16(v)).cpu().numpy()
    want = oracle.attn_prefill(q, k, v)
    check(got, want, "tinyllama prefill")


def test_prefill_llama3_every_query_tile(cuda):
    """4 x 8192 tokens, 32/8 heads, d=128, bf16 inputs (seed 3): the full
    output is computed on the GPU in one launch.  The oracle checks, in all 4
    sequences and all 32 heads, rows 0, 1, 126 and 127 of every 128-row
    query tile -- the first and last row of each tile and the rows at the
    edges of its diagonal (causal) key tile -- so every query tile of every
    CTA tile pair is compared; and one whole (sequence, kv-head group) slab,
    all 8192 rows of the 4 q heads of kv head 5 in the last sequence."""
    import bml_b200
    q, k, v = W.llama3_prefill()
    out = bml_b200.prefill(bits_to_dev(q), bits_to_dev(k), bits_to_dev(v))
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    qf = W.bf16_bits_to_f32(q)
    n, S = q.shape[0], q.shape[1]
    rows = [(sq, t0 + r) for sq in range(n) for t0 in range(0, S, 128) for r in (0, 1, 126, 127)]
    want = oracle.attn_prefill_rows(qf, k, v, rows, dtype=oracle.BF16)
    idx_s = torch.tensor([r[0] for r in rows], device="cuda")
    idx_t = torch.tensor([r[1] for r in rows], device="cuda")
    got = out[idx_s, idx_t].cpu().numpy()
    check(got, want, "first/last/diagonal-edge rows of every query tile")
    slab = [(n - 1, t) for t in range(S)]
    want = oracle.attn_prefill_rows(qf, k, v, slab, heads=(20, 24), dtype=oracle.BF16)
    got = out[n - 1, :, 20:24].cpu().numpy()
    check(got, want, "sequence 3, q heads 20..23, all rows")


@pytest.mark.parametrize("S", [1, 2, 17, 127, 128, 129, 255, 300])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("H,Hkv", [(32, 4), (8, 8), (4, 1)])
def test_prefill_shapes(cuda, S, d, H, Hkv):
    import bml_b200
    rng = np.random.default_rng(S * 131 + d + H)
    n = 2
    q = rng.standard_normal((n, S, H, d), dtype=np.float32)
    k = rng.standard_normal((n, S, Hkv, d), dtype=np.float32)
    v = rng.standard_normal((n, S, Hkv, d), dtype=np.float32)
    # give the oracle the same bf16-rounded values the GPU sees
    qb, kb, vb = (W.f32_to_bf16_bits(x) for x in (q, k, v))
    got = bml_b200.prefill(bits_to_dev(qb), bits_to_dev(kb), bits_to_dev(vb)).cpu().numpy()
    want = oracle.attn_prefill(W.bf16_bits_to_f32(qb), kb, vb, dtype=oracle.BF16)
    check(got, want, f"S={S} d={d} H={H}/{Hkv}")


def torch_attention(q, k, v, causal, scale):
    """fp32 reference: q [n,S,H,d], k/v [n,S,Hkv,d]."""
    n, S, H, d = q.shape
    g = H // k.shape[2]
    kk = k.float().repeat_interleave(g, dim=2)
    vv = v.float().repeat_interleave(g, dim=2)
    s = torch.einsum("nshd,nthd->nhst", q.float(), kk) * scale
    if causal:
        mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("nhst,nthd->nshd", p, vv)


@pytest.mark.parametrize("S", [64, 200, 384])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_non_causal_and_f16(cuda, S, dtype):
    import bml_b200
    g = torch.Generator(device="cuda").manual_seed(S)
    q = torch.randn(2, S, 8, 128, device="cuda", generator=g).to(dtype)
    k = torch.randn(2, S, 2, 128, device="cuda", generator=g).to(dtype)
    v = torch.randn(2, S, 2, 128, device="cuda", generator=g).to(dtype)
    scale = 128 ** -0.5
    for causal in (True, False):
        got = bml_b200.prefill(q, k, v, causal=causal)
        want = torch_attention(q, k, v, causal, scale)
        check(got.cpu().numpy(), want.cpu().numpy(), f"S={S} causal={causal} {dtype}")


def test_prefill_bf16_output_and_repeat(cuda):
    import bml_b200
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(1, 777, 16, 64, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(1, 777, 4, 64, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(1, 777, 4, 64, device="cuda", generator=g).to(torch.bfloat16)
    a = bml_b200.prefill(q, k, v)
    b = bml_b200.prefill(q, k, v)
    c = bml_b200.prefill(q, k, v, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(a, b), "prefill is deterministic"
    assert (c.float() - a).abs().max().item() < 1e-2
