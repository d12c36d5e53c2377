"""The allocation-free decode entry point, bml_attn_decode_batched_noalloc.

It exists for callers that cannot call cudaMalloc -- a runtime whose pool
allocator owns all device memory, or a serving loop that must not pay
cudaMalloc's device-wide synchronisation -- and takes its scratch from the
library's fixed 4 MiB device array.  These tests call it through the C ABI
and check it against bml_attn_decode_batched (the workspace-taking entry
point) on two calls in a row, against the oracle on the 64-sequence ragged
TinyLlama-shaped batch, that bml_attn_noalloc_check reports no timeout
after good calls, and that oversized batches are refused."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from bml_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 1e-4  # the decode tolerance used by the other decode tests


def _batch(seed, lens, n_kv, d, group, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    H = n_kv * group
    q = torch.randn(len(lens), H, d, device="cuda", generator=g)
    ks = [torch.randn(L, n_kv, d, device="cuda", generator=g).to(dtype) for L in lens]
    vs = [torch.randn(L, n_kv, d, device="cuda", generator=g).to(dtype) for L in lens]
    return q, ks, vs


@pytest.mark.parametrize("lens,n_kv,d,group,dtype", [
    ([1, 77, 700, 4096, 33], 4, 64, 8, torch.float16),
    ([8192] * 8, 8, 128, 4, torch.bfloat16),
])
def test_noalloc_matches_workspace_entry_point(cuda, lens, n_kv, d, group, dtype):
    import bml_b200
    import bml_b200._lib as L
    from bml_b200.attention import dtype_code
    q, ks, vs = _batch(sum(lens), lens, n_kv, d, group, dtype)
    batch = bml_b200.SeqBatch(ks, vs)
    want = bml_b200.decode_batched(q, batch)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):  # two calls in a row share (and must reset) the scratch
        out = torch.full_like(q, float("nan"))
        st = L.lib().bml_attn_decode_batched_noalloc(
            batch.descs, len(lens), q.shape[1], n_kv, d, dtype_code(dtype), -1.0,
            C.c_void_p(q.data_ptr()), C.c_void_p(out.data_ptr()), stream)
        assert st == L.BML_OK, L.last_error()
        torch.cuda.synchronize()
        err = (out - want).abs().max().item()
        assert err < TOL, err
    assert L.lib().bml_attn_noalloc_check(stream) == L.BML_OK, L.last_error()


def test_noalloc_matches_oracle_on_ragged_batch(cuda):
    """64 sequences of U[128, 4096] positions (seed 2), f16 KV, 32 q / 4 kv
    heads, d = 64: two calls in a row against the oracle, then the check."""
    import bml_b200
    import bml_b200._lib as L
    from bml_b200.attention import dtype_code
    q, ks, vs = W.batched_tinyllama()
    want = oracle.attn_decode_batched(q, ks, vs)
    batch = bml_b200.SeqBatch([torch.from_numpy(k).cuda() for k in ks], [torch.from_numpy(v).cuda() for v in vs])
    qd = torch.from_numpy(q).cuda()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        out = torch.full_like(qd, float("nan"))
        st = L.lib().bml_attn_decode_batched_noalloc(batch.descs, len(batch), 32, 4, 64, dtype_code(torch.float16),
                                                     -1.0, C.c_void_p(qd.data_ptr()), C.c_void_p(out.data_ptr()),
                                                     stream)
        assert st == L.BML_OK, L.last_error()
        err = np.abs(out.cpu().numpy() - want).max()
        assert err < TOL, err
    assert L.lib().bml_attn_noalloc_check(stream) == L.BML_OK, L.last_error()


def test_noalloc_refuses_batches_beyond_its_scratch(cuda):
    import bml_b200._lib as L
    lens = [16] * 256
    descs = (L.bml_seq_desc * 256)(*[L.bml_seq_desc(16, 16, n, 0) for n in lens])
    st = L.lib().bml_attn_decode_batched_noalloc(descs, 256, 64, 8, 128, L.BML_BF16, -1.0, 16, 16, None)
    assert st == L.BML_E_INVALID
    assert "maximum" in L.last_error()


def test_noalloc_python_wrapper(cuda):
    import bml_b200
    q, ks, vs = _batch(7, [300, 5], 2, 128, 4, torch.bfloat16)
    a = bml_b200.decode_batched(q, ks, vs)
    b = bml_b200.attention.decode_batched_noalloc(q, ks, vs)
    torch.cuda.synchronize()
    assert (a - b).abs().max().item() < TOL
    assert np.isfinite(b.cpu().numpy()).all()
