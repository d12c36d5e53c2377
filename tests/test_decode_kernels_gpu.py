"""GPU parity of both decode kernels for 16-bit caches, and the bounded
waits of the tensor-core kernel.

bml_attn_decode_batched takes the bulk-copy warp-MMA kernel (claimed tiles,
in-kernel merge) for 16-bit caches with 512..2048-byte position rows; the
CUDA-core kernel serves f32 caches and every other row size.  The test-only
entry point bml_diag_decode_batched (include/bml_diag.h) forces the
CUDA-core kernel for 16-bit caches too, so both are checked against the
oracle on the same inputs: ragged lengths around every tile edge, many
sequences, the decode tolerance 1e-4.  It also sets the wait limit and can
make the tensor-core kernel's producer fill no stage: its consumers' first
wait then runs out, the kernel returns by itself and the host reads
BML_E_TIMEOUT -- the failure path of a device wait, without any fault."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from bml_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 1e-4
EDGE = [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 129, 1000, 4099]
CASES = [("bf16", 128, 8, 4), ("f16", 128, 8, 4), ("bf16", 64, 4, 8), ("f16", 64, 8, 2), ("bf16", 128, 2, 4),
         ("f16", 128, 4, 1)]


def _case(dtype, d, n_kv, group):
    rng = np.random.default_rng(7 + d + n_kv + group)
    lens = EDGE + [int(x) for x in rng.integers(1, 300, 60)]
    H = n_kv * group
    q = rng.standard_normal((len(lens), H, d), dtype=np.float32)
    ks, vs, kd, vd, code = [], [], [], [], None
    for L in lens:
        k = rng.standard_normal((L, n_kv, d), dtype=np.float32)
        v = rng.standard_normal((L, n_kv, d), dtype=np.float32)
        if dtype == "f16":
            k, v = k.astype(np.float16), v.astype(np.float16)
            kd.append(torch.from_numpy(k).cuda())
            vd.append(torch.from_numpy(v).cuda())
        else:
            k, v, code = W.f32_to_bf16_bits(k), W.f32_to_bf16_bits(v), oracle.BF16
            kd.append(torch.from_numpy(k.view(np.int16)).cuda().view(torch.bfloat16))
            vd.append(torch.from_numpy(v.view(np.int16)).cuda().view(torch.bfloat16))
        ks.append(k)
        vs.append(v)
    return q, ks, vs, kd, vd, code


def _diag(batch, q, out, ws, kernel, wait_ns=0, flags=0):
    import bml_b200._lib as L
    from bml_b200.attention import dtype_code
    st = L.lib().bml_diag_decode_batched(batch.descs, len(batch), q.shape[1], batch.n_kv, batch.head_dim,
                                         dtype_code(batch.dtype), -1.0, C.c_void_p(q.data_ptr()),
                                         C.c_void_p(out.data_ptr()), ws.ptr, ws.nbytes, kernel, wait_ns, flags,
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == L.BML_OK, L.last_error()


@pytest.mark.parametrize("kernel", ["default", "cuda_core"])
@pytest.mark.parametrize("dtype,d,n_kv,group", CASES)
def test_decode_kernel_parity(cuda, kernel, dtype, d, n_kv, group):
    import bml_b200
    import bml_b200._lib as L
    q, ks, vs, kd, vd, code = _case(dtype, d, n_kv, group)
    batch = bml_b200.SeqBatch(kd, vd)
    qd = torch.from_numpy(q).cuda()
    out = torch.full_like(qd, float("nan"))
    ws = bml_b200.Workspace().ensure(len(batch), q.shape[1], d)
    k = L.BML_DIAG_DECODE_DEFAULT if kernel == "default" else L.BML_DIAG_DECODE_CUDA_CORE
    _diag(batch, qd, out, ws, k)
    want = oracle.attn_decode_batched(q, ks, vs, dtype=code)
    assert np.abs(out.cpu().numpy() - want).max() < TOL
    ws.check()


def test_stalled_wait_reports_timeout_and_context_stays_usable(cuda):
    """The producer fills no stage (a flag that nothing sets), so each
    consumer warp's first wait runs into a 20 ms limit; the launch ends by
    itself, the workspace's error word reads BML_E_TIMEOUT once (the check
    clears it), and the next decode on the same workspace is correct."""
    import bml_b200
    import bml_b200._lib as L
    q, ks, vs, kd, vd, code = _case("bf16", 128, 8, 4)
    batch = bml_b200.SeqBatch(kd, vd)
    qd = torch.from_numpy(q).cuda()
    out = torch.empty_like(qd)
    ws = bml_b200.Workspace().ensure(len(batch), q.shape[1], 128)
    _diag(batch, qd, out, ws, L.BML_DIAG_DECODE_DEFAULT, wait_ns=20_000_000, flags=L.BML_DIAG_STALL)
    torch.cuda.synchronize()
    with pytest.raises(L.BmlError) as e:
        ws.check()
    assert e.value.status == L.BML_E_TIMEOUT
    ws.check()  # cleared by the first check
    got = bml_b200.decode_batched(qd, batch, workspace=ws).cpu().numpy()
    want = oracle.attn_decode_batched(q, ks, vs, dtype=code)
    assert np.abs(got - want).max() < TOL
    ws.check()


def test_device_exp2_error_bound(cuda):
    """The SFU exponential (ex2.approx) every decode, merge and prefill
    softmax uses, against CUDA's exp2f over the range the softmax feeds it."""
    import bml_b200._lib as L
    x = torch.linspace(-125.5, 10.0, 200002, device="cuda", dtype=torch.float32)
    out = torch.empty_like(x)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.lib().bml_diag_exp2(C.c_void_p(x.data_ptr()), x.numel(), C.c_void_p(out.data_ptr()), st) == 0
    want = torch.exp2(x.double())
    rel = ((out.double() - want).abs() / want).max().item()
    assert rel < 2e-6, rel
