"""GPU parity of the weight path against the oracle's restatement of
gguf_compiler.rs: read_tensor_f32 (:351-470) bit for bit on random bytes
(every f16 scale pattern, truncated data, element counts that are not a
multiple of 32), and matmul_f64 (:1239-1255) read straight from the stored
tensor -- by the staged kernel (n_out % 256 == 0) and the direct one --
within 1e-6 of sum_i |x_i W_ij| (terms and partial sums are f32 on the
device, f64 in the reference) plus 1e-12."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def dev_bytes(b: bytes) -> torch.Tensor:
    return torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).cuda()


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    na, nb = np.isnan(a), np.isnan(b)
    return a.shape == b.shape and np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32),
                                                                             b[~nb].view(np.uint32))


def quant_bytes(rng, gguf_type, n_blocks, sane=True):
    bb = 18 if gguf_type == oracle.GGUF_Q4_0 else 34
    raw = rng.integers(0, 256, n_blocks * bb, dtype=np.uint8)
    if sane:  # finite scales of a realistic size
        sc = (rng.standard_normal(n_blocks) * 0.02).astype(np.float16).view(np.uint16)
        raw.reshape(n_blocks, bb)[:, 0] = sc & 0xFF
        raw.reshape(n_blocks, bb)[:, 1] = sc >> 8
    return raw.tobytes()


@pytest.mark.parametrize("gguf_type", [oracle.GGUF_Q4_0, oracle.GGUF_Q8_0])
@pytest.mark.parametrize("n_elems,cut", [(32 * 4096, 0), (32 * 1000 + 17, 0), (32 * 64, 7), (31, 0)])
def test_read_tensor_quantized_bit_exact(cuda, gguf_type, n_elems, cut):
    import bml_b200
    rng = np.random.default_rng(n_elems + gguf_type + cut)
    data = quant_bytes(rng, gguf_type, max(1, n_elems // 32), sane=False)  # every scale bit pattern
    if cut:
        data = data[:len(data) - cut]
    want = oracle.read_tensor_f32(data, gguf_type, n_elems)
    got = bml_b200.read_tensor_f32(dev_bytes(data), gguf_type, n_elems).cpu().numpy()
    assert same_bits(got, want)


@pytest.mark.parametrize("gguf_type,n", [(oracle.GGUF_F16, 65536), (oracle.GGUF_F32, 1001)])
def test_read_tensor_plain_types(cuda, gguf_type, n):
    import bml_b200
    if gguf_type == oracle.GGUF_F16:
        data = np.arange(n, dtype=np.uint16).tobytes() + b"\x01"  # every pattern + a stray byte
    else:
        data = np.random.default_rng(1).standard_normal(n).astype(np.float32).tobytes()
    want = oracle.read_tensor_f32(data, gguf_type, n)
    got = bml_b200.read_tensor_f32(dev_bytes(data), gguf_type, n).cpu().numpy()
    assert same_bits(got, want)


def weight_bytes(rng, gguf_type, n_in, n_out):
    n = n_in * n_out
    if gguf_type in (oracle.GGUF_Q4_0, oracle.GGUF_Q8_0):
        return quant_bytes(rng, gguf_type, n // 32)
    w = (rng.standard_normal(n) * 0.05).astype(np.float32)
    return (w.astype(np.float16) if gguf_type == oracle.GGUF_F16 else w).tobytes()


@pytest.mark.parametrize("gguf_type,n_in,n_out,x_len", [
    (oracle.GGUF_Q4_0, 4096, 4096, 4096),
    (oracle.GGUF_Q4_0, 4096, 1024, 4096),
    (oracle.GGUF_Q8_0, 2048, 5632, 2048),
    (oracle.GGUF_Q4_0, 64, 96, 100),      # x longer than n_in
    (oracle.GGUF_Q8_0, 300, 64, 200),     # x shorter than n_in
    (oracle.GGUF_F16, 512, 1000, 512),    # n_out not a multiple of 32
    (oracle.GGUF_F32, 777, 333, 777),
    (oracle.GGUF_F32, 1, 1, 1),
    (oracle.GGUF_F16, 520, 768, 520),     # staged kernel, f16
    (oracle.GGUF_F32, 300, 512, 300),     # staged kernel, f32
    (oracle.GGUF_Q4_0, 37, 2304, 37),     # staged, a partial last tile, one row range
])
def test_matmul_f64_matches_oracle(cuda, gguf_type, n_in, n_out, x_len):
    import bml_b200
    rng = np.random.default_rng(n_in * 7 + n_out + gguf_type)
    data = weight_bytes(rng, gguf_type, n_in, n_out)
    x = rng.standard_normal(x_len)
    w_vals = oracle.read_tensor_f32(data, gguf_type, n_in * n_out)
    want = oracle.matmul_f64(w_vals, n_in, n_out, x)
    r = min(n_in, x_len)
    bound = np.abs(x[:r]) @ np.abs(w_vals[:r * n_out].reshape(r, n_out).astype(np.float64))
    wt = bml_b200.WeightTensor(dev_bytes(data), gguf_type, [n_in, n_out])
    got = wt.matmul_f64(torch.from_numpy(x).cuda()).cpu().numpy()
    err = np.abs(got - want)
    assert np.all(err <= 1e-6 * bound + 1e-12), float((err / (bound + 1e-30)).max())
    # deterministic: the same call gives the same bits
    again = wt.matmul_f64(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.array_equal(got.view(np.uint64), again.view(np.uint64))


def test_matmul_truncated_f32_tensor(cuda):
    """Values past the data count as zero (the reference would read on into
    the next tensor of its pool; a well-formed file never gets there)."""
    import bml_b200
    rng = np.random.default_rng(9)
    n_in, n_out = 64, 48
    w = rng.standard_normal(n_in * n_out).astype(np.float32)
    data = w.tobytes()[:4 * (n_in * n_out - 100)]
    x = rng.standard_normal(n_in)
    want = oracle.matmul_f64(np.frombuffer(data, np.float32), n_in, n_out, x)
    got = bml_b200.WeightTensor(dev_bytes(data), oracle.GGUF_F32, [n_in, n_out]).matmul_f64(
        torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.allclose(got, want, rtol=1e-5, atol=1e-9)
