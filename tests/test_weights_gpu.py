"""GPU parity of the weight path against the oracle's restatement of
gguf_compiler.rs: read_tensor_f32 (:351-470) bit for bit on random bytes
(every f16 scale pattern, truncated data, element counts that are not a
multiple of 32), and matmul_f64 (:1239-1255) read straight from the stored
tensor -- by the staged kernel (n_out % 256 == 0) and the direct one --
within 1e-6 of sum_i |x_i W_ij| (terms and partial sums are f32 on the
device, f64 in the reference) plus 1e-12.  The Q4_0 projection is also
pinned bit for bit to a CPU emulation of its own arithmetic order (f32
terms and row-phase chains, f64 phase and range sums), and the
static-weights entry (programmatic dependent launch) to the plain one."""
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


def q4_kernel_emulation(data: bytes, n_in: int, n_out: int, x: np.ndarray, num_sms: int) -> np.ndarray:
    """The staged Q4_0 projection's arithmetic, step for step, on the CPU:
    row ranges as the launch plans them (1024-column tiles, at most 4 CTAs
    an SM, >= 64 rows a range, <= 160 ranges); in each range, for each row
    phase p (rows r0 + p, r0 + p + 8, ...) and column, an f32 chain
    acc = fmaf(f32(f32(x_r) * scale), q - 8, acc) in row order; the 8 phase
    sums added in f64 in phase order from 0.0; the ranges combined as
    sum over groups g (ranges g, g+8, ... in order, from 0.0), groups added in
    order.  fmaf is emulated exactly: the f64 sum of an f32 and an exact
    28-bit product is exact at these magnitudes, so one rounding to f32
    follows."""
    rows = min(n_in, x.size)
    raw = np.frombuffer(data, dtype=np.uint8).reshape(-1, 18)[: n_in * n_out // 32]
    scale = raw[:, :2].copy().view(np.float16).astype(np.float32).reshape(n_in, n_out // 32)
    qb = raw[:, 2:]
    q = np.empty((raw.shape[0], 32), np.int64)
    q[:, 0::2] = qb & 15
    q[:, 1::2] = qb >> 4
    qv = (q - 8).reshape(n_in, n_out).astype(np.float64)
    col_tiles = (n_out + 1023) // 1024
    ranges = min((4 * num_sms) // col_tiles, (rows + 63) // 64, 160)
    ranges = max(ranges, 1)
    rpr = (rows + ranges - 1) // ranges
    ranges = (rows + rpr - 1) // rpr
    xf = x[:rows].astype(np.float32)
    parts = []
    for g in range(ranges):
        r0, r1 = g * rpr, min(g * rpr + rpr, rows)
        ph = np.zeros(n_out, np.float64)
        for p in range(8):
            acc = np.zeros(n_out, np.float32)
            for r in range(r0 + p, r1, 8):
                xs = np.repeat(xf[r] * scale[r], 32)  # f32 product, rounded once
                acc = (acc.astype(np.float64) + xs.astype(np.float64) * qv[r]).astype(np.float32)
            ph = ph + acc.astype(np.float64)
        parts.append(ph)
    if ranges == 1:
        return parts[0]
    grp = []
    for g in range(8):
        s = np.zeros(n_out, np.float64)
        for r in range(g, ranges, 8):
            s = s + parts[r]
        grp.append(s)
    t = grp[0]
    for g in range(1, 8):
        t = t + grp[g]
    return t


@pytest.mark.parametrize("n_in,n_out", [(300, 2048), (1000, 768), (64, 1280), (37, 2304)])
def test_matmul_q4_0_bit_exact_to_its_arithmetic(cuda, n_in, n_out):
    import bml_b200
    rng = np.random.default_rng(n_in + 3 * n_out)
    data = quant_bytes(rng, oracle.GGUF_Q4_0, n_in * n_out // 32)
    x = rng.standard_normal(n_in)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    want = q4_kernel_emulation(data, n_in, n_out, x, sms)
    wt = bml_b200.WeightTensor(dev_bytes(data), oracle.GGUF_Q4_0, [n_in, n_out])
    got = wt.matmul_f64(torch.from_numpy(x).cuda(), overlap=False).cpu().numpy()
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), float(np.abs(got - want).max())


@pytest.mark.parametrize("gguf_type,n_in,n_out", [
    (oracle.GGUF_Q4_0, 4096, 14336), (oracle.GGUF_Q4_0, 37, 2304), (oracle.GGUF_Q8_0, 2048, 5632),
    (oracle.GGUF_F16, 520, 768), (oracle.GGUF_F32, 777, 333)])
def test_static_weights_entry_same_bits(cuda, gguf_type, n_in, n_out):
    """bml_matmul_f64_static, launched back to back behind other kernels
    (each x produced by the kernel just before), gives the plain call's bits."""
    import bml_b200
    rng = np.random.default_rng(n_in + n_out + gguf_type)
    data = weight_bytes(rng, gguf_type, n_in, n_out)
    wt = bml_b200.WeightTensor(dev_bytes(data), gguf_type, [n_in, n_out])
    xs = [torch.from_numpy(rng.standard_normal(n_in)).cuda() for _ in range(3)]
    plain = [wt.matmul_f64(x, overlap=False).cpu().numpy() for x in xs]
    outs = []
    for x in xs:
        x2 = x * 1.0  # a kernel that writes x right before the call
        outs.append(wt.matmul_f64(x2, overlap=True))
    torch.cuda.synchronize()
    for a, b in zip(plain, outs):
        assert np.array_equal(a.view(np.uint64), b.cpu().numpy().view(np.uint64))
