"""GGUF upload on the GPU: tensors of a file copied into device memory by
bml_gguf_upload equal the file's bytes (pieces of the 32 MiB staging size
and beyond, one and several host threads), and a projection read from an
uploaded Q4_0 tensor equals the oracle's matmul_f64 over the reference's
dequantisation of the same file bytes (the loader feeding the weight
path, gguf.rs:339-364 -> gguf_compiler.rs:351-470, :1239-1255)."""
import numpy as np
import pytest
import torch

import oracle
from oracle import gguf_oracle as O

pytestmark = pytest.mark.gpu


def q4_bytes(rng, n):
    nb = n // 32
    raw = rng.integers(0, 256, (nb, 18), dtype=np.uint8)
    sc = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint16)
    raw[:, 0], raw[:, 1] = sc & 0xFF, sc >> 8
    return raw.tobytes()


@pytest.fixture(scope="module")
def model_file(tmp_path_factory):
    from bml_b200 import gguf
    rng = np.random.default_rng(21)
    tensors = [
        ("blk.0.attn_q.weight", [4096, 1024], 2, q4_bytes(rng, 4096 * 1024)),
        ("blk.0.ffn_up.weight", [8192, 8192], 2, q4_bytes(rng, 8192 * 8192)),  # 37.7 MB: two pieces
        ("output_norm.weight", [4096], 0, rng.standard_normal(4096).astype(np.float32).tobytes()),
        ("blk.0.attn_k.weight", [512, 256], 1, rng.standard_normal(512 * 256).astype(np.float16).tobytes()),
        ("blk.0.attn_v.weight", [512, 256], 8, bytes(rng.integers(0, 256, 512 * 256 // 32 * 34, dtype=np.uint8))),
        ("iq", [256], 16, b"\0" * 66),
    ]
    p = tmp_path_factory.mktemp("gguf") / "model.gguf"
    gguf.write_gguf(p, [("general.architecture", 8, "llama")], tensors)
    return p, tensors


@pytest.mark.parametrize("threads", [1, 4])
def test_upload_bytes_exact(cuda, model_file, threads):
    from bml_b200 import gguf
    p, tensors = model_file
    raw = open(p, "rb").read()
    parsed = O.parse(raw)
    with gguf.GgufFile(p) as f:
        names = [t[0] for t in tensors[:5]]
        dev = f.upload(names, threads=threads)
        torch.cuda.synchronize()
        for name, _, _, data in tensors[:5]:
            info = O.find_tensor(parsed, name)
            start = parsed["data_offset"] + info["offset"]
            assert dev[name].numel() == len(data)
            assert np.array_equal(dev[name].cpu().numpy(), np.frombuffer(raw[start:start + len(data)], np.uint8))


def test_upload_refusals(cuda, model_file, tmp_path):
    from bml_b200 import _lib, gguf
    p, tensors = model_file
    with gguf.GgufFile(p) as f:
        with pytest.raises(_lib.BmlUnsupported):
            f.upload(["iq"])  # a block layout this library does not know
    # a tensor that runs past the end of the file
    raw = open(p, "rb").read()
    cut = tmp_path / "cut.gguf"
    open(cut, "wb").write(raw[:len(raw) - 4096])
    with gguf.GgufFile(cut) as f:
        with pytest.raises(_lib.BmlInvalid):
            f.upload([f.tensor_infos[-2]])


def test_uploaded_q4_projection_matches_oracle(cuda, model_file):
    from bml_b200 import gguf
    p, tensors = model_file
    name, dims, t, data = tensors[0]
    rng = np.random.default_rng(5)
    x = rng.standard_normal(dims[0])
    with gguf.GgufFile(p) as f:
        w = f.weight(name)
        got = w.matmul_f64(torch.from_numpy(x).cuda()).cpu().numpy()
        view = f.tensor_data(f.find_tensor(name))  # the reference reads quantized data to the end of file
        vals = oracle.read_tensor_f32(view.tobytes(), oracle.GGUF_Q4_0, dims[0] * dims[1])
    want = oracle.matmul_f64(vals, dims[0], dims[1], x)
    bound = np.abs(x) @ np.abs(vals.reshape(dims[0], dims[1]).astype(np.float64))
    assert np.all(np.abs(got - want) <= 1e-6 * bound + 1e-12)
