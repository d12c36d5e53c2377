"""The library's GGUF parser (bml_gguf.h, bml_b200.gguf) against the
oracle's restatement of the reference's GgufParser (crates/parser/src/
gguf.rs): the reference's own synthetic file and the facts its tests check
(gguf.rs:601-790), seeded random files with every metadata type, nested
arrays, invalid UTF-8, repeated keys and names, every tensor type, and the
files the reference rejects.  Host code only: no GPU."""
import os
import struct

import numpy as np
import pytest

from oracle import gguf_oracle as O

G = None


@pytest.fixture(scope="module", autouse=True)
def lib():
    global G
    from bml_b200 import build
    build.build()
    import bml_b200.gguf as gg
    G = gg


def reference_fixture(path):
    """The file create_gguf_with_metadata writes (gguf.rs:601-650): two
    metadata (general.architecture "llama", llama.context_length U32 2048),
    one F32 tensor token_embd.weight of dims [4, 2] at offset 0 holding
    0..7, data section aligned to 32."""
    G.write_gguf(path, [("general.architecture", 8, "llama"), ("llama.context_length", 4, 2048)],
                 [("token_embd.weight", [4, 2], 0, np.arange(8, dtype=np.float32).tobytes())])


def same(f, parsed):
    assert f.header == parsed["header"]
    assert f.data_offset == parsed["data_offset"]
    assert f.metadata_typed == parsed["metadata"]
    assert len(f.tensor_infos) == len(parsed["tensor_infos"])
    raw = open(f._path, "rb").read() if hasattr(f, "_path") else None
    for got, want in zip(f.tensor_infos, parsed["tensor_infos"]):
        assert (got.name, got.n_dims, got.dims, got.data_type, got.offset) == \
               (want["name"], want["n_dims"], want["dims"], want["data_type"], want["offset"])
        view = O.tensor_data(parsed, want)
        assert got.present == (view is not None)
        if view is not None:
            assert (got.data_offset, got.view_len) == view
            data = f.tensor_data(got)
            assert data is not None and data.size == view[1]
            if raw is not None and view[1]:
                assert data[:64].tobytes() == raw[view[0]:view[0] + min(64, view[1])]


def test_reference_fixture(tmp_path):
    p = tmp_path / "meta.gguf"
    reference_fixture(p)
    f = G.GgufFile(p)
    f._path = p
    same(f, O.parse(open(p, "rb").read()))
    # the facts the reference's tests assert (gguf.rs:656-760)
    assert f.header["tensor_count"] == 1 and f.header["metadata_kv_count"] == 2
    assert f.architecture() == "llama"
    assert f.metadata_typed["llama.context_length"] == (4, 2048)
    t = f.find_tensor("token_embd.weight")
    assert (t.name, t.n_dims, t.dims, t.data_type) == ("token_embd.weight", 2, [4, 2], 0)
    data = f.tensor_data(t)
    assert data.size == 32
    assert np.array_equal(data.view(np.float32), np.arange(8, dtype=np.float32))
    assert f.find_tensor("nonexistent") is None
    f.close()


def random_value(rng, t, depth=0):
    if t == 9:
        et = int(rng.integers(0, 13)) if depth < 2 else int(rng.integers(0, 9))
        return (et, [random_value(rng, et, depth + 1) for _ in range(int(rng.integers(0, 4)))])
    if t == 8:
        raw = bytes(rng.integers(0, 256, int(rng.integers(0, 12)), dtype=np.uint8))
        return raw if rng.random() < 0.3 else "tok_" + raw.hex()
    if t == 7:
        return bool(rng.integers(0, 2))
    if t in (6, 12):
        x = float(rng.standard_normal())
        return float(np.float32(x)) if t == 6 else x
    lo, hi = {0: (0, 255), 1: (-128, 127), 2: (0, 65535), 3: (-32768, 32767), 4: (0, 2**32 - 1),
              5: (-2**31, 2**31 - 1), 10: (0, 2**63), 11: (-2**63, 2**63 - 1)}[t]
    return int(rng.integers(lo, hi, dtype=np.int64 if t != 10 else np.uint64))


TENSOR_TYPES = [0, 1, 2, 3, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 19, 20, 23, 24, 25, 26, 27, 28, 29]


@pytest.mark.parametrize("seed", range(12))
def test_random_files_match_oracle(tmp_path, seed):
    rng = np.random.default_rng(seed)
    meta = []
    for k in range(int(rng.integers(0, 20))):
        t = int(rng.integers(0, 13))
        key = f"key.{int(rng.integers(0, 8))}" if rng.random() < 0.3 else f"general.k{k}"  # repeats
        meta.append((key, t, random_value(rng, t)))
    tensors = []
    for k in range(int(rng.integers(0, 10))):
        t = TENSOR_TYPES[int(rng.integers(0, len(TENSOR_TYPES)))]
        dims = [int(rng.integers(1, 5)) * 32 for _ in range(int(rng.integers(1, 4)))]
        name = f"blk.{int(rng.integers(0, 4))}.w" if rng.random() < 0.3 else f"t{k}"
        tensors.append((name, dims, t, bytes(rng.integers(0, 256, int(rng.integers(0, 3000)), dtype=np.uint8))))
    p = tmp_path / f"r{seed}.gguf"
    G.write_gguf(p, meta, tensors)
    raw = open(p, "rb").read()
    if seed % 3 == 0 and len(raw) > 40:  # cut the file: some views vanish or shrink
        raw = raw[:len(raw) - int(rng.integers(1, 2000))]
        open(p, "wb").write(raw)
    try:
        want = O.parse(raw)
    except O.GgufError:
        with pytest.raises(Exception):
            G.GgufFile(p)
        return
    f = G.GgufFile(p)
    f._path = p
    same(f, want)
    for t in tensors:
        got, ref = f.find_tensor(t[0]), O.find_tensor(want, t[0])
        assert (got is None) == (ref is None)
        if got is not None:
            assert got.index == want["tensor_infos"].index(ref)
    f.close()


def header(magic=0x46554747, version=3, nt=0, nkv=0):
    return struct.pack("<IIQQ", magic, version, nt, nkv)


def kv(key, t, payload):
    return struct.pack("<Q", len(key)) + key + struct.pack("<I", t) + payload


@pytest.mark.parametrize("blob", [
    header(magic=0xDEADBEEF),                       # reject_invalid_magic (gguf.rs:779-793)
    header(version=4),
    header()[:20],                                  # shorter than 24 bytes
    header(nkv=1) + kv(b"a", 13, b""),              # unknown metadata type
    header(nkv=1) + kv(b"a", 4, b"\1\0"),           # truncated U32
    header(nkv=1) + kv(b"a", 9, struct.pack("<IQ", 77, 0)),  # empty array of an unknown type
    header(nkv=1) + kv(b"a", 9, struct.pack("<IQ", 4, 1 << 60)),  # array count beyond the file
    header(nt=1) + struct.pack("<Q", 1) + b"w" + struct.pack("<IQIQ", 1, 32, 4, 0),  # tensor type 4
    header(nt=1) + struct.pack("<Q", 1) + b"w" + struct.pack("<I", 3),  # truncated dims
    header(nt=1 << 40),                             # more tensors than the file can hold
])
def test_rejected_files(tmp_path, blob):
    p = tmp_path / "bad.gguf"
    open(p, "wb").write(blob)
    with pytest.raises(O.GgufError):
        O.parse(blob)
    from bml_b200 import _lib
    with pytest.raises(_lib.BmlError):
        G.GgufFile(p)


def test_invalid_utf8_and_last_key_wins(tmp_path):
    p = tmp_path / "u.gguf"
    G.write_gguf(p, [("k", 8, b"ab\xff\xfecd"), ("k", 4, 7), ("x\xe9", 8, "y")], [])
    f = G.GgufFile(p)
    want = O.parse(open(p, "rb").read())
    assert f.metadata_typed == want["metadata"]
    assert f.get_metadata("k") == 7
    assert f.architecture() is None
    f.close()


def test_missing_file_and_sizes(tmp_path):
    from bml_b200 import _lib
    with pytest.raises(_lib.BmlError):
        G.GgufFile(tmp_path / "missing.gguf")
    # exact stored sizes of the block types (what upload copies)
    p = tmp_path / "s.gguf"
    G.write_gguf(p, [], [("q4", [256, 2], 2, b"\0" * 288), ("q8", [64], 8, b"\0" * 68),
                         ("k4", [512], 12, b"\0" * 288), ("iq", [256], 16, b"\0" * 66),
                         ("bf", [3, 5], 29, b"\0" * 30)])
    f = G.GgufFile(p)
    assert [t.nbytes for t in f.tensor_infos] == [288, 68, 288, 0, 30]
    f.close()
