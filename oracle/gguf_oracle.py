"""Pure-Python restatement of the reference's GGUF parser
(crates/parser/src/gguf.rs in SugarFreeDoNoSo/bml), over a file's bytes.

TEST INFRASTRUCTURE ONLY: the checker for the library's parser
(bml_b200/csrc/gguf.cu), never the thing measured or shipped.  Values are
(type id, payload) pairs as the reference's GgufMetadataValue enum holds
them; arrays as (ARRAY, (elem type, [items])).
"""
from __future__ import annotations

import struct

GGUF_MAGIC = 0x46554747  # gguf.rs:25
SUPPORTED_VERSION = 3    # gguf.rs:26
ARRAY, STRING = 9, 8
_SCALAR = {0: ("<B", 1), 1: ("<b", 1), 2: ("<H", 2), 3: ("<h", 2), 4: ("<I", 4), 5: ("<i", 4), 6: ("<f", 4),
           7: (None, 1), 10: ("<Q", 8), 11: ("<q", 8), 12: ("<d", 8)}


class GgufError(ValueError):
    pass


def tensor_type_known(t: int) -> bool:
    """GgufDataType::from_u32 (gguf.rs:77-108)."""
    return t <= 3 or 6 <= t <= 29


def element_size(t: int) -> int:
    """GgufDataType::element_size (gguf.rs:132-143) for tensor type ids."""
    return {0: 4, 26: 4, 1: 2, 25: 2, 29: 2, 24: 1, 27: 8, 28: 8}.get(t, 0)


def is_quantized(t: int) -> bool:
    """GgufDataType::is_quantized (gguf.rs:145-170): the block types and
    F16 / BF16."""
    return 2 <= t <= 23 or t in (1, 29)


def _string(b: bytes, off: int):
    """decode_string (gguf.rs:381-393)."""
    if off + 8 > len(b):
        raise GgufError("offset out of range reading string len")
    n = struct.unpack_from("<Q", b, off)[0]
    if off + 8 + n > len(b):
        raise GgufError("offset out of range reading string data")
    return b[off + 8:off + 8 + n].decode("utf-8", errors="replace"), off + 8 + n


def _value(b: bytes, off: int, t: int):
    """decode_metadata_value (gguf.rs:409-545)."""
    if t in _SCALAR:
        fmt, size = _SCALAR[t]
        if off + size > len(b):
            raise GgufError("offset out of range")
        if t == 7:
            return (t, b[off] != 0), off + 1
        return (t, struct.unpack_from(fmt, b, off)[0]), off + size
    if t == STRING:
        s, off = _string(b, off)
        return (t, s), off
    if t == ARRAY:
        if off + 12 > len(b):
            raise GgufError("offset out of range reading array header")
        et, count = struct.unpack_from("<IQ", b, off)
        off += 12
        items = []
        for _ in range(count):
            v, off = _value(b, off, et)
            items.append(v)
        if et > 12:  # from_metadata_u32 after the loop
            raise GgufError(f"unknown array type {et}")
        return (ARRAY, (et, items)), off
    raise GgufError(f"unknown metadata type {t}")


def parse(b: bytes) -> dict:
    """GgufParser::open (gguf.rs:239-292) over the file's bytes."""
    if len(b) < 24:
        raise GgufError("file too small")
    magic, version, n_tensors, n_kv = struct.unpack_from("<IIQQ", b, 0)
    if magic != GGUF_MAGIC:
        raise GgufError(f"bad magic 0x{magic:08X}")
    if version > SUPPORTED_VERSION:
        raise GgufError(f"unsupported version {version}")
    off = 24
    meta = {}
    for _ in range(n_kv):
        key, off = _string(b, off)
        if off + 4 > len(b):
            raise GgufError("offset out of range reading value type")
        t = struct.unpack_from("<I", b, off)[0]
        v, off = _value(b, off + 4, t)
        meta[key] = v  # HashMap::insert: the last value of a key wins
    infos = []
    for _ in range(n_tensors):  # decode_tensor_info (gguf.rs:548-592)
        name, off = _string(b, off)
        if off + 4 > len(b):
            raise GgufError("offset out of range reading n_dims")
        nd = struct.unpack_from("<I", b, off)[0]
        off += 4
        dims = []
        for _ in range(nd):
            if off + 8 > len(b):
                raise GgufError("offset out of range reading dim")
            dims.append(struct.unpack_from("<Q", b, off)[0])
            off += 8
        if off + 4 > len(b):
            raise GgufError("offset out of range reading data_type")
        t = struct.unpack_from("<I", b, off)[0]
        if not tensor_type_known(t):
            raise GgufError(f"unknown tensor type {t}")
        off += 4
        if off + 8 > len(b):
            raise GgufError("offset out of range reading tensor offset")
        toff = struct.unpack_from("<Q", b, off)[0]
        off += 8
        infos.append({"name": name, "n_dims": nd, "dims": dims, "data_type": t, "offset": toff})
    data_offset = (off + 31) // 32 * 32  # align(offset, 32)
    return {"header": {"magic": magic, "version": version, "tensor_count": n_tensors, "metadata_kv_count": n_kv},
            "metadata": meta, "tensor_infos": infos, "data_offset": data_offset, "size": len(b)}


def find_tensor(parsed: dict, name: str):
    """find_tensor (gguf.rs:332-337): the first tensor of that name."""
    for t in parsed["tensor_infos"]:
        if t["name"] == name:
            return t
    return None


def tensor_data(parsed: dict, info: dict):
    """tensor_data (gguf.rs:339-364) as (start, length), or None."""
    start = parsed["data_offset"] + info["offset"]
    size = parsed["size"]
    if start > size:
        return None
    es = element_size(info["data_type"])
    if es:
        n = 1
        for d in info["dims"]:
            n *= d
        end = start + n * es
        return None if end > size else (start, n * es)
    if is_quantized(info["data_type"]):
        return (start, size - start)
    return None
