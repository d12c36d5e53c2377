"""GGUF files on the B200: the host parser of libbmlattn.so (include/bml_gguf.h)
behind the reference's GgufParser interface, and tensors uploaded to device
memory.

Mirrors crates/parser/src/gguf.rs in SugarFreeDoNoSo/bml: GgufParser::open
(:239-292), header / metadata / tensor_infos / architecture /
get_metadata / find_tensor / tensor_data (:294-364).  Metadata values are
plain Python values (int, float, bool, str, lists for arrays); strings are
decoded as the reference does, replacing invalid UTF-8 (from_utf8_lossy).
`metadata_typed` keeps the GGUF type ids, as the reference's
GgufMetadataValue enum does.

`write_gguf` writes a GGUF v3 file (for fixtures and benchmarks).
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass

import numpy as np

from . import _lib as L

GGUF_MAGIC = 0x46554747
NOT_FOUND = (1 << 64) - 1

# metadata value types (gguf.rs:112-129)
META_U8, META_I8, META_U16, META_I16, META_U32, META_I32, META_F32, META_BOOL = range(8)
META_STRING, META_ARRAY, META_U64, META_I64, META_F64 = 8, 9, 10, 11, 12
_SCALAR_FMT = {META_U8: "<B", META_I8: "<b", META_U16: "<H", META_I16: "<h", META_U32: "<I", META_I32: "<i",
               META_F32: "<f", META_BOOL: "<?", META_U64: "<Q", META_I64: "<q", META_F64: "<d"}


@dataclass
class TensorInfo:
    """GgufTensorInfo (gguf.rs:203-209) plus where its data lies."""
    name: str
    n_dims: int
    dims: list
    data_type: int
    offset: int
    index: int
    present: bool      # tensor_data() is Some
    data_offset: int   # absolute file offset of the data
    view_len: int      # bytes of tensor_data()'s slice
    nbytes: int        # exact stored size (0: a layout this library does not know)


def _text(ptr: int, n: int) -> str:
    return C.string_at(ptr, n).decode("utf-8", errors="replace") if n else ""


class GgufFile:
    """GgufParser: the file memory-mapped and parsed by the library."""

    def __init__(self, path):
        h = C.c_void_p()
        L.call("bml_gguf_open", str(path).encode(), C.byref(h))
        self._h = h
        hd = L.bml_gguf_header()
        L.call("bml_gguf_get_header", self._h, C.byref(hd))
        self.header = {"magic": hd.magic, "version": hd.version, "tensor_count": hd.tensor_count,
                       "metadata_kv_count": hd.metadata_kv_count}
        self.data_offset = hd.data_offset
        self.file_size = hd.file_size
        self._infos = None
        self._meta = None

    def close(self) -> None:
        if self._h:
            L.call("bml_gguf_close", self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- tensors ---------------------------------------------------------
    def _info(self, i: int) -> TensorInfo:
        t = L.bml_gguf_tensor()
        L.call("bml_gguf_tensor_info", self._h, i, C.byref(t))
        return TensorInfo(_text(t.name, t.name_len), t.n_dims, [t.dims[k] for k in range(t.n_dims)], t.type,
                          t.offset, i, bool(t.present), t.data_offset, t.view_len, t.nbytes)

    @property
    def tensor_infos(self) -> list:
        if self._infos is None:
            self._infos = [self._info(i) for i in range(self.header["tensor_count"])]
        return self._infos

    def find_tensor(self, name: str):
        idx = C.c_uint64()
        L.call("bml_gguf_find_tensor", self._h, name.encode(), C.byref(idx))
        return None if idx.value == NOT_FOUND else self.tensor_infos[idx.value]

    def tensor_data(self, info: TensorInfo):
        """Zero-copy uint8 view of tensor_data() (None where the reference
        returns None); valid while the file is open."""
        p, n = C.c_void_p(), C.c_uint64()
        L.call("bml_gguf_tensor_view", self._h, info.index, C.byref(p), C.byref(n))
        if not p.value:
            return None
        if n.value == 0:
            return np.zeros(0, np.uint8)
        return np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p.value))

    # -- metadata --------------------------------------------------------
    def _value(self, i: int, path: list):
        v = L.bml_gguf_value()
        arr = (C.c_uint64 * max(1, len(path)))(*path)
        L.call("bml_gguf_meta_value", self._h, i, arr, len(path), C.byref(v))
        if v.type == META_ARRAY:
            return (META_ARRAY, (v.elem_type, [self._value(i, path + [k]) for k in range(v.len)]))
        if v.type == META_STRING:
            return (META_STRING, _text(v.str, v.len))
        if v.type in (META_F32, META_F64):
            return (v.type, v.f)
        if v.type in (META_I8, META_I16, META_I32, META_I64):
            return (v.type, v.i)
        if v.type == META_BOOL:
            return (v.type, bool(v.u))
        return (v.type, v.u)

    @property
    def metadata_typed(self) -> dict:
        """key -> (type id, value); arrays as (ARRAY, (elem type, [items]));
        a repeated key keeps its last value, as the reference's HashMap."""
        if self._meta is None:
            meta = {}
            for i in range(self.header["metadata_kv_count"]):
                kp, kn = C.c_void_p(), C.c_uint64()
                L.call("bml_gguf_meta_key", self._h, i, C.byref(kp), C.byref(kn))
                meta[_text(kp.value, kn.value)] = self._value(i, [])
            self._meta = meta
        return self._meta

    @property
    def metadata(self) -> dict:
        return {k: plain(v) for k, v in self.metadata_typed.items()}

    def get_metadata(self, key: str):
        v = self.metadata_typed.get(key)
        return None if v is None else plain(v)

    def architecture(self):
        """general.architecture when it is a string (gguf.rs:319-325)."""
        v = self.metadata_typed.get("general.architecture")
        return v[1] if v is not None and v[0] == META_STRING else None

    # -- device upload ---------------------------------------------------
    def upload(self, infos, device=None, threads: int = 0) -> dict:
        """Copies tensors (TensorInfo or names) into fresh device buffers
        (uint8 torch tensors of nbytes each, on `device`); name -> tensor."""
        import torch
        infos = [self.find_tensor(i) if isinstance(i, str) else i for i in infos]
        if any(i is None for i in infos):
            raise KeyError("tensor not found")
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index or 0)
        out = {i.name: torch.empty(i.nbytes, dtype=torch.uint8, device=dev) for i in infos}
        idx = (C.c_uint64 * max(1, len(infos)))(*[i.index for i in infos])
        dst = (C.c_void_p * max(1, len(infos)))(*[out[i.name].data_ptr() for i in infos])
        with torch.cuda.device(dev):
            torch.cuda.current_stream().synchronize()  # the buffers exist before the copies start
            L.call("bml_gguf_upload", self._h, idx, len(infos), dst, threads)
        return out

    def weight(self, name: str, device=None):
        """A WeightTensor of the named tensor, uploaded."""
        from .weights import WeightTensor
        info = self.find_tensor(name)
        if info is None:
            raise KeyError(name)
        return WeightTensor(self.upload([info], device)[name], info.data_type, info.dims)


def plain(v):
    t, x = v
    if t == META_ARRAY:
        return [plain(e) for e in x[1]]
    return x


# ---------------------------------------------------------------------------
# writer
# ---------------------------------------------------------------------------
def _w_str(out: bytearray, s) -> None:
    b = s.encode() if isinstance(s, str) else bytes(s)
    out += struct.pack("<Q", len(b)) + b


def _w_value(out: bytearray, t: int, x) -> None:
    if t == META_STRING:
        _w_str(out, x)
    elif t == META_ARRAY:
        et, items = x
        out += struct.pack("<IQ", et, len(items))
        for it in items:
            _w_value(out, et, it)
    else:
        out += struct.pack(_SCALAR_FMT[t], x)


def write_gguf(path, metadata, tensors, version: int = 3) -> None:
    """Writes a GGUF file.  metadata: list of (key, type id, value) (arrays
    as (elem type, [items])); tensors: list of (name, dims, type id, bytes)
    laid out in order from the 32-byte aligned data section, each padded to
    32 bytes."""
    out = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, version, len(tensors), len(metadata)))
    for k, t, x in metadata:
        _w_str(out, k)
        out += struct.pack("<I", t)
        _w_value(out, t, x)
    off = 0
    for name, dims, ttype, data in tensors:
        _w_str(out, name)
        out += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", ttype, off)
        off += (memoryview(data).nbytes + 31) // 32 * 32
    out += b"\0" * ((-len(out)) % 32)
    with open(path, "wb") as f:
        f.write(out)
        for _, _, _, data in tensors:
            nb = memoryview(data).nbytes
            f.write(data)
            f.write(b"\0" * ((-nb) % 32))
