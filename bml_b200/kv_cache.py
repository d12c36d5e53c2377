"""HashConsedKV on the GPU: the Python mirror of the reference struct
(crates/compiler/src/kv_cache.rs:25-181 in SugarFreeDoNoSo/bml) over the
bml_kv_* entry points.  Method names, argument order and results follow the
Rust API; index errors the Rust code panics on raise BmlInvalid (an
IndexError-like ValueError)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L
from .attention import _need, _ptr, _stream, dtype_code

_NAMES = {"f32": L.BML_F32, "f16": L.BML_F16, "bf16": L.BML_BF16,
          torch.float32: L.BML_F32, torch.float16: L.BML_F16, torch.bfloat16: L.BML_BF16}
_TORCH = {L.BML_F32: torch.float32, L.BML_F16: torch.float16, L.BML_BF16: torch.bfloat16}


class _DevArray:
    """Minimal __cuda_array_interface__ exporter so torch can view the
    library-owned layer buffers without a copy."""

    def __init__(self, ptr: int, shape, typestr: str, owner):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}
        self._owner = owner


class HashConsedKV:
    """KV cache: per-layer K and V buffers [max_seq_len][n_kv_heads][head_dim]
    on one GPU, ring slot pos % max_seq_len (kv_cache.rs:83)."""

    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, max_seq_len: int,
                 dtype="f32", device: int | None = None):
        self._h = None
        dev = torch.cuda.current_device() if device is None else int(device)
        desc = L.bml_kv_desc(n_layers, n_kv_heads, head_dim, max_seq_len, _NAMES[dtype], dev)
        h = C.c_void_p()
        L.call("bml_kv_create", C.byref(desc), C.byref(h))
        self._h = h
        self.n_layers, self.n_kv_heads, self.head_dim, self.max_seq_len = (
            n_layers, n_kv_heads, head_dim, max_seq_len)
        self.dtype_code = _NAMES[dtype]
        self.device = torch.device("cuda", dev)

    def close(self) -> None:
        h, self._h = self._h, None
        if h:
            L.call("bml_kv_destroy", h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # kv_cache.rs:82-101 ------------------------------------------------------
    def _store(self, which, layer, pos, kv_head, data):
        a = np.ascontiguousarray(np.asarray(data, dtype=np.float32)).reshape(-1)
        L.call("bml_kv_store", self._h, which, layer, pos, kv_head, a.ctypes.data, a.size)

    def store_k(self, layer: int, pos: int, kv_head: int, data) -> None:
        self._store(L.WHICH_K, layer, pos, kv_head, data)

    def store_v(self, layer: int, pos: int, kv_head: int, data) -> None:
        self._store(L.WHICH_V, layer, pos, kv_head, data)

    # kv_cache.rs:111-124 -----------------------------------------------------
    def _load(self, which, layer, pos, kv_head) -> np.ndarray:
        out = np.empty(self.head_dim, np.float32)
        L.call("bml_kv_load", self._h, which, layer, pos, kv_head, out.ctypes.data)
        return out

    def load_k(self, layer: int, pos: int, kv_head: int) -> np.ndarray:
        return self._load(L.WHICH_K, layer, pos, kv_head)

    def load_v(self, layer: int, pos: int, kv_head: int) -> np.ndarray:
        return self._load(L.WHICH_V, layer, pos, kv_head)

    # kv_cache.rs:135-141 -----------------------------------------------------
    def dot_qk(self, q, layer: int, pos: int, kv_head: int) -> float:
        a = np.ascontiguousarray(np.asarray(q, dtype=np.float32)).reshape(-1)
        out = C.c_float()
        L.call("bml_kv_dot_qk", self._h, a.ctypes.data, a.size, layer, pos, kv_head, C.byref(out))
        return float(out.value)

    # kv_cache.rs:148-180 -----------------------------------------------------
    def _stats(self, which):
        u, t, r = C.c_uint64(), C.c_uint64(), C.c_double()
        L.call("bml_kv_stats", self._h, which, C.byref(u), C.byref(t), C.byref(r))
        return (u.value, t.value, r.value)

    def k_stats(self):
        return self._stats(L.WHICH_K)

    def v_stats(self):
        return self._stats(L.WHICH_V)

    def byte_size(self) -> int:
        out = C.c_uint64()
        L.call("bml_kv_byte_size", self._h, C.byref(out))
        return out.value

    def current_pos(self) -> int:
        out = C.c_uint32()
        L.call("bml_kv_current_pos", self._h, C.byref(out))
        return out.value

    def advance(self) -> None:
        L.call("bml_kv_advance", self._h)

    def advance_by(self, n: int) -> None:
        L.call("bml_kv_advance_by", self._h, n)

    # device-side extensions --------------------------------------------------
    def layer_tensor(self, which: int, layer: int) -> torch.Tensor:
        """Zero-copy torch view of one layer's K (which=0) or V (1) buffer."""
        p = C.c_void_p()
        L.call("bml_kv_layer_ptr", self._h, which, layer, C.byref(p))
        typestr = {L.BML_F32: "<f4", L.BML_F16: "<f2", L.BML_BF16: "<f2"}[self.dtype_code]
        arr = _DevArray(p.value, (self.max_seq_len, self.n_kv_heads, self.head_dim), typestr, self)
        with torch.cuda.device(self.device):
            t = torch.as_tensor(arr, device=self.device)
        if self.dtype_code == L.BML_BF16:
            t = t.view(torch.bfloat16)
        return t

    def append(self, layer: int, pos: int, k: torch.Tensor, v: torch.Tensor, stream=None) -> None:
        """Device store of all kv heads at pos (gguf_compiler.rs:994-1006 in
        one launch).  k, v: [n_kv_heads, head_dim] CUDA tensors."""
        _need(k, "k")
        _need(v, "v", k.dtype)
        if k.numel() != self.n_kv_heads * self.head_dim or v.numel() != k.numel():
            raise ValueError("k/v must hold n_kv_heads * head_dim values")
        L.call("bml_kv_append", self._h, layer, pos, _ptr(k), _ptr(v), dtype_code(k.dtype),
               _stream(stream))

    def append_rope(self, layer: int, pos: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    stream=None) -> torch.Tensor:
        """RoPE on q (in place) and k, then k and v stored at pos: the
        projection tail of gguf_compiler.rs:984-1006 with apply_rope_inplace
        (:1290-1317) in one launch.  q [n_heads, head_dim], k/v [n_kv_heads,
        head_dim], all f32 CUDA tensors; returns q."""
        _need(q, "q", torch.float32)
        _need(k, "k", torch.float32)
        _need(v, "v", torch.float32)
        if k.numel() != self.n_kv_heads * self.head_dim or v.numel() != k.numel():
            raise ValueError("k/v must hold n_kv_heads * head_dim values")
        if q.numel() % self.head_dim != 0:
            raise ValueError("q must hold n_heads * head_dim values")
        L.call("bml_kv_append_rope", self._h, layer, pos, _ptr(q), q.numel() // self.head_dim, _ptr(k), _ptr(v),
               _stream(stream))
        return q

    def attention(self, q: torch.Tensor, layer: int, pos: int, scale: float = -1.0,
                  out: torch.Tensor | None = None, stream=None, wrap_compat: bool = False) -> torch.Tensor:
        """The attention block of forward_layer_cached (gguf_compiler.rs:
        1008-1050) for the token at `pos`: q [n_heads, head_dim] f32 CUDA
        tensor -> [n_heads, head_dim] f32.  pos >= max_seq_len is refused
        unless wrap_compat, which reproduces the reference's loop over
        positions 0..pos read through slot p % max_seq_len (kv_cache.rs:83)."""
        _need(q, "q", torch.float32)
        n_heads = q.numel() // self.head_dim
        if out is None:
            out = torch.empty(n_heads, self.head_dim, dtype=torch.float32, device=q.device)
        L.call("bml_attn_decode_wrap" if wrap_compat else "bml_attn_decode", self._h, layer, pos, n_heads,
               float(scale), _ptr(q), _ptr(out), _stream(stream))
        return out
