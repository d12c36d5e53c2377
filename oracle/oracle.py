"""ctypes front end of the C oracle (bml_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never the thing
measured or shipped.  Each function names the reference code it restates;
the restatement itself lives in bml_oracle.c.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libbmloracle.so")
_lock = threading.Lock()
_lib = None

F32, F16, BF16 = 0, 1, 2
K, V = 0, 1
# GGUF tensor type ids read by read_tensor_f32 (crates/parser/src/gguf.rs:36-43)
GGUF_F32, GGUF_F16, GGUF_Q4_0, GGUF_Q8_0 = 0, 1, 2, 8


def build(force: bool = False) -> str:
    """Compiles bml_oracle.c with the committed Makefile (gcc, -O2,
    -ffp-contract=off, OpenMP)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "bml_oracle.c"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = C.CDLL(_LIB_PATH)
            vp, u32, i32, f64p = C.c_void_p, C.c_uint32, C.c_int, C.c_void_p
            L.orc_kv_new.restype = vp
            L.orc_kv_new.argtypes = [u32, u32, u32, u32]
            L.orc_kv_free.argtypes = [vp]
            L.orc_kv_store.restype = i32
            L.orc_kv_store.argtypes = [vp, i32, u32, u32, u32, vp, C.c_size_t]
            L.orc_kv_load.restype = i32
            L.orc_kv_load.argtypes = [vp, i32, u32, u32, u32, vp]
            L.orc_kv_dot_qk.restype = C.c_float
            L.orc_kv_dot_qk.argtypes = [vp, vp, C.c_size_t, u32, u32, u32]
            L.orc_kv_stats.argtypes = [vp, i32, vp, vp, vp]
            L.orc_kv_byte_size.restype = C.c_uint64
            L.orc_kv_byte_size.argtypes = [vp]
            L.orc_kv_current_pos.restype = u32
            L.orc_kv_current_pos.argtypes = [vp]
            L.orc_kv_advance.argtypes = [vp]
            L.orc_kv_advance_by.argtypes = [vp, u32]
            L.orc_kv_buffer.restype = vp
            L.orc_kv_buffer.argtypes = [vp, i32, u32]
            L.orc_softmax_f32.restype = C.c_size_t
            L.orc_softmax_f32.argtypes = [vp, C.c_size_t, vp]
            L.orc_rope_inplace_f64.argtypes = [vp, C.c_size_t, C.c_size_t, C.c_size_t]
            L.orc_rope_rows_f32.argtypes = [vp, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t]
            L.orc_attn_decode.restype = i32
            L.orc_attn_decode.argtypes = [vp, vp, vp, i32, u32, u32, u32, u32, u32,
                                          C.c_double, f64p, i32]
            L.orc_attn_decode_batched.restype = i32
            L.orc_attn_decode_batched.argtypes = [vp, vp, vp, vp, u32, i32, u32, u32, u32,
                                                  C.c_double, f64p, i32]
            L.orc_attn_prefill.restype = i32
            L.orc_attn_prefill.argtypes = [vp, vp, vp, i32, u32, u32, u32, u32, u32,
                                           C.c_double, u32, u32, f64p, i32]
            L.orc_attn_prefill_rows.restype = i32
            L.orc_attn_prefill_rows.argtypes = [vp, vp, vp, i32, u32, u32, u32, u32, u32, C.c_double, vp,
                                                u32, u32, u32, f64p, i32]
            L.orc_attn_decode_literal.restype = i32
            L.orc_attn_decode_literal.argtypes = [vp, vp, vp, u32, u32, u32, u32, u32, u32,
                                                  u32, f64p]
            L.orc_num_threads.restype = i32
            L.orc_gguf_f16_to_f32.restype = C.c_float
            L.orc_gguf_f16_to_f32.argtypes = [C.c_uint16]
            L.orc_read_tensor_f32.restype = C.c_int64
            L.orc_read_tensor_f32.argtypes = [vp, C.c_uint64, i32, C.c_uint64, vp]
            L.orc_matmul_f64.argtypes = [vp, C.c_uint64, C.c_uint64, C.c_uint64, vp, C.c_uint64, vp]
            _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _dtype_code(a: np.ndarray) -> int:
    """f32 arrays are f32; uint16 arrays carry f16 or bf16 bits and must be
    tagged by the caller; np.float16 is f16."""
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    raise TypeError(f"pass f32/f16 arrays or (uint16 bits, dtype code): {a.dtype}")


class HashConsedKV:
    """Mirror of kv_cache.rs:25-181 over the C restatement."""

    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, max_seq_len: int):
        self._L = lib()
        self._h = self._L.orc_kv_new(n_layers, n_kv_heads, head_dim, max_seq_len)
        self.n_layers, self.n_kv_heads, self.head_dim, self.max_seq_len = (
            n_layers, n_kv_heads, head_dim, max_seq_len)

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            self._L.orc_kv_free(h)

    def _store(self, which, layer, pos, kv_head, data):
        a = np.ascontiguousarray(np.asarray(data, dtype=np.float32))
        if self._L.orc_kv_store(self._h, which, layer, pos, kv_head, _ptr(a), a.size) != 0:
            raise IndexError("store out of range (the reference panics here)")

    def store_k(self, layer, pos, kv_head, data):
        self._store(K, layer, pos, kv_head, data)

    def store_v(self, layer, pos, kv_head, data):
        self._store(V, layer, pos, kv_head, data)

    def _load(self, which, layer, pos, kv_head):
        out = np.empty(self.head_dim, np.float32)
        if self._L.orc_kv_load(self._h, which, layer, pos, kv_head, _ptr(out)) != 0:
            raise IndexError("load out of range (the reference panics here)")
        return out

    def load_k(self, layer, pos, kv_head):
        return self._load(K, layer, pos, kv_head)

    def load_v(self, layer, pos, kv_head):
        return self._load(V, layer, pos, kv_head)

    def dot_qk(self, q, layer, pos, kv_head) -> float:
        a = np.ascontiguousarray(np.asarray(q, dtype=np.float32))
        return float(self._L.orc_kv_dot_qk(self._h, _ptr(a), a.size, layer, pos, kv_head))

    def _stats(self, which):
        u, t, r = C.c_uint64(), C.c_uint64(), C.c_double()
        self._L.orc_kv_stats(self._h, which, C.byref(u), C.byref(t), C.byref(r))
        return (u.value, t.value, r.value)

    def k_stats(self):
        return self._stats(K)

    def v_stats(self):
        return self._stats(V)

    def byte_size(self) -> int:
        return int(self._L.orc_kv_byte_size(self._h))

    def current_pos(self) -> int:
        return int(self._L.orc_kv_current_pos(self._h))

    def advance(self):
        self._L.orc_kv_advance(self._h)

    def advance_by(self, n):
        self._L.orc_kv_advance_by(self._h, n)

    def buffer(self, which: int, layer: int) -> np.ndarray:
        """Copy of one layer's flat buffer [max_seq_len][n_kv][head_dim]."""
        n = self.max_seq_len * self.n_kv_heads * self.head_dim
        p = self._L.orc_kv_buffer(self._h, which, layer)
        return np.ctypeslib.as_array((C.c_float * n).from_address(p)).copy().reshape(
            self.max_seq_len, self.n_kv_heads, self.head_dim)

    def attention(self, q, layer, pos, n_heads, n_threads=1) -> np.ndarray:
        """gguf_compiler.rs:1008-1050 at `pos` over this cache's layer."""
        qa = np.ascontiguousarray(np.asarray(q, dtype=np.float32)).reshape(-1)
        out = np.empty(n_heads * self.head_dim, np.float64)
        kb = self._L.orc_kv_buffer(self._h, K, layer)
        vb = self._L.orc_kv_buffer(self._h, V, layer)
        rc = self._L.orc_attn_decode(_ptr(qa), kb, vb, F32, self.max_seq_len, self.n_kv_heads,
                                     self.head_dim, n_heads, pos, -1.0, _ptr(out), n_threads)
        if rc != 0:
            raise ValueError("rejected shape")
        return out.reshape(n_heads, self.head_dim)


def softmax_f32(scores) -> np.ndarray:
    """kv_cache.rs:188-200."""
    a = np.ascontiguousarray(np.asarray(scores, dtype=np.float32))
    out = np.empty_like(a)
    if a.size:
        lib().orc_softmax_f32(_ptr(a), a.size, _ptr(out))
    return out


def rope_inplace_f64(x: np.ndarray, pos: int, head_dim: int) -> np.ndarray:
    """gguf_compiler.rs:1290-1317 on an f64 vector (in place)."""
    assert x.dtype == np.float64 and x.flags["C_CONTIGUOUS"]
    lib().orc_rope_inplace_f64(_ptr(x), x.size, pos, head_dim)
    return x


def rope_rows_f32(x: np.ndarray, head_dim: int, pos0: int = 0) -> np.ndarray:
    """RoPE on rows [n_rows][row_len] of f32 at positions pos0 + r, computed in
    f64 as the reference does; x is modified in place."""
    assert x.dtype == np.float32 and x.flags["C_CONTIGUOUS"]
    rows = x.shape[0]
    row_len = x.size // rows
    lib().orc_rope_rows_f32(_ptr(x), rows, row_len, pos0, head_dim)
    return x


def attn_decode(q, k, v, pos=None, scale=-1.0, dtype=None, n_threads=1) -> np.ndarray:
    """One token over one cache (gguf_compiler.rs:1008-1050).
    q [n_heads, d] f32; k, v [max_seq_len, n_kv, d] (f32, f16, or uint16 bf16
    bits with dtype=BF16); pos defaults to the last position."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    code = dtype if dtype is not None else _dtype_code(k)
    S, n_kv, d = k.shape
    n_heads = q.shape[0]
    if pos is None:
        pos = S - 1
    out = np.empty((n_heads, d), np.float64)
    rc = lib().orc_attn_decode(_ptr(q), _ptr(k), _ptr(v), code, S, n_kv, d, n_heads, pos,
                               float(scale), _ptr(out), n_threads)
    if rc != 0:
        raise ValueError("rejected shape")
    return out


def attn_decode_batched(q, ks, vs, scale=-1.0, dtype=None, n_threads=0) -> np.ndarray:
    """Batched decode: q [n_seqs, n_heads, d]; ks/vs lists of [L_i, n_kv, d]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    n_seqs, n_heads, d = q.shape
    ks = [np.ascontiguousarray(a) for a in ks]
    vs = [np.ascontiguousarray(a) for a in vs]
    code = dtype if dtype is not None else _dtype_code(ks[0])
    n_kv = ks[0].shape[1]
    lens = np.array([a.shape[0] for a in ks], np.uint32)
    kp = (C.c_void_p * n_seqs)(*[a.ctypes.data for a in ks])
    vp_ = (C.c_void_p * n_seqs)(*[a.ctypes.data for a in vs])
    out = np.empty((n_seqs, n_heads, d), np.float64)
    rc = lib().orc_attn_decode_batched(_ptr(q), C.addressof(kp), C.addressof(vp_), _ptr(lens),
                                       n_seqs, code, n_kv, d, n_heads, float(scale), _ptr(out),
                                       n_threads)
    if rc != 0:
        raise ValueError("rejected shape")
    return out


def attn_prefill(q, k, v, scale=-1.0, rows=None, dtype=None, n_threads=0) -> np.ndarray:
    """Causal prefill = per-token loop (gguf_compiler.rs:946-958).
    q [n_seqs, S, n_heads, d] f32; k, v [n_seqs, S, n_kv, d].  rows=(lo, hi)
    restricts the computed query rows; other rows of the result are NaN."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    code = dtype if dtype is not None else _dtype_code(k)
    n_seqs, S, n_heads, d = q.shape
    n_kv = k.shape[2]
    lo, hi = rows if rows is not None else (0, S)
    out = np.full(q.shape, np.nan, np.float64)
    rc = lib().orc_attn_prefill(_ptr(q), _ptr(k), _ptr(v), code, n_seqs, S, n_heads, n_kv, d,
                                float(scale), lo, hi, _ptr(out), n_threads)
    if rc != 0:
        raise ValueError("rejected shape")
    return out


def attn_prefill_rows(q, k, v, rows, heads=None, scale=-1.0, dtype=None, n_threads=0) -> np.ndarray:
    """Causal prefill at chosen query rows: rows is a list of (sequence,
    position); returns [len(rows), h_hi - h_lo, d] for heads=(h_lo, h_hi)
    (default all), the values attn_prefill gives at those rows."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    code = dtype if dtype is not None else _dtype_code(k)
    n_seqs, S, n_heads, d = q.shape
    n_kv = k.shape[2]
    h_lo, h_hi = heads if heads is not None else (0, n_heads)
    r = np.ascontiguousarray(np.asarray(rows, dtype=np.uint32).reshape(-1, 2))
    out = np.empty((r.shape[0], h_hi - h_lo, d), np.float64)
    rc = lib().orc_attn_prefill_rows(_ptr(q), _ptr(k), _ptr(v), code, n_seqs, S, n_heads, n_kv, d,
                                     float(scale), _ptr(r), r.shape[0], h_lo, h_hi, _ptr(out), n_threads)
    if rc != 0:
        raise ValueError("rejected shape")
    return out


def attn_decode_literal(q, k, v, pos, heads=None) -> np.ndarray:
    """The reference's literal per-load heap-copy pattern, f32 cache only."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    S, n_kv, d = k.shape
    n_heads = q.shape[0]
    h_lo, h_hi = heads if heads is not None else (0, n_heads)
    out = np.full((n_heads, d), np.nan, np.float64)
    rc = lib().orc_attn_decode_literal(_ptr(q), _ptr(k), _ptr(v), S, n_kv, d, n_heads, h_lo,
                                       h_hi, pos, _ptr(out))
    if rc != 0:
        raise ValueError("rejected shape")
    return out


def num_threads() -> int:
    return int(lib().orc_num_threads())


def f16_to_f32(h: int) -> float:
    """gguf_compiler.rs:373-403."""
    return float(lib().orc_gguf_f16_to_f32(h))


def read_tensor_f32(data, gguf_type: int, n_elems: int) -> np.ndarray:
    """read_tensor_f32 (gguf_compiler.rs:351-369) with dequantize_q4_0 /
    dequantize_q8_0 (:405-470): the tensor's bytes -> its f32 values."""
    buf = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8))
    cap = max(int(n_elems), buf.size // 2 + 1)
    out = np.zeros(cap, np.float32)
    n = lib().orc_read_tensor_f32(_ptr(buf) if buf.size else None, buf.size, gguf_type, n_elems, _ptr(out))
    if n < 0:
        raise ValueError(f"GGUF type {gguf_type} is not read by the reference")
    return out[:n]


def matmul_f64(w: np.ndarray, n_in: int, n_out: int, x: np.ndarray) -> np.ndarray:
    """matmul_f64 (gguf_compiler.rs:1239-1255): y = x . W, W [n_in, n_out]
    indexed i*n_out + j over the tensor's f32 values, f64 accumulation."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty(n_out, np.float64)
    lib().orc_matmul_f64(_ptr(w), w.size, n_in, n_out, _ptr(x), x.size, _ptr(y))
    return y
