"""Torch-facing wrappers of the attention entry points of libbmlattn.so.

torch is used for device memory and streams only; every computation runs in
the library's own sm_100a kernels.  Function names follow the reference
(crates/compiler/src/kv_cache.rs, crates/compiler/src/gguf_compiler.rs in
SugarFreeDoNoSo/bml) where one exists.
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import torch

from . import _lib as L

_DT = {torch.float32: L.BML_F32, torch.float16: L.BML_F16, torch.bfloat16: L.BML_BF16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def _stream(stream=None) -> C.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _ptr(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def _need(t: torch.Tensor, name: str, dtype=None, ndim=None) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dims, got {tuple(t.shape)}")


# ---------------------------------------------------------------------------
# softmax_f32 (kv_cache.rs:188-200)
# ---------------------------------------------------------------------------
def softmax_f32(x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Row-wise softmax_f32 over the last dimension of an f32 CUDA tensor."""
    _need(x, "x", torch.float32)
    if out is None:
        out = torch.empty_like(x)
    n = x.shape[-1] if x.dim() else 1
    rows = x.numel() // n if n else 0
    L.call("bml_softmax_f32", _ptr(x), rows, n, _ptr(out), _stream(stream))
    return out


# ---------------------------------------------------------------------------
# Decode workspace
# ---------------------------------------------------------------------------
class Workspace:
    """Device scratch for the split-K decode kernels (partial slots, merge
    tickets, error word).  Zero-filled at allocation; every call leaves it
    ready for the next.  Calls sharing one workspace must not overlap."""

    def __init__(self, device=None):
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   torch.device(device).index or 0)
        self.buf = torch.zeros(0, dtype=torch.uint8, device=self.device)
        self._sized = None  # the last (n_seqs, n_heads, head_dim) ensured

    def ensure(self, n_seqs: int, n_heads: int, head_dim: int) -> "Workspace":
        if self._sized == (n_seqs, n_heads, head_dim):
            return self
        size = C.c_size_t()
        L.call("bml_attn_decode_workspace_size", n_seqs, n_heads, head_dim, self.device.index,
               C.byref(size))
        if self.buf.numel() < size.value:
            self.buf = torch.zeros(size.value, dtype=torch.uint8, device=self.device)
        self._sized = (n_seqs, n_heads, head_dim)
        return self

    @property
    def ptr(self) -> C.c_void_p:
        return _ptr(self.buf)

    @property
    def nbytes(self) -> int:
        return self.buf.numel()

    def check(self, stream=None) -> None:
        """Raises BmlError(BML_E_TIMEOUT) if a bounded device wait gave up."""
        L.call("bml_attn_workspace_check", self.ptr, self.nbytes, _stream(stream))


_workspaces: dict[int, Workspace] = {}


def default_workspace(device_index: int) -> Workspace:
    ws = _workspaces.get(device_index)
    if ws is None:
        ws = _workspaces[device_index] = Workspace(device_index)
    return ws


# ---------------------------------------------------------------------------
# Sequence batches
# ---------------------------------------------------------------------------
class SeqBatch:
    """A batch of per-sequence KV caches, each [len, n_kv, d] contiguous on
    one device (or one [n_seqs, len, n_kv, d] tensor).  Holds the C
    descriptor array so repeated decode steps pay no per-call packing."""

    def __init__(self, ks: Sequence[torch.Tensor] | torch.Tensor,
                 vs: Sequence[torch.Tensor] | torch.Tensor):
        if isinstance(ks, torch.Tensor) and ks.dim() == 4:
            ks = list(ks.unbind(0))
            vs = list(vs.unbind(0))
        if len(ks) != len(vs) or not ks:
            raise ValueError("need matching, non-empty K and V lists")
        k0 = ks[0]
        self.n_kv, self.head_dim = int(k0.shape[1]), int(k0.shape[2])
        self.dtype = k0.dtype
        self.device = k0.device
        for i, (k, v) in enumerate(zip(ks, vs)):
            if k.dim() != 3 or tuple(k.shape) != tuple(v.shape):
                raise ValueError(f"sequence {i}: K/V shapes {tuple(k.shape)} / {tuple(v.shape)}")
            if (k.shape[1], k.shape[2]) != (self.n_kv, self.head_dim) or k.dtype != self.dtype:
                raise ValueError(f"sequence {i}: mismatched kv heads / head_dim / dtype")
            _need(k, f"K[{i}]")
            _need(v, f"V[{i}]")
        self.ks, self.vs = list(ks), list(vs)  # keep the storage alive
        self.lens = [int(k.shape[0]) for k in ks]
        self.descs = (L.bml_seq_desc * len(ks))(
            *[L.bml_seq_desc(k.data_ptr(), v.data_ptr(), int(k.shape[0]), 0) for k, v in zip(ks, vs)])

    def __len__(self) -> int:
        return len(self.ks)

    @property
    def kv_bytes(self) -> int:
        es = torch.tensor([], dtype=self.dtype).element_size()
        return 2 * sum(self.lens) * self.n_kv * self.head_dim * es


def _as_batch(ks, vs) -> SeqBatch:
    return ks if isinstance(ks, SeqBatch) else SeqBatch(ks, vs)


# ---------------------------------------------------------------------------
# Decode (gguf_compiler.rs:1008-1050 for a batch of sequences)
# ---------------------------------------------------------------------------
def decode_batched(q: torch.Tensor, ks, vs=None, scale: float = -1.0, out: torch.Tensor | None = None,
                   workspace: Workspace | None = None, stream=None) -> torch.Tensor:
    """Split-K flash decoding.  q [n_seqs, n_heads, d] f32; ks/vs a SeqBatch
    or per-sequence [L_i, n_kv, d] tensors.  Returns out [n_seqs, n_heads, d]
    f32.  scale < 0 selects 1/sqrt(d)."""
    b = _as_batch(ks, vs)
    _need(q, "q", torch.float32, 3)
    n_seqs, n_heads, d = q.shape
    if n_seqs != len(b) or d != b.head_dim:
        raise ValueError(f"q {tuple(q.shape)} does not match the batch ({len(b)} seqs, d={b.head_dim})")
    if out is None:
        out = torch.empty_like(q)
    else:
        _need(out, "out", torch.float32)
    ws = (workspace or default_workspace(q.device.index)).ensure(n_seqs, n_heads, d)
    L.call("bml_attn_decode_batched", b.descs, n_seqs, n_heads, b.n_kv, d, dtype_code(b.dtype),
           float(scale), _ptr(q), _ptr(out), ws.ptr, ws.nbytes, _stream(stream))
    return out


def decode_batched_noalloc(q: torch.Tensor, ks, vs=None, scale: float = -1.0,
                           out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """decode_batched without a workspace, for callers that cannot allocate
    device memory (a pool allocator that owns all of it, or a serving loop
    that must not pay cudaMalloc's device-wide synchronisation).  Scratch is
    the library's fixed 4 MiB device array: larger batches raise
    BmlInvalid, and calls that overlap in time on the GPU race (serialise
    them).  The first call on a device should come before any stream
    capture."""
    b = _as_batch(ks, vs)
    _need(q, "q", torch.float32, 3)
    n_seqs, n_heads, d = q.shape
    if n_seqs != len(b) or d != b.head_dim:
        raise ValueError("q does not match the batch")
    if out is None:
        out = torch.empty_like(q)
    else:
        _need(out, "out", torch.float32)
    L.call("bml_attn_decode_batched_noalloc", b.descs, n_seqs, n_heads, b.n_kv, d, dtype_code(b.dtype),
           float(scale), _ptr(q), _ptr(out), _stream(stream))
    return out


def decode_partial(q: torch.Tensor, ks, vs=None, scale: float = -1.0,
                   workspace: Workspace | None = None, stream=None,
                   m: torch.Tensor | None = None, l: torch.Tensor | None = None,
                   o: torch.Tensor | None = None):
    """KV-split partials (m, l, o) of each sequence's slice: m, l [n_seqs,
    n_heads] (m in log2 units), o [n_seqs, n_heads, d] normalised by l.
    Output tensors may be passed in (e.g. views of one packed buffer)."""
    b = _as_batch(ks, vs)
    _need(q, "q", torch.float32, 3)
    n_seqs, n_heads, d = q.shape
    if n_seqs != len(b) or d != b.head_dim:
        raise ValueError("q does not match the batch")
    m = torch.empty(n_seqs, n_heads, dtype=torch.float32, device=q.device) if m is None else m
    l_ = torch.empty_like(m) if l is None else l
    o = torch.empty_like(q) if o is None else o
    for t, n in ((m, "m"), (l_, "l"), (o, "o")):
        _need(t, n, torch.float32)
    if m.numel() != n_seqs * n_heads or l_.numel() != m.numel() or o.numel() != q.numel():
        raise ValueError("partial output shapes do not match q")
    ws = (workspace or default_workspace(q.device.index)).ensure(n_seqs, n_heads, d)
    L.call("bml_attn_decode_partial", b.descs, n_seqs, n_heads, b.n_kv, d, dtype_code(b.dtype),
           float(scale), _ptr(q), _ptr(m), _ptr(l_), _ptr(o), ws.ptr, ws.nbytes, _stream(stream))
    return m, l_, o


def merge_lse(m: torch.Tensor, l_: torch.Tensor, o: torch.Tensor, out: torch.Tensor | None = None,
              stream=None) -> torch.Tensor:
    """Log-sum-exp merge of stacked partials: m, l [P, ...rows], o [P, ...rows, d]."""
    for t, n in ((m, "m"), (l_, "l"), (o, "o")):
        _need(t, n, torch.float32)
    n_parts = m.shape[0]
    d = o.shape[-1]
    n_rows = m.numel() // n_parts
    if o.numel() != n_parts * n_rows * d or l_.shape != m.shape:
        raise ValueError("partial shapes do not match")
    if out is None:
        out = torch.empty(o.shape[1:], dtype=torch.float32, device=o.device)
    L.call("bml_attn_merge_lse", _ptr(m), _ptr(l_), _ptr(o), n_parts, n_rows, d, _ptr(out),
           _stream(stream))
    return out


def merge_lse_packed(parts: torch.Tensor, n_rows: int, head_dim: int,
                     out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Merge of n_parts packed partials laid out [part][m (n_rows) | l
    (n_rows) | o (n_rows*head_dim)], as an all-gather of one packed buffer
    per rank produces them.  Returns [n_rows, head_dim] (or fills out)."""
    _need(parts, "parts", torch.float32)
    n_parts = parts.shape[0] if parts.dim() > 1 else 1
    if parts.numel() != n_parts * n_rows * (head_dim + 2):
        raise ValueError("packed partial size mismatch")
    if out is None:
        out = torch.empty(n_rows, head_dim, dtype=torch.float32, device=parts.device)
    else:
        _need(out, "out", torch.float32)
    L.call("bml_attn_merge_lse_packed", _ptr(parts), n_parts, n_rows, head_dim, _ptr(out),
           _stream(stream))
    return out


# ---------------------------------------------------------------------------
# Prefill (gguf_compiler.rs:946-958 token loop, all tokens at once)
# ---------------------------------------------------------------------------
def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float = -1.0,
            causal: bool = True, out_dtype: torch.dtype = torch.float32,
            out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Causal prefill on the tcgen05 kernel.  q [n_seqs, S, n_heads, d],
    k/v [n_seqs, S, n_kv, d], all bf16 (or all f16).  Returns
    [n_seqs, S, n_heads, d] in out_dtype (f32 or the input dtype)."""
    _need(q, "q", None, 4)
    _need(k, "k", q.dtype, 4)
    _need(v, "v", q.dtype, 4)
    n_seqs, S, n_heads, d = q.shape
    if k.shape != v.shape or k.shape[0] != n_seqs or k.shape[1] != S or k.shape[3] != d:
        raise ValueError(f"k/v shape {tuple(k.shape)} does not match q {tuple(q.shape)}")
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
    else:
        _need(out, "out", out_dtype)
    L.call("bml_attn_prefill", _ptr(q), _ptr(k), _ptr(v), n_seqs, S, n_heads, int(k.shape[2]), d,
           dtype_code(q.dtype), float(scale), 1 if causal else 0, _ptr(out), dtype_code(out_dtype),
           _stream(stream))
    return out
