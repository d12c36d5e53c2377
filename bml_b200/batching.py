"""Continuous batching of decode steps over per-request KV caches.

The reference serves one request at a time: its HTTP server holds the
InferenceCompiler behind a global Mutex and runs a whole generation per
request (crates/api/src/main.rs:33-36, :266-354), rejecting requests beyond
MAX_PENDING_REQUESTS = 64 (:31, :181-194).  DecodeBatcher is the batched
caller: requests join and leave between steps, and one step of every active
request's layer is two launches -- the batched K/V append (with RoPE, as
gguf_compiler.rs:984-1006 and :1290-1317 do per request) and the batched
split-K decode over every request's cache (gguf_compiler.rs:1008-1050 per
request).

Storage: each request owns K and V tensors [n_layers, capacity, n_kv, d] in
the cache dtype on one device; the descriptor arrays the C entry points take
are kept per layer and rebuilt only when the set of requests changes.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from .attention import Workspace, _need, _ptr, _stream, dtype_code

MAX_PENDING_REQUESTS = 64  # crates/api/src/main.rs:31


class AtCapacity(RuntimeError):
    """A request beyond max_requests (the reference answers 429,
    crates/api/src/main.rs:183-194)."""


def _len_view(arr, n: int) -> np.ndarray:
    """Writable uint32 view of the len fields of a bml_seq_desc array (numpy
    cannot read ctypes' structure format, so view the words)."""
    words = C.sizeof(L.bml_seq_desc) // 4
    flat = (C.c_uint32 * (words * n)).from_address(C.addressof(arr))
    return np.ctypeslib.as_array(flat).reshape(n, words)[:, L.bml_seq_desc.len.offset // 4]


@dataclass
class _Request:
    k: torch.Tensor  # [n_layers, capacity, n_kv, d]
    v: torch.Tensor
    length: int      # positions committed (all layers)


class DecodeBatcher:
    """One decode step at a time for a changing set of requests.

    Per token: for every layer, ``step(layer, q, k_new, v_new)`` stores each
    active request's new K/V row at its position (its current length) and
    returns attention over positions [0, length] for all of them; after the
    last layer, ``advance()`` commits the position (forward_cached runs
    forward_layer_cached for every layer at position pos, then advances the
    cache, gguf_compiler.rs:946-958).  Rows of q, k_new, v_new and of the result
    follow ``active`` (the order of ``add``, with removed requests taken
    out)."""

    def __init__(self, n_layers: int, n_heads: int, n_kv_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.bfloat16, device=None, rope: bool = True,
                 max_requests: int = MAX_PENDING_REQUESTS, scale: float = -1.0):
        if n_heads % n_kv_heads:
            raise ValueError("n_heads must be a multiple of n_kv_heads")
        if rope and head_dim % 2:
            raise ValueError("RoPE needs an even head_dim")
        dtype_code(dtype)
        self.n_layers, self.n_heads, self.n_kv, self.head_dim = n_layers, n_heads, n_kv_heads, head_dim
        self.dtype, self.rope, self.scale = dtype, rope, float(scale)
        self.max_requests = max_requests
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   torch.device(device).index or 0)
        self.workspace = Workspace(self.device)
        self._reqs: dict = {}
        self._order: list = []
        self._descs = None   # per-layer ctypes arrays of bml_seq_desc
        self._lens = None    # per-layer numpy views of their len fields
        self._host_lens = np.zeros(0, np.uint32)
        self._caps = np.zeros(0, np.uint32)
        self._full = False
        self._ws_n = -1

    # -- membership -------------------------------------------------------
    @property
    def active(self) -> list:
        return list(self._order)

    def __len__(self) -> int:
        return len(self._order)

    def length(self, rid) -> int:
        return self._reqs[rid].length

    def add(self, rid, capacity: int, k_prompt: torch.Tensor | None = None,
            v_prompt: torch.Tensor | None = None) -> None:
        """Admits request `rid` with room for `capacity` positions.  The
        prompt's K/V ([n_layers, P, n_kv, d], e.g. from a prefill) become
        its first P positions.  Raises AtCapacity beyond max_requests."""
        if rid in self._reqs:
            raise KeyError(f"request {rid!r} is already active")
        if len(self._order) >= self.max_requests:
            raise AtCapacity(f"{len(self._order)} requests active (max {self.max_requests})")
        shape = (self.n_layers, capacity, self.n_kv, self.head_dim)
        # uninitialised: a row is written (prompt copy or append) before any
        # kernel reads it, and no kernel reads past a request's length
        k = torch.empty(shape, dtype=self.dtype, device=self.device)
        v = torch.empty(shape, dtype=self.dtype, device=self.device)
        n = 0
        if k_prompt is not None:
            if v_prompt is None or k_prompt.shape != v_prompt.shape:
                raise ValueError("k_prompt and v_prompt must match")
            n = int(k_prompt.shape[1])
            if (k_prompt.dim() != 4 or k_prompt.shape[0] != self.n_layers or n > capacity
                    or tuple(k_prompt.shape[2:]) != (self.n_kv, self.head_dim)):
                raise ValueError(f"prompt K/V {tuple(k_prompt.shape)} does not fit {shape}")
            k[:, :n].copy_(k_prompt)
            v[:, :n].copy_(v_prompt)
        self._reqs[rid] = _Request(k, v, n)
        self._order.append(rid)
        self._descs = None

    def remove(self, rid) -> None:
        """Drops request `rid` and frees its cache (stream-ordered)."""
        del self._reqs[rid]
        self._order.remove(rid)
        self._descs = None

    def _build(self) -> None:
        n = len(self._order)
        row = self.n_kv * self.head_dim * torch.tensor([], dtype=self.dtype).element_size()
        self._descs, self._lens = [], []
        for layer in range(self.n_layers):
            arr = (L.bml_seq_desc * max(n, 1))()
            for i, rid in enumerate(self._order):
                r = self._reqs[rid]
                off = layer * r.k.shape[1] * row
                arr[i] = L.bml_seq_desc(r.k.data_ptr() + off, r.v.data_ptr() + off, r.length, 0)
            self._descs.append(arr)
            self._lens.append(_len_view(arr, max(n, 1))[:n])
        self._host_lens = np.array([self._reqs[r].length for r in self._order], np.uint32)
        self._caps = np.array([self._reqs[r].k.shape[1] for r in self._order], np.uint32)
        self._full = bool((self._host_lens >= self._caps).any())

    # -- one layer of one token -------------------------------------------
    def step(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
             out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """q [n_active, n_heads, d] f32 (rotated in place when rope=True);
        k_new, v_new [n_active, n_kv, d] (f32 with RoPE, else f32/f16/bf16).
        Returns the attention output [n_active, n_heads, d] f32."""
        n = len(self._order)
        if n == 0:
            raise ValueError("no active requests")
        if not 0 <= layer < self.n_layers:
            raise ValueError(f"layer {layer} out of range")
        if self._descs is None:
            self._build()
        _need(q, "q", torch.float32, 3)
        _need(k_new, "k_new", ndim=3)
        _need(v_new, "v_new", k_new.dtype, 3)
        if tuple(q.shape) != (n, self.n_heads, self.head_dim) or \
                tuple(k_new.shape) != (n, self.n_kv, self.head_dim) or k_new.shape != v_new.shape:
            raise ValueError(f"q {tuple(q.shape)} / k_new {tuple(k_new.shape)} do not match "
                             f"{n} requests x ({self.n_heads}|{self.n_kv}, {self.head_dim})")
        if self._full:
            rid = self._order[int(np.nonzero(self._host_lens >= self._caps)[0][0])]
            raise ValueError(f"request {rid!r} is full ({self._reqs[rid].length} positions)")
        lens = self._lens[layer]
        descs = self._descs[layer]
        st = _stream(stream)
        lens[:] = self._host_lens              # append row = current length
        if self.rope:
            if k_new.dtype != torch.float32:
                raise TypeError("RoPE append takes f32 k_new / v_new")
            L.call("bml_kv_append_rope_batched", descs, n, self.n_heads, self.n_kv, self.head_dim,
                   dtype_code(self.dtype), _ptr(q), _ptr(k_new), _ptr(v_new), st)
        else:
            L.call("bml_kv_append_batched", descs, n, self.n_kv, self.head_dim, dtype_code(self.dtype),
                   _ptr(k_new), _ptr(v_new), dtype_code(k_new.dtype), st)
        lens[:] = self._host_lens + 1          # attend over [0, length]
        if out is None:
            out = torch.empty_like(q)
        else:
            _need(out, "out", torch.float32, 3)
        if self._ws_n != n:
            self.workspace.ensure(n, self.n_heads, self.head_dim)
            self._ws_n = n
        ws = self.workspace
        L.call("bml_attn_decode_batched", descs, n, self.n_heads, self.n_kv, self.head_dim,
               dtype_code(self.dtype), self.scale, _ptr(q), _ptr(out), ws.ptr, ws.nbytes, st)
        return out

    def advance(self) -> None:
        """Commits the token stored by the last step of every layer."""
        for rid in self._order:
            self._reqs[rid].length += 1
        self._host_lens = self._host_lens + 1
        self._full = bool((self._host_lens >= self._caps).any())

    def cache(self, rid, layer: int):
        """(K, V) views [length, n_kv, d] of request `rid`'s layer."""
        r = self._reqs[rid]
        return r.k[layer, :r.length], r.v[layer, :r.length]
