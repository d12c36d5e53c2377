"""Multi-GPU partitioning of the decode path (one process per GPU).

Two ways the path shards, neither of which exists in the reference (its
attention runs in one thread of one process):

* Batched decode: sequences are independent, so they are dealt to GPUs by
  longest-processing-time first (work ~ cached length) and each GPU runs
  its own batch.  No collective.
* Long-context decode: one sequence's KV length is cut into contiguous
  ranges, one per GPU.  Each GPU computes the (m, l, o) partial of its
  range (bml_attn_decode_partial), the packed partials are all-gathered
  over NCCL (NVLink), and every GPU merges them in rank order
  (bml_attn_merge_lse_packed), so all ranks hold bit-identical outputs.
"""
from __future__ import annotations

from typing import Callable, Sequence


def lpt_partition(lengths: Sequence[int], n_parts: int) -> list[list[int]]:
    """Deals sequence indices to n_parts bins, longest first, each to the
    currently lightest bin (lowest bin index on ties).  Indices inside a bin
    are returned in ascending order."""
    if n_parts < 1:
        raise ValueError("n_parts must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    loads = [0] * n_parts
    bins: list[list[int]] = [[] for _ in range(n_parts)]
    for i in order:
        b = min(range(n_parts), key=lambda j: (loads[j], j))
        bins[b].append(i)
        loads[b] += int(lengths[i])
    return [sorted(b) for b in bins]


def kv_split_ranges(length: int, n_parts: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) ranges covering [0, length), sizes differing by at
    most one position; a range may be empty only if length < n_parts."""
    if n_parts < 1 or length < 0:
        raise ValueError("bad split")
    base, extra = divmod(length, n_parts)
    out, lo = [], 0
    for r in range(n_parts):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def packed_size(n_rows: int, head_dim: int) -> int:
    """Floats in one packed partial: m [n_rows] | l [n_rows] | o [n_rows, d]."""
    return n_rows * (head_dim + 2)


class KVSplitDecode:
    """One decode step of a sequence whose KV is split across the ranks of a
    process group.  Every rank calls it with the same q and its own slice.

    `pg` is the torch.distributed module (or None for one rank).  The
    partial and merge backends default to the CUDA library; tests on CPU
    pass restatements instead, so the exchange logic runs under gloo."""

    def __init__(self, pg, world: int, n_heads: int, head_dim: int, device,
                 partial_fn: Callable | None = None, merge_fn: Callable | None = None):
        import torch
        self.pg, self.world, self.n_heads, self.d = pg, world, n_heads, head_dim
        self.device = device
        self.partial_fn = partial_fn
        self.merge_fn = merge_fn
        self._packed = None
        self._gathered = None
        self._torch = torch

    def _buffers(self, n_rows: int):
        torch = self._torch
        size = packed_size(n_rows, self.d)
        if self._packed is None or self._packed.numel() != size:
            self._packed = torch.empty(size, dtype=torch.float32, device=self.device)
            self._gathered = torch.empty(self.world * size, dtype=torch.float32, device=self.device)
        return self._packed, self._gathered

    def __call__(self, q, batch, workspace=None, out=None):
        torch = self._torch
        if self.world == 1 and self.partial_fn is None and self.merge_fn is None:
            # one rank holds the whole sequence: the plain decode, whose slot
            # merge already yields the final output (no partial, no merge)
            from .attention import decode_batched
            return decode_batched(q, batch, out=out, workspace=workspace)
        n_seqs = q.shape[0]
        n_rows = n_seqs * self.n_heads
        packed, gathered = self._buffers(n_rows)
        m = packed[:n_rows].view(n_seqs, self.n_heads)
        l_ = packed[n_rows:2 * n_rows].view(n_seqs, self.n_heads)
        o = packed[2 * n_rows:].view(n_seqs, self.n_heads, self.d)
        if self.partial_fn is None:
            from .attention import decode_partial
            decode_partial(q, batch, workspace=workspace, m=m, l=l_, o=o)
        else:
            self.partial_fn(q, batch, m, l_, o)
        if self.world > 1:
            self.pg.all_gather_into_tensor(gathered, packed)
            parts = gathered.view(self.world, -1)
        else:
            parts = packed.view(1, -1)
        if out is None:
            out = torch.empty(n_seqs, self.n_heads, self.d, dtype=torch.float32, device=self.device)
        if self.merge_fn is None:
            from .attention import merge_lse_packed
            merge_lse_packed(parts, n_rows, self.d, out=out)
        else:
            self.merge_fn(parts, n_rows, self.d, out)
        return out
