"""Multi-GPU partitioning of the decode path (one process per GPU).

Two ways the path shards, neither of which exists in the reference (its
attention runs in one thread of one process):

* Batched decode: sequences are independent, so they are dealt to GPUs by
  longest-processing-time first (work ~ cached length) and each GPU runs
  its own batch.  No collective.
* Long-context decode: one sequence's KV length is cut into contiguous
  ranges, one per GPU.  By default (fused) each GPU decodes its range and,
  inside the same kernel, exchanges its per-(q head, 32 dims) partials with
  every other GPU over peer memory and merges them in rank order
  (bml_attn_decode_kvsplit).  The other form computes each range's (m, l, o)
  partial (bml_attn_decode_partial), all-gathers the packed partials over
  NCCL and merges them (bml_attn_merge_lse_packed).  Either way all ranks
  hold bit-identical outputs.
"""
from __future__ import annotations

import time
from typing import Callable, Sequence


class RankFailure(RuntimeError):
    """A peer rank of a KV-split decode stopped answering: it missed a
    health check within the timeout, or a collective with it failed.  The
    reference's counterpart is its worker HealthCheck message
    (crates/runtime/src/net.rs) and the CLI's exit on a TCP error."""

    def __init__(self, msg: str, rank: int | None = None):
        super().__init__(msg)
        self.rank = rank


class SplitMismatch(RuntimeError):
    """The ranks of a KV-split decode disagree on the split (world size,
    head shape or total KV length), so their partials would not merge."""


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
    pass restatements instead, so the exchange logic runs under gloo.

    Failure detection (all on the host; nothing waits on the GPU):
    * the first call checks that every rank has the same plan (world size,
      q heads, head_dim, total KV length); SplitMismatch otherwise;
    * health_check(), called by every rank between steps (the same number of
      times), publishes this rank's check count in the process group's
      key-value store and waits (bounded) until every peer has published
      the same count; RankFailure names a peer that did not answer in time;
    * a collective that fails (a peer left, or the process group's own
      timeout ran out) is raised as RankFailure.
    """

    def __init__(self, pg, world: int, n_heads: int, head_dim: int, device,
                 partial_fn: Callable | None = None, merge_fn: Callable | None = None,
                 store=None, health_timeout_s: float = 10.0, fused: bool = True):
        import torch
        self.pg, self.world, self.n_heads, self.d = pg, world, n_heads, head_dim
        self.device = device
        self.partial_fn = partial_fn
        self.merge_fn = merge_fn
        self.store = store
        self.health_timeout_s = health_timeout_s
        self.rank = pg.get_rank() if pg is not None and world > 1 else 0
        self.steps = 0
        self._checks = 0
        self._plan_checked = world == 1
        self._packed = None
        self._gathered = None
        self._torch = torch
        # the exchange inside the decode kernel: CUDA library, several ranks
        self.fused = fused and world > 1 and partial_fn is None and merge_fn is None
        self._peer = None

    def _open_peer(self):
        """Creates this rank's exchange buffer and maps every rank's
        (handles all-gathered through the process group)."""
        import ctypes as C

        from . import _lib as L
        h = C.c_void_p()
        dev = self._torch.device(self.device).index or 0
        L.call("bml_kvsplit_create", dev, self.rank, self.world, self.n_heads, self.d, C.byref(h))
        buf = (C.c_char * L.BML_KVSPLIT_HANDLE_BYTES)()
        try:
            L.call("bml_kvsplit_handle", h, buf, L.BML_KVSPLIT_HANDLE_BYTES)
            mine = bytes(buf)
            every = [None] * self.world
            self._collective("exchange-handle all-gather", self.pg.all_gather_object, every, mine)
            blob = b"".join(every)
            L.call("bml_kvsplit_open", h, blob, len(blob))
        except Exception:
            L.call("bml_kvsplit_destroy", h)
            raise
        self._peer = h

    def close(self) -> None:
        """Unmaps the peers' exchange buffers and frees this rank's."""
        if self._peer is not None:
            from . import _lib as L
            L.call("bml_kvsplit_destroy", self._peer)
            self._peer = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _buffers(self, n_rows: int):
        torch = self._torch
        size = packed_size(n_rows, self.d)
        if self._packed is None or self._packed.numel() != size:
            self._packed = torch.empty(size, dtype=torch.float32, device=self.device)
            self._gathered = torch.empty(self.world * size, dtype=torch.float32, device=self.device)
        return self._packed, self._gathered

    def _collective(self, what: str, fn, *args):
        try:
            return fn(*args)
        except (RuntimeError, ValueError, OSError) as e:  # gloo / NCCL errors, timeouts
            raise RankFailure(f"rank {self.rank}: {what} failed ({type(e).__name__}: {e})") from e

    def check_plan(self, total_len: int) -> None:
        """All ranks agree on (world, n_heads, head_dim, total_len)."""
        torch = self._torch
        mine = torch.tensor([self.world, self.n_heads, self.d, int(total_len)], dtype=torch.int64,
                            device=self.device)
        every = torch.empty(self.world * 4, dtype=torch.int64, device=self.device)
        self._collective("plan all-gather", self.pg.all_gather_into_tensor, every, mine)
        rows = every.view(self.world, 4).cpu().tolist()
        if any(r != rows[0] for r in rows):
            raise SplitMismatch(f"rank {self.rank}: split plans differ across ranks "
                                f"(world, n_heads, head_dim, total_len): {rows}")
        self._plan_checked = True

    def _store(self):
        if self.store is not None:
            return self.store
        from torch.distributed import distributed_c10d as c10d
        return c10d._get_default_store()

    def health_check(self, timeout_s: float | None = None) -> None:
        """Publishes this rank's health-check count and waits until every
        peer has published at least the same count (each call needs a fresh
        answer from every peer); RankFailure names the first peer still
        missing when the timeout runs out."""
        if self.world == 1:
            return
        self._checks += 1
        store = self._store()
        deadline = time.monotonic() + (self.health_timeout_s if timeout_s is None else timeout_s)
        pending = [r for r in range(self.world) if r != self.rank]
        try:
            store.set(f"bml/kvsplit/{self.rank}", str(self._checks))
        except (RuntimeError, OSError) as e:  # the store's host rank is gone
            raise RankFailure(f"rank {self.rank}: key-value store unreachable ({e})", rank=0) from e
        while pending:
            still = []
            for r in pending:
                key = f"bml/kvsplit/{r}"
                try:
                    seen = store.check([key]) and int(store.get(key).decode()) >= self._checks
                except (RuntimeError, OSError) as e:
                    raise RankFailure(f"rank {self.rank}: key-value store unreachable ({e})", rank=0) from e
                if not seen:
                    still.append(r)
            pending = still
            if pending and time.monotonic() > deadline:
                raise RankFailure(f"rank {self.rank}: rank {pending[0]} missed health check {self._checks} "
                                  f"(after {self.steps} steps)", rank=pending[0])
            if pending:
                time.sleep(0.01)

    def _fused_step(self, q, batch, workspace, out):
        import ctypes as C

        from . import _lib as L
        from .attention import _need, _ptr, _stream, default_workspace, dtype_code
        torch = self._torch
        if self._peer is None:
            self._open_peer()
        _need(q, "q", torch.float32, 3)
        if q.shape[0] != 1 or len(batch) != 1:
            raise ValueError("the fused KV split takes one sequence")
        if out is None:
            out = torch.empty_like(q)
        ws = (workspace or default_workspace(q.device.index)).ensure(1, self.n_heads, self.d)
        L.call("bml_attn_decode_kvsplit", self._peer, batch.descs, self.n_heads, batch.n_kv, self.d,
               dtype_code(batch.dtype), C.c_float(-1.0), _ptr(q), _ptr(out), ws.ptr, ws.nbytes, _stream(None))
        self.steps += 1
        return out

    def __call__(self, q, batch, workspace=None, out=None, total_len: int | None = None):
        torch = self._torch
        if self.world == 1 and self.partial_fn is None and self.merge_fn is None:
            # one rank holds the whole sequence: the plain decode, whose
            # in-kernel merge already yields the final output
            from .attention import decode_batched
            return decode_batched(q, batch, out=out, workspace=workspace)
        if not self._plan_checked:
            self.check_plan(total_len if total_len is not None else -1)
        if self.fused:
            return self._fused_step(q, batch, workspace, out)
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
            self._collective("partials all-gather", self.pg.all_gather_into_tensor, gathered, packed)
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
        self.steps += 1
        return out
