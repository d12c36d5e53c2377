"""Multi-rank host logic on CPU: world-size-2 gloo process groups.

The GPU exchange (KVSplitDecode) runs here with CPU restatements of the
partial and merge kernels plugged in, so the split ranges, the packed
all-gather layout and the rank-order merge are exercised end to end and
compared with the oracle's single-pass attention."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from bml_b200 import sharding


def test_lpt_partition_balances_and_covers():
    lens = [int(x) for x in np.random.default_rng(2).integers(128, 4097, 64)]
    for n in (1, 2, 4, 8):
        bins = sharding.lpt_partition(lens, n)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(64))
        loads = [sum(lens[i] for i in b) for b in bins]
        assert max(loads) - min(loads) <= max(lens)
    assert sharding.lpt_partition([5, 5, 5], 2) == [[0, 2], [1]]


def test_kv_split_ranges():
    for L in (1, 7, 131072, 131073):
        for n in (1, 2, 3, 8):
            r = sharding.kv_split_ranges(L, n)
            assert r[0][0] == 0 and r[-1][1] == L
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            sizes = [b - a for a, b in r]
            assert max(sizes) - min(sizes) <= 1


def np_partial(q, k, v, scale):
    """(m, l, o) of one slice in the kernels' convention: m is the max of
    scale*log2(e)*q.k, l = sum 2^(s-m), o = sum 2^(s-m) v / l."""
    n_heads, d = q.shape
    g = n_heads // k.shape[1]
    c = scale * np.log2(np.e)
    m = np.empty(n_heads)
    l_ = np.empty(n_heads)
    o = np.empty((n_heads, d))
    for h in range(n_heads):
        s = (k[:, h // g, :].astype(np.float64) @ q[h].astype(np.float64)) * c
        m[h] = s.max()
        w = np.exp2(s - m[h])
        l_[h] = w.sum()
        o[h] = (w[:, None] * v[:, h // g, :]).sum(0) / l_[h]
    return m, l_, o


def np_merge_packed(parts, n_rows, d, out):
    P = parts.shape[0]
    m = parts[:, :n_rows].double()
    l_ = parts[:, n_rows:2 * n_rows].double()
    o = parts[:, 2 * n_rows:].double().view(P, n_rows, d)
    M = m.max(0).values
    f = torch.exp2(m - M) * l_
    res = (o * f[..., None]).sum(0) / f.sum(0)[..., None]
    out.copy_(res.view(out.shape).float())


def _worker(rank, world, port, q, k, v, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = sharding.kv_split_ranges(k.shape[0], world)[rank]
        scale = 1.0 / np.sqrt(q.shape[-1])

        def partial_fn(qq, batch, m, l_, o):
            mm, ll, oo = np_partial(q[0], batch[0], batch[1], scale)
            m.copy_(torch.from_numpy(mm).view_as(m))
            l_.copy_(torch.from_numpy(ll).view_as(l_))
            o.copy_(torch.from_numpy(oo).view_as(o))

        step = sharding.KVSplitDecode(dist, world, q.shape[1], q.shape[2], torch.device("cpu"),
                                      partial_fn=partial_fn, merge_fn=np_merge_packed)
        out = step(torch.from_numpy(q), (k[lo:hi], v[lo:hi]))
        ret[rank] = out.numpy().copy()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_kv_split_exchange_matches_oracle(world):
    rng = np.random.default_rng(4)
    L, n_kv, d, H = 1000, 2, 32, 8
    q = rng.standard_normal((1, H, d), dtype=np.float32)
    k = rng.standard_normal((L, n_kv, d), dtype=np.float32)
    v = rng.standard_normal((L, n_kv, d), dtype=np.float32)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        ret = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, q, k, v, ret)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        outs = [ret[r] for r in range(world)]
    want = oracle.attn_decode(q[0], k, v)
    for o in outs:
        np.testing.assert_allclose(o[0], want, atol=1e-5)
    # every rank merged the same gathered partials in rank order
    np.testing.assert_array_equal(outs[0], outs[1])


def _lpt_worker(rank, world, port, lens, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = sharding.lpt_partition(lens, world)[rank]
        t = torch.tensor([sum(lens[i] for i in mine)], dtype=torch.int64)
        dist.all_reduce(t)
        ret[rank] = (mine, int(t.item()))
    finally:
        dist.destroy_process_group()


def test_batched_sharding_is_consistent_across_ranks():
    """Every rank derives the same plan with no exchange; together the
    shards cover each sequence exactly once."""
    lens = [int(x) for x in np.random.default_rng(2).integers(128, 4097, 64)]
    ctx = mp.get_context("spawn")
    port = _free_port()
    with ctx.Manager() as mgr:
        ret = mgr.dict()
        procs = [ctx.Process(target=_lpt_worker, args=(r, 2, port, lens, ret)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        a, b = ret[0], ret[1]
    assert sorted(a[0] + b[0]) == list(range(64))
    assert a[1] == b[1] == sum(lens)


# ---------------------------------------------------------------------------
# Failure detection on the host (no GPU involved): a rank that leaves between
# steps, and ranks that disagree on the split.
# ---------------------------------------------------------------------------
def _failure_worker(rank, world, port, mode, q, k, v, ret):
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    total = k.shape[0] + (rank if mode == "mismatch" else 0)  # a rank with a different length
    lo, hi = sharding.kv_split_ranges(k.shape[0], world)[rank]
    scale = 1.0 / np.sqrt(q.shape[-1])

    def partial_fn(qq, batch, m, l_, o):
        mm, ll, oo = np_partial(q[0], batch[0], batch[1], scale)
        m.copy_(torch.from_numpy(mm).view_as(m))
        l_.copy_(torch.from_numpy(ll).view_as(l_))
        o.copy_(torch.from_numpy(oo).view_as(o))

    step = sharding.KVSplitDecode(dist, world, q.shape[1], q.shape[2], torch.device("cpu"),
                                  partial_fn=partial_fn, merge_fn=np_merge_packed, health_timeout_s=3.0)
    try:
        if mode == "mismatch":
            try:
                step(torch.from_numpy(q), (k[lo:hi], v[lo:hi]), total_len=total)
                ret[rank] = ("no error",)
            except sharding.SplitMismatch as e:
                ret[rank] = ("SplitMismatch", str(e))
            return
        # mode "leave": one good step with a health check on both ranks
        step(torch.from_numpy(q), (k[lo:hi], v[lo:hi]), total_len=total)
        step.health_check()
        if rank == 1:
            ret[1] = ("left",)
            os._exit(0)  # leaves between steps: nothing of it is in flight
        t0 = time.monotonic()
        try:
            step.health_check()
            hc = ("no error", time.monotonic() - t0)
        except sharding.RankFailure as e:
            hc = ("RankFailure", time.monotonic() - t0, e.rank)
        t0 = time.monotonic()
        try:
            step(torch.from_numpy(q), (k[lo:hi], v[lo:hi]), total_len=total)
            st = ("no error", time.monotonic() - t0)
        except sharding.RankFailure as e:
            st = ("RankFailure", time.monotonic() - t0)
        ret[0] = (hc, st)
    finally:
        if mode == "leave":
            os._exit(0)  # the group has lost a rank: leave without a collective teardown
        dist.destroy_process_group()


def _run_failure(mode):
    rng = np.random.default_rng(5)
    L, n_kv, d, H = 300, 2, 32, 8
    q = rng.standard_normal((1, H, d), dtype=np.float32)
    k = rng.standard_normal((L, n_kv, d), dtype=np.float32)
    v = rng.standard_normal((L, n_kv, d), dtype=np.float32)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        ret = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_failure_worker, args=(r, 2, port, mode, q, k, v, ret)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(90)
            if p.is_alive():
                p.kill()
                pytest.fail(f"{mode}: a rank did not finish within 90 s")
        return dict(ret)


def test_rank_that_leaves_is_detected_within_the_timeout():
    """Rank 1 leaves between steps.  Rank 0's health check names it within
    its 3 s limit, and the next step's all-gather fails with RankFailure
    within the process group's 10 s timeout instead of waiting forever."""
    ret = _run_failure("leave")
    assert ret[1] == ("left",)
    hc, st = ret[0]
    assert hc[0] == "RankFailure" and hc[2] == 1 and hc[1] < 6.0, hc
    assert st[0] == "RankFailure" and st[1] < 30.0, st


def test_mismatched_split_is_refused_on_every_rank():
    """Ranks that disagree on the total KV length stop at the first call's
    plan check with SplitMismatch, before any partial is exchanged."""
    ret = _run_failure("mismatch")
    assert ret[0][0] == "SplitMismatch" and ret[1][0] == "SplitMismatch", ret
