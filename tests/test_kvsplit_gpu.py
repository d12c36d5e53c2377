"""KV split of one long sequence over two GPUs with the exchange inside the
decode kernel (bml_attn_decode_kvsplit through KVSplitDecode(fused=True)).

Two processes, one GPU each; a gloo group carries only the exchange-buffer
handles.  Each rank decodes its contiguous half of a seeded bf16 cache and
swaps per-(q head, 32 dims) partials with the other over peer memory; both
must then hold the oracle's single-pass attention over the whole sequence
(decode tolerance 1e-4), bit-identical between the ranks, on three calls in
a row (the exchange slots alternate between two parities) and on three
replays of a CUDA graph holding two calls (the exchange's epoch is kept on
the device).  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from bml_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q, k, v, ret):
    import datetime

    import torch.distributed as dist

    import bml_b200
    from bml_b200 import sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev = torch.device("cuda", rank)
        lo, hi = sharding.kv_split_ranges(k.shape[0], world)[rank]
        kd = torch.from_numpy(np.ascontiguousarray(k[lo:hi]).view(np.int16)).to(dev).view(torch.bfloat16)
        vd = torch.from_numpy(np.ascontiguousarray(v[lo:hi]).view(np.int16)).to(dev).view(torch.bfloat16)
        batch = bml_b200.SeqBatch([kd], [vd])
        qd = torch.from_numpy(q[None]).to(dev)
        ws = bml_b200.Workspace(dev).ensure(1, q.shape[0], q.shape[1])
        step = sharding.KVSplitDecode(dist, world, q.shape[0], q.shape[1], dev, fused=True)
        outs = []
        for _ in range(3):
            out = step(qd, batch, ws, total_len=k.shape[0])
            torch.cuda.synchronize(dev)
            outs.append(out.cpu().numpy().copy())
        ws.check()
        # two calls captured in a CUDA graph and replayed: the exchange epoch
        # lives on the device, so every replay takes fresh epochs
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(cap):
            with torch.cuda.graph(g, stream=cap):
                o1 = step(qd, batch, ws, total_len=k.shape[0])
                o2 = step(qd, batch, ws, total_len=k.shape[0])
        torch.cuda.current_stream(dev).wait_stream(cap)
        for _ in range(3):
            o1.zero_()
            o2.zero_()
            g.replay()
            torch.cuda.synchronize(dev)
            outs.append(o1.cpu().numpy().copy())
            outs.append(o2.cpu().numpy().copy())
        ws.check()
        del g
        step.close()
        ret[rank] = outs
    finally:
        dist.destroy_process_group()


def test_kv_split_over_two_gpus_matches_oracle(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    q, k, v = W.longctx_decode(length=20000)
    want = oracle.attn_decode_batched(q[None], [k], [v], dtype=oracle.BF16)[0]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        ret = mgr.dict()
        port = _port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, q, k, v, ret)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            if p.is_alive():
                p.kill()
                pytest.fail("a rank did not finish within 300 s")
            assert p.exitcode == 0
        outs = [ret[r] for r in range(2)]
    for rank_outs in outs:
        for o in rank_outs:
            assert np.abs(o[0] - want).max() < TOL
    for a, b in zip(outs[0], outs[1]):
        np.testing.assert_array_equal(a, b)
