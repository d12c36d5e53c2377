#!/usr/bin/env python
"""Benchmark of the GQA attention hot path on B200.

One step = one pass of the hot path over one batch of synthetic input that
is already resident in HBM.  Workloads (--workload):

  llama3_decode (default)  Llama-3-8B-shaped decode: 32 sequences x 8192
                           cached positions per GPU, 32 q / 8 kv heads,
                           d=128, bf16 KV, f32 q/out.  Metric: HBM GB/s of
                           algorithmic bytes (K+V read once, q read, out
                           written).  N GPUs = N independent batches
                           ("weak": sequences shard with no collective).
  batched_tinyllama        64 ragged sequences (U[128,4096], f16 KV,
                           TinyLlama heads) sharded over the GPUs by
                           longest-processing-time ("strong").
  longctx                  one 131072-position sequence (Llama-3 heads,
                           bf16) split along its KV length over the GPUs;
                           per-GPU (m, l, o) partials all-gathered over
                           NCCL and merged ("strong"); one GPU runs the
                           plain decode of the whole sequence.
  llama3_prefill           causal prefill 4 x 8192, 32/8 heads, d=128,
                           bf16 operands (TFLOP/s of 4*d*H*causal pairs);
                           the 32 (sequence, kv-head group) units are dealt
                           over the GPUs ("strong", no collective).
  gemv                     the projections of Llama-3-8B layers (q, k, v, o
                           4096x4096/1024; gate, up 4096x14336; down
                           14336x4096) as Q4_0 tensors read in place by
                           matmul_f64 (x . W, the reference's indexing); a
                           step is one layer's 7 projections, cycling over 4
                           layers of distinct weights (490 MB > L2).  Metric:
                           HBM GB/s of stored weight bytes + x/y ("weak").
  gguf_load                a GGUF file of 8 Llama-3-8B layers' projections
                           (Q4_0, 0.98 GB) uploaded to the device by
                           bml_gguf_upload (memory-mapped file, pinned
                           staging, 8 host threads).  Metric: GB/s of tensor
                           bytes into device memory (page cache warm).
  serving                  continuous batching (DecodeBatcher): 32 requests
                           of Llama-3-8B shape (32 layers, 32/8 heads,
                           d=128, bf16 KV), prompts U[1024,4096]; a step is
                           one token of every request through all 32 layers
                           (RoPE append + decode per layer); every 8 steps
                           the longest request leaves and a new one joins.
                           Metric: HBM GB/s of algorithmic bytes ("weak").

The default decode line also carries, measured in the same run at the same
GPU count, a "prefill" object (llama3_prefill split by (sequence x kv-head
group), strong), a "batched_tinyllama" object (strong) and a "longctx"
object (strong).

--impl reference times the CPU restatement of the reference's attention
(oracle/, the reference is Rust and cannot be built here) on the host cores
over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# nominal B200 figures, reported beside the measured-peak fractions
SPEC_PEAKS = {"hbm_gbs": 8000.0, "bf16_tflops": 2250.0}

DECODE_METRIC = "GQA decode-attn HBM GB/s (% peak) + prefill TFLOP/s"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def decode_kernel_name(kv_dtype, head_dim: int, n_kv: int, group: int) -> str:
    """Kernel that bml_attn_decode_batched launches for a shape: the
    bulk-copy warp-MMA kernel (dynamic schedule) for 16-bit caches with
    512..2048-byte position rows, the CUDA-core kernel otherwise (mirrors
    decode_select in bml_b200/csrc/decode.cu)."""
    import torch
    row = n_kv * head_dim * 2
    mma = (kv_dtype in (torch.float16, torch.bfloat16) and head_dim in (64, 128) and group in (1, 2, 4, 8)
           and n_kv in (1, 2, 4, 8) and 512 <= row <= 2048)
    return "decode_bulk_kernel" if mma else "decode_kernel"


def profile_traffic(name: str):
    """traffic_bytes_per_launch recorded from an ncu capture in profiles/."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except (OSError, ValueError, IndexError):
        pass
    return None


def host_threads() -> int:
    """Every host core this process may run on (torchrun sets
    OMP_NUM_THREADS=1, which must not throttle the CPU baseline)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU during the timed
    region.  NVML is polled from a thread (about every millisecond), so even
    a few-millisecond timed loop gets samples; without NVML, nvidia-smi's
    200 ms sampling is the fallback.  Read-only: nothing is set."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, torch_index: int):
        import threading
        self.proc = None
        self.t0 = self.t1 = None
        self.samples = []  # (sm_mhz, max_mhz, power_w, reason bits)
        self.stop_ev = threading.Event()
        self.thread = None
        try:
            import torch
            props = torch.cuda.get_device_properties(torch_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        except Exception as e:
            log("clock sampler unavailable:", e)
            return
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def poll():
                while not self.stop_ev.is_set():
                    if self.t0 is not None and self.t1 is None:
                        try:
                            self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)), smax,
                                                 pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                                 int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))))
                        except pynvml.NVMLError:
                            pass
                    time.sleep(0.0005)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception as e:  # no NVML: nvidia-smi
            log("NVML unavailable, sampling with nvidia-smi:", e)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", bus], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception as e:  # no nvidia-smi: report no clocks
            log("clock sampler unavailable:", e)

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        import datetime
        if self.thread is not None:
            self.stop_ev.set()
            self.thread.join(timeout=2)
            sm = [x[0] for x in self.samples]
            reasons = sorted({n for x in self.samples for bit, n in self.REASONS.items() if x[3] & bit})
            return {"sm_mhz": statistics.median(sm) if sm else None,
                    "sm_max_mhz": max(x[1] for x in self.samples) if sm else None,
                    "power_w_max": round(max(x[2] for x in self.samples), 1) if sm else None,
                    "reasons": reasons, "samples": len(sm), "source": "nvml"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                continue
            # keep only samples taken inside the timed region
            if self.t0 is not None and not (self.t0 - 0.05 <= ts <= (self.t1 or ts) + 0.05):
                continue
            f = f[1:]
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
class Dist:
    def __init__(self, n_gpus: int):
        import torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}")
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist
        else:
            torch.cuda.set_device(0)
        self.device = torch.device("cuda", torch.cuda.current_device())

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def timed_loop(fn, steps: int, warmup: int, dist: Dist, sampler_index: int):
    """W untimed steps, then K steps bracketed by barrier + synchronize, timed
    with CUDA events on the launching stream; max over ranks."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    sampler = ClockSampler(sampler_index)
    time.sleep(0.25)  # let the sampler start before the timed region
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.mark_start()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    sampler.mark_end()
    clocks = sampler.stop()
    dist.barrier()
    ms = start.elapsed_time(end)
    return dist.max(ms), clocks


def kernel_ms(fn, reps: int = 30) -> float:
    """Average device duration of one launch of fn (events around each)."""
    import torch
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in ev:
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev) / reps


def graph_of(fn, calls: int):
    """A CUDA graph of `calls` consecutive calls of fn (captured once; fn's
    own Python state advances during the capture only).  Short decode steps
    are replayed this way, as a serving loop would, so that the host's
    per-call cost does not set the step time."""
    import torch
    g = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            for _ in range(calls):
                fn()
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()
    return g


# ---------------------------------------------------------------------------
# workloads on the device
# ---------------------------------------------------------------------------
def gen_normal(shape, dtype, device, gen):
    import torch
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)


def build_llama3_decode(dev, seed, n_seqs=32, length=8192):
    import torch

    import bml_b200
    gen = torch.Generator(device=dev).manual_seed(seed)
    H, Hkv, d = 32, 8, 128
    ks = [gen_normal((length, Hkv, d), torch.bfloat16, dev, gen) for _ in range(n_seqs)]
    vs = [gen_normal((length, Hkv, d), torch.bfloat16, dev, gen) for _ in range(n_seqs)]
    q = gen_normal((n_seqs, H, d), torch.float32, dev, gen)
    batch = bml_b200.SeqBatch(ks, vs)
    return q, batch, H


def build_batched_tinyllama(dev, rank, world, copy=0):
    """The ragged batch of this rank; `copy` draws other values of the same
    shapes (a second copy lets a timed loop alternate between two batches
    whose bytes together exceed twice the L2)."""
    import numpy as np
    import torch

    import bml_b200
    from bml_b200 import sharding
    from bml_b200 import workloads as W
    lens = W.batched_lengths()
    mine = sharding.lpt_partition([int(x) for x in lens], world)[rank]
    gen = torch.Generator(device=dev).manual_seed(2 + 1000 * rank + 100000 * copy)
    H, Hkv, d = 32, 4, 64
    ks = [gen_normal((int(lens[i]), Hkv, d), torch.float16, dev, gen) for i in mine]
    vs = [gen_normal((int(lens[i]), Hkv, d), torch.float16, dev, gen) for i in mine]
    q = gen_normal((len(mine), H, d), torch.float32, dev, gen)
    return q, bml_b200.SeqBatch(ks, vs), H, int(np.sum(lens))


def decode_step_bytes(batch, n_heads):
    return batch.kv_bytes + len(batch) * n_heads * batch.head_dim * 8


# ---------------------------------------------------------------------------
# CPU baseline (oracle) on a bounded sample
# ---------------------------------------------------------------------------
def cpu_decode_sample(workload: str, budget_s: float, threads: int = 0):
    """Times the oracle (all host threads, or `threads`) on a bounded sample
    of the workload; returns (GB/s, threads, description)."""
    import numpy as np

    import oracle
    from bml_b200 import workloads as W
    threads = threads or host_threads()
    if workload == "batched_tinyllama":
        q, ks, vs = W.batched_tinyllama(n_seqs=8)
        code, nkv, d, es = None, 4, 64, 2
        desc = "first 8 of the 64 ragged f16 sequences (seed 2)"
    elif workload == "longctx":
        q1, k, v = W.longctx_decode(length=16384)
        q, ks, vs = q1[None], [k], [v]
        code, nkv, d, es = oracle.BF16, 8, 128, 2
        desc = "first 16384 of 131072 positions (seed 4)"
    else:
        q, k, v = W.llama3_decode(n_seqs=2)
        ks, vs = list(k), list(v)
        code, nkv, d, es = oracle.BF16, 8, 128, 2
        desc = "2 of the 32 sequences x 8192 positions (seed 3)"
    n_heads = q.shape[1]
    total = sum(x.shape[0] for x in ks)
    nbytes = W.decode_bytes(total, nkv, d, es, len(ks), n_heads)
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.attn_decode_batched(q, ks, vs, dtype=code, n_threads=threads)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / reps
    return nbytes / dt / 1e9, threads, f"{desc}, {reps} passes, {dt * 1e3:.1f} ms/pass"


def cpu_literal_sample(workload: str, budget_s: float):
    """The reference's literal access pattern (a heap copy per load_k, and per
    load_v inside the head_dim loop; f32 cache as HashConsedKV holds it) on
    one thread, over the first sequence of the workload's sample, as many q
    heads as the budget allows; returns (GB/s of the whole sequence at the
    time per head x n_heads, description)."""
    import numpy as np

    import oracle
    from bml_b200 import workloads as W
    if workload == "batched_tinyllama":
        q, ks, vs = W.batched_tinyllama(n_seqs=1)
        q1, k, v = q[0], ks[0].astype(np.float32), vs[0].astype(np.float32)
        nkv, d = 4, 64
    else:
        if workload == "longctx":
            q1, k, v = W.longctx_decode(length=8192)
        else:
            q, kk, vv = W.llama3_decode(n_seqs=1)
            q1, k, v = q[0], kk[0], vv[0]

        def widen(bits):
            return (np.ascontiguousarray(bits).view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        k, v = widen(k), widen(v)
        nkv, d = 8, 128
    n_heads, L = q1.shape[0], k.shape[0]
    t0 = time.perf_counter()
    h = 0
    while h < n_heads:
        oracle.attn_decode_literal(q1, k, v, pos=L - 1, heads=(h, h + 1))
        h += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    per_head = (time.perf_counter() - t0) / h
    nbytes = W.decode_bytes(L, nkv, d, 2, 1, n_heads)  # bytes of the stored (16-bit) cache
    return (nbytes / (per_head * n_heads) / 1e9,
            f"1 thread, sequence 0 ({L} positions), {h} of {n_heads} q heads, "
            f"{per_head * 1e3:.0f} ms/head")


def cpu_prefill_sample(budget_s: float):
    """Oracle on the last 16 query rows of one head group... of the 4x8192
    prefill; returns TFLOP/s (causal pairs actually computed)."""
    import oracle
    from bml_b200 import workloads as W
    threads = host_threads()
    S = 8192
    q, k, v = W.llama3_prefill(n_seqs=1, seq_len=S)
    rows = (S - 16, S)
    pairs = sum(t + 1 for t in range(*rows))
    flops = 4 * 128 * 32 * pairs
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.attn_prefill(W.bf16_bits_to_f32(q), k, v, dtype=oracle.BF16, rows=rows, n_threads=threads)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / reps
    return flops / dt / 1e12, threads, f"query rows {rows[0]}..{rows[1] - 1} of one 8192-token sequence, all 32 heads, {reps} passes"


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------
def prefill_units(rank: int, world: int, n: int = 4, n_kv: int = 8):
    """This rank's share of a prefill of n sequences with n_kv kv heads, cut
    into n * n_kv (sequence, kv-head group) units dealt out in contiguous
    runs: (first sequence, sequences, first kv head, kv heads).  For world
    in 1, 2, 4, 8 and 4 x 8 units a share is whole sequences or a run of kv
    heads of one sequence, so it is one launch."""
    units = n * n_kv
    if units % world:
        raise SystemExit(f"{units} prefill units do not split over {world} ranks")
    per = units // world
    u0 = rank * per
    if per >= n_kv:
        if per % n_kv or u0 % n_kv:
            raise SystemExit("prefill share is not whole sequences")
        return u0 // n_kv, per // n_kv, 0, n_kv
    if n_kv % per:
        raise SystemExit("prefill share straddles sequences")
    return u0 // n_kv, 1, u0 % n_kv, per


def run_prefill(dev, steps, warmup, dist, peaks, n=4, S=8192):
    """Causal prefill of n x S tokens (Llama-3-8B heads) split over the ranks
    by (sequence x kv-head group) with no collective ("strong": the total
    work is fixed).  Each rank holds the q/k/v of its own units only."""
    import torch

    import bml_b200
    from bml_b200 import workloads as W
    H, Hkv, d = 32, 8, 128
    G = H // Hkv
    s0, ns, h0, nh = prefill_units(dist.rank, dist.world, n, Hkv)
    gen = torch.Generator(device=dev).manual_seed(3 + 1000 * dist.rank)
    q = gen_normal((ns, S, nh * G, d), torch.bfloat16, dev, gen)
    k = gen_normal((ns, S, nh, d), torch.bfloat16, dev, gen)
    v = gen_normal((ns, S, nh, d), torch.bfloat16, dev, gen)
    out = torch.empty(ns, S, nh * G, d, dtype=torch.float32, device=dev)
    fn = lambda: bml_b200.prefill(q, k, v, out=out)  # noqa: E731
    try:
        fn()
        torch.cuda.synchronize()
    except bml_b200.BmlUnsupported as e:
        return {"unavailable": str(e)}
    # the kernel alone (10 launches) before the long loop heats the GPU into
    # its power cap: the burst figure; the loop gives the sustained one
    for _ in range(max(1, warmup)):
        fn()
    torch.cuda.synchronize()
    kms = kernel_ms(fn, 10)
    ms, clocks = timed_loop(fn, steps, warmup, dist, dist.local)
    flops_total = W.prefill_flops(n, S, H, d)
    flops_mine = W.prefill_flops(ns, S, nh * G, d)
    tflops = flops_total * steps / (ms * 1e-3) / 1e12
    ach = flops_mine / (kms * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    peak_s = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    loop_rank = flops_mine * steps / (ms * 1e-3) / 1e12
    return {"metric": "causal prefill TFLOP/s", "value": round(tflops, 2), "unit": "TFLOP/s",
            "ms_per_step": round(ms / steps, 4), "steps": steps, "scaling": "strong",
            "config": {"workload": "llama3_prefill", "n_seqs": n, "seq_len": S, "n_heads": H,
                       "n_kv_heads": Hkv, "head_dim": d, "causal": True, "dtype": "bf16",
                       "split": f"{n * Hkv} (sequence, kv-head group) units over {dist.world} GPU(s), no collective",
                       "rank0_share": {"first_seq": s0, "seqs": ns, "first_kv_head": h0, "kv_heads": nh}},
            "roofline": {"bound": "tensor", "achieved": round(ach, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(ach / peak, 4), "frac_spec": round(ach / SPEC_PEAKS["bf16_tflops"], 4),
                         "peak_kind": "measured cuBLAS bf16 burst (kernel timed alone, 10 launches)",
                         "loop_per_gpu": round(loop_rank, 2),
                         "loop_frac_sustained": round(loop_rank / peak_s, 4),
                         "traffic": profile_traffic("prefill_tcgen05_llama3.txt") if dist.world == 1 else None,
                         "kernel": "prefill_kernel", "kernel_ms": round(kms, 4),
                         "algorithmic_flops_per_launch": flops_mine},
            "clocks": clocks}


def run_tinyllama_obj(dev, steps, warmup, dist, peaks, cpu_budget):
    """The 64-sequence ragged TinyLlama-shaped batch (U[128,4096], f16 KV),
    sequences dealt over the ranks by longest-processing-time ("strong", no
    collective)."""
    import torch

    import bml_b200
    # two copies of the batch, alternated: 147 MB a step is only a little
    # above the 126 MB L2, so a step never follows one that read its bytes
    copies = [build_batched_tinyllama(dev, dist.rank, dist.world, c) for c in range(2)]
    q, batch, H, _ = copies[0]
    ws = bml_b200.Workspace(dev).ensure(len(batch), H, batch.head_dim)
    out = torch.empty_like(q)
    state = {"i": 0}

    def fn():
        qc, bc = copies[state["i"] & 1][:2]
        state["i"] += 1
        bml_b200.decode_batched(qc, bc, out=out, workspace=ws)

    fn()
    fn()
    torch.cuda.synchronize()
    g = graph_of(fn, 2)  # copy 0 then copy 1
    reps = max(1, steps // 2)
    ms, clocks = timed_loop(g.replay, reps, max(1, warmup // 2), dist, dist.local)
    steps = 2 * reps
    step_bytes = decode_step_bytes(batch, H)
    total = dist.sum(step_bytes)
    kms_each = kernel_ms(fn)
    ws.check()
    del g
    kms = ms / steps  # one launch a step: the launch's average duration over the timed region
    ach = step_bytes / (kms * 1e-3) / 1e9
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    res = {"metric": "batched decode HBM GB/s", "value": round(total * steps / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
           "ms_per_step": round(ms / steps, 5), "steps": steps, "scaling": "strong",
           "config": {"workload": "batched_tinyllama", "n_seqs": 64, "n_seqs_rank0": len(batch),
                      "lengths": "U[128,4096] seed 2", "n_heads": H, "n_kv_heads": 4, "head_dim": 64,
                      "kv_dtype": "f16", "sharding": f"LPT over {dist.world} GPU(s), no collective",
                      "launch": "CUDA graph of two steps (the two batch copies), replayed",
                      "l2": "two copies of the 147 MB batch alternated (294 MB, all ranks) vs 126 MB L2"},
           "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(ach / hbm, 4), "frac_spec": round(ach / SPEC_PEAKS["hbm_gbs"], 4),
                        "traffic": profile_traffic("decode_batched_tinyllama.txt") if dist.world == 1 else None,
                        "kernel": "decode_bulk_kernel", "kernel_ms": round(kms, 5),
                        "kernel_ms_events_each": round(kms_each, 5),
                        "algorithmic_bytes_per_launch": step_bytes},
           "clocks": clocks}
    if dist.world == 1 and cpu_budget > 0:
        v, thr, desc = cpu_decode_sample("batched_tinyllama", cpu_budget)
        res["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": thr, "kind": "port", "sample": desc}
    return res


def run_b200(args):
    import torch

    import bml_b200
    dist = Dist(args.gpus)
    dev = dist.device
    peaks, peak_kind = load_peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    res = {"n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
           "vs_baseline": None, "data": "synthetic: seeded N(0,1) on the device (torch generator)",
           "peak_source": f"{peak_kind} ({PEAKS_PATH if peak_kind == 'measured' else 'fallback'})"}
    wl = args.workload
    cpu = 0.0 if args.no_cpu or dist.world > 1 else args.cpu_budget
    if wl == "llama3_prefill":
        pre = run_prefill(dev, args.steps, args.warmup, dist, peaks, args.prefill_n, args.prefill_s)
        res.update(pre)
        res.update({"metric": DECODE_METRIC, "dtype": "bf16", "gpu_launches": args.steps})
        emit(res, dist)
        return
    if wl == "batched_tinyllama":
        obj = run_tinyllama_obj(dev, args.steps, args.warmup, dist, peaks, cpu)
        res.update(obj)
        res.update({"metric": DECODE_METRIC, "dtype": "f32 (f16 KV)", "gpu_launches": args.steps})
        emit(res, dist)
        return
    if wl == "longctx":
        return run_longctx(args, dist, peaks, res)
    if wl == "serving":
        return run_serving(args, dist, peaks, res)
    if wl == "gemv":
        return run_gemv(args, dist, peaks, res)
    if wl == "gguf_load":
        return run_gguf_load(args, dist, peaks, res)
    if wl != "llama3_decode":
        raise SystemExit(f"unknown workload {wl}")

    q, batch, H = build_llama3_decode(dev, 3 + 1000 * dist.rank)
    cfg = {"workload": "llama3_decode", "n_seqs_per_gpu": len(batch), "context": 8192, "n_heads": H,
           "n_kv_heads": 8, "head_dim": 128, "kv_dtype": "bf16",
           "l2": "inputs larger than L2 (1 GiB of KV per step vs 126 MB)"}
    ws = bml_b200.Workspace(dev).ensure(len(batch), H, batch.head_dim)
    out = torch.empty_like(q)
    fn = lambda: bml_b200.decode_batched(q, batch, out=out, workspace=ws)  # noqa: E731
    fn()
    torch.cuda.synchronize()
    ms, clocks = timed_loop(fn, args.steps, args.warmup, dist, dist.local)
    step_bytes = decode_step_bytes(batch, H)
    total_bytes = dist.sum(step_bytes)
    gbs = total_bytes * args.steps / (ms * 1e-3) / 1e9
    kms_each = kernel_ms(fn)
    kms = ms / args.steps  # one launch a step: its average duration over the timed region
    ach = step_bytes / (kms * 1e-3) / 1e9
    ws.check()

    # end to end through the public API with host buffers
    e2e = e2e_decode(q, batch, ws, args, dist, step_bytes)

    res.update({
        "metric": DECODE_METRIC, "value": round(gbs, 1), "unit": "GB/s",
        "ms_per_step": round(ms / args.steps, 5), "scaling": "weak", "dtype": "f32 (bf16 KV)", "config": cfg,
        "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(ach / hbm, 4), "frac_spec": round(ach / SPEC_PEAKS["hbm_gbs"], 4),
                     "traffic": profile_traffic("decode_llama3_decode.txt"),
                     "kernel": decode_kernel_name(batch.dtype, batch.head_dim, batch.n_kv, H // batch.n_kv),
                     "kernel_ms": round(kms, 5), "kernel_ms_events_each": round(kms_each, 5),
                     "algorithmic_bytes_per_launch": step_bytes},
        # per step: one decode_bulk_kernel (partials merged in the same launch)
        "clocks": clocks, "e2e": e2e, "gpu_launches": args.steps,
    })
    del q, batch, ws, out
    torch.cuda.empty_cache()
    if dist.world == 1 and not args.no_cpu:
        v, thr, desc = cpu_decode_sample(wl, args.cpu_budget * 0.7)
        v1, _, desc1 = cpu_decode_sample(wl, args.cpu_budget * 0.3, threads=1)
        vl, descl = cpu_literal_sample(wl, min(4.0, args.cpu_budget * 0.2))
        res["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": thr, "kind": "port",
                               "sample": desc, "value_1core": round(v1, 4), "sample_1core": desc1,
                               "value_literal": round(vl, 6), "sample_literal": descl}
    if not args.no_prefill:
        pre = run_prefill(dev, max(3, args.prefill_steps), 3, dist, peaks)
        if dist.world == 1 and not args.no_cpu and "value" in pre:
            pv, pthr, pdesc = cpu_prefill_sample(args.cpu_budget / 2)
            pre["cpu_baseline"] = {"value": round(pv, 5), "unit": "TFLOP/s", "cores": pthr, "kind": "port",
                                   "sample": pdesc}
        res["prefill"] = pre
        res["gpu_launches"] += pre.get("steps", 0)
        torch.cuda.empty_cache()
    if not args.no_sub:
        sub_steps = max(args.steps, args.sub_steps)
        tiny = run_tinyllama_obj(dev, sub_steps, max(3, args.warmup), dist, peaks, cpu / 2)
        res["batched_tinyllama"] = tiny
        res["gpu_launches"] += sub_steps
        torch.cuda.empty_cache()
        lc = run_longctx_obj(dev, sub_steps, max(3, args.warmup), dist, peaks, cpu / 2, args.kvsplit)
        res["gpu_launches"] += sub_steps * lc.pop("launches_per_step")
        res["longctx"] = lc
    emit(res, dist)


def e2e_decode(q, batch, ws, args, dist, step_bytes):
    """Each step: pinned host q -> device, decode through the C ABI, result
    -> pinned host, stream synchronised (the host holds the result)."""
    import torch

    import bml_b200
    q_host = q.cpu().pin_memory()
    out_host = torch.empty_like(q_host).pin_memory()
    q_dev = torch.empty_like(q)
    out_dev = torch.empty_like(q)
    stream = torch.cuda.current_stream()

    def step():
        q_dev.copy_(q_host, non_blocking=True)
        bml_b200.decode_batched(q_dev, batch, out=out_dev, workspace=ws)
        out_host.copy_(out_dev, non_blocking=True)
        stream.synchronize()

    n = max(10, min(args.steps, 500))
    for _ in range(3):
        step()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = dist.max(a.elapsed_time(b))
    total = dist.sum(step_bytes)
    return {"value": round(total * n / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": q_host.numel() * 4, "d2h_bytes_per_step": out_host.numel() * 4,
            "steps": n, "ms_per_step": round(ms / n, 5)}


def run_longctx_obj(dev, steps, warmup, dist, peaks, cpu_budget, kvsplit="peer"):
    """One 131072-position sequence (Llama-3-8B heads, bf16 KV) split along
    its KV length over the ranks; per-rank (m, l, o) partials exchanged and
    merged ("strong").  One GPU runs the plain decode of the whole
    sequence."""
    import torch

    import bml_b200
    from bml_b200 import sharding
    total_len, H, Hkv, d = 131072, 32, 8, 128
    lo, hi = sharding.kv_split_ranges(total_len, dist.world)[dist.rank]
    gen = torch.Generator(device=dev).manual_seed(4)
    # every rank draws the whole sequence's q; its KV slice is its own draw
    q = gen_normal((1, H, d), torch.float32, dev, gen)
    gen.manual_seed(4 + 1000 * (dist.rank + 1))
    k = gen_normal((hi - lo, Hkv, d), torch.bfloat16, dev, gen)
    v = gen_normal((hi - lo, Hkv, d), torch.bfloat16, dev, gen)
    batch = bml_b200.SeqBatch([k], [v])
    ws = bml_b200.Workspace(dev).ensure(1, H, d)
    merged = torch.empty(1, H, d, dtype=torch.float32, device=dev)
    step = sharding.KVSplitDecode(dist.pg, dist.world, H, d, dev, fused=kvsplit == "peer")
    fn = lambda: step(q, batch, ws, out=merged, total_len=total_len)  # noqa: E731
    fn()
    torch.cuda.synchronize()
    graphed = not (dist.world > 1 and kvsplit == "nccl")  # NCCL's collective stays outside graphs
    if graphed:
        g = graph_of(fn, 2)
        reps = max(1, steps // 2)
        ms, clocks = timed_loop(g.replay, reps, max(1, warmup // 2), dist, dist.local)
        steps = 2 * reps
        del g
    else:
        ms, clocks = timed_loop(fn, steps, warmup, dist, dist.local)
    step_bytes = decode_step_bytes(batch, H)
    total = dist.sum(step_bytes)
    gbs = total * steps / (ms * 1e-3) / 1e9
    if dist.world > 1 and kvsplit == "nccl":
        kfn = lambda: bml_b200.decode_partial(q, batch, workspace=ws)  # noqa: E731
        kms_each = kernel_ms(kfn)
        kms = kms_each  # the decode launch alone (the step also has NCCL and a merge)
    else:  # one launch: the whole step (with the exchange inside it on several GPUs)
        kms_each = kernel_ms(fn)
        kms = ms / steps  # the launch's average duration over the timed region
    ws.check()
    ach = step_bytes / (kms * 1e-3) / 1e9
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    res = {"metric": "sequence-split decode HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
           "ms_per_step": round(ms / steps, 5), "steps": steps, "scaling": "strong",
           "config": {"workload": "longctx", "context": total_len, "n_heads": H, "n_kv_heads": Hkv,
                      "head_dim": d, "kv_dtype": "bf16",
                      "split": ("one GPU: the whole sequence, plain decode" if dist.world == 1 else
                                f"KV length over {dist.world} GPUs; per-(head, 32 dims) partials exchanged over "
                                "peer memory and merged inside the decode kernel" if kvsplit == "peer" else
                                f"KV length over {dist.world} GPUs, NCCL all_gather of (m, l, o) + LSE merge"),
                      "l2": "512 MiB of KV (K + V) per step, all ranks",
                      "launch": "CUDA graph of two steps, replayed" if graphed else "one call a step"},
           "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(ach / hbm, 4), "frac_spec": round(ach / SPEC_PEAKS["hbm_gbs"], 4),
                        "traffic": profile_traffic("decode_longctx.txt") if dist.world == 1 else None,
                        "kernel": "decode_bulk_kernel", "kernel_ms": round(kms, 5),
                        "kernel_ms_events_each": round(kms_each, 5),
                        "algorithmic_bytes_per_launch": step_bytes},
           # per step: decode_bulk_kernel; with the NCCL exchange also
           # merge_lse_packed_kernel, with NCCL's all-gather between
           "launches_per_step": 2 if dist.world > 1 and kvsplit == "nccl" else 1,
           "clocks": clocks}
    if dist.world > 1:
        step.close()
    if dist.world == 1 and cpu_budget > 0:
        v, thr, desc = cpu_decode_sample("longctx", cpu_budget)
        res["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": thr, "kind": "port", "sample": desc}
    return res


def run_longctx(args, dist, peaks, res):
    obj = run_longctx_obj(dist.device, args.steps, args.warmup, dist, peaks, 0 if args.no_cpu else args.cpu_budget,
                          args.kvsplit)
    res.update(obj)
    res["metric"] = DECODE_METRIC
    res["dtype"] = "f32 (bf16 KV)"
    res["gpu_launches"] = args.steps * obj.pop("launches_per_step")
    emit(res, dist)


# Llama-3-8B projections: (name, n_in, n_out) in the reference's (dims[0],
# dims[1]) terms
GEMV_LAYER = [("attn_q", 4096, 4096), ("attn_k", 4096, 1024), ("attn_v", 4096, 1024), ("attn_output", 4096, 4096),
              ("ffn_gate", 4096, 14336), ("ffn_up", 4096, 14336), ("ffn_down", 14336, 4096)]


def q4_0_bytes(n_elems: int, gen, dev):
    """Random Q4_0 tensor bytes on the device: N(0, 0.02) f16 scales, random
    nibbles."""
    import torch
    nb = n_elems // 32
    raw = torch.randint(0, 256, (nb, 18), dtype=torch.uint8, device=dev, generator=gen)
    sc = (torch.randn(nb, device=dev, generator=gen) * 0.02).to(torch.float16).view(torch.int16)
    raw[:, 0] = (sc & 0xFF).to(torch.uint8)
    raw[:, 1] = ((sc >> 8) & 0xFF).to(torch.uint8)
    return raw.reshape(-1)


def cpu_gemv_sample(budget_s: float):
    """The oracle's matmul_f64 over the dequantised f32 values of the
    attn_q tensor (the reference's arithmetic and loop order, one thread)."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(7)
    n_in, n_out = 4096, 4096
    nb = n_in * n_out // 32
    raw = rng.integers(0, 256, (nb, 18), dtype=np.uint8)
    sc = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint16)
    raw[:, 0], raw[:, 1] = sc & 0xFF, sc >> 8
    w = oracle.read_tensor_f32(raw.tobytes(), oracle.GGUF_Q4_0, n_in * n_out)
    x = rng.standard_normal(n_in)
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.matmul_f64(w, n_in, n_out, x)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / reps
    nbytes = nb * 18 + (n_in + n_out) * 8
    return nbytes / dt / 1e9, 1, f"attn_q 4096x4096 Q4_0 (f32 values, 1 thread), {reps} passes, {dt * 1e3:.1f} ms/pass"


def run_gemv(args, dist, peaks, res):
    import torch

    import bml_b200
    dev = dist.device
    gen = torch.Generator(device=dev).manual_seed(8 + 1000 * dist.rank)
    n_layers = 4
    layers = [[bml_b200.WeightTensor(q4_0_bytes(a * b, gen, dev), bml_b200.weights.GGUF_Q4_0, [a, b])
               for _, a, b in GEMV_LAYER] for _ in range(n_layers)]
    xs = {a: gen_normal((a,), torch.float64, dev, gen) for _, a, _ in GEMV_LAYER}
    ys = [torch.empty(b, dtype=torch.float64, device=dev) for _, _, b in GEMV_LAYER]
    state = {"t": 0}

    def step():
        ws = layers[state["t"] % n_layers]
        state["t"] += 1
        for w, y in zip(ws, ys):
            w.matmul_f64(xs[w.n_in], out=y)

    # A layer's projections are a handful of ~5-30 us kernels, shorter than
    # the host time of launching them one by one from Python, so a step
    # replays a CUDA graph of the layer's launches (one graph per layer of
    # weights), as a model's decode loop would.
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    graphs = []
    cap = torch.cuda.Stream(device=dev)
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        for li in range(n_layers):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                for w, y in zip(layers[li], ys):
                    w.matmul_f64(xs[w.n_in], out=y)
            graphs.append(g)
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()

    def step_graph():
        graphs[state["t"] % n_layers].replay()
        state["t"] += 1

    ms, clocks = timed_loop(step_graph, args.steps, args.warmup, dist, dist.local)
    step_bytes = sum(w.nbytes + (w.n_in + w.n_out) * 8 for w in layers[0])
    total = dist.sum(step_bytes)
    gbs = total * args.steps / (ms * 1e-3) / 1e9
    # the largest projection alone: a graph of 16 launch pairs (gemv + range
    # reduce) cycling over the 4 layers' copies so that each streams from HBM
    bigs = [layers[i][5] for i in range(n_layers)]
    kg = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(kg, stream=cap):
            for i in range(16):
                bigs[i % n_layers].matmul_f64(xs[4096], out=ys[5])
    torch.cuda.synchronize()
    kg.replay()
    torch.cuda.synchronize()
    kms = kernel_ms(kg.replay, reps=10) / 16
    big_bytes = bigs[0].nbytes + (bigs[0].n_in + bigs[0].n_out) * 8
    ach = big_bytes / (kms * 1e-3) / 1e9
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])

    # end to end through the public API, launched from Python one call at a
    # time (no graph): x from pinned host memory each step, the last y back
    xh = {a: t.cpu().pin_memory() for a, t in xs.items()}
    yh = torch.empty(GEMV_LAYER[-1][2], dtype=torch.float64).pin_memory()
    stream = torch.cuda.current_stream()

    def step_e2e():
        for a in xs:
            xs[a].copy_(xh[a], non_blocking=True)
        step()
        yh.copy_(ys[-1], non_blocking=True)
        stream.synchronize()

    n = max(10, min(args.steps, 200))
    for _ in range(3):
        step_e2e()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n):
        step_e2e()
    b.record(stream)
    torch.cuda.synchronize()
    ems = dist.max(a.elapsed_time(b))
    e2e = {"value": round(total * n / (ems * 1e-3) / 1e9, 1), "unit": "GB/s",
           "h2d_bytes_per_step": sum(t.numel() * 8 for t in xh.values()), "d2h_bytes_per_step": yh.numel() * 8,
           "steps": n, "ms_per_step": round(ems / n, 5)}
    res.update({"metric": "Q4_0 projection (matmul_f64) HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
                "ms_per_step": round(ms / args.steps, 5), "scaling": "weak", "dtype": "f32 terms, f64 sums (Q4_0 W)",
                "config": {"workload": "gemv", "model": "Llama-3-8B projections", "layers_cycled": n_layers,
                           "tensors": [f"{nm} {a}x{b}" for nm, a, b in GEMV_LAYER], "quant": "Q4_0",
                           "l2": "4 layers of distinct weights, 490 MB cycled > 126 MB L2"},
                "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(ach / hbm, 4), "frac_spec": round(ach / SPEC_PEAKS["hbm_gbs"], 4),
                             "traffic": None,
                             "kernel": "gemv_staged_kernel<Q4_0> + gemv_reduce_kernel (ffn_up 4096x14336)",
                             "kernel_ms": round(kms, 5), "algorithmic_bytes_per_launch": big_bytes},
                "timing": "device time of CUDA-graph replays of each layer's launches",
                "clocks": clocks, "e2e": e2e, "gpu_launches": args.steps * 2 * len(GEMV_LAYER)})
    del graphs, kg
    if dist.world == 1 and not args.no_cpu:
        v, thr, desc = cpu_gemv_sample(args.cpu_budget)
        res["cpu_baseline"] = {"value": round(v, 4), "unit": "GB/s", "cores": thr, "kind": "port", "sample": desc}
    emit(res, dist)


def cpu_gguf_sample(path, budget_s: float):
    """What the reference does with a loaded tensor: read_tensor_f32 into
    its f32 pool (the oracle's dequantize_q4_0, one thread)."""
    import oracle
    from bml_b200 import gguf
    with gguf.GgufFile(path) as f:
        info = f.find_tensor("blk.0.attn_q.weight")
        view = f.tensor_data(info)[:info.nbytes].tobytes()
    n = info.dims[0] * info.dims[1]
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.read_tensor_f32(view, oracle.GGUF_Q4_0, n)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / reps
    return len(view) / dt / 1e9, 1, f"attn_q 4096x4096 Q4_0 to f32 (1 thread), {reps} passes, {dt * 1e3:.1f} ms/pass"


def run_gguf_load(args, dist, peaks, res):
    import tempfile

    import numpy as np
    import torch

    from bml_b200 import gguf
    dev = dist.device
    n_layers = 8
    rng = np.random.default_rng(9 + dist.rank)
    block = rng.integers(0, 256, 32 << 20, dtype=np.uint8)  # 32 MiB of random bytes, reused
    tensors = []
    for layer in range(n_layers):
        for nm, a, b in GEMV_LAYER:
            nbytes = a * b // 32 * 18
            reps = -(-nbytes // block.size)
            tensors.append((f"blk.{layer}.{nm}.weight", [a, b], 2, np.tile(block, reps)[:nbytes]))
    tmpdir = tempfile.mkdtemp(prefix="bml_gguf_")
    path = os.path.join(tmpdir, f"model_{dist.rank}.gguf")
    gguf.write_gguf(path, [("general.architecture", 8, "llama"), ("llama.block_count", 4, n_layers)], tensors)
    del tensors
    f = gguf.GgufFile(path)
    infos = f.tensor_infos
    bufs = [torch.empty(i.nbytes, dtype=torch.uint8, device=dev) for i in infos]
    import ctypes as C
    from bml_b200 import _lib as L
    idx = (C.c_uint64 * len(infos))(*[i.index for i in infos])
    dst = (C.c_void_p * len(infos))(*[b.data_ptr() for b in bufs])
    total_bytes = sum(i.nbytes for i in infos)
    torch.cuda.synchronize()

    def step():
        L.call("bml_gguf_upload", f._h, idx, len(infos), dst, args.gguf_threads)

    ms, clocks = timed_loop(step, args.steps, args.warmup, dist, dist.local)
    gbs = dist.sum(total_bytes) * args.steps / (ms * 1e-3) / 1e9
    # the copy engine's own rate: one 256 MiB pinned buffer to the device
    pin = torch.empty(256 << 20, dtype=torch.uint8).pin_memory()
    dbuf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    dbuf.copy_(pin, non_blocking=True)
    torch.cuda.synchronize()
    h2d_ms = kernel_ms(lambda: dbuf.copy_(pin, non_blocking=True), reps=10)
    h2d = pin.numel() / (h2d_ms * 1e-3) / 1e9
    ach = total_bytes / (ms / args.steps * 1e-3) / 1e9
    ok = all(torch.equal(bufs[k][:64].cpu(), torch.from_numpy(f.tensor_data(infos[k])[:64].copy())) for k in (0, -1))
    res.update({"metric": "GGUF upload GB/s (host file -> device)", "value": round(gbs, 2), "unit": "GB/s",
                "ms_per_step": round(ms / args.steps, 3), "scaling": "weak", "dtype": "u8 (Q4_0 bytes)",
                "config": {"workload": "gguf_load", "tensors": len(infos), "file_bytes": f.file_size,
                           "tensor_bytes": total_bytes, "layers": n_layers, "threads": args.gguf_threads,
                           "page_cache": "warm",
                           "bytes_verified": bool(ok)},
                "roofline": {"bound": "h2d", "achieved": round(ach, 2), "peak": round(h2d, 2), "unit": "GB/s",
                             "frac": round(ach / h2d, 4), "traffic": None,
                             "peak_source": "pinned 256 MiB cudaMemcpyAsync to the device, measured in this run"},
                "clocks": clocks,
                "e2e": {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": total_bytes,
                        "d2h_bytes_per_step": 0},
                "gpu_launches": 0})
    if dist.world == 1 and not args.no_cpu:
        v, thr, desc = cpu_gguf_sample(path, args.cpu_budget)
        res["cpu_baseline"] = {"value": round(v, 4), "unit": "GB/s", "cores": thr, "kind": "port", "sample": desc}
    f.close()
    os.remove(path)
    os.rmdir(tmpdir)
    emit(res, dist)


def run_serving(args, dist, peaks, res):
    """DecodeBatcher over 32 Llama-3-shaped requests; one step = one token of
    every request through all layers, with a leave + join every 8 steps."""
    import numpy as np
    import torch

    import bml_b200
    dev = dist.device
    n_req, n_layers, H, Hkv, d = 32, 32, 32, 8, 128
    row = Hkv * d * 2
    rng = np.random.default_rng(6 + 1000 * dist.rank)
    lens0 = [int(x) for x in rng.integers(1024, 4097, n_req)]
    total_steps = args.steps + args.warmup + 8
    cap = ((max(lens0) + total_steps + 255) // 256) * 256
    gen = torch.Generator(device=dev).manual_seed(6 + 1000 * dist.rank)
    k_prompt = gen_normal((n_layers, 4096, Hkv, d), torch.bfloat16, dev, gen)
    v_prompt = gen_normal((n_layers, 4096, Hkv, d), torch.bfloat16, dev, gen)
    b = bml_b200.DecodeBatcher(n_layers, H, Hkv, d, dtype=torch.bfloat16, device=dev, rope=True)
    next_id = [0]

    def join(L):
        b.add(next_id[0], cap, k_prompt[:, :L], v_prompt[:, :L])
        next_id[0] += 1

    for L in lens0:
        join(L)
    q = gen_normal((n_layers, n_req, H, d), torch.float32, dev, gen)
    kn = gen_normal((n_layers, n_req, Hkv, d), torch.float32, dev, gen)
    vn = gen_normal((n_layers, n_req, Hkv, d), torch.float32, dev, gen)
    out = torch.empty(n_req, H, d, dtype=torch.float32, device=dev)
    state = {"t": 0, "bytes": 0}
    # per request and layer: KV read over len+1 positions, q read, out
    # written, and the append (q read+write, k/v f32 read, k/v bf16 write)
    per_layer_fixed = H * d * 4 * 2 + H * d * 4 * 2 + 2 * Hkv * d * 4 + 2 * row

    def token():
        if state["t"] and state["t"] % 8 == 0:
            longest = max(b.active, key=b.length)
            b.remove(longest)
            join(int(rng.integers(1024, 4097)))
        state["bytes"] += n_layers * sum(2 * (b.length(r) + 1) * row + per_layer_fixed for r in b.active)
        for layer in range(n_layers):
            b.step(layer, q[layer], kn[layer], vn[layer], out=out)
        b.advance()
        state["t"] += 1

    token()
    torch.cuda.synchronize()
    state["bytes"] = 0
    for _ in range(args.warmup):
        token()
    torch.cuda.synchronize()
    warm_bytes = state["bytes"]
    ms, clocks = timed_loop(token, args.steps, 0, dist, dist.local)
    step_bytes = (state["bytes"] - warm_bytes) / args.steps
    total = dist.sum(step_bytes)
    gbs = total * args.steps / (ms * 1e-3) / 1e9
    b.workspace.check()

    # end to end: each token's q/k/v of every layer from pinned host memory,
    # the last layer's attention output back to the host
    qh, kh, vh = q.cpu().pin_memory(), kn.cpu().pin_memory(), vn.cpu().pin_memory()
    oh = torch.empty(n_req, H, d, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream()

    def token_e2e():
        q.copy_(qh, non_blocking=True)
        kn.copy_(kh, non_blocking=True)
        vn.copy_(vh, non_blocking=True)
        token()
        oh.copy_(out, non_blocking=True)
        stream.synchronize()

    n = max(5, min(args.steps, 100))
    for _ in range(2):
        token_e2e()
    dist.barrier()
    torch.cuda.synchronize()
    b0 = state["bytes"]
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n):
        token_e2e()
    e.record(stream)
    torch.cuda.synchronize()
    ems = dist.max(a.elapsed_time(e))
    e2e = {"value": round(dist.sum((state["bytes"] - b0) / n) * n / (ems * 1e-3) / 1e9, 1), "unit": "GB/s",
           "h2d_bytes_per_step": (qh.numel() + kh.numel() + vh.numel()) * 4, "d2h_bytes_per_step": oh.numel() * 4,
           "steps": n, "ms_per_step": round(ems / n, 4),
           "tokens_per_s": round(dist.sum(n_req) * n / (ems * 1e-3), 1)}
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    ach = step_bytes / (ms / args.steps * 1e-3) / 1e9
    res.update({"metric": DECODE_METRIC, "value": round(gbs, 1), "unit": "GB/s",
                "ms_per_step": round(ms / args.steps, 5), "scaling": "weak", "dtype": "f32 (bf16 KV)",
                "config": {"workload": "serving", "n_requests": n_req, "n_layers": n_layers, "n_heads": H,
                           "n_kv_heads": Hkv, "head_dim": d, "kv_dtype": "bf16", "prompts": "U[1024,4096] seed 6",
                           "churn": "longest request leaves, a new one joins, every 8 steps",
                           "tokens_per_s": round(dist.sum(n_req) * args.steps / (ms * 1e-3), 1),
                           "l2": "~10 GB of KV read per step vs 126 MB L2"},
                "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(ach / hbm, 4), "frac_spec": round(ach / SPEC_PEAKS["hbm_gbs"], 4),
                             "traffic": None,
                             "kernel": "decode_bulk_kernel + slot_merge_kernel + rope_append_rows_kernel, 32 layers per step",
                             "algorithmic_bytes_per_step": round(step_bytes)},
                "clocks": clocks, "e2e": e2e, "gpu_launches": args.steps * n_layers * 3})
    emit(res, dist)


def run_reference(args):
    """CPU restatement of the reference path, timed on the host cores.  Under
    torchrun only rank 0 works; the others exit at once."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl = args.workload
    threads = host_threads()
    total = args.steps + args.warmup
    per_step = max(0.05, min(2.0, 60.0 / max(total, 1)))
    if wl == "llama3_prefill":
        unit, metric_v = "TFLOP/s", None
        vals = []
        for i in range(total):
            v, thr, desc = cpu_prefill_sample(per_step)
            if i >= args.warmup:
                vals.append(v)
    else:
        unit = "GB/s"
        vals = []
        for i in range(total):
            v, thr, desc = cpu_decode_sample(wl, per_step)
            if i >= args.warmup:
                vals.append(v)
    metric_v = statistics.median(vals)
    line = {"impl": "reference", "metric": DECODE_METRIC, "value": round(metric_v, 4), "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "vs_baseline": None, "dtype": "f32 dot / f64 P.V (reference arithmetic)",
            "data": "synthetic: seeded N(0,1) (numpy PCG64)",
            "config": {"workload": wl},
            "cpu_baseline": {"value": round(metric_v, 4), "unit": unit, "cores": threads, "kind": "port",
                             "sample": desc + f"; median of {len(vals)} steps"},
            "e2e": {"value": round(metric_v, 4), "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "reference is Rust (no cargo/rustc here): timed via the C restatement in oracle/"}
    print(json.dumps(line), flush=True)


def emit(res, dist):
    if dist.rank == 0:
        print(json.dumps(res), flush=True)
    dist.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="llama3_decode",
                    choices=["llama3_decode", "batched_tinyllama", "longctx", "llama3_prefill", "serving", "gemv",
                             "gguf_load"])
    ap.add_argument("--prefill-steps", type=int, default=200)
    ap.add_argument("--prefill-n", type=int, default=4, help="prefill sequences (llama3_prefill)")
    ap.add_argument("--prefill-s", type=int, default=8192, help="prefill tokens per sequence")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-sub", action="store_true",
                    help="default line without its batched_tinyllama and longctx objects")
    ap.add_argument("--kvsplit", default="peer", choices=["peer", "nccl"],
                    help="longctx over several GPUs: exchange inside the decode kernel (peer) or NCCL all-gather")
    ap.add_argument("--sub-steps", type=int, default=500,
                    help="timed steps of the batched_tinyllama and longctx objects (at least --steps)")
    ap.add_argument("--gguf-threads", type=int, default=8, help="host threads of bml_gguf_upload (gguf_load)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        log("warm-up raised to 3 steps (minimum)")
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
