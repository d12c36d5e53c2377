"""GPU parity of each decode kernel family for 16-bit caches.

By default the library picks the TMA warp-MMA kernel for launches of up to
64 sequences and the bulk-copy warp-MMA kernel for larger ones;
BML_DECODE_KERNEL=tma / =bulk / =mma / =cuda forces one family (the
cp.async warp-MMA kernel is the fallback of both), and the library reads it
once per process, so each family runs in a child process.  Same oracle and 1e-4 tolerance as
test_decode_gpu.py, on ragged lengths around every tile edge, more than 64
sequences (the TMA kernel's per-launch limit) and a 2-slot split-K merge."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, ROOT)
import oracle
import bml_b200
from bml_b200 import workloads as W

EDGE = [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 129, 1000, 4099]
worst = 0.0
cases = [("bf16", 128, 8, 4), ("f16", 128, 8, 4), ("bf16", 64, 4, 8), ("f16", 64, 8, 2), ("bf16", 128, 2, 4),
         ("f16", 128, 4, 1)]
for dtype, d, n_kv, group in cases:
    rng = np.random.default_rng(7 + d + n_kv + group)
    lens = EDGE + list(rng.integers(1, 300, 60))  # 75 sequences: more than one TMA launch
    H = n_kv * group
    q = rng.standard_normal((len(lens), H, d), dtype=np.float32)
    ks, vs, kd, vd, code = [], [], [], [], None
    for L in lens:
        k = rng.standard_normal((int(L), n_kv, d), dtype=np.float32)
        v = rng.standard_normal((int(L), n_kv, d), dtype=np.float32)
        if dtype == "f16":
            k, v = k.astype(np.float16), v.astype(np.float16)
            kd.append(torch.from_numpy(k).cuda()); vd.append(torch.from_numpy(v).cuda())
        else:
            k, v, code = W.f32_to_bf16_bits(k), W.f32_to_bf16_bits(v), oracle.BF16
            kd.append(torch.from_numpy(k.view(np.int16)).cuda().view(torch.bfloat16))
            vd.append(torch.from_numpy(v.view(np.int16)).cuda().view(torch.bfloat16))
        ks.append(k); vs.append(v)
    got = bml_b200.decode_batched(torch.from_numpy(q).cuda(), kd, vd).cpu().numpy()
    want = oracle.attn_decode_batched(q, ks, vs, dtype=code)
    worst = max(worst, float(np.abs(got - want).max()))
print("WORST", worst)
"""


@pytest.mark.parametrize("family", ["auto", "bulk", "tma", "mma", "cuda"])
def test_decode_family_parity(cuda, family):
    env = dict(os.environ, BML_DECODE_KERNEL=family)
    res = subprocess.run([sys.executable, "-c", "ROOT = %r\n" % ROOT + CHILD], env=env, capture_output=True,
                         text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    worst = float(res.stdout.strip().split()[-1])
    assert worst < 1e-4, worst
