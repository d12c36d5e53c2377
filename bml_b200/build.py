"""Builds libbmlattn.so (the CUDA library behind include/bml_attn.h) in-tree
for sm_100a with nvcc.  No JIT cache is involved: the .so sits next to this
file and travels with the source tree."""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libbmlattn.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


BUILD_DIR = os.path.join(HERE, "_build")
FLAGS = ["-std=c++17", "-O3", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden"]


def headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(HERE, "..", "include", "*.h"))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(d) > t for d in sources() + headers())


def _object(src: str, newest_header: float, force: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
    if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header):
        cmd = [nvcc_path(), *FLAGS, "-c", "-o", obj + ".tmp", src]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        os.replace(obj + ".tmp", obj)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles every csrc/*.cu to an object (in parallel, each only when it
    or a header changed) and links libbmlattn.so."""
    if not force and not needs_build():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    os.makedirs(BUILD_DIR, exist_ok=True)
    newest = max((os.path.getmtime(h) for h in headers()), default=0.0)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda f: _object(f, newest, force, verbose), srcs))
    subprocess.run([nvcc_path(), *ARCH, "-shared", "-o", LIB + ".tmp", *objs], check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
