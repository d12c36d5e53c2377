"""The C++ mirror of the Rust API (include/bml_attn.hpp): the reference's
kv_cache.rs tests ported to C++, compiled against libbmlattn.so here and run
on the GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "test_kv_cache.cpp")
EXE = os.path.join(ROOT, "tests", "cpp", "test_kv_cache")


def build_exe():
    from bml_b200 import build
    lib = build.build()
    libdir = os.path.dirname(lib)
    cmd = [build.nvcc_path(), "-std=c++17", "-O2", "-x", "cu", SRC, "-o", EXE,
           f"-L{libdir}", "-lbmlattn", f"-Xlinker=-rpath={libdir}"]
    subprocess.run(cmd, check=True)
    return EXE


def test_cpp_mirror_compiles():
    """Compiles on CPU (nvcc is present here)."""
    assert os.path.exists(build_exe())


@pytest.mark.gpu
def test_cpp_reference_kv_tests_on_gpu(cuda):
    exe = build_exe()
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("ok ") == 9, r.stdout
