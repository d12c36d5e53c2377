"""The C ABI: the library loads, exports exactly what include/*.h
(bml_attn.h, bml_weights.h, bml_gguf.h and the test-only bml_diag.h) declares, and rejects bad arguments on the host
(no GPU needed: nothing is launched before validation passes)."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("bml_attn.h", "bml_weights.h", "bml_gguf.h",
                                                      "bml_diag.h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(bml_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def L():
    from bml_b200 import build
    build.build()
    import bml_b200._lib as lib
    return lib


def test_header_and_binding_agree(L):
    assert declared_functions() == sorted(L.SIGNATURES)


def test_library_exports_every_declared_symbol(L):
    lib = L.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (bml_[a-z0-9_]+)$", out, flags=re.M))
    assert exported == set(declared_functions())


def test_version_and_empty_error(L):
    assert b"sm_100a" in L.lib().bml_version()


def test_invalid_arguments_rejected_on_host(L):
    lib = L.lib()
    # n_heads not a multiple of n_kv (gguf_compiler.rs:1011 would mis-index)
    seqs = (L.bml_seq_desc * 1)(L.bml_seq_desc(16, 16, 8, 0))
    st = lib.bml_attn_decode_batched(seqs, 1, 6, 4, 64, L.BML_BF16, -1.0, 16, 16, 16, 1 << 20, None)
    assert st == L.BML_E_INVALID
    assert "multiple" in L.last_error()
    # zero-length sequence: the reference always attends over [0, pos]
    seqs = (L.bml_seq_desc * 1)(L.bml_seq_desc(16, 16, 0, 0))
    st = lib.bml_attn_decode_batched(seqs, 1, 32, 4, 64, L.BML_F16, -1.0, 16, 16, 16, 1 << 20, None)
    assert st == L.BML_E_INVALID
    # unsupported head_dim
    st = lib.bml_attn_decode_batched(seqs, 1, 32, 4, 96, L.BML_F16, -1.0, 16, 16, 16, 1 << 20, None)
    assert st == L.BML_E_UNSUPPORTED
    # misaligned q
    seqs = (L.bml_seq_desc * 1)(L.bml_seq_desc(16, 16, 4, 0))
    st = lib.bml_attn_decode_batched(seqs, 1, 32, 4, 64, L.BML_F16, -1.0, 20, 16, 16, 1 << 20, None)
    assert st == L.BML_E_INVALID
    # too small a workspace
    st = lib.bml_attn_decode_batched(seqs, 1, 32, 4, 64, L.BML_F16, -1.0, 16, 16, 16, 64, None)
    assert st == L.BML_E_INVALID and "workspace" in L.last_error()
    # prefill shape checks
    st = lib.bml_attn_prefill(16, 16, 16, 1, 8, 6, 4, 64, L.BML_BF16, -1.0, 1, 16, L.BML_F32, None)
    assert st == L.BML_E_INVALID
    st = lib.bml_attn_prefill(16, 16, 16, 1, 8, 32, 4, 64, L.BML_F32, -1.0, 1, 16, L.BML_F32, None)
    assert st == L.BML_E_UNSUPPORTED
    # kv handle creation with a zero dimension
    h = C.c_void_p()
    desc = L.bml_kv_desc(1, 0, 64, 16, L.BML_F32, 0)
    assert lib.bml_kv_create(C.byref(desc), C.byref(h)) == L.BML_E_INVALID
    assert not h.value
    # merge with zero parts
    assert lib.bml_attn_merge_lse(16, 16, 16, 0, 4, 64, 16, None) == L.BML_E_INVALID
    # softmax of an empty row is a valid no-op (kv_cache.rs:189-191)
    assert lib.bml_softmax_f32(None, 1, 0, None, None) == L.BML_OK


def test_workspace_size_query(L):
    size = C.c_size_t()
    assert L.lib().bml_attn_decode_workspace_size(64, 32, 64, 0, C.byref(size)) == L.BML_OK
    assert size.value > 64 * 32 * 66 * 4
    big = C.c_size_t()
    L.lib().bml_attn_decode_workspace_size(100000, 32, 64, 0, C.byref(big))
    assert big.value < (1 << 30)  # launches are chunked, scratch does not grow without bound


def test_python_errors_are_typed(L):
    import bml_b200
    with pytest.raises(bml_b200.BmlInvalid):
        L.call("bml_attn_merge_lse", 16, 16, 16, 0, 4, 64, 16, None)


def test_weight_path_rejects_on_host(L):
    lib = L.lib()
    n = C.c_uint64()
    # a GGUF type the reference does not read (Q4_K)
    assert lib.bml_read_tensor_f32(16, 144, 12, 256, 16, C.byref(n), None) == L.BML_E_UNSUPPORTED
    # quantized tensor with n_out not a multiple of 32
    assert lib.bml_matmul_f64(16, 18 * 8, L.GGUF_Q4_0, 16, 16, 16, 16, 16, None, 0, None) == L.BML_E_UNSUPPORTED
    # misaligned F32 weights
    assert lib.bml_matmul_f64(18, 64, L.GGUF_F32, 4, 4, 16, 4, 16, None, 0, None) == L.BML_E_INVALID
    # the static-weights entry validates the same way
    assert lib.bml_matmul_f64_static(16, 18 * 8, L.GGUF_Q4_0, 16, 16, 16, 16, 16, None, 0, None) == L.BML_E_UNSUPPORTED
    assert lib.bml_matmul_f64_static(18, 64, L.GGUF_F32, 4, 4, 16, 4, 16, None, 0, None) == L.BML_E_INVALID
    size = C.c_size_t()
    assert lib.bml_matmul_workspace_size(4096, C.byref(size)) == L.BML_OK and size.value == 160 * 4096 * 8


def test_rust_binding_declares_every_product_entry_point():
    """crates/bml-attn-cuda/src/ffi.rs (the binding a bml maintainer adds)
    declares exactly the product entry points of bml_attn.h, bml_weights.h
    and bml_gguf.h; the test-only bml_diag.h is left out."""
    text = open(os.path.join(ROOT, "crates", "bml-attn-cuda", "src", "ffi.rs")).read()
    rust = set(re.findall(r"pub fn (bml_[a-z0-9_]+)\s*\(", text))
    product = set()
    for h in ("bml_attn.h", "bml_weights.h", "bml_gguf.h"):
        t = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", h)).read(), flags=re.S)
        product |= set(re.findall(r"\b(bml_[a-z0-9_]+)\s*\(", t))
    assert rust == product, (sorted(product - rust), sorted(rust - product))
