"""ctypes binding of libbmlattn.so (include/bml_attn.h).

Loading fails loudly when the library has not been built: there is no CPU
fallback anywhere in this package."""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbmlattn.so")

BML_OK, BML_E_INVALID, BML_E_CUDA, BML_E_NCCL, BML_E_TIMEOUT, BML_E_OOM, BML_E_UNSUPPORTED = range(7)
BML_F32, BML_F16, BML_BF16 = 0, 1, 2
WHICH_K, WHICH_V = 0, 1

_STATUS_NAMES = {0: "BML_OK", 1: "BML_E_INVALID", 2: "BML_E_CUDA", 3: "BML_E_NCCL",
                 4: "BML_E_TIMEOUT", 5: "BML_E_OOM", 6: "BML_E_UNSUPPORTED"}


class BmlError(RuntimeError):
    """A non-OK bml_status, with the library's bml_last_error() message."""

    def __init__(self, status: int, fn: str, msg: str):
        super().__init__(f"{fn}: {_STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class BmlInvalid(BmlError, ValueError):
    """BML_E_INVALID: where the reference would panic on a bad index/shape."""


class BmlUnsupported(BmlError, NotImplementedError):
    """BML_E_UNSUPPORTED: a valid shape this library has no kernel for."""


class bml_kv_desc(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("max_seq_len", C.c_uint32), ("dtype", C.c_int), ("device", C.c_int32)]


class bml_seq_desc(C.Structure):
    _fields_ = [("k_dev", C.c_void_p), ("v_dev", C.c_void_p), ("len", C.c_uint32),
                ("reserved", C.c_uint32)]


class bml_gguf_header(C.Structure):
    _fields_ = [("magic", C.c_uint32), ("version", C.c_uint32), ("tensor_count", C.c_uint64),
                ("metadata_kv_count", C.c_uint64), ("data_offset", C.c_uint64), ("file_size", C.c_uint64)]


class bml_gguf_tensor(C.Structure):
    _fields_ = [("name", C.c_void_p), ("name_len", C.c_uint64), ("n_dims", C.c_uint32), ("type", C.c_uint32),
                ("dims", C.POINTER(C.c_uint64)), ("offset", C.c_uint64), ("present", C.c_int32),
                ("data_offset", C.c_uint64), ("view_len", C.c_uint64), ("nbytes", C.c_uint64)]


class bml_gguf_value(C.Structure):
    _fields_ = [("type", C.c_uint32), ("elem_type", C.c_uint32), ("len", C.c_uint64), ("u", C.c_uint64),
                ("i", C.c_int64), ("f", C.c_double), ("str", C.c_void_p)]


# name -> (restype, argtypes); mirrors include/bml_attn.h, bml_weights.h,
# bml_gguf.h and bml_diag.h one to one.
_vp, _u32, _i32, _st, _sz = C.c_void_p, C.c_uint32, C.c_int32, C.c_int32, C.c_size_t
GGUF_F32, GGUF_F16, GGUF_Q4_0, GGUF_Q8_0 = 0, 1, 2, 8  # include/bml_weights.h
SIGNATURES = {
    "bml_last_error": (C.c_char_p, []),
    "bml_version": (C.c_char_p, []),
    "bml_kv_create": (_st, [C.POINTER(bml_kv_desc), C.POINTER(_vp)]),
    "bml_kv_destroy": (_st, [_vp]),
    "bml_kv_store": (_st, [_vp, C.c_int, _u32, _u32, _u32, _vp, _sz]),
    "bml_kv_load": (_st, [_vp, C.c_int, _u32, _u32, _u32, _vp]),
    "bml_kv_dot_qk": (_st, [_vp, _vp, _sz, _u32, _u32, _u32, C.POINTER(C.c_float)]),
    "bml_kv_stats": (_st, [_vp, C.c_int, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                           C.POINTER(C.c_double)]),
    "bml_kv_byte_size": (_st, [_vp, C.POINTER(C.c_uint64)]),
    "bml_kv_current_pos": (_st, [_vp, C.POINTER(_u32)]),
    "bml_kv_advance": (_st, [_vp]),
    "bml_kv_advance_by": (_st, [_vp, _u32]),
    "bml_kv_layer_ptr": (_st, [_vp, C.c_int, _u32, C.POINTER(_vp)]),
    "bml_kv_append": (_st, [_vp, _u32, _u32, _vp, _vp, C.c_int, _vp]),
    "bml_kv_append_rope": (_st, [_vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp]),
    "bml_kv_append_batched": (_st, [C.POINTER(bml_seq_desc), _u32, _u32, _u32, C.c_int, _vp, _vp, C.c_int,
                                    _vp]),
    "bml_kv_append_rope_batched": (_st, [C.POINTER(bml_seq_desc), _u32, _u32, _u32, _u32, C.c_int, _vp, _vp,
                                         _vp, _vp]),
    "bml_attn_decode": (_st, [_vp, _u32, _u32, _u32, C.c_float, _vp, _vp, _vp]),
    "bml_attn_decode_wrap": (_st, [_vp, _u32, _u32, _u32, C.c_float, _vp, _vp, _vp]),
    "bml_attn_decode_workspace_size": (_st, [_u32, _u32, _u32, _i32, C.POINTER(_sz)]),
    "bml_attn_decode_batched": (_st, [C.POINTER(bml_seq_desc), _u32, _u32, _u32, _u32, C.c_int,
                                      C.c_float, _vp, _vp, _vp, _sz, _vp]),
    "bml_attn_decode_batched_noalloc": (_st, [C.POINTER(bml_seq_desc), _u32, _u32, _u32, _u32, C.c_int,
                                              C.c_float, _vp, _vp, _vp]),
    "bml_attn_decode_partial": (_st, [C.POINTER(bml_seq_desc), _u32, _u32, _u32, _u32, C.c_int,
                                      C.c_float, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "bml_attn_merge_lse": (_st, [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp]),
    "bml_attn_merge_lse_packed": (_st, [_vp, _u32, _u32, _u32, _vp, _vp]),
    "bml_attn_prefill": (_st, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, C.c_int, C.c_float,
                               C.c_int, _vp, C.c_int, _vp]),
    "bml_softmax_f32": (_st, [_vp, _u32, _u32, _vp, _vp]),
    # include/bml_weights.h
    "bml_read_tensor_f32": (_st, [_vp, C.c_uint64, _i32, C.c_uint64, _vp, C.POINTER(C.c_uint64), _vp]),
    "bml_matmul_workspace_size": (_st, [C.c_uint64, C.POINTER(_sz)]),
    "bml_matmul_f64": (_st, [_vp, C.c_uint64, _i32, C.c_uint64, C.c_uint64, _vp, C.c_uint64, _vp, _vp, _sz, _vp]),
    "bml_matmul_f64_static": (_st, [_vp, C.c_uint64, _i32, C.c_uint64, C.c_uint64, _vp, C.c_uint64, _vp, _vp, _sz, _vp]),
    # include/bml_gguf.h
    "bml_gguf_open": (_st, [C.c_char_p, C.POINTER(_vp)]),
    "bml_gguf_close": (_st, [_vp]),
    "bml_gguf_get_header": (_st, [_vp, C.POINTER(bml_gguf_header)]),
    "bml_gguf_tensor_info": (_st, [_vp, C.c_uint64, C.POINTER(bml_gguf_tensor)]),
    "bml_gguf_find_tensor": (_st, [_vp, C.c_char_p, C.POINTER(C.c_uint64)]),
    "bml_gguf_tensor_view": (_st, [_vp, C.c_uint64, C.POINTER(_vp), C.POINTER(C.c_uint64)]),
    "bml_gguf_meta_key": (_st, [_vp, C.c_uint64, C.POINTER(_vp), C.POINTER(C.c_uint64)]),
    "bml_gguf_meta_find": (_st, [_vp, C.c_char_p, C.POINTER(C.c_uint64)]),
    "bml_gguf_meta_value": (_st, [_vp, C.c_uint64, C.POINTER(C.c_uint64), _u32, C.POINTER(bml_gguf_value)]),
    "bml_gguf_upload": (_st, [_vp, C.POINTER(C.c_uint64), _u32, C.POINTER(_vp), _u32]),
    "bml_attn_workspace_check": (_st, [_vp, _sz, _vp]),
    "bml_attn_noalloc_check": (_st, [_vp]),
    "bml_kvsplit_create": (_st, [_i32, _u32, _u32, _u32, _u32, C.POINTER(_vp)]),
    "bml_kvsplit_handle": (_st, [_vp, _vp, _sz]),
    "bml_kvsplit_open": (_st, [_vp, _vp, _sz]),
    "bml_attn_decode_kvsplit": (_st, [_vp, C.POINTER(bml_seq_desc), _u32, _u32, _u32, C.c_int, C.c_float, _vp,
                                      _vp, _vp, _sz, _vp]),
    "bml_kvsplit_destroy": (_st, [_vp]),
    # include/bml_diag.h (test-only)
    "bml_diag_exp2": (_st, [_vp, _u32, _vp, _vp]),
    "bml_diag_decode_batched": (_st, [C.POINTER(bml_seq_desc), _u32, _u32, _u32, _u32, C.c_int,
                                      C.c_float, _vp, _vp, _vp, _sz, C.c_int, C.c_uint64, _u32, _vp]),
}

BML_DIAG_DECODE_DEFAULT, BML_DIAG_DECODE_CUDA_CORE = 0, 1  # include/bml_diag.h
BML_DIAG_STALL = 1
BML_KVSPLIT_HANDLE_BYTES = 64  # include/bml_attn.h

_lock = threading.Lock()
_lib = None


def lib() -> C.CDLL:
    """The loaded library; raises if it was never built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m bml_b200.build` "
                    "(or __graft_entry__.build()); this package has no CPU fallback")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    return lib().bml_last_error().decode()


def check(status: int, fn: str) -> None:
    if status == BML_OK:
        return
    msg = last_error()
    if status == BML_E_INVALID:
        raise BmlInvalid(status, fn, msg)
    if status == BML_E_UNSUPPORTED:
        raise BmlUnsupported(status, fn, msg)
    raise BmlError(status, fn, msg)


_fns: dict = {}


def call(fn: str, *args) -> None:
    f = _fns.get(fn)
    if f is None:
        f = _fns[fn] = getattr(lib(), fn)
    check(f(*args), fn)
