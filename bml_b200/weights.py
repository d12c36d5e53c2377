"""Torch-facing wrappers of the weight path (include/bml_weights.h): GGUF
tensor dequantisation and the x . W projections on the device.

Mirrors crates/compiler/src/gguf_compiler.rs in SugarFreeDoNoSo/bml:
read_tensor_f32 (:351-369, with dequantize_q4_0 / dequantize_q8_0 at
:405-470) and InferenceCompiler::matmul_f64 (:1239-1255), which reads the
weight pool at i*n_out + j with (n_in, n_out) = (dims[0], dims[1])
(load_tensor, :1333-1358).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .attention import _stream

GGUF_F32, GGUF_F16, GGUF_Q4_0, GGUF_Q8_0 = L.GGUF_F32, L.GGUF_F16, L.GGUF_Q4_0, L.GGUF_Q8_0
_BLOCK_BYTES = {GGUF_Q4_0: 18, GGUF_Q8_0: 34}


def _bytes(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA tensor")
    return t.view(torch.uint8) if t.dtype != torch.uint8 else t


def values_read(gguf_type: int, data_len: int, n_elems: int) -> int:
    """How many values read_tensor_f32 returns (gguf_compiler.rs:351-369)."""
    if gguf_type == GGUF_F32:
        return data_len // 4
    if gguf_type == GGUF_F16:
        return data_len // 2
    if gguf_type in _BLOCK_BYTES:
        return n_elems
    raise L.BmlUnsupported(L.BML_E_UNSUPPORTED, "read_tensor_f32", f"GGUF type {gguf_type}")


def read_tensor_f32(data: torch.Tensor, gguf_type: int, n_elems: int, out: torch.Tensor | None = None,
                    stream=None) -> torch.Tensor:
    """A tensor's stored bytes (device) -> its f32 values, as the reference's
    read_tensor_f32 decodes them (bit for bit)."""
    b = _bytes(data, "data")
    n = values_read(gguf_type, b.numel(), n_elems)
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device=b.device)
    elif out.dtype != torch.float32 or out.numel() < n or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous f32 tensor of at least {n} values")
    got = C.c_uint64()
    L.call("bml_read_tensor_f32", C.c_void_p(b.data_ptr()), b.numel(), gguf_type, n_elems,
           C.c_void_p(out.data_ptr()), C.byref(got), _stream(stream))
    return out[:got.value]


class WeightTensor:
    """One weight tensor on the device as stored in the GGUF file (quantized
    blocks stay quantized), with the reference's (n_in, n_out) view."""

    def __init__(self, data: torch.Tensor, gguf_type: int, dims):
        self.data = _bytes(data, "data")
        self.gguf_type = int(gguf_type)
        dims = [int(d) for d in dims]
        # load_tensor (gguf_compiler.rs:1341-1352)
        self.n_in, self.n_out = (dims[0], dims[1]) if len(dims) >= 2 else ((dims[0], 1) if dims else (0, 1))
        self.n_elems = 1
        for d in dims:
            self.n_elems *= d
        values_read(self.gguf_type, self.data.numel(), self.n_elems)  # rejects unread types
        self._ws = None

    @property
    def nbytes(self) -> int:
        return self.data.numel()

    def to_f32(self, stream=None) -> torch.Tensor:
        return read_tensor_f32(self.data, self.gguf_type, self.n_elems, stream=stream)

    def matmul_f64(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None,
                   overlap: bool = True) -> torch.Tensor:
        """y = x . W (gguf_compiler.rs:1239-1255); x, y f64 device vectors.

        overlap: the tensor's bytes are not written by the kernel launched
        just before (a WeightTensor's data is written once, by its upload),
        so the call may start streaming them while that kernel ends
        (bml_matmul_f64_static; same result bits).  False gives the plain
        bml_matmul_f64."""
        if not isinstance(x, torch.Tensor) or not x.is_cuda or x.dtype != torch.float64 or not x.is_contiguous():
            raise ValueError("x must be a contiguous f64 CUDA vector")
        if out is None:
            out = torch.empty(self.n_out, dtype=torch.float64, device=x.device)
        if self._ws is None:
            size = C.c_size_t()
            L.call("bml_matmul_workspace_size", self.n_out, C.byref(size))
            self._ws = torch.empty(size.value, dtype=torch.uint8, device=x.device)
        L.call("bml_matmul_f64_static" if overlap else "bml_matmul_f64", C.c_void_p(self.data.data_ptr()), self.nbytes,
               self.gguf_type, self.n_in, self.n_out,
               C.c_void_p(x.data_ptr()), x.numel(), C.c_void_p(out.data_ptr()), C.c_void_p(self._ws.data_ptr()),
               self._ws.numel(), _stream(stream))
        return out


def matmul_f64(w: WeightTensor, x: torch.Tensor, out: torch.Tensor | None = None, stream=None,
               overlap: bool = True) -> torch.Tensor:
    return w.matmul_f64(x, out=out, stream=stream, overlap=overlap)
