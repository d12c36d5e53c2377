"""bml_b200: B200-native (sm_100a) GQA attention over the KV cache, a drop-in
for the attention hot path of SugarFreeDoNoSo/bml.

The compute lives in libbmlattn.so (C ABI: include/bml_attn.h).  This
package is its host-side mirror of the reference interface:

  HashConsedKV       crates/compiler/src/kv_cache.rs:25-181
  softmax_f32        crates/compiler/src/kv_cache.rs:188-200
  HashConsedKV.attention / decode_batched
                     attention block of gguf_compiler.rs:1008-1050
  prefill            the forward_cached token loop, gguf_compiler.rs:946-958
  decode_partial / merge_lse
                     KV-split flash decoding (no reference counterpart)
  DecodeBatcher      continuous batching of decode steps, the batched form
                     of crates/api/src/main.rs:266-354's one-request loop
  read_tensor_f32 / WeightTensor.matmul_f64
                     gguf_compiler.rs:351-470 and :1239-1255 on the device
"""
from ._lib import BmlError, BmlInvalid, BmlUnsupported, last_error  # noqa: F401
from .attention import (SeqBatch, Workspace, decode_batched, decode_partial,  # noqa: F401
                        merge_lse, merge_lse_packed, prefill, softmax_f32)
from .kv_cache import HashConsedKV  # noqa: F401
from .batching import AtCapacity, DecodeBatcher, MAX_PENDING_REQUESTS  # noqa: F401
from .weights import WeightTensor, matmul_f64, read_tensor_f32  # noqa: F401
