// ffi.rs -- one declaration per entry point of include/bml_attn.h,
// bml_weights.h and bml_gguf.h (libbmlattn.so).
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

pub type bml_status = i32;
pub const BML_OK: bml_status = 0;
pub const BML_E_INVALID: bml_status = 1;
pub const BML_E_CUDA: bml_status = 2;
pub const BML_E_TIMEOUT: bml_status = 4;
pub const BML_E_OOM: bml_status = 5;
pub const BML_E_UNSUPPORTED: bml_status = 6;
#[repr(C)] #[derive(Clone, Copy)] pub enum bml_dtype { F32 = 0, F16 = 1, BF16 = 2 }
#[repr(C)] pub struct bml_kv { _p: [u8; 0] }
#[repr(C)] pub struct bml_kv_desc {
    pub n_layers: u32, pub n_kv_heads: u32, pub head_dim: u32, pub max_seq_len: u32,
    pub dtype: bml_dtype, pub device: i32,
}
#[repr(C)] pub struct bml_seq_desc { pub k_dev: *const c_void, pub v_dev: *const c_void, pub len: u32, pub reserved: u32 }
#[repr(C)] pub struct bml_gguf { _p: [u8; 0] }
#[repr(C)] pub struct bml_kvsplit { _p: [u8; 0] }
pub const BML_KVSPLIT_HANDLE_BYTES: usize = 64;
#[repr(C)] pub struct bml_gguf_header {
    pub magic: u32, pub version: u32, pub tensor_count: u64, pub metadata_kv_count: u64,
    pub data_offset: u64, pub file_size: u64,
}
#[repr(C)] pub struct bml_gguf_tensor {
    pub name: *const c_char, pub name_len: u64, pub n_dims: u32, pub type_: u32, pub dims: *const u64,
    pub offset: u64, pub present: i32, pub data_offset: u64, pub view_len: u64, pub nbytes: u64,
}
#[repr(C)] pub struct bml_gguf_value {
    pub type_: u32, pub elem_type: u32, pub len: u64, pub u: u64, pub i: i64, pub f: f64, pub str_: *const c_char,
}

extern "C" {
    pub fn bml_last_error() -> *const c_char;
    pub fn bml_version() -> *const c_char;
    pub fn bml_kv_create(desc: *const bml_kv_desc, out: *mut *mut bml_kv) -> bml_status;
    pub fn bml_kv_destroy(kv: *mut bml_kv) -> bml_status;
    pub fn bml_kv_store(kv: *mut bml_kv, which: c_int, layer: u32, pos: u32, kv_head: u32,
                        data: *const f32, len: usize) -> bml_status;
    pub fn bml_kv_load(kv: *const bml_kv, which: c_int, layer: u32, pos: u32, kv_head: u32,
                       out: *mut f32) -> bml_status;
    pub fn bml_kv_dot_qk(kv: *const bml_kv, q: *const f32, q_len: usize, layer: u32, pos: u32,
                         kv_head: u32, out: *mut f32) -> bml_status;
    pub fn bml_kv_stats(kv: *const bml_kv, which: c_int, unique: *mut u64, total: *mut u64,
                        ratio: *mut f64) -> bml_status;
    pub fn bml_kv_byte_size(kv: *const bml_kv, out: *mut u64) -> bml_status;
    pub fn bml_kv_current_pos(kv: *const bml_kv, out: *mut u32) -> bml_status;
    pub fn bml_kv_advance(kv: *mut bml_kv) -> bml_status;
    pub fn bml_kv_advance_by(kv: *mut bml_kv, n: u32) -> bml_status;
    pub fn bml_kv_layer_ptr(kv: *const bml_kv, which: c_int, layer: u32, out: *mut *mut c_void) -> bml_status;
    pub fn bml_kv_append(kv: *mut bml_kv, layer: u32, pos: u32, k: *const c_void, v: *const c_void,
                         src: bml_dtype, stream: *mut c_void) -> bml_status;
    pub fn bml_kv_append_rope(kv: *mut bml_kv, layer: u32, pos: u32, q: *mut f32, n_heads: u32,
                              k: *const f32, v: *const f32, stream: *mut c_void) -> bml_status;
    pub fn bml_kv_append_batched(seqs: *const bml_seq_desc, n_seqs: u32, n_kv: u32, head_dim: u32,
                                 kv: bml_dtype, k: *const c_void, v: *const c_void, src: bml_dtype,
                                 stream: *mut c_void) -> bml_status;
    pub fn bml_kv_append_rope_batched(seqs: *const bml_seq_desc, n_seqs: u32, n_heads: u32, n_kv: u32,
                                      head_dim: u32, kv: bml_dtype, q: *mut f32, k: *const f32,
                                      v: *const f32, stream: *mut c_void) -> bml_status;
    pub fn bml_attn_decode(kv: *mut bml_kv, layer: u32, pos: u32, n_heads: u32, scale: f32,
                           q: *const f32, out: *mut f32, stream: *mut c_void) -> bml_status;
    pub fn bml_attn_decode_wrap(kv: *mut bml_kv, layer: u32, pos: u32, n_heads: u32, scale: f32,
                                q: *const f32, out: *mut f32, stream: *mut c_void) -> bml_status;
    pub fn bml_attn_decode_workspace_size(n_seqs: u32, n_heads: u32, head_dim: u32, device: i32,
                                          bytes: *mut usize) -> bml_status;
    pub fn bml_attn_decode_batched(seqs: *const bml_seq_desc, n_seqs: u32, n_heads: u32, n_kv: u32,
                                   head_dim: u32, kv: bml_dtype, scale: f32, q: *const f32,
                                   out: *mut f32, ws: *mut c_void, ws_bytes: usize,
                                   stream: *mut c_void) -> bml_status;
    pub fn bml_attn_decode_batched_noalloc(seqs: *const bml_seq_desc, n_seqs: u32, n_heads: u32,
                                           n_kv: u32, head_dim: u32, kv: bml_dtype, scale: f32,
                                           q: *const f32, out: *mut f32,
                                           stream: *mut c_void) -> bml_status;
    pub fn bml_attn_decode_partial(seqs: *const bml_seq_desc, n_seqs: u32, n_heads: u32, n_kv: u32,
                                   head_dim: u32, kv: bml_dtype, scale: f32, q: *const f32,
                                   m: *mut f32, l: *mut f32, o: *mut f32, ws: *mut c_void,
                                   ws_bytes: usize, stream: *mut c_void) -> bml_status;
    pub fn bml_attn_merge_lse(m: *const f32, l: *const f32, o: *const f32, n_parts: u32, n_rows: u32,
                              head_dim: u32, out: *mut f32, stream: *mut c_void) -> bml_status;
    pub fn bml_attn_merge_lse_packed(parts: *const f32, n_parts: u32, n_rows: u32, head_dim: u32,
                                     out: *mut f32, stream: *mut c_void) -> bml_status;
    pub fn bml_attn_prefill(q: *const c_void, k: *const c_void, v: *const c_void, n_seqs: u32,
                            seq_len: u32, n_heads: u32, n_kv: u32, head_dim: u32, input: bml_dtype,
                            scale: f32, causal: c_int, out: *mut c_void, out_dtype: bml_dtype,
                            stream: *mut c_void) -> bml_status;
    pub fn bml_softmax_f32(x: *const f32, n_rows: u32, n: u32, out: *mut f32,
                           stream: *mut c_void) -> bml_status;
    pub fn bml_attn_workspace_check(ws: *mut c_void, bytes: usize, stream: *mut c_void) -> bml_status;
    pub fn bml_attn_noalloc_check(stream: *mut c_void) -> bml_status;
    pub fn bml_kvsplit_create(device: i32, rank: u32, world: u32, n_heads: u32, head_dim: u32,
                              out: *mut *mut bml_kvsplit) -> bml_status;
    pub fn bml_kvsplit_handle(h: *const bml_kvsplit, handle: *mut c_void, bytes: usize) -> bml_status;
    pub fn bml_kvsplit_open(h: *mut bml_kvsplit, handles: *const c_void, bytes: usize) -> bml_status;
    pub fn bml_attn_decode_kvsplit(h: *mut bml_kvsplit, slice: *const bml_seq_desc, n_heads: u32, n_kv: u32,
                                   head_dim: u32, kv: bml_dtype, scale: f32, q: *const f32, out: *mut f32,
                                   ws: *mut c_void, ws_bytes: usize, stream: *mut c_void) -> bml_status;
    pub fn bml_kvsplit_destroy(h: *mut bml_kvsplit) -> bml_status;

    // include/bml_weights.h -- read_tensor_f32 / matmul_f64 on the device
    pub fn bml_read_tensor_f32(data: *const c_void, data_len: u64, gguf_type: i32, n_elems: u64,
                               out: *mut f32, n_values: *mut u64, stream: *mut c_void) -> bml_status;
    pub fn bml_matmul_workspace_size(n_out: u64, bytes: *mut usize) -> bml_status;
    pub fn bml_matmul_f64(w: *const c_void, data_len: u64, gguf_type: i32, n_in: u64, n_out: u64,
                          x: *const f64, x_len: u64, y: *mut f64, ws: *mut c_void, ws_bytes: usize,
                          stream: *mut c_void) -> bml_status;
    pub fn bml_matmul_f64_static(w: *const c_void, data_len: u64, gguf_type: i32, n_in: u64, n_out: u64,
                                 x: *const f64, x_len: u64, y: *mut f64, ws: *mut c_void, ws_bytes: usize,
                                 stream: *mut c_void) -> bml_status;

    // include/bml_gguf.h -- GgufParser + upload to the device
    pub fn bml_gguf_open(path: *const c_char, out: *mut *mut bml_gguf) -> bml_status;
    pub fn bml_gguf_close(g: *mut bml_gguf) -> bml_status;
    pub fn bml_gguf_get_header(g: *const bml_gguf, out: *mut bml_gguf_header) -> bml_status;
    pub fn bml_gguf_tensor_info(g: *const bml_gguf, index: u64, out: *mut bml_gguf_tensor) -> bml_status;
    pub fn bml_gguf_find_tensor(g: *const bml_gguf, name: *const c_char, index: *mut u64) -> bml_status;
    pub fn bml_gguf_tensor_view(g: *const bml_gguf, index: u64, ptr: *mut *const c_void,
                                len: *mut u64) -> bml_status;
    pub fn bml_gguf_meta_key(g: *const bml_gguf, index: u64, key: *mut *const c_char,
                             key_len: *mut u64) -> bml_status;
    pub fn bml_gguf_meta_find(g: *const bml_gguf, key: *const c_char, index: *mut u64) -> bml_status;
    pub fn bml_gguf_meta_value(g: *const bml_gguf, index: u64, path: *const u64, depth: u32,
                               out: *mut bml_gguf_value) -> bml_status;
    pub fn bml_gguf_upload(g: *mut bml_gguf, indices: *const u64, n: u32, dst: *const *mut c_void,
                           threads: u32) -> bml_status;
}
