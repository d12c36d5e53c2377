// lib.rs -- safe wrapper keeping the reference's HashConsedKV signatures
// (crates/compiler/src/kv_cache.rs:53-180 in SugarFreeDoNoSo/bml) over the
// device-resident cache of libbmlattn.so.  BML_E_INVALID panics, exactly
// where the reference's slice indexing would.
pub mod ffi;
use ffi::*;

fn check(s: bml_status) {
    if s == BML_OK { return; }
    let msg = unsafe { std::ffi::CStr::from_ptr(bml_last_error()) }.to_string_lossy().into_owned();
    // BML_E_INVALID is exactly where kv_cache.rs panics (slice index out of range)
    panic!("bml-attn: {msg}");
}

/// Drop-in for crates/compiler/src/kv_cache.rs::HashConsedKV, backed by HBM.
pub struct HashConsedKV { raw: *mut bml_kv, head_dim: u32 }

impl HashConsedKV {
    pub fn new(n_layers: u32, n_kv_heads: u32, head_dim: u32, max_seq_len: u32) -> Self {
        let d = bml_kv_desc { n_layers, n_kv_heads, head_dim, max_seq_len, dtype: bml_dtype::F32, device: 0 };
        let mut raw = std::ptr::null_mut();
        check(unsafe { bml_kv_create(&d, &mut raw) });
        Self { raw, head_dim }
    }
    pub fn store_k(&mut self, layer: u32, pos: u32, kv_head: u32, data: &[f32]) {
        check(unsafe { bml_kv_store(self.raw, 0, layer, pos, kv_head, data.as_ptr(), data.len()) });
    }
    pub fn store_v(&mut self, layer: u32, pos: u32, kv_head: u32, data: &[f32]) {
        check(unsafe { bml_kv_store(self.raw, 1, layer, pos, kv_head, data.as_ptr(), data.len()) });
    }
    pub fn load_k(&self, layer: u32, pos: u32, kv_head: u32) -> Vec<f32> {
        let mut v = vec![0.0; self.head_dim as usize];
        check(unsafe { bml_kv_load(self.raw, 0, layer, pos, kv_head, v.as_mut_ptr()) });
        v
    }
    pub fn load_v(&self, layer: u32, pos: u32, kv_head: u32) -> Vec<f32> {
        let mut v = vec![0.0; self.head_dim as usize];
        check(unsafe { bml_kv_load(self.raw, 1, layer, pos, kv_head, v.as_mut_ptr()) });
        v
    }
    pub fn dot_qk(&self, q: &[f32], layer: u32, pos: u32, kv_head: u32) -> f32 {
        let mut out = 0.0;
        check(unsafe { bml_kv_dot_qk(self.raw, q.as_ptr(), q.len(), layer, pos, kv_head, &mut out) });
        out
    }
    pub fn k_stats(&self) -> (usize, usize, f64) { self.stats(0) }
    pub fn v_stats(&self) -> (usize, usize, f64) { self.stats(1) }
    fn stats(&self, which: i32) -> (usize, usize, f64) {
        let (mut u, mut t, mut r) = (0u64, 0u64, 0f64);
        check(unsafe { bml_kv_stats(self.raw, which, &mut u, &mut t, &mut r) });
        (u as usize, t as usize, r)
    }
    pub fn byte_size(&self) -> usize {
        let mut b = 0u64;
        check(unsafe { bml_kv_byte_size(self.raw, &mut b) });
        b as usize
    }
    pub fn current_pos(&self) -> u32 {
        let mut p = 0;
        check(unsafe { bml_kv_current_pos(self.raw, &mut p) });
        p
    }
    pub fn advance(&mut self) { check(unsafe { bml_kv_advance(self.raw) }) }
    pub fn advance_by(&mut self, n: u32) { check(unsafe { bml_kv_advance_by(self.raw, n) }) }
    pub fn raw(&mut self) -> *mut bml_kv { self.raw }
}

impl Drop for HashConsedKV {
    fn drop(&mut self) { unsafe { bml_kv_destroy(self.raw); } }
}
