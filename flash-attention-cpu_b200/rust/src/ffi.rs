//! Declarations of the C ABI (include/fa_b200.h) that this crate binds.
use std::os::raw::{c_char, c_int, c_void};

/// `fa_config`: the crate's `FlashAttentionConfig` as a C struct.
#[repr(C)]
pub struct FaConfig {
    pub block_size_q: usize,
    pub block_size_kv: usize,
    pub causal: u8,
}

pub type SingleFn = unsafe extern "C" fn(
    q: *const f32,
    q_len: usize,
    k: *const f32,
    k_len: usize,
    v: *const f32,
    v_len: usize,
    seq_len_q: usize,
    seq_len_k: usize,
    d_head: usize,
    config: *const FaConfig,
    out: *mut f32,
    out_len: usize,
) -> c_int;

pub type MultiFn = unsafe extern "C" fn(
    q: *const f32,
    q_len: usize,
    k: *const f32,
    k_len: usize,
    v: *const f32,
    v_len: usize,
    batch: usize,
    heads: usize,
    seq_len_q: usize,
    seq_len_k: usize,
    d_head: usize,
    config: *const FaConfig,
    out: *mut f32,
    out_len: usize,
) -> c_int;

extern "C" {
    pub fn fa_flash_attention_v1(q: *const f32, q_len: usize, k: *const f32, k_len: usize,
        v: *const f32, v_len: usize, seq_len_q: usize, seq_len_k: usize, d_head: usize,
        config: *const FaConfig, out: *mut f32, out_len: usize) -> c_int;
    pub fn fa_flash_attention_v2(q: *const f32, q_len: usize, k: *const f32, k_len: usize,
        v: *const f32, v_len: usize, seq_len_q: usize, seq_len_k: usize, d_head: usize,
        config: *const FaConfig, out: *mut f32, out_len: usize) -> c_int;
    pub fn fa_flash_attention_v3(q: *const f32, q_len: usize, k: *const f32, k_len: usize,
        v: *const f32, v_len: usize, seq_len_q: usize, seq_len_k: usize, d_head: usize,
        config: *const FaConfig, out: *mut f32, out_len: usize) -> c_int;
    pub fn fa_flash_attention_multihead_v1(q: *const f32, q_len: usize, k: *const f32,
        k_len: usize, v: *const f32, v_len: usize, batch: usize, heads: usize,
        seq_len_q: usize, seq_len_k: usize, d_head: usize, config: *const FaConfig,
        out: *mut f32, out_len: usize) -> c_int;
    pub fn fa_flash_attention_multihead_v2(q: *const f32, q_len: usize, k: *const f32,
        k_len: usize, v: *const f32, v_len: usize, batch: usize, heads: usize,
        seq_len_q: usize, seq_len_k: usize, d_head: usize, config: *const FaConfig,
        out: *mut f32, out_len: usize) -> c_int;
    pub fn fa_flash_attention_multihead_v3(q: *const f32, q_len: usize, k: *const f32,
        k_len: usize, v: *const f32, v_len: usize, batch: usize, heads: usize,
        seq_len_q: usize, seq_len_k: usize, d_head: usize, config: *const FaConfig,
        out: *mut f32, out_len: usize) -> c_int;
    pub fn fa_forward_device(q: *const f32, k: *const f32, v: *const f32, out: *mut f32,
        lse: *mut f32, batch_heads: usize, seq_len_q: usize, seq_len_k: usize, d_head: usize,
        causal: c_int, stream: *mut c_void) -> c_int;
    pub fn fa_flash_attention_multihead_lse(q: *const f32, k: *const f32, v: *const f32,
        batch_heads: usize, seq_len_q: usize, seq_len_k: usize, d_head: usize, causal: c_int,
        out: *mut f32, lse: *mut f32) -> c_int;
    pub fn fa_flash_attention_backward(q: *const f32, k: *const f32, v: *const f32,
        out: *const f32, lse: *const f32, dout: *const f32, dq: *mut f32, dk: *mut f32,
        dv: *mut f32, batch_heads: usize, seq_len_q: usize, seq_len_k: usize, d_head: usize,
        causal: c_int) -> c_int;
    pub fn fa_sync_status(stream: *mut c_void) -> c_int;
    pub fn fa_set_precision(precision: c_int) -> c_int;
    pub fn fa_set_devices(devices: *const c_int, n: c_int) -> c_int;
    pub fn fa_last_error() -> *const c_char;
}
