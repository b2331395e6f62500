//! The `flash-attention-cpu` crate's public API, with the attention forward
//! running on NVIDIA B200 GPUs (hand-written sm_100a CUDA in libfa_b200.so,
//! reached through the C ABI of include/fa_b200.h).
//!
//! Same items, signatures and behaviour as the crate (src/lib.rs:60-87):
//! `FlashAttentionConfig` (default 64 / 128 / false), `flash_attention_v1`,
//! `_v2`, `_v3` and their `_multihead` forms (also under the modules `v1`,
//! `v2`, `v3`), the aliases `flash_attention` / `flash_attention_multihead`
//! (v2), and the `naive` module.  A length mismatch panics with the crate's
//! messages; a zero-sized dimension returns with `out` untouched.  v1, v2
//! and v3 compute the same function and run the same GPU kernels.  The
//! block sizes are accepted and do not change the result.
//!
//! Beyond the crate, [`gpu`] sets the arithmetic (TF32, error-compensated
//! 3xTF32 (the default), f32), the devices a call spreads over, and gives the
//! device-resident forward.  Any failure other than a length mismatch (no
//! usable GPU, a CUDA error, a kernel's bounded wait running out) panics with
//! the library's message: there is no CPU fallback.
#![warn(missing_docs)]

mod ffi;
pub mod naive;

use std::ffi::CStr;

/// Tuning knobs of the crate (src/common.rs:16-36).  On the GPU the tiling
/// does not depend on them; they are validated and passed along.
#[derive(Debug, Clone, Copy)]
pub struct FlashAttentionConfig {
    /// Query rows per tile (`Br`).
    pub block_size_q: usize,
    /// Key/value rows per inner tile (`Bc`).
    pub block_size_kv: usize,
    /// Query position `i` sees key positions `<= i` only (top-left aligned).
    pub causal: bool,
}

impl Default for FlashAttentionConfig {
    fn default() -> Self {
        FlashAttentionConfig { block_size_q: 64, block_size_kv: 128, causal: false }
    }
}

fn to_c(config: &FlashAttentionConfig) -> ffi::FaConfig {
    ffi::FaConfig {
        block_size_q: config.block_size_q,
        block_size_kv: config.block_size_kv,
        causal: config.causal as u8,
    }
}

fn last_error() -> String {
    // SAFETY: fa_last_error returns a NUL-terminated thread-local string that
    // stays valid until the next library call on this thread.
    unsafe { CStr::from_ptr(ffi::fa_last_error()) }.to_string_lossy().into_owned()
}

fn check(rc: i32) {
    if rc != 0 {
        panic!("flash-attention (B200): {}", last_error());
    }
}

#[allow(clippy::too_many_arguments)]
fn single(f: ffi::SingleFn, q: &[f32], k: &[f32], v: &[f32], seq_len_q: usize,
          seq_len_k: usize, d_head: usize, config: &FlashAttentionConfig, out: &mut [f32]) {
    assert_eq!(q.len(), seq_len_q * d_head, "q shape mismatch");
    assert_eq!(k.len(), seq_len_k * d_head, "k shape mismatch");
    assert_eq!(v.len(), seq_len_k * d_head, "v shape mismatch");
    assert_eq!(out.len(), seq_len_q * d_head, "out shape mismatch");
    if seq_len_q == 0 || seq_len_k == 0 || d_head == 0 {
        return;
    }
    let c = to_c(config);
    // SAFETY: every pointer comes with the length of its slice, and `out` is
    // borrowed mutably for the whole (synchronous) call.
    let rc = unsafe {
        f(q.as_ptr(), q.len(), k.as_ptr(), k.len(), v.as_ptr(), v.len(), seq_len_q, seq_len_k,
          d_head, &c, out.as_mut_ptr(), out.len())
    };
    check(rc);
}

#[allow(clippy::too_many_arguments)]
fn multi(f: ffi::MultiFn, q: &[f32], k: &[f32], v: &[f32], batch: usize, heads: usize,
         seq_len_q: usize, seq_len_k: usize, d_head: usize, config: &FlashAttentionConfig,
         out: &mut [f32]) {
    let (per_q, per_k) = (seq_len_q * d_head, seq_len_k * d_head);
    assert_eq!(q.len(), batch * heads * per_q);
    assert_eq!(k.len(), batch * heads * per_k);
    assert_eq!(v.len(), batch * heads * per_k);
    assert_eq!(out.len(), batch * heads * per_q);
    if batch * heads == 0 || seq_len_q == 0 || seq_len_k == 0 || d_head == 0 {
        return;
    }
    let c = to_c(config);
    // SAFETY: as in `single`.
    let rc = unsafe {
        f(q.as_ptr(), q.len(), k.as_ptr(), k.len(), v.as_ptr(), v.len(), batch, heads,
          seq_len_q, seq_len_k, d_head, &c, out.as_mut_ptr(), out.len())
    };
    check(rc);
}

macro_rules! variant_module {
    ($m:ident, $single:ident, $multi:ident, $csingle:ident, $cmulti:ident, $doc:literal) => {
        #[doc = $doc]
        pub mod $m {
            use super::{ffi, multi, single, FlashAttentionConfig};

            /// Single-head attention: `q`/`out` are `[seq_len_q, d_head]`, `k`/`v`
            /// `[seq_len_k, d_head]`, row-major f32.
            #[allow(clippy::too_many_arguments)]
            pub fn $single(q: &[f32], k: &[f32], v: &[f32], seq_len_q: usize, seq_len_k: usize,
                           d_head: usize, config: &FlashAttentionConfig, out: &mut [f32]) {
                single(ffi::$csingle, q, k, v, seq_len_q, seq_len_k, d_head, config, out)
            }

            /// Batched multi-head attention on `[batch, heads, seq, d_head]` buffers.
            #[allow(clippy::too_many_arguments)]
            pub fn $multi(q: &[f32], k: &[f32], v: &[f32], batch: usize, heads: usize,
                          seq_len_q: usize, seq_len_k: usize, d_head: usize,
                          config: &FlashAttentionConfig, out: &mut [f32]) {
                multi(ffi::$cmulti, q, k, v, batch, heads, seq_len_q, seq_len_k, d_head,
                      config, out)
            }
        }
    };
}

variant_module!(v1, flash_attention_v1, flash_attention_multihead_v1, fa_flash_attention_v1,
                fa_flash_attention_multihead_v1, "The crate's v1 entry points (src/v1.rs).");
variant_module!(v2, flash_attention_v2, flash_attention_multihead_v2, fa_flash_attention_v2,
                fa_flash_attention_multihead_v2, "The crate's v2 entry points (src/v2.rs).");
variant_module!(v3, flash_attention_v3, flash_attention_multihead_v3, fa_flash_attention_v3,
                fa_flash_attention_multihead_v3, "The crate's v3 entry points (src/v3.rs).");

pub use v1::{flash_attention_multihead_v1, flash_attention_v1};
pub use v2::{flash_attention_multihead_v2, flash_attention_v2};
pub use v3::{flash_attention_multihead_v3, flash_attention_v3};
pub use v2::flash_attention_multihead_v2 as flash_attention_multihead;
pub use v2::flash_attention_v2 as flash_attention;

/// Controls and calls of the GPU library that the crate has no counterpart for.
pub mod gpu {
    use super::{check, ffi};
    use std::os::raw::c_void;

    /// Arithmetic of the tensor-core path.
    #[derive(Debug, Clone, Copy, PartialEq, Eq)]
    pub enum Precision {
        /// tcgen05 kind::tf32: max abs error <= 2e-3.
        Tf32 = 0,
        /// Error-compensated hi*hi + hi*lo + lo*hi (the default): <= 2e-5.
        ThreeXTf32 = 1,
        /// f32 FMA on the CUDA cores.
        Fp32 = 2,
    }

    /// Sets the arithmetic of later calls (process-wide).
    pub fn set_precision(p: Precision) {
        // SAFETY: plain value argument.
        check(unsafe { ffi::fa_set_precision(p as i32) });
    }

    /// Devices the slice calls spread over (contiguous (batch, head) ranges per
    /// device; a long single head splits its keys).  Empty: one device.
    pub fn set_devices(devices: &[i32]) {
        // SAFETY: pointer and length of a live slice.
        check(unsafe { ffi::fa_set_devices(devices.as_ptr(), devices.len() as i32) });
    }

    /// The multihead forward on device memory, enqueued on `stream` (a
    /// cudaStream_t; null = the legacy default stream).  `lse` may be null.
    ///
    /// # Safety
    /// `q`, `out` must point to `batch*heads*seq_len_q*d_head` f32 of device
    /// memory, `k`, `v` to `batch*heads*seq_len_k*d_head`, `lse` (if not null)
    /// to `batch*heads*seq_len_q`, all on the current device and alive until
    /// the stream reaches the call.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn flash_attention_multihead_device(q: *const f32, k: *const f32, v: *const f32,
                                                   out: *mut f32, lse: *mut f32, batch: usize,
                                                   heads: usize, seq_len_q: usize,
                                                   seq_len_k: usize, d_head: usize, causal: bool,
                                                   stream: *mut c_void) {
        // SAFETY: the caller guarantees the buffers (see above).
        let rc = unsafe {
            ffi::fa_forward_device(q, k, v, out, lse, batch * heads, seq_len_q, seq_len_k, d_head,
                                   causal as i32, stream)
        };
        check(rc);
    }

    /// The multihead forward on host slices that also returns the row LSE
    /// (natural log of each row's scaled-score sum), as the backward needs it.
    /// Panics on a shape mismatch, like the crate's entry points.
    #[allow(clippy::too_many_arguments)]
    pub fn flash_attention_multihead_lse(q: &[f32], k: &[f32], v: &[f32], batch: usize,
                                         heads: usize, seq_len_q: usize, seq_len_k: usize,
                                         d_head: usize, causal: bool) -> (Vec<f32>, Vec<f32>) {
        let bh = batch * heads;
        assert_eq!(q.len(), bh * seq_len_q * d_head, "q shape mismatch");
        assert_eq!(k.len(), bh * seq_len_k * d_head, "k shape mismatch");
        assert_eq!(v.len(), bh * seq_len_k * d_head, "v shape mismatch");
        let mut out = vec![0.0f32; q.len()];
        let mut lse = vec![0.0f32; bh * seq_len_q];
        // SAFETY: every pointer covers the length checked above.
        check(unsafe {
            ffi::fa_flash_attention_multihead_lse(q.as_ptr(), k.as_ptr(), v.as_ptr(), bh,
                                                  seq_len_q, seq_len_k, d_head, causal as i32,
                                                  out.as_mut_ptr(), lse.as_mut_ptr())
        });
        (out, lse)
    }

    /// Gradients (dq, dk, dv) of the forward from its output `out`, row `lse`
    /// and the output gradient `dout` (the crate itself is forward-only).  At
    /// `Precision::Tf32` the tcgen05 kernels run (d_head 32, 64, 96, 128);
    /// otherwise exact f32 on the CUDA cores.
    #[allow(clippy::too_many_arguments)]
    pub fn flash_attention_backward(q: &[f32], k: &[f32], v: &[f32], out: &[f32], lse: &[f32],
                                    dout: &[f32], batch: usize, heads: usize, seq_len_q: usize,
                                    seq_len_k: usize, d_head: usize, causal: bool)
                                    -> (Vec<f32>, Vec<f32>, Vec<f32>) {
        let bh = batch * heads;
        let nq = bh * seq_len_q * d_head;
        let nk = bh * seq_len_k * d_head;
        assert_eq!(q.len(), nq, "q shape mismatch");
        assert_eq!(k.len(), nk, "k shape mismatch");
        assert_eq!(v.len(), nk, "v shape mismatch");
        assert_eq!(out.len(), nq, "out shape mismatch");
        assert_eq!(lse.len(), bh * seq_len_q, "lse shape mismatch");
        assert_eq!(dout.len(), nq, "dout shape mismatch");
        let (mut dq, mut dk, mut dv) = (vec![0.0f32; nq], vec![0.0f32; nk], vec![0.0f32; nk]);
        // SAFETY: every pointer covers the length checked above.
        check(unsafe {
            ffi::fa_flash_attention_backward(q.as_ptr(), k.as_ptr(), v.as_ptr(), out.as_ptr(),
                                             lse.as_ptr(), dout.as_ptr(), dq.as_mut_ptr(),
                                             dk.as_mut_ptr(), dv.as_mut_ptr(), bh, seq_len_q,
                                             seq_len_k, d_head, causal as i32)
        });
        (dq, dk, dv)
    }

    /// Waits for `stream` and panics if a kernel of this library hit its
    /// bounded-wait limit (how the asynchronous device calls report failures).
    ///
    /// # Safety
    /// `stream` must be a live cudaStream_t of the current device (or null).
    pub unsafe fn sync_status(stream: *mut c_void) {
        // SAFETY: the caller guarantees the stream.
        check(unsafe { ffi::fa_sync_status(stream) });
    }
}
