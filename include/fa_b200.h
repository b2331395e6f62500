/*
 * fa_b200.h -- C ABI of the B200 FlashAttention forward.
 *
 * A drop-in for the public API of the `flash-attention-cpu` crate (v0.2.0):
 * every crate entry point for the attention forward has one C function here
 * that a Rust (or any FFI) binding calls with the slice pointers and lengths.
 * The crate's shape checks, zero-dimension early return and block-size clamp
 * are honoured on this side; every compute step runs on the GPU in
 * hand-written sm_100a CUDA.  There is no CPU fallback: without a usable GPU
 * the calls return FA_ERR_NO_DEVICE.
 *
 * Conventions shared by every function below:
 *   - Tensors are f32, row-major, [heads, seq, d_head] (single-head calls:
 *     [seq, d_head]); K and V have seq_len_k rows, Q and OUT seq_len_q rows.
 *   - Causal masking is top-left aligned: query i sees key j iff j <= i
 *     (src/naive.rs:37-40, tests/correctness.rs:184-194), also when
 *     seq_len_q != seq_len_k.
 *   - Return value is an fa_status; on failure fa_last_error() returns a
 *     thread-local message.  A shape mismatch returns FA_ERR_SHAPE with the
 *     crate's assert message ("q shape mismatch", ...; src/common.rs:51-54).
 *   - Host-pointer calls are synchronous: OUT is complete when they return.
 *   - block_size_q / block_size_kv are accepted and validated (0 is clamped to
 *     1, src/v2.rs:172-173) but the GPU tiling does not depend on them, so
 *     results are identical for every block size.
 */
#ifndef FA_B200_H
#define FA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors `FlashAttentionConfig { block_size_q, block_size_kv, causal }`
 * (src/common.rs:16-22); fa_config_default() mirrors its Default impl
 * (src/common.rs:24-36: 64 / 128 / false). */
typedef struct fa_config {
  size_t block_size_q;
  size_t block_size_kv;
  uint8_t causal;
} fa_config;

typedef enum fa_status {
  FA_OK = 0,
  FA_ERR_SHAPE = 1,       /* length mismatch: the crate panics here */
  FA_ERR_ARG = 2,         /* null pointer / bad enum / size overflow */
  FA_ERR_CUDA = 3,        /* CUDA runtime error (message has details) */
  FA_ERR_TIMEOUT = 4,     /* a bounded in-kernel wait expired */
  FA_ERR_NO_DEVICE = 5,   /* no usable sm_100 GPU: there is no CPU fallback */
  FA_ERR_UNSUPPORTED = 6  /* shape outside what any kernel handles */
} fa_status;

/* Arithmetic of the tensor-core path.  Not part of the crate's config struct
 * (adding a field would break the crate's struct literals), so it is set out
 * of band: fa_set_precision() or the FA_B200_PRECISION environment variable
 * ("tf32", "3xtf32", "fp32"), read once at first use. */
typedef enum fa_precision {
  FA_PREC_TF32 = 0,   /* tcgen05 kind::tf32 MMAs: max abs err <= 2e-3 */
  FA_PREC_3XTF32 = 1, /* error-compensated (hi*hi + hi*lo + lo*hi): <= 2e-5 */
  FA_PREC_FP32 = 2    /* plain f32 FMA on the CUDA cores (exact f32) */
} fa_precision;

/* Default precision: FA_PREC_3XTF32, so the crate's own 1e-5 known-answer
 * test (tests/correctness.rs:240-263) passes through this library. */
FA_API fa_config fa_config_default(void);

/* ---- crate API, host slices (synchronous) ------------------------------ */

/* Replace flash_attention_v1 / _v2 / _v3 (src/v1.rs:51-60, src/v2.rs:49-58,
 * src/v3.rs:61-70).  The three schedules compute the same function; on the GPU
 * they run the same kernel family.  `fa_flash_attention` is the crate alias
 * `flash_attention` -> v2 (src/lib.rs:87). */
FA_API int fa_flash_attention_v1(const float* q, size_t q_len, const float* k, size_t k_len,
                          const float* v, size_t v_len, size_t seq_len_q,
                          size_t seq_len_k, size_t d_head, const fa_config* config,
                          float* out, size_t out_len);
FA_API int fa_flash_attention_v2(const float* q, size_t q_len, const float* k, size_t k_len,
                          const float* v, size_t v_len, size_t seq_len_q,
                          size_t seq_len_k, size_t d_head, const fa_config* config,
                          float* out, size_t out_len);
FA_API int fa_flash_attention_v3(const float* q, size_t q_len, const float* k, size_t k_len,
                          const float* v, size_t v_len, size_t seq_len_q,
                          size_t seq_len_k, size_t d_head, const fa_config* config,
                          float* out, size_t out_len);
FA_API int fa_flash_attention(const float* q, size_t q_len, const float* k, size_t k_len,
                       const float* v, size_t v_len, size_t seq_len_q, size_t seq_len_k,
                       size_t d_head, const fa_config* config, float* out, size_t out_len);

/* Replace flash_attention_multihead_v1 / _v2 / _v3 (src/v1.rs:134-159,
 * src/v2.rs:132-157, src/v3.rs:144-169; fan-out src/common.rs:72-101) and
 * the alias flash_attention_multihead -> v2 (src/lib.rs:86).  Buffers are
 * [batch, heads, seq, d_head]. */
FA_API int fa_flash_attention_multihead_v1(const float* q, size_t q_len, const float* k,
                                    size_t k_len, const float* v, size_t v_len,
                                    size_t batch, size_t heads, size_t seq_len_q,
                                    size_t seq_len_k, size_t d_head,
                                    const fa_config* config, float* out, size_t out_len);
FA_API int fa_flash_attention_multihead_v2(const float* q, size_t q_len, const float* k,
                                    size_t k_len, const float* v, size_t v_len,
                                    size_t batch, size_t heads, size_t seq_len_q,
                                    size_t seq_len_k, size_t d_head,
                                    const fa_config* config, float* out, size_t out_len);
FA_API int fa_flash_attention_multihead_v3(const float* q, size_t q_len, const float* k,
                                    size_t k_len, const float* v, size_t v_len,
                                    size_t batch, size_t heads, size_t seq_len_q,
                                    size_t seq_len_k, size_t d_head,
                                    const fa_config* config, float* out, size_t out_len);
FA_API int fa_flash_attention_multihead(const float* q, size_t q_len, const float* k,
                                 size_t k_len, const float* v, size_t v_len, size_t batch,
                                 size_t heads, size_t seq_len_q, size_t seq_len_k,
                                 size_t d_head, const fa_config* config, float* out,
                                 size_t out_len);

/* Same as fa_flash_attention_multihead_v2, plus the row log-sum-exp
 * lse[bh*seq_len_q] = log(sum_j exp(s_ij)) of the scaled scores (natural log;
 * -inf for a row that sees no key).  lse may be NULL.  No crate counterpart:
 * the crate does not expose the LSE; it is the parity side channel and the
 * input of the KV-split combine. */
FA_API int fa_flash_attention_multihead_lse(const float* q, const float* k, const float* v,
                                     size_t batch_heads, size_t seq_len_q,
                                     size_t seq_len_k, size_t d_head, int causal,
                                     float* out, float* lse);

/* ---- device-resident API (asynchronous on `stream`) -------------------- */

/* The multihead forward on DEVICE buffers of the current device, enqueued on
 * `stream` (a cudaStream_t; NULL = legacy default stream).  No crate
 * counterpart: it is the device-resident caller of the same kernels that the
 * host-slice calls use, for callers whose tensors already live in HBM. */
FA_API int fa_forward_device(const float* q, const float* k, const float* v, float* out,
                      float* lse, size_t batch_heads, size_t seq_len_q,
                      size_t seq_len_k, size_t d_head, int causal, void* stream);

/* Partial forward over the key range held in k/v (seq_len_k rows) whose first
 * key sits at global position k_offset, for queries whose first row sits at
 * global position q_offset (causal masking compares global positions).
 * Writes the range-normalised output and its LSE (-inf, zeros where a row sees
 * none of these keys).  Device buffers, async.  Used by the KV-range split
 * across GPUs; fa_lse_combine_device merges the partials. */
FA_API int fa_forward_partial_device(const float* q, const float* k, const float* v,
                              float* out, float* lse, size_t batch_heads,
                              size_t seq_len_q, size_t seq_len_k, size_t d_head,
                              int causal, size_t q_offset, size_t k_offset, void* stream);

/* Merge n_parts partial results, stored part-major as o_parts[n][rows][d] and
 * lse_parts[n][rows], into out[rows][d] and lse_out[rows] (nullable):
 * lse = log(sum_p exp(lse_p)), out = sum_p exp(lse_p - lse) * o_p.
 * Parts with lse_p = -inf get weight 0 (no NaN from -inf - -inf).  Device
 * buffers, async. */
FA_API int fa_lse_combine_device(const float* o_parts, const float* lse_parts, size_t n_parts,
                          size_t rows, size_t d_head, float* out, float* lse_out,
                          void* stream);

/* Allocation-free variant of the decode (few query rows) forward, for callers
 * that cannot allocate device memory while they run: code under an allocator
 * that forbids new device allocations, or a runtime that owns all device
 * memory and hands out only its own buffers.  No counterpart in the reference
 * (the crate never allocates device memory).  Same inputs, outputs and results
 * as fa_forward_device for seq_len_q <= 16, d_head % 4 == 0, d_head <= 256,
 * batch_heads <= 65535; the split partials live in a fixed 4 MiB device array
 * of this library (held on every GPU that loads it until exit) instead of a
 * per-call allocation, and a shape needing more than that is rejected with
 * FA_ERR_UNSUPPORTED.  The first call on a device looks the array's address
 * up (a CUDA runtime query, no allocation); make that first call before any
 * stream capture.  All calls on a device share the array: calls whose kernels
 * overlap on the GPU race (serialise them on one stream).  q, k, v and out
 * must be 16-byte aligned (the kernel reads them with 16-byte vector loads);
 * other pointers are refused with FA_ERR_UNSUPPORTED before any device call.
 * The device set by fa_set_device applies, as for every other call.  Device
 * buffers, asynchronous on `stream`. */
FA_API int fa_forward_decode_noalloc(const float* q, const float* k, const float* v, float* out,
                                     float* lse, size_t batch_heads, size_t seq_len_q,
                                     size_t seq_len_k, size_t d_head, int causal, void* stream);

/* ---- backward pass (no crate counterpart: the crate is forward-only) ------ */

/* Gradients of the forward: given Q, K, V, the forward output O and its row
 * LSE (from fa_flash_attention_multihead_lse / fa_forward_device) and dO,
 * writes dQ [bh, seq_len_q, d_head], dK and dV [bh, seq_len_k, d_head]; d_head
 * <= 128.  At FA_PREC_TF32 with d_head in {32, 64, 96, 128} and 16-byte
 * aligned buffers the tcgen05 kernels run (TF32 operands, f32 accumulation);
 * otherwise exact f32 on the CUDA cores.  Same causal convention as the
 * forward (top-left).  Device buffers, async on `stream`; a bounded-wait
 * failure surfaces through fa_sync_status. */
FA_API int fa_backward_device(const float* q, const float* k, const float* v, const float* out,
                              const float* lse, const float* dout, float* dq, float* dk,
                              float* dv, size_t batch_heads, size_t seq_len_q, size_t seq_len_k,
                              size_t d_head, int causal, void* stream);
/* The same on host buffers (synchronous; copies in and out). */
FA_API int fa_flash_attention_backward(const float* q, const float* k, const float* v,
                                       const float* out, const float* lse, const float* dout,
                                       float* dq, float* dk, float* dv, size_t batch_heads,
                                       size_t seq_len_q, size_t seq_len_k, size_t d_head,
                                       int causal);

/* Waits for `stream` and reports whether any kernel this library enqueued on
 * the current device has hit its bounded-wait limit since the last check
 * (FA_ERR_TIMEOUT; the flag is then cleared).  The device-resident calls are
 * asynchronous, so this is where their in-kernel failures surface. */
FA_API int fa_sync_status(void* stream);

/* Test hook of the failure path (no crate counterpart).  With skip_block >= 0,
 * one softmax thread (warp) of the first CTA (pair) of every later
 * tensor-core launch does not announce P of key block `skip_block` (counted
 * from the CTA's first block), so the MMA issuer's bounded wait for it runs
 * out: the kernel raises its abort flag, every role leaves, in-flight copies
 * and MMAs are drained, tensor memory is freed, and the call reports
 * FA_ERR_TIMEOUT.  wait_ns sets the limit of those abortable waits (0: the
 * default of 2 s).  fa_test_stall(-1, 0) restores normal operation.  Only
 * software arrives are withheld: no copy or MMA completion is skipped. */
FA_API int fa_test_stall(int skip_block, unsigned long long wait_ns);

/* ---- library control ---------------------------------------------------- */
FA_API int fa_set_precision(int precision); /* fa_precision */
FA_API int fa_get_precision(void);
/* Device used by the host-slice calls (default: the CUDA current device). */
FA_API int fa_set_device(int device);
/* Devices the host-slice calls (fa_flash_attention*, _multihead*, _lse) spread
 * over, one process driving them all.  The crate fans its (batch, head) slices
 * out over every core (src/common.rs:72-101); with n > 1 devices these calls
 * give each device a contiguous range of slices (its own copies over its own
 * host link, its own kernels; no collective), and a call with fewer slices
 * than devices on long sequences (seq_len_q > 16, seq_len_k >= 2048 per
 * device, seq_len_q*seq_len_k*d_head >= 8e9: the crate's single-head
 * flash_attention_v2 on a long head, src/v2.rs:49-121) splits each slice's
 * keys over the devices and merges the partial outputs by log-sum-exp after
 * peer copies of the partials.  Results equal the one-device results to
 * within the precision mode's tolerance.  A device may be listed more than
 * once (its entries then share that GPU).  n == 1 is fa_set_device(devices[0]);
 * n == 0 returns to one device.  Overrides FA_B200_DEVICES ("0,1,2,3" or
 * "all", read at first use).  The device-resident calls are unaffected. */
FA_API int fa_set_devices(const int* devices, int n);
/* Copies up to `capacity` entries of the device list into `devices` and
 * returns its length (0: one device, see fa_set_device). */
FA_API int fa_get_devices(int* devices, int capacity);
FA_API int fa_device_count(void);
/* Thread-local message of the last failure on this thread ("" if none). */
FA_API const char* fa_last_error(void);
/* Number of kernels this library has launched in this process. */
FA_API uint64_t fa_launch_count(void);
/* Name of the kernel family the last successful call on this thread used
 * ("tcgen05_tf32", "tcgen05_3xtf32", "simt_fp32", "decode_splitkv", ...). */
FA_API const char* fa_last_path(void);
/* Page-locks (pins) `bytes` of host memory at `ptr` for the copy engines, so
 * host-slice calls on buffers inside it move data at the full PCIe rate
 * instead of through the library's pinned staging slots.  For buffers a caller
 * reuses across many calls.  Not in the crate's API (it has no device).
 * Memory that is already pinned is accepted as it is. */
FA_API int fa_pin_host(void* ptr, size_t bytes);
/* Undoes fa_pin_host (`ptr` as given to it). */
FA_API int fa_unpin_host(void* ptr);
/* Frees cached staging buffers, and the calling thread's streams, events and
 * pinned status word (created again on the next call). */
FA_API void fa_shutdown(void);

#ifdef __cplusplus
}
#endif
#endif /* FA_B200_H */
