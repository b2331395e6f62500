// flash_attention.hpp -- C++ mirror of the `flash-attention-cpu` crate's public
// API (src/lib.rs:78-87) over the B200 C ABI (include/fa_b200.h).
//
// Same names, argument order and meaning as the crate:
//   FlashAttentionConfig{block_size_q, block_size_kv, causal} (default 64/128/false)
//   flash_attention_v1 / _v2 / _v3(q, k, v, seq_len_q, seq_len_k, d_head, config, out)
//   flash_attention_multihead_v1 / _v2 / _v3(q, k, v, batch, heads, seq_len_q,
//                                            seq_len_k, d_head, config, out)
//   flash_attention = flash_attention_v2; flash_attention_multihead = _multihead_v2
// Slices are std::span<const float> / std::span<float> (the crate's &[f32] /
// &mut [f32]).  Where the crate panics -- a length mismatch, src/common.rs:51-54
// and 87-90 -- these functions throw flash_attention_cpu::Panic with the same
// message; a zero dimension returns without touching `out` (src/common.rs:56).
// Every other failure (no GPU, CUDA error, bounded-wait timeout) throws
// flash_attention_cpu::Error.  All compute runs on the GPU; there is no CPU path.
// Link with -lfa_b200 (flash-attention-cpu_b200/lib).
#pragma once

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <limits>
#include <span>
#include <vector>
#include <stdexcept>
#include <string>

#include "../../include/fa_b200.h"

namespace flash_attention_cpu {

struct FlashAttentionConfig {
  std::size_t block_size_q = 64;
  std::size_t block_size_kv = 128;
  bool causal = false;
};

class Panic : public std::logic_error {
 public:
  using std::logic_error::logic_error;
};

class Error : public std::runtime_error {
 public:
  Error(int status, const std::string& msg) : std::runtime_error(msg), status(status) {}
  int status;
};

namespace detail {
inline void check(int rc) {
  if (rc == FA_OK) return;
  const std::string msg = fa_last_error();
  if (rc == FA_ERR_SHAPE) throw Panic(msg);
  throw Error(rc, msg);
}
inline fa_config to_c(const FlashAttentionConfig& c) {
  fa_config r;
  r.block_size_q = c.block_size_q;
  r.block_size_kv = c.block_size_kv;
  r.causal = c.causal ? 1 : 0;
  return r;
}
using SingleFn = int (*)(const float*, size_t, const float*, size_t, const float*, size_t, size_t,
                         size_t, size_t, const fa_config*, float*, size_t);
using MultiFn = int (*)(const float*, size_t, const float*, size_t, const float*, size_t, size_t,
                        size_t, size_t, size_t, size_t, const fa_config*, float*, size_t);
inline void single(SingleFn fn, std::span<const float> q, std::span<const float> k,
                   std::span<const float> v, std::size_t sq, std::size_t sk, std::size_t d,
                   const FlashAttentionConfig& cfg, std::span<float> out) {
  const fa_config c = to_c(cfg);
  check(fn(q.data(), q.size(), k.data(), k.size(), v.data(), v.size(), sq, sk, d, &c, out.data(),
           out.size()));
}
inline void multi(MultiFn fn, std::span<const float> q, std::span<const float> k,
                  std::span<const float> v, std::size_t batch, std::size_t heads, std::size_t sq,
                  std::size_t sk, std::size_t d, const FlashAttentionConfig& cfg,
                  std::span<float> out) {
  const fa_config c = to_c(cfg);
  check(fn(q.data(), q.size(), k.data(), k.size(), v.data(), v.size(), batch, heads, sq, sk, d,
           &c, out.data(), out.size()));
}
}  // namespace detail

#define FA_CPP_SINGLE(name)                                                                \
  inline void name(std::span<const float> q, std::span<const float> k,                   \
                   std::span<const float> v, std::size_t seq_len_q, std::size_t seq_len_k, \
                   std::size_t d_head, const FlashAttentionConfig& config,                \
                   std::span<float> out) {                                                \
    detail::single(&fa_##name, q, k, v, seq_len_q, seq_len_k, d_head, config, out);       \
  }
FA_CPP_SINGLE(flash_attention_v1)
FA_CPP_SINGLE(flash_attention_v2)
FA_CPP_SINGLE(flash_attention_v3)
FA_CPP_SINGLE(flash_attention)
#undef FA_CPP_SINGLE

#define FA_CPP_MULTI(name)                                                                   \
  inline void name(std::span<const float> q, std::span<const float> k,                     \
                   std::span<const float> v, std::size_t batch, std::size_t heads,          \
                   std::size_t seq_len_q, std::size_t seq_len_k, std::size_t d_head,        \
                   const FlashAttentionConfig& config, std::span<float> out) {              \
    detail::multi(&fa_##name, q, k, v, batch, heads, seq_len_q, seq_len_k, d_head, config, \
                  out);                                                                     \
  }
FA_CPP_MULTI(flash_attention_multihead_v1)
FA_CPP_MULTI(flash_attention_multihead_v2)
FA_CPP_MULTI(flash_attention_multihead_v3)
FA_CPP_MULTI(flash_attention_multihead)
#undef FA_CPP_MULTI

// ---- the crate's `naive` module (src/naive.rs:14-75) -------------------------
// Textbook attention that materialises the [seq_len_q, seq_len_k] score
// matrix.  In the crate it is public CPU code used as a correctness oracle and
// a benchmark comparison point; it stays CPU code here (an API item of the
// crate, not a fallback of the GPU forward, which never calls it).
namespace naive {
inline void naive_attention(std::span<const float> q, std::span<const float> k,
                            std::span<const float> v, std::size_t seq_len_q,
                            std::size_t seq_len_k, std::size_t d_head, bool causal,
                            std::span<float> out) {
  if (q.size() != seq_len_q * d_head) throw Panic("assertion failed: q.len() == seq_len_q * d_head");
  if (k.size() != seq_len_k * d_head) throw Panic("assertion failed: k.len() == seq_len_k * d_head");
  if (v.size() != seq_len_k * d_head) throw Panic("assertion failed: v.len() == seq_len_k * d_head");
  if (out.size() != seq_len_q * d_head)
    throw Panic("assertion failed: out.len() == seq_len_q * d_head");
  const float scale = 1.0f / std::sqrt(static_cast<float>(d_head));
  std::vector<float> p(seq_len_k);
  for (std::size_t i = 0; i < seq_len_q; i++) {
    const float* qi = q.data() + i * d_head;
    // scaled scores of row i, -inf past the diagonal when causal
    float m = -std::numeric_limits<float>::infinity();
    for (std::size_t j = 0; j < seq_len_k; j++) {
      if (causal && j > i) {
        p[j] = -std::numeric_limits<float>::infinity();
        continue;
      }
      const float* kj = k.data() + j * d_head;
      float dot = 0.0f;
      for (std::size_t c = 0; c < d_head; c++) dot += qi[c] * kj[c];
      p[j] = dot * scale;
      m = std::max(m, p[j]);
    }
    // softmax of the row (a row that sees no key keeps probability 0)
    float sum = 0.0f;
    for (std::size_t j = 0; j < seq_len_k; j++) {
      p[j] = std::exp(p[j] - m);
      sum += p[j];
    }
    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
    float* o = out.data() + i * d_head;
    std::fill(o, o + d_head, 0.0f);
    for (std::size_t j = 0; j < seq_len_k; j++) {
      const float w = p[j] * inv;
      if (w == 0.0f) continue;
      const float* vj = v.data() + j * d_head;
      for (std::size_t c = 0; c < d_head; c++) o[c] += w * vj[c];
    }
  }
}
}  // namespace naive

// ---- beyond the crate's API (this library's additions) ---------------------

// The multihead forward that also returns each row's LSE (natural log of the
// scaled-score row sum), as the backward needs it.  out: [batch*heads*seq_len_q*d_head],
// lse: [batch*heads*seq_len_q].
inline void flash_attention_multihead_lse(std::span<const float> q, std::span<const float> k,
                                          std::span<const float> v, std::size_t batch_heads,
                                          std::size_t seq_len_q, std::size_t seq_len_k,
                                          std::size_t d_head, bool causal, std::span<float> out,
                                          std::span<float> lse) {
  const std::size_t nq = batch_heads * seq_len_q * d_head, nk = batch_heads * seq_len_k * d_head;
  if (q.size() != nq) throw Panic("q shape mismatch");
  if (k.size() != nk) throw Panic("k shape mismatch");
  if (v.size() != nk) throw Panic("v shape mismatch");
  if (out.size() != nq) throw Panic("out shape mismatch");
  if (lse.size() != batch_heads * seq_len_q) throw Panic("lse shape mismatch");
  detail::check(fa_flash_attention_multihead_lse(q.data(), k.data(), v.data(), batch_heads,
                                                 seq_len_q, seq_len_k, d_head, causal ? 1 : 0,
                                                 out.data(), lse.data()));
}

// Gradients dq, dk, dv of the forward (exact f32), from its out and lse.
inline void flash_attention_backward(std::span<const float> q, std::span<const float> k,
                                     std::span<const float> v, std::span<const float> out,
                                     std::span<const float> lse, std::span<const float> dout,
                                     std::size_t batch_heads, std::size_t seq_len_q,
                                     std::size_t seq_len_k, std::size_t d_head, bool causal,
                                     std::span<float> dq, std::span<float> dk,
                                     std::span<float> dv) {
  const std::size_t nq = batch_heads * seq_len_q * d_head, nk = batch_heads * seq_len_k * d_head;
  if (q.size() != nq || out.size() != nq || dout.size() != nq || dq.size() != nq)
    throw Panic("q/out/dout/dq shape mismatch");
  if (k.size() != nk || v.size() != nk || dk.size() != nk || dv.size() != nk)
    throw Panic("k/v/dk/dv shape mismatch");
  if (lse.size() != batch_heads * seq_len_q) throw Panic("lse shape mismatch");
  detail::check(fa_flash_attention_backward(q.data(), k.data(), v.data(), out.data(), lse.data(),
                                            dout.data(), dq.data(), dk.data(), dv.data(),
                                            batch_heads, seq_len_q, seq_len_k, d_head,
                                            causal ? 1 : 0));
}

// Pins a host buffer for the lifetime of the object (fa_pin_host), so host-slice
// calls on it copy at the full PCIe rate.
class PinnedRange {
 public:
  explicit PinnedRange(std::span<float> s) : p_(s.data()) { detail::check(fa_pin_host(p_, s.size_bytes())); }
  ~PinnedRange() { fa_unpin_host(p_); }
  PinnedRange(const PinnedRange&) = delete;
  PinnedRange& operator=(const PinnedRange&) = delete;

 private:
  void* p_;
};

}  // namespace flash_attention_cpu
