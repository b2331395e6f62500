// C++ port of the crate's integration tests (tests/correctness.rs) against the
// C++ API mirror (flash-attention-cpu_b200/cpp/flash_attention.hpp), checked
// against the test-only naive oracle (oracle/fa_oracle.c), as the crate checks
// against its own naive module.  `correctness_port cpu` runs only the cases that
// need no GPU (shape panics, zero-sized dimensions); no argument runs all.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <functional>
#include <string>
#include <vector>

#include "../../flash-attention-cpu_b200/cpp/flash_attention.hpp"

extern "C" void oracle_naive_f32(const float* q, const float* k, const float* v, size_t sq,
                                 size_t sk, size_t d, int causal, float* out);

using namespace flash_attention_cpu;
using Vec = std::vector<float>;

static int g_failed = 0, g_run = 0;
#define CHECK(cond, ...)                         \
  do {                                           \
    ++g_run;                                     \
    if (!(cond)) {                               \
      ++g_failed;                                \
      std::printf("FAIL %s:%d: ", __FILE__, __LINE__); \
      std::printf(__VA_ARGS__);                  \
      std::printf("\n");                         \
    }                                            \
  } while (0)

// uniform(-1, 1) from a splitmix64 stream (the crate's StdRng stream is Rust-only)
static Vec random_vec(size_t n, uint64_t shift) {
  uint64_t s = 0xC0FFEEull ^ shift;
  Vec v(n);
  for (auto& x : v) {
    s += 0x9E3779B97F4A7C15ull;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    x = (float)((double)(z >> 11) / 9007199254740992.0 * 2.0 - 1.0);
  }
  return v;
}
static float max_abs_diff(const float* a, const float* b, size_t n) {
  float m = 0.f;
  for (size_t i = 0; i < n; i++) m = std::fmax(m, std::fabs(a[i] - b[i]));
  return m;
}

using SingleFn = void (*)(std::span<const float>, std::span<const float>, std::span<const float>,
                          std::size_t, std::size_t, std::size_t, const FlashAttentionConfig&,
                          std::span<float>);
static const SingleFn kVariants[3] = {flash_attention_v1, flash_attention_v2, flash_attention_v3};
static const char* kNames[3] = {"v1", "v2", "v3"};

static void run_case(size_t sq, size_t sk, size_t d, size_t br, size_t bc, bool causal) {
  Vec q = random_vec(sq * d, 1), k = random_vec(sk * d, 2), v = random_vec(sk * d, 3);
  Vec want(sq * d);
  oracle_naive_f32(q.data(), k.data(), v.data(), sq, sk, d, causal, want.data());
  for (int i = 0; i < 3; i++) {
    Vec out(sq * d, 0.f);
    kVariants[i](q, k, v, sq, sk, d, FlashAttentionConfig{br, bc, causal}, out);
    const float diff = max_abs_diff(out.data(), want.data(), out.size());
    CHECK(diff < 1e-3f, "%s sq=%zu sk=%zu d=%zu br=%zu bc=%zu causal=%d diff %g", kNames[i], sq,
          sk, d, br, bc, (int)causal, diff);
  }
}

static bool panics(const std::function<void()>& f) {
  try {
    f();
  } catch (const Panic&) {
    return true;
  }
  return false;
}

static void cpu_cases() {
  // shape_mismatches_panic (:396-433)
  const size_t sq = 4, sk = 4, d = 8;
  Vec q = random_vec(sq * d, 1), k = random_vec(sk * d, 2), v = random_vec(sk * d, 3);
  for (int i = 0; i < 3; i++) {
    Vec out(sq * d);
    std::span<const float> qs(q), ks(k), vs(v);
    CHECK(panics([&] { kVariants[i](qs.first(q.size() - 1), ks, vs, sq, sk, d, {}, out); }),
          "%s q", kNames[i]);
    CHECK(panics([&] { kVariants[i](qs, ks.first(k.size() - 1), vs, sq, sk, d, {}, out); }),
          "%s k", kNames[i]);
    CHECK(panics([&] { kVariants[i](qs, ks, vs.first(v.size() - 1), sq, sk, d, {}, out); }),
          "%s v", kNames[i]);
    CHECK(panics([&] {
            kVariants[i](qs, ks, vs, sq, sk, d, {}, std::span<float>(out).first(out.size() - 1));
          }),
          "%s out", kNames[i]);
  }
  // multihead_shape_mismatch_panics (:435-459)
  Vec qm = random_vec(2 * 2 * 4 * 8, 1), km = random_vec(2 * 2 * 4 * 8, 2);
  Vec outm(2 * 2 * 4 * 8);
  for (auto fn : {flash_attention_multihead_v1, flash_attention_multihead_v2,
                  flash_attention_multihead_v3})
    CHECK(panics([&] {
            fn(std::span<const float>(qm).first(qm.size() - 1), km, km, 2, 2, 4, 4, 8, {}, outm);
          }),
          "multihead q");
  // zero_sized_dimensions_leave_out_untouched (:461-504)
  for (int i = 0; i < 3; i++) {
    Vec e, kk = random_vec(4 * 8, 2), out;
    kVariants[i](e, kk, kk, 0, 4, 8, {}, out);
    Vec q2 = random_vec(4 * 8, 4), out2(4 * 8, 12.5f);
    kVariants[i](q2, e, e, 4, 0, 8, {}, out2);
    bool same = true;
    for (float x : out2) same = same && x == 12.5f;
    CHECK(same, "%s sk=0 must leave out untouched", kNames[i]);
    kVariants[i](e, e, e, 4, 4, 0, {}, out);
  }
  // the crate's `naive` module (src/naive.rs:14-75) on the CPU, against the
  // oracle's restatement of it, over the ragged and causal shapes of the
  // crate's tests; and its length asserts
  const size_t shapes[][3] = {{17, 23, 32}, {1, 1, 16}, {1, 50, 33}, {50, 1, 33},
                              {97, 131, 17}, {10, 40, 32}, {64, 64, 64}};
  for (const auto& sh : shapes)
    for (bool causal : {false, true}) {
      const size_t a = sh[0], b = sh[1], dd = sh[2];
      Vec nq = random_vec(a * dd, 7), nk = random_vec(b * dd, 8), nv = random_vec(b * dd, 9);
      Vec got(a * dd, -1.f), want(a * dd);
      naive::naive_attention(nq, nk, nv, a, b, dd, causal, got);
      oracle_naive_f32(nq.data(), nk.data(), nv.data(), a, b, dd, causal, want.data());
      CHECK(max_abs_diff(got.data(), want.data(), got.size()) < 1e-5f, "naive %zu %zu %zu %d",
            a, b, dd, (int)causal);
    }
  Vec nout(sq * d);
  CHECK(panics([&] {
          naive::naive_attention(std::span<const float>(q).first(q.size() - 1), k, v, sq, sk, d,
                                 false, nout);
        }),
        "naive q");
}

static void gpu_cases() {
  run_case(64, 64, 64, 32, 32, false);  // matches_naive_exact_block_multiples
  run_case(128, 128, 64, 64, 64, false);
  for (auto c : {std::vector<size_t>{17, 23, 32, 8, 8}, {1, 1, 16, 8, 8}, {1, 50, 33, 16, 16},
                 {50, 1, 33, 16, 16}, {97, 131, 17, 32, 40}, {200, 200, 128, 64, 128}})
    run_case(c[0], c[1], c[2], c[3], c[4], false);  // matches_naive_ragged_sizes
  for (size_t b : {3, 5, 6, 7})
    for (bool causal : {false, true}) {
      run_case(23, 29, 24, b, 12, causal);  // block_size_q_not_a_multiple_of_four
      run_case(29, 23, 24, 12, b, causal);  // block_size_kv_not_a_multiple_of_four
    }
  run_case(64, 64, 64, 32, 32, true);  // matches_naive_causal
  run_case(97, 97, 33, 16, 24, true);
  run_case(1, 1, 16, 8, 8, true);
  run_case(5, 5, 8, 64, 64, true);
  run_case(10, 40, 32, 4, 8, true);  // causal_asymmetric_seq_lens
  run_case(10, 10, 8, 1024, 1024, false);  // single_block_bigger_than_everything
  run_case(10, 10, 8, 1024, 1024, true);
  {  // multihead_matches_per_head_naive (:204-238)
    const size_t b = 2, h = 3, sq = 37, sk = 50, d = 16;
    Vec q = random_vec(b * h * sq * d, 21), k = random_vec(b * h * sk * d, 22),
        v = random_vec(b * h * sk * d, 23);
    for (auto fn : {flash_attention_multihead_v1, flash_attention_multihead_v2,
                    flash_attention_multihead_v3, flash_attention_multihead}) {
      Vec out(b * h * sq * d);
      fn(q, k, v, b, h, sq, sk, d, FlashAttentionConfig{8, 12, true}, out);
      for (size_t bh = 0; bh < b * h; bh++) {
        Vec want(sq * d);
        oracle_naive_f32(q.data() + bh * sq * d, k.data() + bh * sk * d, v.data() + bh * sk * d,
                         sq, sk, d, 1, want.data());
        const float diff = max_abs_diff(out.data() + bh * sq * d, want.data(), sq * d);
        CHECK(diff < 1e-3f, "multihead head %zu diff %g", bh, diff);
      }
    }
  }
  {  // causal_first_query_equals_first_value_row (:240-263), 1e-5
    const size_t s = 256, d = 64;
    Vec q = random_vec(s * d, 30), k = random_vec(s * d, 31), v = random_vec(s * d, 32);
    for (int i = 0; i < 3; i++)
      for (auto bb : {std::pair<size_t, size_t>{64, 128}, {32, 32}, {1024, 1024}, {1, 1}}) {
        Vec out(s * d);
        kVariants[i](q, k, v, s, s, d, FlashAttentionConfig{bb.first, bb.second, true}, out);
        const float diff = max_abs_diff(out.data(), v.data(), d);
        CHECK(diff < 1e-5f, "%s row0 diff %g", kNames[i], diff);
      }
  }
  {  // output_is_finite (:265-293)
    Vec q = random_vec(40 * 32, 10), k = random_vec(40 * 32, 11), v = random_vec(40 * 32, 12);
    for (int i = 0; i < 3; i++) {
      Vec out(40 * 32);
      FlashAttentionConfig cfg;
      cfg.causal = true;
      kVariants[i](q, k, v, 40, 40, 32, cfg, out);
      bool fin = true;
      for (float x : out) fin = fin && std::isfinite(x);
      CHECK(fin, "%s non-finite output", kNames[i]);
    }
  }
  {  // v1_v2_v3_mutually_agree (:295-375): v2 vs v3 < 1e-5
    const size_t cs[4][6] = {{64, 64, 64, 32, 32, 0}, {97, 131, 17, 32, 40, 1},
                             {5, 5, 8, 64, 64, 1}, {200, 200, 128, 64, 128, 1}};
    for (auto& c : cs) {
      Vec q = random_vec(c[0] * c[2], 1), k = random_vec(c[1] * c[2], 2),
          v = random_vec(c[1] * c[2], 3);
      Vec o[3];
      for (int i = 0; i < 3; i++) {
        o[i].assign(c[0] * c[2], 0.f);
        kVariants[i](q, k, v, c[0], c[1], c[2], FlashAttentionConfig{c[3], c[4], c[5] != 0}, o[i]);
      }
      CHECK(max_abs_diff(o[0].data(), o[1].data(), o[0].size()) < 1e-3f, "v1 v2");
      CHECK(max_abs_diff(o[0].data(), o[2].data(), o[0].size()) < 1e-3f, "v1 v3");
      CHECK(max_abs_diff(o[1].data(), o[2].data(), o[0].size()) < 1e-5f, "v2 v3");
    }
  }
  for (bool causal : {false, true}) run_case(23, 29, 16, 0, 0, causal);  // zero_block_size_is_clamped
  {  // this library's additions: LSE, backward, pinned buffers (known answers)
    // One key: P = 1, so out = v, lse = scale*q.k, dv = dout, dq = dk = 0.
    const size_t d = 16;
    Vec q = random_vec(d, 40), k = random_vec(d, 41), v = random_vec(d, 42), dout = random_vec(d, 43);
    Vec out(d), lse(1), dq(d), dk(d), dv(d);
    const int old = fa_get_precision();
    fa_set_precision(FA_PREC_FP32);
    flash_attention_multihead_lse(q, k, v, 1, 1, 1, d, false, out, lse);
    float dot = 0.f;
    for (size_t i = 0; i < d; i++) dot += q[i] * k[i];
    CHECK(max_abs_diff(out.data(), v.data(), d) < 1e-6f, "one-key out");
    CHECK(std::fabs(lse[0] - dot / std::sqrt(16.0f)) < 1e-5f, "one-key lse %g", lse[0]);
    flash_attention_backward(q, k, v, out, lse, dout, 1, 1, 1, d, false, dq, dk, dv);
    Vec zero(d, 0.f);
    CHECK(max_abs_diff(dv.data(), dout.data(), d) < 1e-6f, "one-key dv");
    CHECK(max_abs_diff(dq.data(), zero.data(), d) < 1e-6f, "one-key dq");
    CHECK(max_abs_diff(dk.data(), zero.data(), d) < 1e-6f, "one-key dk");
    fa_set_precision(old);
    // pinned buffers give what pageable ones give
    const size_t bh = 4, s = 300, dd = 64;
    Vec a = random_vec(bh * s * dd, 50), b = random_vec(bh * s * dd, 51), c = random_vec(bh * s * dd, 52);
    Vec o1(bh * s * dd), o2(bh * s * dd);
    flash_attention_multihead_v2(a, b, c, 1, bh, s, s, dd, FlashAttentionConfig{64, 128, true}, o1);
    {
      PinnedRange pa(a), pb(b), pc(c), po(o2);
      flash_attention_multihead_v2(a, b, c, 1, bh, s, s, dd, FlashAttentionConfig{64, 128, true}, o2);
    }
    CHECK(max_abs_diff(o1.data(), o2.data(), o1.size()) == 0.f, "pinned vs pageable");
  }
}

int main(int argc, char** argv) {
  const bool cpu_only = argc > 1 && std::string(argv[1]) == "cpu";
  cpu_cases();
  if (!cpu_only) gpu_cases();
  std::printf("%d checks, %d failed\n", g_run, g_failed);
  return g_failed ? 1 : 0;
}
