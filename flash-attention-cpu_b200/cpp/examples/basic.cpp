// The crate's API from C++ on the GPU (the C++ counterpart of the crate's
// examples/basic.rs): one head, plain and causal; a batched multi-head call;
// the three schedules agreeing; the CPU naive oracle beside the GPU result.
// Build: g++ -std=c++20 basic.cpp -L../../lib -lfa_b200 -Wl,-rpath,../../lib
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "../flash_attention.hpp"

namespace fac = flash_attention_cpu;

// deterministic values in (-1, 1) from a 64-bit linear congruential sequence
static std::vector<float> values(std::size_t n, std::uint64_t seed) {
  std::uint64_t s = seed ^ 0x5DEECE66Dull;
  std::vector<float> v(n);
  for (float& x : v) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    x = static_cast<float>(s >> 40) / static_cast<float>(1u << 24) * 2.0f - 1.0f;
  }
  return v;
}

static float max_diff(const float* a, const float* b, std::size_t n) {
  float m = 0.0f;
  for (std::size_t i = 0; i < n; i++) m = std::fmax(m, std::fabs(a[i] - b[i]));
  return m;
}

int main() {
  const std::size_t s = 256, d = 64;
  auto q = values(s * d, 1), k = values(s * d, 2), v = values(s * d, 3);
  std::vector<float> out(s * d), want(s * d);

  fac::flash_attention(q, k, v, s, s, d, {}, out);
  fac::naive::naive_attention(q, k, v, s, s, d, false, want);
  const float e1 = max_diff(out.data(), want.data(), out.size());
  std::printf("single head: out[0][0..4] = %.6f %.6f %.6f %.6f, max |gpu - naive| = %.2e\n",
              out[0], out[1], out[2], out[3], e1);

  fac::FlashAttentionConfig causal;
  causal.causal = true;
  fac::flash_attention(q, k, v, s, s, d, causal, out);
  const float e2 = max_diff(out.data(), v.data(), d);
  std::printf("causal: row 0 equals V row 0 to %.2e\n", e2);

  const std::size_t b = 4, h = 8, n = b * h * s * d;
  auto mq = values(n, 4), mk = values(n, 5), mv = values(n, 6);
  std::vector<float> mo(n);
  fac::flash_attention_multihead(mq, mk, mv, b, h, s, s, d, causal, mo);
  std::printf("multihead [%zu, %zu, %zu, %zu]: out[0][0..4] = %.6f %.6f %.6f %.6f\n", b, h, s,
              d, mo[0], mo[1], mo[2], mo[3]);

  std::vector<float> o1(s * d), o3(s * d);
  fac::flash_attention_v1(q, k, v, s, s, d, causal, o1);
  fac::flash_attention_v3(q, k, v, s, s, d, causal, o3);
  const float e3 = max_diff(o1.data(), o3.data(), o1.size());
  std::printf("v1 vs v3: max diff %.2e\n", e3);
  // the library's default precision (3xTF32) keeps the crate's 1e-5 checks
  const bool ok = e1 < 1e-5f && e2 < 1e-5f && e3 == 0.0f;
  std::printf("%s\n", ok ? "ok" : "MISMATCH");
  return ok ? 0 : 1;
}
