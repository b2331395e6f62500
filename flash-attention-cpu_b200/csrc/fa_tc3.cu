// Error-compensated ("3xTF32") tensor-core attention forward for sm_100a.
//
// Every f32 operand x is split as x = hi + lo with hi = x with its low 13
// mantissa bits cleared (exactly representable in TF32, whatever rounding the
// tensor core applies) and lo = x - hi (exact).  Each product a*b is formed as
// hi_a*hi_b + hi_a*lo_b + lo_a*hi_b with three kind::tf32 MMAs accumulating in
// f32 in TMEM; the dropped lo*lo term and the truncation of lo leave a relative
// error near 2^-21, which keeps the output within 2e-5 of f32 attention.
//
//   K, V  hi is read straight from K and V: the tensor core reads an f32
//         operand of a kind::tf32 MMA by dropping its low 13 mantissa bits,
//         which is exactly hi (the 2e-5 parity tests would show a rounding
//         tensor core as a 2^-11 error).  lo is written once per call by
//         split_lo into workspace planes.  All four load by TMA like the TF32
//         kernel (K-major 128B swizzle for K, MN-major 128B/32B-atom for V).
//   Q     split by the softmax warps and staged in TMEM: hi [0,D), lo [D,2D).
//   P     written back to TMEM as hi (over S) and lo (next BK columns).
//
// One CTA = one 128-row query tile, warp roles as in the TF32 kernel (K and V
// producers, a warp-uniform MMA issuer, one softmax warpgroup).  TMEM columns:
// Q hi/lo [0, 2D), O [2D, 3D), then NSB buffers of (S/P hi, P lo), BK each.
// For D = 128 this fills 512 columns with one S buffer (QK^T of the next tile
// then follows PV of the current one); D = 64 keeps two buffers.
#include "fa_tc_ptx.cuh"

namespace fa {
namespace {

// lo = x - hi for K and V ([0, n4) from k, [n4, 2 n4) from v), one pass.
__global__ void __launch_bounds__(256) split_lo(const float4* __restrict__ k,
                                                const float4* __restrict__ v,
                                                float4* __restrict__ lo, size_t n4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < 2 * n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const float4 x = i < n4 ? k[i] : v[i - n4];
    float4 l;
    l.x = x.x - __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
    l.y = x.y - __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
    l.z = x.z - __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
    l.w = x.w - __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
    lo[i] = l;
  }
}

__device__ __forceinline__ float hi_part(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

template <int D, int BK, int NKS, int NVS, int NSB>
struct Tc3Cfg {
  static constexpr int kChunks = D / 32;
  static constexpr int kKBytes = BK * D * 4;  // one plane of a K tile
  static constexpr int kVBytes = BK * D * 4;
  static constexpr int kOffK = 0;                           // NKS x (hi, lo)
  static constexpr int kOffV = kOffK + NKS * 2 * kKBytes;   // NVS x (hi, lo)
  static constexpr int kOffBar = kOffV + NVS * 2 * kVBytes;
  static constexpr int kNumBars = 1 + 2 * NKS + 2 * NVS + 2 * NSB + 4;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
  static constexpr int kTmemColsUsed = 3 * D + NSB * 2 * BK;
  static constexpr int kTmemCols = kTmemColsUsed <= 256 ? 256 : 512;
  static_assert(kTmemColsUsed <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared-memory budget");
  static_assert(BK % 32 == 0 && D % 32 == 0, "tile shape");
};

template <int D, int BK, int NKS, int NVS, int NSB>
__global__ void __launch_bounds__(kThreads, 1)
    tc_fwd_3xtf32(const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                  const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl,
                  FwdParams p, float* split_o, float* split_lse) {
  using C = Tc3Cfg<D, BK, NKS, NVS, NSB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sK = sbase + C::kOffK;
  const uint32_t sV = sbase + C::kOffV;
  const uint32_t bar0 = sbase + C::kOffBar;
  const uint32_t bar_q_full = bar0;
  auto bar_k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto bar_k_empty = [&](int s) { return bar0 + 8u * (1 + NKS + s); };
  auto bar_v_full = [&](int s) { return bar0 + 8u * (1 + 2 * NKS + s); };
  auto bar_v_empty = [&](int s) { return bar0 + 8u * (1 + 2 * NKS + NVS + s); };
  constexpr uint32_t kB2 = 1 + 2 * NKS + 2 * NVS;
  auto bar_s_full = [&](int b) { return bar0 + 8u * (kB2 + b); };
  auto bar_p_full = [&](int b) { return bar0 + 8u * (kB2 + NSB + b); };
  const uint32_t bar_o_done = bar0 + 8u * (kB2 + 2 * NSB);
  const uint32_t bar_drain = bar0 + 8u * (kB2 + 2 * NSB + 1);
  const uint32_t bar_o_final = bar0 + 8u * (kB2 + 2 * NSB + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffBar + C::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blockIdx.x runs over (slice, tile).  Causal: heaviest tiles of all
  // slices first, for the balance of the last wave.  Non-causal tiles cost the
  // same, so the tiles of a slice are adjacent and the CTAs resident at one
  // time share few slices' K/V planes through L2 (measured on one B200:
  // 256 x 1024 x 64 142 -> 165 TFLOP/s; the slice-adjacent order on the causal
  // 32 x 4096 x 128 ran 186 -> 165, its heavy tiles landing in the last wave).
  const int n_qt = (p.sq + kBM - 1) / kBM;
  const unsigned lin = blockIdx.x;
  const int bh = p.causal ? (int)(lin % (unsigned)p.bh) : (int)(lin / (unsigned)n_qt);
  const int qt = p.causal ? n_qt - 1 - (int)(lin / (unsigned)p.bh) : (int)(lin % (unsigned)n_qt);
  const int q0 = qt * kBM;
  const int q_rows = min(kBM, p.sq - q0);
  int kend = p.sk;
  if (p.causal) kend = causal_limit(p.q_offset + q0 + q_rows - 1, p.k_offset, p.sk);
  // blockIdx.z: the part of the key range this CTA covers (gridDim.z parts);
  // with more than one part the range-normalised O and LSE go to split_o /
  // split_lse ([part][bh][sq]) for the LSE combine.
  const int nb = (kend + BK - 1) / BK;
  const int j0 = (int)((long long)blockIdx.z * nb / gridDim.z);
  const int n_kv = (int)((long long)(blockIdx.z + 1) * nb / gridDim.z) - j0;
  const bool to_split = gridDim.z > 1;
  const size_t zrow = ((size_t)blockIdx.z * p.bh + bh) * p.sq;  // row base in split space

  if (threadIdx.x == 0) {
    mbar_init(bar_q_full, 128);
    for (int s = 0; s < NKS; s++) {
      mbar_init(bar_k_full(s), 1);
      mbar_init(bar_k_empty(s), 1);
    }
    for (int s = 0; s < NVS; s++) {
      mbar_init(bar_v_full(s), 1);
      mbar_init(bar_v_empty(s), 1);
    }
    for (int b = 0; b < NSB; b++) {
      mbar_init(bar_s_full(b), 1);
      mbar_init(bar_p_full(b), 128);
    }
    mbar_init(bar_o_done, 1);
    mbar_init(bar_drain, 1);
    mbar_init(bar_o_final, 1);
    *abort_flag = (*(volatile int*)p.err != 0) ? 1 : 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_qh = tmem, t_ql = tmem + (uint32_t)D;
  const uint32_t t_o = tmem + (uint32_t)(2 * D);
  auto t_s = [&](int b) { return tmem + (uint32_t)(3 * D + b * 2 * BK); };  // S / P hi
  auto t_pl = [&](int b) { return tmem + (uint32_t)(3 * D + b * 2 * BK + BK); };
  const bool skip = *abort_flag != 0;

  if (warp == 0 || warp == 2) {
    // ------------------------------ TMA producers: warp 0 K (hi, lo), warp 2 V (hi, lo)
    const bool is_k = warp == 0;
    const int NS = is_k ? NKS : NVS;
    if (lane == 0 && !skip) {
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; j++) {
        const int s = j % NS;
        const uint32_t full = is_k ? bar_k_full(s) : bar_v_full(s);
        const uint32_t empty = is_k ? bar_k_empty(s) : bar_v_empty(s);
        if (j >= NS) ok = mbar_wait(empty, ((j / NS) & 1) ^ 1, abort_flag, p.err, p.wait_ns);
        if (!ok) break;
        mbar_expect_tx(full, 2 * C::kKBytes);
        const uint32_t base = (is_k ? sK : sV) + s * 2 * C::kKBytes;
        for (int c = 0; c < C::kChunks; c++) {
          tma_load_3d(base + c * BK * 128, is_k ? &tmKh : &tmVh, full, 32 * c, (j0 + j) * BK, bh);
          tma_load_3d(base + C::kKBytes + c * BK * 128, is_k ? &tmKl : &tmVl, full, 32 * c,
                      (j0 + j) * BK, bh);
        }
        issued = j + 1;
      }
      volatile int no_abort = 0;
      for (int j = max(0, issued - NS); j < issued; j++)
        mbar_wait(is_k ? bar_k_full(j % NS) : bar_v_full(j % NS), (j / NS) & 1, &no_abort, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (warp-uniform; one elected lane issues)
    if (!skip) {
      constexpr uint32_t idesc_qk = instr_desc(kBM, BK, false);
      constexpr uint32_t idesc_pv = instr_desc(kBM, D, true);
      bool ok = __all_sync(0xffffffffu, mbar_wait(bar_q_full, 0, abort_flag, p.err, p.wait_ns));
      tc_fence_after();
      auto issue_pv = [&](int jj) -> bool {
        const int b = jj % NSB, s = jj % NVS;
        if (!__all_sync(0xffffffffu, mbar_wait(bar_p_full(b), (jj / NSB) & 1, abort_flag, p.err, p.wait_ns)))
          return false;
        if (!__all_sync(0xffffffffu, mbar_wait(bar_v_full(s), (jj / NVS) & 1, abort_flag, p.err, p.wait_ns)))
          return false;
        tc_fence_after();
        const uint64_t vh = smem_desc(sV + s * 2 * C::kVBytes, BK * 128, 512, kLayoutSw128Base32);
        const uint64_t vl = vh + (uint64_t)(C::kVBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < BK / 8; kk++) {
          const uint64_t o = (uint64_t)(kk * 64);
          mma_ts_elect(t_o, t_s(b) + kk * 8, vh + o, idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
          mma_ts_elect(t_o, t_s(b) + kk * 8, vl + o, idesc_pv, 1u);
          mma_ts_elect(t_o, t_pl(b) + kk * 8, vh + o, idesc_pv, 1u);
        }
        tc_commit_elect(bar_v_empty(s));
        tc_commit_elect(bar_o_done);
        return true;
      };
      for (int j = 0; j < n_kv && ok; j++) {
        const int s = j % NKS, b = j % NSB;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_k_full(s), (j / NKS) & 1, abort_flag, p.err, p.wait_ns));
        if (!ok) break;
        if (NSB == 1 && j > 0) {
          // single S buffer: PV(j-1) must have been issued (it reads P from it);
          // MMAs of one thread run in issue order, so S(j) may follow at once.
          ok = issue_pv(j - 1);
          if (!ok) break;
        }
        tc_fence_after();
        const uint64_t kh = smem_desc(sK + s * 2 * C::kKBytes, 16, 1024, kLayoutSw128);
        const uint64_t kl = kh + (uint64_t)(C::kKBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++) {
          const uint64_t o = (uint64_t)(((kk >> 2) * BK * 128 + (kk & 3) * 32) >> 4);
          mma_ts_elect(t_s(b), t_qh + kk * 8, kh + o, idesc_qk, kk > 0 ? 1u : 0u);
          mma_ts_elect(t_s(b), t_qh + kk * 8, kl + o, idesc_qk, 1u);
          mma_ts_elect(t_s(b), t_ql + kk * 8, kh + o, idesc_qk, 1u);
        }
        tc_commit_elect(bar_s_full(b));
        tc_commit_elect(bar_k_empty(s));
        if (NSB > 1 && j > 0) ok = issue_pv(j - 1);
      }
      if (ok && n_kv > 0 && issue_pv(n_kv - 1)) tc_commit_elect(bar_o_final);
      tc_commit_elect(bar_drain);
      volatile int no_abort = 0;
      mbar_wait(bar_drain, 0, &no_abort, p.err);
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------ softmax warpgroup: thread = query row
    const int quarter = warp - kSoftmaxWarp0;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const long long qg = p.q_offset + q0 + r;
    const float c_log2 = p.scale_log2;
    bool ok = !skip;
    if (ok) {
      const bool valid = r < q_rows;
      const float4* qrow = reinterpret_cast<const float4*>(p.q + ((size_t)bh * p.sq + q0 + r) * D);
#pragma unroll
      for (int c = 0; c < D / 32; c++) {
        uint32_t rh[32], rl[32];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float4 v4 = valid ? __ldg(qrow + c * 8 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
          const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
          for (int t = 0; t < 4; t++) {
            const float h = hi_part(vv[t]);
            rh[4 * e + t] = __float_as_uint(h);
            rl[4 * e + t] = __float_as_uint(vv[t] - h);
          }
        }
        tmem_st32(t_qh + lane_off + c * 32, rh);
        tmem_st32(t_ql + lane_off + c * 32, rl);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_q_full);
    }
    float m = -INFINITY, l = 0.0f;
    for (int j = 0; j < n_kv && ok; j++) {
      const int b = j % NSB;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full(b), (j / NSB) & 1, abort_flag, p.err, p.wait_ns));
      if (!ok) break;
      tc_fence_after();
      float x[BK];
      {
        uint32_t sr[BK];
#pragma unroll
        for (int c = 0; c < BK / 32; c++)
          tmem_ld32(t_s(b) + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + c * 32));
        tmem_wait_ld_regs(sr);
#pragma unroll
        for (int e = 0; e < BK; e++) x[e] = __uint_as_float(sr[e]);
      }
      const int kbase = (j0 + j) * BK;
      int lim = min(BK, p.sk - kbase);
      if (p.causal) lim = min(lim, causal_limit(qg, p.k_offset + kbase, BK));
      if (!__all_sync(0xffffffffu, lim == BK)) {
#pragma unroll
        for (int e = 0; e < BK; e++) x[e] = (e < lim) ? x[e] : -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < BK; e++) mx = fmaxf(mx, x[e]);
      const float m_new = fmaxf(m, __fmul_rn(mx, c_log2));
      float corr = 1.0f;
      bool need = false;
      if (m == -INFINITY) {
        m = m_new;
      } else if (m_new > m + kRescaleLog2) {
        need = true;
        // an exact power of two, so the rescaled O and l stay exact
        corr = exp2f(floorf(m - m_new));
        m = m - floorf(m - m_new);
      }
      if (__any_sync(0xffffffffu, need)) {
        // O is being accumulated by PV(j-1); with one S buffer PV(j-1) was
        // issued before S(j), so it has completed once S(j) is visible.
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o_done, (j - 1) & 1, abort_flag, p.err, p.wait_ns));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; c++) {
          uint32_t rr[32];
          tmem_ld32(t_o + lane_off + c * 32, rr);
          tmem_wait_ld_regs(rr);
#pragma unroll
          for (int e = 0; e < 32; e++) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * corr);
          tmem_st32(t_o + lane_off + c * 32, rr);
        }
        l *= corr;
      }
      // The exponent argument is round(x*c) - m with both steps rounded on their
      // own (no FMA), and m was formed as round(max x * c): the row's maximum
      // then gives exactly 2^0.  A fused x*c - m would leave the rounding
      // residual of x*c, which at large scores (|x*c| ~ 1e14, ulp ~ 1e7)
      // turns 2^residual into 0 or inf.
      const float neg_m = (m == -INFINITY) ? 0.0f : -m;
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < BK / 32; c++) {
        uint32_t rh[32], rl[32];
#pragma unroll
        for (int e = 0; e < 32; e++) {
          const float pe = exp2f(__fadd_rn(__fmul_rn(x[c * 32 + e], c_log2), neg_m));
          const float h = hi_part(pe);
          rs[e & 3] += pe;
          rh[e] = __float_as_uint(h);
          rl[e] = __float_as_uint(pe - h);
        }
        tmem_st32(t_s(b) + lane_off + c * 32, rh);
        tmem_st32(t_pl(b) + lane_off + c * 32, rl);
      }
      l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      tmem_wait_st();
      tc_fence_before();
      // (test hook: one thread of the first CTA withholds its arrive)
      if (!(p.test_skip == j && threadIdx.x == 128 && blockIdx.x == 0 && blockIdx.z == 0))
        mbar_arrive(bar_p_full(b));
    }
    if (n_kv > 0) {
      const bool w = ok ? mbar_wait(bar_o_final, 0, abort_flag, p.err, p.wait_ns) : false;
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tc_fence_after();
      const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
      const bool row_ok = r < q_rows;
      float* orow = to_split ? split_o + (zrow + q0 + r) * D : p.o + ((size_t)bh * p.sq + q0 + r) * D;
#pragma unroll
      for (int c = 0; c < D / 32; c++) {
        uint32_t rr[32];
        if (n_kv > 0) {
          tmem_ld32(t_o + lane_off + c * 32, rr);
          tmem_wait_ld_regs(rr);
        } else {
#pragma unroll
          for (int e = 0; e < 32; e++) rr[e] = 0u;
        }
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4 v4 = make_float4(__uint_as_float(rr[e]) * inv_l, __uint_as_float(rr[e + 1]) * inv_l,
                                    __uint_as_float(rr[e + 2]) * inv_l,
                                    __uint_as_float(rr[e + 3]) * inv_l);
            *reinterpret_cast<float4*>(orow + c * 32 + e) = v4;
          }
        }
      }
      if (row_ok && (to_split || p.lse))
        (to_split ? split_lse + zrow : p.lse + (size_t)bh * p.sq)[q0 + r] =
            l > 0.0f ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)C::kTmemCols)
                 : "memory");
  }
}

template <int D, int BK, int NKS, int NVS, int NSB>
cudaError_t launch_3x(const FwdParams& p, float* ws, int n_split, cudaStream_t s) {
  using C = Tc3Cfg<D, BK, NKS, NVS, NSB>;
  const size_t n = (size_t)p.bh * p.sk * D;  // floats per K (or V) plane
  float* kl = ws;
  float* vl = ws + n;
  split_lo<<<148 * 8, 256, 0, s>>>(reinterpret_cast<const float4*>(p.k),
                                   reinterpret_cast<const float4*>(p.v),
                                   reinterpret_cast<float4*>(ws), n / 4);
  count_launch(1);
  CUtensorMap mkh, mkl, mvh, mvl;
  if (!make_map(&mkh, p.k, D, p.sk, p.bh, BK, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mkl, kl, D, p.sk, p.bh, BK, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mvh, p.v, D, p.sk, p.bh, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
      !make_map(&mvl, vl, D, p.sk, p.bh, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(tc_fwd_3xtf32<D, BK, NKS, NVS, NSB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  const size_t rows = (size_t)p.bh * p.sq;
  float* split_o = n_split > 1 ? ws + 2 * n : nullptr;
  float* split_lse = n_split > 1 ? split_o + (size_t)n_split * rows * D : nullptr;
  const long long n_ctas = (long long)p.bh * ((p.sq + kBM - 1) / kBM);
  if (n_ctas > INT32_MAX) return cudaErrorInvalidValue;
  dim3 grid((unsigned)n_ctas, 1, n_split);
  tc_fwd_3xtf32<D, BK, NKS, NVS, NSB><<<grid, kThreads, C::kSmemBytes, s>>>(mkh, mkl, mvh, mvl, p,
                                                                            split_o, split_lse);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || n_split == 1) return e;
  return launch_combine(split_o, split_lse, n_split, (long long)rows, D, p.o, p.lse, s);
}

}  // namespace

// Key-range parts per CTA tile: with fewer CTAs (one per 128-row tile) than
// half the SMs, each tile's key blocks are divided over up to 64 CTAs so that
// the launch fills the SMs, while every part keeps at least 4 blocks of 64 keys
// (measured on one B200: 1 x 128 x 2048 keys 45 -> 34 us, 1 x 100 x 32768 keys
// 124 -> 70 us against 8 blocks and 16 parts at most).
static int tc3_pick_splits(const FwdParams& p, int num_sms) {
  const long long ctas = (long long)p.bh * ((p.sq + kBM - 1) / kBM);
  if (ctas * 2 > num_sms) return 1;
  int kend = p.sk;
  if (p.causal) kend = causal_limit(p.q_offset + p.sq - 1, p.k_offset, p.sk);
  const long long nb = (kend + 63) / 64;
  long long split = num_sms / ctas;
  if (split > nb / 4) split = nb / 4;
  if (split > 64) split = 64;
  return split < 1 ? 1 : (int)split;
}

size_t tc3_workspace_floats(const FwdParams& p, int num_sms) {
  const int split = tc3_pick_splits(p, num_sms);
  size_t f = 2 * (size_t)p.bh * p.sk * p.d;  // lo planes of K and V
  if (split > 1) f += (size_t)split * p.bh * p.sq * (p.d + 1);
  return f;
}

cudaError_t launch_tc3(const FwdParams& p, float* ws, int num_sms, cudaStream_t s) {
  const int split = tc3_pick_splits(p, num_sms);
  if (p.d == 128) return launch_3x<128, 64, 2, 1, 1>(p, ws, split, s);
  if (p.d == 64) return launch_3x<64, 64, 3, 3, 2>(p, ws, split, s);
  return cudaErrorInvalidValue;
}

}  // namespace fa
