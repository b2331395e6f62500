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
  grid_dep_wait();  // (launched with launch_pdl)
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
  // (launched with launch_pdl: nothing below runs before the previous kernel on
  // the stream has completed; a CTA's set-up takes ~0.2 us, so little is lost)
  grid_dep_wait();
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
    *abort_flag = (*(volatile int*)p.err != 0) ? 1 : 0;  // an earlier CTA failed: skip work
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
          const float pe = ex2(__fadd_rn(__fmul_rn(x[c * 32 + e], c_log2), neg_m));
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

// ===========================================================================
// CTA-pair form (cta_group::2, M = 256) for launches of more than 128 query
// rows.  Same arithmetic as tc_fwd_3xtf32; what changes is where the operands
// live, so that two S buffers fit in tensor memory and QK^T of the next key
// block runs while the softmax works on the current one:
//
//   Q     the raw Q tile is TMA-loaded into this CTA's shared memory (128 rows
//         x D, 128B swizzle).  At each tile change the softmax warps write Q hi
//         into tensor memory [0, D) (A operand of the hi*hi and hi*lo MMAs)
//         and Q lo over the raw tile in place (A operand of the lo*hi MMA, from
//         shared memory: only one of the three MMAs pays for reading A there).
//   K, V  raw (hi) and lo planes by TMA; each CTA holds half of every K block
//         (BK/2 keys) and half of every V block's columns (D/2).
//   TMEM  Q hi [0, D), O [D, 2D), then NSB buffers of (S / P hi, P lo).
//
// Roles (8 warps): warp 0 K producer, warp 1 MMA issuer (leader CTA), warp 2
// V producer, warp 3 Q loader, warps 4-7 softmax (thread = query row).  The
// Q buffer is refilled once every QK^T MMA of a tile has completed (the MMA
// warp commits q_smem_empty to both CTAs after the tile's last QK^T), a whole
// tile's PV and epilogue ahead of its use.  O leaves by per-row stores.
template <int D, int BK, int NKS, int NVS, int NSB>
struct Tc3PairCfg {
  static constexpr int kKHalf = BK / 2;           // keys of a K block held per CTA
  static constexpr int kDHalf = D / 2;            // V columns held per CTA
  static constexpr int kKPlane = kKHalf * D * 4;  // one plane (hi or lo) per CTA
  static constexpr int kVPlane = BK * kDHalf * 4;
  static constexpr int kQBytes = kBM * D * 4;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;           // NKS x (hi, lo)
  static constexpr int kOffV = kOffK + NKS * 2 * kKPlane;  // NVS x (hi, lo)
  static constexpr int kOffBar = kOffV + NVS * 2 * kVPlane;
  static constexpr int kNumBars = 1 + 2 * NKS + 2 * NVS + 2 * NSB + 5 + (NSB - 1);
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
  static constexpr int kTmemColsUsed = 2 * D + NSB * 2 * BK;
  static constexpr int kTmemCols = kTmemColsUsed <= 256 ? 256 : 512;
  static_assert(D % 64 == 0 && D <= 128, "pair kernel: D in {64, 128}");
  static_assert(BK % 64 == 0, "pair kernel: BK a multiple of 64");
  static_assert(kTmemColsUsed <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared-memory budget");
};

template <int D, int BK, int NKS, int NVS, int NSB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    tc_fwd_3xtf32_pair(const __grid_constant__ CUtensorMap tmKh,
                       const __grid_constant__ CUtensorMap tmKl,
                       const __grid_constant__ CUtensorMap tmVh,
                       const __grid_constant__ CUtensorMap tmVl,
                       const __grid_constant__ CUtensorMap tmQ, FwdParams p, int n_pairs,
                       int n_split, float* split_o, float* split_lse) {
  using C = Tc3PairCfg<D, BK, NKS, NVS, NSB>;
  // (launched with launch_pdl: nothing below runs before the previous kernel on
  // the stream has completed; a CTA's set-up takes ~0.2 us, so little is lost)
  grid_dep_wait();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + C::kOffQ;
  const uint32_t sK = sbase + C::kOffK;
  const uint32_t sV = sbase + C::kOffV;
  const uint32_t bar0 = sbase + C::kOffBar;
  // q_full: Q lo staged in TMEM by the softmax warps of both CTAs (leader waits)
  const uint32_t bar_q_full = bar0;
  auto bar_k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto bar_k_empty = [&](int s) { return bar0 + 8u * (1 + NKS + s); };
  auto bar_v_full = [&](int s) { return bar0 + 8u * (1 + 2 * NKS + s); };
  auto bar_v_empty = [&](int s) { return bar0 + 8u * (1 + 2 * NKS + NVS + s); };
  constexpr uint32_t kB2 = 1 + 2 * NKS + 2 * NVS;
  auto bar_s_full = [&](int b) { return bar0 + 8u * (kB2 + b); };
  auto bar_p_full = [&](int b) { return bar0 + 8u * (kB2 + NSB + b); };
  // o_done(b) completes once per PV of the blocks G with G % NSB == b.  A K
  // slot is free once the QK^T that read it has completed, and a V slot once
  // its PV has: with as many slots as S buffers, slot G % NSB frees exactly
  // when S buffer G % NSB fills (s_full) or PV(G) completes (o_done), so the
  // producers wait on those and no separate "empty" barriers are committed.
  auto bar_o_done = [&](int b) {
    return bar0 + 8u * (b == 0 ? kB2 + 2 * NSB : kB2 + 2 * NSB + 4 + b);
  };
  constexpr bool kKShare = NKS == NSB, kVShare = NVS == NSB;
  const uint32_t bar_drain = bar0 + 8u * (kB2 + 2 * NSB + 1);
  const uint32_t bar_o_final = bar0 + 8u * (kB2 + 2 * NSB + 2);  // once per tile
  const uint32_t bar_q_smem_full = bar0 + 8u * (kB2 + 2 * NSB + 3);   // Q landed (local TMA)
  const uint32_t bar_q_smem_empty = bar0 + 8u * (kB2 + 2 * NSB + 4);  // tile's QK^T done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffBar + C::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto at_leader = [&](uint32_t bar) { return map_to_rank(bar, 0); };
  auto at_peer = [&](uint32_t bar) { return map_to_rank(bar, 1); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cid = (int)(blockIdx.x >> 1), n_clusters = (int)(gridDim.x >> 1);
  const int n_work = n_pairs * p.bh * n_split;
  struct Tile {
    int bh, q0_pair, q0, q_rows, j0, n_kv, z;
  };
  auto work_of = [&](int k) { return k * n_clusters + ((k & 1) ? n_clusters - 1 - cid : cid); };
  auto tile_of = [&](int w) {
    Tile t;
    int sp = 0;
    if (n_split > 1) {
      const int wq = w / n_split;
      sp = w - wq * n_split;
      w = wq;
    }
    int pair;
    if (p.causal) {  // heaviest pairs first
      const int wq = w / p.bh;
      pair = n_pairs - 1 - wq;
      t.bh = w - wq * p.bh;
    } else {  // the pairs of a slice together (they share its K/V through L2)
      const int wq = w / n_pairs;
      pair = w - wq * n_pairs;
      t.bh = wq;
    }
    t.q0_pair = pair * 2 * kBM;
    t.q0 = t.q0_pair + (int)rank * kBM;
    t.q_rows = max(0, min(kBM, p.sq - t.q0));
    const int pair_rows = min(2 * kBM, p.sq - t.q0_pair);
    int kend = p.sk;
    if (p.causal) kend = causal_limit(p.q_offset + t.q0_pair + pair_rows - 1, p.k_offset, p.sk);
    const int nb = (kend + BK - 1) / BK;
    if (n_split > 1) {
      t.j0 = sp * nb / n_split;
      t.n_kv = (sp + 1) * nb / n_split - t.j0;
    } else {
      t.j0 = 0;
      t.n_kv = nb;
    }
    t.z = sp * p.bh + t.bh;
    return t;
  };

  if (threadIdx.x == 0) {
    mbar_init(bar_q_full, 8);  // 4 softmax warps x 2 CTAs
    for (int s = 0; s < NKS; s++) {
      mbar_init(bar_k_full(s), 2);
      mbar_init(bar_k_empty(s), 1);
    }
    for (int s = 0; s < NVS; s++) {
      mbar_init(bar_v_full(s), 2);
      mbar_init(bar_v_empty(s), 1);
    }
    for (int b = 0; b < NSB; b++) {
      mbar_init(bar_s_full(b), 1);
      mbar_init(bar_p_full(b), 8);
    }
    for (int b = 0; b < NSB; b++) mbar_init(bar_o_done(b), 1);
    mbar_init(bar_drain, 1);
    mbar_init(bar_o_final, 1);
    mbar_init(bar_q_smem_full, 1);
    mbar_init(bar_q_smem_empty, 1);
    *abort_flag = (*(volatile int*)p.err != 0) ? 1 : 0;  // an earlier CTA failed: skip work
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_qh = tmem;  // Q hi (A of hi*hi and hi*lo); Q lo lives in shared memory
  const uint32_t t_o = tmem + (uint32_t)D;
  auto t_s = [&](int b) { return tmem + (uint32_t)(2 * D + b * 2 * BK); };  // S / P hi
  auto t_pl = [&](int b) { return tmem + (uint32_t)(2 * D + b * 2 * BK + BK); };
  const bool skip = *abort_flag != 0;

  if (warp == 0 || warp == 2) {
    // ------------------------------ TMA producers: warp 0 K halves, warp 2 V halves
    const bool is_k = warp == 0;
    const int NS = is_k ? NKS : NVS;
    if (lane == 0 && !skip) {
      int G = 0;
      bool ok = true;
      for (int k = 0; k * n_clusters < n_work && ok; k++) {
        const int w = work_of(k);
        if (w >= n_work) continue;
        const Tile t = tile_of(w);
        for (int j = 0; j < t.n_kv && ok; j++, G++) {
          const int s = G % NS;
          if (G >= NS) {
            const uint32_t empty = is_k ? (kKShare ? bar_s_full(G % NSB) : bar_k_empty(s))
                                        : (kVShare ? bar_o_done(G % NSB) : bar_v_empty(s));
            ok = mbar_wait(empty, ((G / NS) & 1) ^ 1, abort_flag, p.err, p.wait_ns);
          }
          if (!ok) break;
          const uint32_t full = at_leader(is_k ? bar_k_full(s) : bar_v_full(s));
          if (is_k) {
            mbar_expect_tx_cluster(full, 2 * C::kKPlane);
            const uint32_t base = sK + s * 2 * C::kKPlane;
            const int y = (t.j0 + j) * BK + (int)rank * C::kKHalf;
            for (int c = 0; c < D / 32; c++) {
              tma_load_3d_pair(base + c * C::kKHalf * 128, &tmKh, full, 32 * c, y, t.bh);
              tma_load_3d_pair(base + C::kKPlane + c * C::kKHalf * 128, &tmKl, full, 32 * c, y,
                               t.bh);
            }
          } else {
            mbar_expect_tx_cluster(full, 2 * C::kVPlane);
            const uint32_t base = sV + s * 2 * C::kVPlane;
            const int y = (t.j0 + j) * BK;
            for (int c = 0; c < C::kDHalf / 32; c++) {
              const int x = (int)rank * C::kDHalf + 32 * c;
              tma_load_3d_pair(base + c * BK * 128, &tmVh, full, x, y, t.bh);
              tma_load_3d_pair(base + C::kVPlane + c * BK * 128, &tmVl, full, x, y, t.bh);
            }
          }
        }
      }
      // no TMA write may land after the CTAs exit, even when a consumer aborted
      volatile int no_abort = 0;
      if (leader)
        for (int g = max(0, G - NS); g < G; g++)
          mbar_wait(is_k ? bar_k_full(g % NS) : bar_v_full(g % NS), (g / NS) & 1, &no_abort,
                    p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (leader CTA; one elected lane issues)
    if (leader && !skip) {
      constexpr uint32_t idesc_qk = instr_desc(2 * kBM, BK, false);
      constexpr uint32_t idesc_pv = instr_desc(2 * kBM, D, true);
      auto commit_both = [&](uint32_t bar) {
        tc_commit_pair_elect(bar);
        tc_commit_pair_elect(at_peer(bar));
      };
      const uint64_t qdesc = smem_desc(sQ, 16, 1024, kLayoutSw128);
      // K(G) known to have landed (checked while waiting for an earlier P)
      bool k_known = false;
      // PV of global block G (block j of its tile): O (+)= P(G) V(G), three
      // terms.  While waiting for P(G) it also checks V(G) and, when poll_k,
      // K(G + 2), the block of the next QK^T.
      auto issue_pv = [&](int G, int j, bool poll_k) -> bool {
        const int b = G % NSB, sv = G % NVS, gk = G + 2;
        bool kd = false;
        const bool w = mbar_wait2_poll(bar_p_full(b), (G / NSB) & 1, bar_v_full(sv), (G / NVS) & 1,
                                       bar_k_full(gk % NKS), (gk / NKS) & 1, poll_k, &kd,
                                       abort_flag, p.err, p.wait_ns);
        if (!__all_sync(0xffffffffu, w)) return false;
        k_known = __all_sync(0xffffffffu, kd);
        tc_fence_after();
        const uint64_t vh =
            smem_desc(sV + sv * 2 * C::kVPlane, BK * 128, 512, kLayoutSw128Base32);
        const uint64_t vl = vh + (uint64_t)(C::kVPlane >> 4);
#pragma unroll
        for (int kk = 0; kk < BK / 8; kk++) {
          const uint64_t o = (uint64_t)(kk * 64);
          mma_ts_pair_elect(t_o, t_s(b) + kk * 8, vh + o, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          mma_ts_pair_elect(t_o, t_s(b) + kk * 8, vl + o, idesc_pv, 1u);
          mma_ts_pair_elect(t_o, t_pl(b) + kk * 8, vh + o, idesc_pv, 1u);
        }
        if (!kVShare) commit_both(bar_v_empty(sv));
        commit_both(bar_o_done(G % NSB));
        return true;
      };
      bool ok = true;
      int G = 0, it = 0;
      for (int k = 0; k * n_clusters < n_work && ok; k++) {
        const int w = work_of(k);
        if (w >= n_work) continue;
        const Tile t = tile_of(w);
        ok = __all_sync(0xffffffffu, mbar_wait_cl(bar_q_full, it & 1, abort_flag, p.err, p.wait_ns));
        if (!ok) break;
        tc_fence_after();
        for (int j = 0; j < t.n_kv && ok; j++) {
          const int Gj = G + j, s = Gj % NKS, b = Gj % NSB;
          if (!k_known)
            ok = __all_sync(0xffffffffu, mbar_wait(bar_k_full(s), (Gj / NKS) & 1, abort_flag, p.err,
                                                   p.wait_ns));
          k_known = false;
          if (!ok) break;
          tc_fence_after();
          const uint64_t kh = smem_desc(sK + s * 2 * C::kKPlane, 16, 1024, kLayoutSw128);
          const uint64_t kl = kh + (uint64_t)(C::kKPlane >> 4);
#pragma unroll
          for (int kk = 0; kk < D / 8; kk++) {
            const uint64_t ko = (uint64_t)(((kk >> 2) * C::kKHalf * 128 + (kk & 3) * 32) >> 4);
            const uint64_t qo = (uint64_t)(((kk >> 2) * kBM * 128 + (kk & 3) * 32) >> 4);
            // hi*hi and hi*lo with A = Q hi from TMEM, lo*hi with A = Q lo from
            // shared memory (an SS MMA reads 32 B per row of A and B from shared
            // memory, a TS one only B's)
            mma_ts_pair_elect(t_s(b), t_qh + kk * 8, kh + ko, idesc_qk, kk > 0 ? 1u : 0u);
            mma_ts_pair_elect(t_s(b), t_qh + kk * 8, kl + ko, idesc_qk, 1u);
            mma_ss_pair_elect(t_s(b), qdesc + qo, kh + ko, idesc_qk, 1u);
          }
          commit_both(bar_s_full(b));
          if (!kKShare) commit_both(bar_k_empty(s));
          if (j == t.n_kv - 1) commit_both(bar_q_smem_empty);  // the tile's last QK^T
          // (the next QK^T is S(Gj + 1) = block (Gj - 1) + 2, in this tile if j + 1 < n_kv)
          if (j > 0) ok = issue_pv(Gj - 1, j - 1, j + 1 < t.n_kv);
        }
        if (!ok) break;
        if (t.n_kv == 0) commit_both(bar_q_smem_empty);
        if (t.n_kv > 0) ok = issue_pv(G + t.n_kv - 1, t.n_kv - 1, false);
        k_known = false;
        if (!ok) break;
        commit_both(bar_o_final);
        G += t.n_kv;
        it++;
      }
      commit_both(bar_drain);
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------ Q loader (one lane): this CTA's 128 rows of
    // each tile into the Q buffer, once the previous tile's QK^T has read it
    if (lane == 0 && !skip) {
      bool ok = true;
      int it = 0, qit = 0;
      auto load_q = [&](const Tile& q) {
        mbar_expect_tx(bar_q_smem_full, C::kQBytes);
        for (int c = 0; c < D / 32; c++)
          tma_load_3d(sQ + c * (kBM * 128), &tmQ, bar_q_smem_full, 32 * c, q.q0, q.bh);
        qit++;
      };
      auto next_work = [&](int k) {
        for (int k2 = k + 1; k2 * n_clusters < n_work; k2++)
          if (work_of(k2) < n_work) return k2;
        return -1;
      };
      const int k0 = next_work(-1);
      if (k0 >= 0) load_q(tile_of(work_of(k0)));
      for (int k = k0; k >= 0 && ok; k = next_work(k)) {
        const int kn = next_work(k);
        if (kn < 0) break;
        ok = mbar_wait(bar_q_smem_empty, it & 1, abort_flag, p.err, p.wait_ns);
        if (!ok) break;
        load_q(tile_of(work_of(kn)));
        it++;
      }
      volatile int no_abort = 0;
      if (qit > 0) mbar_wait(bar_q_smem_full, (qit - 1) & 1, &no_abort, p.err);
    }
    __syncwarp();
  } else {
    // ------------------------------ softmax warpgroup: thread = query row
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float c_log2 = p.scale_log2;
    auto warp_arrive_leader = [&](uint32_t bar) {
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(bar);
        else
          mbar_arrive_remote(at_leader(bar));
      }
    };
    bool ok = !skip;
    bool have_prev = false;
    Tile pt{};
    int pit = 0;
    float pm = -INFINITY, pl = 0.0f;
    // The previous tile's O (scaled by 1/l) and LSE to global memory.
    auto epilogue = [&]() {
      if (!ok) return;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_o_final, pit & 1, abort_flag, p.err, p.wait_ns));
      if (!ok) return;
      tc_fence_after();
      const float inv_l = pl > 0.0f ? 1.0f / pl : 0.0f;
      const bool row_ok = r < pt.q_rows;
      float* orow = split_o ? split_o + ((size_t)pt.z * p.sq + pt.q0 + r) * D
                            : p.o + ((size_t)pt.bh * p.sq + pt.q0 + r) * D;
#pragma unroll
      for (int c = 0; c < D / 32; c++) {
        uint32_t rr[32];
        if (pt.n_kv > 0) {
          tmem_ld32(t_o + lane_off + c * 32, rr);
          tmem_wait_ld_regs(rr);
        } else {
#pragma unroll
          for (int e = 0; e < 32; e++) rr[e] = 0u;
        }
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(orow + c * 32 + e) =
                make_float4(__uint_as_float(rr[e]) * inv_l, __uint_as_float(rr[e + 1]) * inv_l,
                            __uint_as_float(rr[e + 2]) * inv_l, __uint_as_float(rr[e + 3]) * inv_l);
        }
      }
      if (row_ok && (split_lse || p.lse))
        (split_lse ? split_lse + (size_t)pt.z * p.sq : p.lse + (size_t)pt.bh * p.sq)[pt.q0 + r] =
            pl > 0.0f ? (pm + log2f(pl)) * 0.69314718055994530942f : -INFINITY;
      tc_fence_before();  // O reads done before the next PV may overwrite it
    };
    int G = 0, it = 0;
    for (int k = 0; k * n_clusters < n_work && ok; k++) {
      const int w = work_of(k);
      if (w >= n_work) continue;
      const Tile t = tile_of(w);
      const long long qg = p.q_offset + t.q0 + r;
      // Q hi of this tile into TMEM and Q lo over the raw Q in shared memory
      // (each thread its own row, in place).  The previous tile's QK^T MMAs,
      // which read the old Q hi and lo, have completed: its last S was visible
      // to this warpgroup.
      ok = __all_sync(0xffffffffu, mbar_wait(bar_q_smem_full, it & 1, abort_flag, p.err,
                                             p.wait_ns));
      if (!ok) break;
      {
        uint8_t* qrow = smem + C::kOffQ + r * 128;
#pragma unroll
        for (int c = 0; c < D / 32; c++) {
          uint32_t rh[32];
#pragma unroll
          for (int e = 0; e < 8; e++) {
            float4* unit = reinterpret_cast<float4*>(qrow + c * (kBM * 128) + ((e ^ (r & 7)) << 4));
            const float4 v4 = *unit;
            const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
            float lo[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
              const float h = hi_part(vv[u]);
              rh[4 * e + u] = __float_as_uint(h);
              lo[u] = vv[u] - h;
            }
            *unit = make_float4(lo[0], lo[1], lo[2], lo[3]);
          }
          tmem_st32(t_qh + lane_off + c * 32, rh);
        }
        tmem_wait_st();
        fence_proxy_async_smem();  // Q lo in shared memory is read by the tensor core
        tc_fence_before();
        // release at cluster scope: the leader's MMAs read this CTA's Q lo
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_release(at_leader(bar_q_full));
      }
      if (have_prev) epilogue();
      if (!ok) break;
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j < t.n_kv && ok; j++) {
        const int Gj = G + j, b = Gj % NSB;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full(b), (Gj / NSB) & 1, abort_flag, p.err,
                                               p.wait_ns));
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
        const int kbase = (t.j0 + j) * BK;
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
          corr = exp2f(floorf(m - m_new));  // an exact power of two
          m = m - floorf(m - m_new);
        }
        if (__any_sync(0xffffffffu, need)) {
          // O is being accumulated by PV(G-1): wait for it, then rescale in TMEM
          ok = __all_sync(0xffffffffu, mbar_wait(bar_o_done((Gj - 1) % NSB), ((Gj - 1) / NSB) & 1,
                                                 abort_flag, p.err, p.wait_ns));
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
        // exponent round(x*c) - m, each step rounded on its own (see tc_fwd_3xtf32)
        const float neg_m = (m == -INFINITY) ? 0.0f : -m;
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < BK / 32; c++) {
          uint32_t rh[32], rl[32];
#pragma unroll
          for (int e = 0; e < 32; e++) {
            const float pe = ex2(__fadd_rn(__fmul_rn(x[c * 32 + e], c_log2), neg_m));
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
        // (test hook: the first softmax warp of the first pair's leader
        // withholds its arrive)
        if (!(p.test_skip == Gj && blockIdx.x == 0 && warp == kSoftmaxWarp0))
          warp_arrive_leader(bar_p_full(b));
      }
      G += t.n_kv;
      have_prev = true;
      pt = t;
      pit = it;
      pm = m;
      pl = l;
      it++;
    }
    if (have_prev && ok) epilogue();
  }
  // Every MMA of the pair completes before either CTA frees TMEM or exits.
  if (warp == 1 && lane == 0 && !skip) {
    volatile int no_abort = 0;
    mbar_wait(bar_drain, 0, &no_abort, p.err);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)C::kTmemCols)
                 : "memory");
  }
}

template <int D, int BK, int NKS, int NVS, int NSB>
cudaError_t launch_3x_pair(const FwdParams& p, float* ws, int n_split, int num_sms,
                           cudaStream_t s) {
  using C = Tc3PairCfg<D, BK, NKS, NVS, NSB>;
  const size_t n = (size_t)p.bh * p.sk * D;  // floats per K (or V) plane
  float* kl = ws;
  float* vl = ws + n;
  {
    cudaError_t le = launch_pdl(split_lo, dim3(148 * 8), dim3(256), 0, s,
                                reinterpret_cast<const float4*>(p.k),
                                reinterpret_cast<const float4*>(p.v), reinterpret_cast<float4*>(ws),
                                n / 4);
    if (le != cudaSuccess) return le;
  }
  count_launch(1);
  CUtensorMap mkh, mkl, mvh, mvl, mq;
  if (!make_map(&mkh, p.k, D, p.sk, p.bh, BK / 2, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mkl, kl, D, p.sk, p.bh, BK / 2, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mvh, p.v, D, p.sk, p.bh, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
      !make_map(&mvl, vl, D, p.sk, p.bh, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
      !make_map(&mq, p.q, D, p.sq, p.bh, kBM, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(tc_fwd_3xtf32_pair<D, BK, NKS, NVS, NSB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  const long long rows = (long long)p.bh * p.sq;
  float* split_o = n_split > 1 ? ws + 2 * n : nullptr;
  float* split_lse = n_split > 1 ? split_o + (size_t)n_split * rows * D : nullptr;
  const int n_pairs = (p.sq + 2 * kBM - 1) / (2 * kBM);
  const long long n_work = (long long)n_pairs * p.bh * n_split;
  if (n_work > INT32_MAX) return cudaErrorInvalidValue;
  const int n_clusters = (int)(n_work < num_sms / 2 ? n_work : num_sms / 2);
  cudaError_t le = launch_pdl(tc_fwd_3xtf32_pair<D, BK, NKS, NVS, NSB>, dim3(2 * n_clusters),
                              dim3(kThreads), C::kSmemBytes, s, mkh, mkl, mvh, mvl, mq, p, n_pairs,
                              n_split, split_o, split_lse);
  if (le != cudaSuccess) return le;
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || n_split == 1) return e;
  return launch_combine(split_o, split_lse, n_split, rows, D, p.o, p.lse, s);
}

template <int D, int BK, int NKS, int NVS, int NSB>
cudaError_t launch_3x(const FwdParams& p, float* ws, int n_split, cudaStream_t s) {
  using C = Tc3Cfg<D, BK, NKS, NVS, NSB>;
  const size_t n = (size_t)p.bh * p.sk * D;  // floats per K (or V) plane
  float* kl = ws;
  float* vl = ws + n;
  {
    cudaError_t le = launch_pdl(split_lo, dim3(148 * 8), dim3(256), 0, s,
                                reinterpret_cast<const float4*>(p.k),
                                reinterpret_cast<const float4*>(p.v), reinterpret_cast<float4*>(ws),
                                n / 4);
    if (le != cudaSuccess) return le;
  }
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
  cudaError_t le = launch_pdl(tc_fwd_3xtf32<D, BK, NKS, NVS, NSB>, grid, dim3(kThreads), C::kSmemBytes,
                              s, mkh, mkl, mvh, mvl, p, split_o, split_lse);
  if (le != cudaSuccess) return le;
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || n_split == 1) return e;
  return launch_combine(split_o, split_lse, n_split, (long long)rows, D, p.o, p.lse, s);
}

}  // namespace

// Key-range parts per CTA tile (single-CTA kernel, up to 128 query rows):
// with fewer CTAs (one per 128-row tile) than half the SMs, each tile's key
// blocks are divided over up to 64 CTAs so that the launch fills the SMs,
// while every part keeps at least 4 blocks of 64 keys (measured on one B200:
// 1 x 128 x 2048 keys 45 -> 34 us, 1 x 100 x 32768 keys 124 -> 70 us against 8
// blocks and 16 parts at most).  Pair kernel (more rows): work units of 256
// rows; when they are at most half the SM pairs, each unit's key blocks are
// divided so the units fill the pairs, keeping at least 8 blocks of 64 keys
// per part, at most 16 parts.
static int tc3_pick_splits(const FwdParams& p, int num_sms) {
  int kend = p.sk;
  if (p.causal) kend = causal_limit(p.q_offset + p.sq - 1, p.k_offset, p.sk);
  const long long nb = (kend + 63) / 64;
  if (p.sq > kBM && (p.d == 64 || p.d == 128)) {
    const long long n_work = (long long)((p.sq + 2 * kBM - 1) / (2 * kBM)) * p.bh;
    const long long clusters = num_sms / 2;
    if (n_work > 2 * clusters) return 1;
    if (n_work * 2 > clusters) {
      // one or two rounds of tiles: split the keys when the schedule model
      // (pair_schedule_makespan, shared with the TF32 pair kernel) says the
      // shorter longest cluster pays for the merge
      const double t_blk = p.d == 128 ? 1.8 : 1.0;  // us per 64-key block, one B200
      double best = 0.0;
      int best_s = 1;
      for (int sp = 1; sp <= 3; sp++) {
        const double t = pair_schedule_makespan(p, sp, (int)clusters, 64, 2.0) * t_blk +
                         (sp > 1 ? merge_cost_us(p, sp) : 0.0);
        if (sp == 1 || t < best) {
          best = t;
          best_s = sp;
        }
      }
      return best_s;
    }
    long long split = clusters / n_work;
    if (split > nb / 8) split = nb / 8;
    if (split > 16) split = 16;
    return split < 1 ? 1 : (int)split;
  }
  const long long ctas = (long long)p.bh * ((p.sq + kBM - 1) / kBM);
  if (ctas * 2 > num_sms) return 1;
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
  if (p.sq > kBM) {
    if (p.d == 128) return launch_3x_pair<128, 64, 2, 2, 2>(p, ws, split, num_sms, s);
    if (p.d == 64) return launch_3x_pair<64, 64, 3, 3, 3>(p, ws, split, num_sms, s);
  }
  if (p.d == 128) return launch_3x<128, 64, 2, 1, 1>(p, ws, split, s);
  if (p.d == 64) return launch_3x<64, 64, 3, 3, 2>(p, ws, split, s);
  // d = 32, 96: the single-CTA kernel at every length (see tc_supported)
  if (p.d == 96) return launch_3x<96, 64, 2, 1, 1>(p, ws, split, s);
  if (p.d == 32) return launch_3x<32, 64, 3, 3, 2>(p, ws, split, s);
  return cudaErrorInvalidValue;
}

}  // namespace fa
