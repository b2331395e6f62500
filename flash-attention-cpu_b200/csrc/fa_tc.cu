// Tensor-core attention forward for sm_100a (B200): tcgen05 TF32 MMAs with
// the accumulators in tensor memory (TMEM), TMA tile loads into 128-byte
// swizzled shared memory, and warp-specialised roles on an mbarrier pipeline.
// Two kernels share the design:
//
// tc_fwd_tf32 (up to 128 query rows): one CTA per 128-row tile of a slice,
// with blockIdx.z parts of the key range for launches that leave SMs idle.
//   warp 0 (one lane)  K producer: K tiles of BK keys through an NKS-deep ring.
//   warp 2 (one lane)  V producer: V sub-tiles of VK keys through an NVS-deep
//                      ring (separate rings, so a K slot frees as soon as its
//                      QK^T MMA has read it, before PV).
//   warp 1             MMA issuer (warp-uniform, one elected lane issues):
//                      S_b = Q K_j^T into TMEM buffer b = j % 2, then
//                      O += P_{j-1} V_{j-1} with P read straight from TMEM
//                      (the .kind::tf32 "A from TMEM" form).  Issuing S_j
//                      before PV_{j-1} lets QK^T of the next tile run while the
//                      softmax warps work on the current one (the mechanism
//                      behind the crate's v3 software pipelining,
//                      src/v3.rs:445-483).
//   warps 4-7          softmax, one query row per thread: Q staged into TMEM
//                      (scaled by scale*log2 e, rounded to TF32), then per
//                      tile tcgen05.ld the score row, mask (causal diagonal
//                      tiles and keys past seq_len_k, src/v2.rs:268-287),
//                      running max, exp2, row sum, P written back over S in
//                      TMEM (src/v2.rs:289-339).  O is rescaled in TMEM only
//                      when the running max grows by more than 2^8 (lazy
//                      rescaling); O and l share the same stale max, so the
//                      final out = O / l (src/v2.rs:375-382) is exact.
//   TMEM columns: Q [0, D), O [D, 2D), S/P buffers [2D + b*BK, 2D + (b+1)*BK).
//
// tc_fwd_tf32_pair (more than 128 query rows): a persistent CTA pair
// (cta_group::2, M = 256) per SM pair looping over 256-row work tiles; each SM
// holds half of every K tile and half of every V tile's columns.  Warp 3 moves
// O out and the next tile's Q in through one shared-memory buffer, and two
// softmax warpgroups split each row's columns.  The kernel's own comment has
// the details.
//
// Causal runs never load or multiply key tiles wholly past a tile's last row
// (src/v2.rs:210-212), and the heaviest tiles are dispatched first.
//
// Shared-memory layouts (all 1024-byte aligned, 32 f32 = 128 B per swizzle row):
//   K  [D/32 chunks][BK keys][32]    K-major B operand of QK^T, 128B swizzle
//                                    (16-byte granules XOR row%8)
//   V  [D/32 chunks][VK keys][32]    MN-major B operand of PV (d contiguous).
//                                    An MN-major TF32 operand must use the
//                                    "128B swizzle, 32B atom" layout (32-byte
//                                    granules XOR row%4; K grouped by 4 rows,
//                                    512 B apart), which TMA writes with
//                                    CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
//   Q / O (pair kernel) [D/32 chunks][128 rows][32], 128B swizzle.
#include "fa_tc_ptx.cuh"

#include <algorithm>
#include <vector>

namespace fa {
namespace {


// D: head size.  BK: keys per K tile (the N of the QK^T MMA).  VK: keys per V
// sub-tile (BK/VK sub-tiles per K tile, so V slots free up in finer steps).
// NKS / NVS: depth of the K and V rings.
template <int D, int BK, int VK, int NKS, int NVS>
struct TcCfg {
  static constexpr int kChunks = D / 32;
  static constexpr int kVS = BK / VK;
  static constexpr int kKBytes = BK * D * 4;
  static constexpr int kVBytes = VK * D * 4;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + NKS * kKBytes;
  static constexpr int kOffBar = kOffV + NVS * kVBytes;
  static constexpr int kNumBars = 1 + 2 * NKS + 2 * NVS + 2 + 2 + 1 + 1 + 1;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + align slack
  // TMEM columns: Q [0, D), O [D, 2D), S/P buffers [2D, 2D + 2*BK)
  static constexpr int kTmemColsUsed = 2 * D + 2 * BK;
  static constexpr int kTmemCols = kTmemColsUsed <= 32 ? 32 : kTmemColsUsed <= 64 ? 64
                                   : kTmemColsUsed <= 128 ? 128 : kTmemColsUsed <= 256 ? 256 : 512;
  static_assert(D % 32 == 0 && D <= 128, "D must be a multiple of 32, at most 128");
  static_assert(BK % 32 == 0 && BK <= 256, "BK must be a multiple of 32");
  static_assert(BK % VK == 0 && VK % 8 == 0, "V sub-tiles must divide the K tile");
  static_assert(kTmemColsUsed <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared-memory budget");
};

// ---- the kernel ------------------------------------------------------------
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <int D, int BK, int VK, int NKS, int NVS>
__global__ void __launch_bounds__(kThreads, 1)
    tc_fwd_tf32(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                FwdParams p, float* split_o, float* split_lse) {
  using C = TcCfg<D, BK, VK, NKS, NVS>;
  constexpr int VS = C::kVS;
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
  const uint32_t bar_q_full = bar0;  // Q staged in TMEM by the softmax warps
  auto bar_k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto bar_k_empty = [&](int s) { return bar0 + 8u * (1 + NKS + s); };
  auto bar_v_full = [&](int s) { return bar0 + 8u * (1 + 2 * NKS + s); };
  auto bar_v_empty = [&](int s) { return bar0 + 8u * (1 + 2 * NKS + NVS + s); };
  constexpr uint32_t kB2 = 1 + 2 * NKS + 2 * NVS;
  auto bar_s_full = [&](int b) { return bar0 + 8u * (kB2 + b); };
  auto bar_p_full = [&](int b) { return bar0 + 8u * (kB2 + 2 + b); };
  // o_done completes once per PV.  A wait on it for PV_{j-1} at softmax step j
  // is unambiguous: S_j was issued after PV_{j-2}, so when S_j is visible at
  // most PV_{j-1} and PV_j remain, and PV_j cannot start before P_j exists.
  const uint32_t bar_o_done = bar0 + 8u * (kB2 + 4);
  const uint32_t bar_drain = bar0 + 8u * (kB2 + 5);
  // Single-use barrier for "the last PV has completed".  The per-PV o_done
  // barrier cannot serve the epilogue: when the softmax loop ends, the last two
  // PVs may both be pending, and a parity wait cannot tell phase n from n-2.
  const uint32_t bar_o_final = bar0 + 8u * (kB2 + 6);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffBar + C::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int n_qt = gridDim.y;
  const int qt = n_qt - 1 - (int)blockIdx.y;  // heaviest causal tiles dispatched first
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
  const size_t zrow = (size_t)(blockIdx.z * gridDim.x + bh) * p.sq;

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
    for (int b = 0; b < 2; b++) {
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
  const uint32_t t_q = tmem;                        // Q tile (A operand of QK^T)
  const uint32_t t_o = tmem + (uint32_t)D;          // O accumulator
  auto t_s = [&](int b) { return tmem + (uint32_t)(2 * D + b * BK); };
  const bool skip = *abort_flag != 0;

  if (warp == 0) {
    // ------------------------------ TMA producer, K ring
    // K and V have separate producers so a K load never waits behind a V slot
    // (V slots free only after PV, K slots right after QK^T).
    if (lane == 0 && !skip) {
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; j++) {
        const int sk = j % NKS;
        if (j >= NKS) ok = mbar_wait(bar_k_empty(sk), ((j / NKS) & 1) ^ 1, abort_flag, p.err, p.wait_ns);
        if (!ok) break;
        mbar_expect_tx(bar_k_full(sk), C::kKBytes);
        for (int c = 0; c < C::kChunks; c++)
          tma_load_3d(sK + sk * C::kKBytes + c * BK * 128, &tmK, bar_k_full(sk), 32 * c,
                      (j0 + j) * BK, bh);
        issued = j + 1;
      }
      // Wait (bounded, ignoring the abort flag) for the last load of every
      // slot, so no TMA write can land after the CTA exits even when a
      // consumer role aborted.  On the normal path these have all completed.
      volatile int no_abort = 0;
      for (int j = max(0, issued - NKS); j < issued; j++)
        mbar_wait(bar_k_full(j % NKS), (j / NKS) & 1, &no_abort, p.err);
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------ TMA producer, V ring (VK-key sub-tiles)
    if (lane == 0 && !skip) {
      int issued = 0;
      bool ok = true;
      const int n_v = n_kv * VS;
      for (int g = 0; g < n_v && ok; g++) {
        const int sv = g % NVS;
        if (g >= NVS) ok = mbar_wait(bar_v_empty(sv), ((g / NVS) & 1) ^ 1, abort_flag, p.err, p.wait_ns);
        if (!ok) break;
        mbar_expect_tx(bar_v_full(sv), C::kVBytes);
        for (int c = 0; c < C::kChunks; c++)
          tma_load_3d(sV + sv * C::kVBytes + c * VK * 128, &tmV, bar_v_full(sv), 32 * c,
                      j0 * BK + g * VK, bh);
        issued = g + 1;
      }
      volatile int no_abort = 0;
      for (int g = max(0, issued - NVS); g < issued; g++)
        mbar_wait(bar_v_full(g % NVS), (g / NVS) & 1, &no_abort, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (whole warp; one elected lane issues)
    if (!skip) {
      constexpr uint32_t idesc_qk = instr_desc(kBM, BK, false);
      constexpr uint32_t idesc_pv = instr_desc(kBM, D, true);
      bool ok = __all_sync(0xffffffffu, mbar_wait(bar_q_full, 0, abort_flag, p.err, p.wait_ns));
      tc_fence_after();
      auto issue_pv = [&](int jj) -> bool {
        const int b = jj & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(bar_p_full(b), (jj >> 1) & 1, abort_flag, p.err, p.wait_ns)))
          return false;
#pragma unroll
        for (int h = 0; h < VS; h++) {
          const int g = jj * VS + h, sv = g % NVS;
          if (!__all_sync(0xffffffffu, mbar_wait(bar_v_full(sv), (g / NVS) & 1, abort_flag, p.err, p.wait_ns)))
            return false;
          tc_fence_after();
          // 8 keys = two 4-row groups (SBO = 512 B); 32-column chunks LBO apart
          const uint64_t vdesc =
              smem_desc(sV + sv * C::kVBytes, VK * 128, 512, kLayoutSw128Base32);
#pragma unroll
          for (int kk = 0; kk < VK / 8; kk++)
            mma_ts_elect(t_o, t_s(b) + h * VK + kk * 8, vdesc + (uint64_t)(kk * 64), idesc_pv,
                         (jj > 0 || h > 0 || kk > 0) ? 1u : 0u);
          tc_commit_elect(bar_v_empty(sv));
        }
        tc_commit_elect(bar_o_done);
        return true;
      };
      for (int j = 0; j < n_kv && ok; j++) {
        const int s = j % NKS, b = j & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_k_full(s), (j / NKS) & 1, abort_flag, p.err, p.wait_ns));
        if (!ok) break;
        tc_fence_after();
        const uint64_t kdesc = smem_desc(sK + s * C::kKBytes, 16, 1024, kLayoutSw128);
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++)
          mma_ts_elect(t_s(b), t_q + kk * 8,
                       kdesc + (uint64_t)(((kk >> 2) * BK * 128 + (kk & 3) * 32) >> 4), idesc_qk,
                       kk > 0 ? 1u : 0u);
        tc_commit_elect(bar_s_full(b));
        tc_commit_elect(bar_k_empty(s));
        if (j > 0) ok = issue_pv(j - 1);
      }
      if (ok && n_kv > 0 && issue_pv(n_kv - 1)) tc_commit_elect(bar_o_final);
      // Drain: all MMAs issued by this warp complete before TMEM is freed.
      tc_commit_elect(bar_drain);
      volatile int no_abort = 0;
      mbar_wait(bar_drain, 0, &no_abort, p.err);
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------ softmax warpgroup: thread = query row
    const int quarter = warp - kSoftmaxWarp0;  // == warp % 4: TMEM lanes 32*quarter..
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const long long qg = p.q_offset + q0 + r;
    const float c_log2 = p.scale_log2;
    bool ok = !skip;
    // Stage this row of Q into TMEM, multiplied by scale*log2(e) and rounded to
    // TF32 (round-to-nearest): the scores then come out in log2 units.
    if (ok) {
      const bool valid = r < q_rows;
      const float4* qrow = reinterpret_cast<const float4*>(p.q + ((size_t)bh * p.sq + q0 + r) * D);
#pragma unroll
      for (int c = 0; c < D / 32; c++) {
        uint32_t rr[32];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float4 v4 = valid ? __ldg(qrow + c * 8 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
          rr[4 * e + 0] = to_tf32_rna(v4.x * c_log2);
          rr[4 * e + 1] = to_tf32_rna(v4.y * c_log2);
          rr[4 * e + 2] = to_tf32_rna(v4.z * c_log2);
          rr[4 * e + 3] = to_tf32_rna(v4.w * c_log2);
        }
        tmem_st32(t_q + lane_off + c * 32, rr);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_q_full);
    }
    float m = -INFINITY;  // running max in log2 units (possibly stale by < 2^8)
    float l = 0.0f;
    for (int j = 0; j < n_kv && ok; j++) {
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full(b), (j >> 1) & 1, abort_flag, p.err, p.wait_ns));
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
      // visible keys of this row in tile j: [0, lim); mask only partial tiles
      const int kbase = (j0 + j) * BK;
      int lim = min(BK, p.sk - kbase);
      if (p.causal) lim = min(lim, causal_limit(qg, p.k_offset + kbase, BK));
      if (!__all_sync(0xffffffffu, lim == BK)) {
#pragma unroll
        for (int e = 0; e < BK; e++) x[e] = (e < lim) ? x[e] : -INFINITY;
      }
      float mx[4];
#pragma unroll
      for (int t = 0; t < 4; t++) mx[t] = -INFINITY;
#pragma unroll
      for (int e = 0; e < BK; e += 8) {
        const int t = (e >> 3) & 3;
        mx[t] = fmax3(mx[t], x[e], x[e + 1]);
        mx[t] = fmax3(mx[t], x[e + 2], x[e + 3]);
        mx[t] = fmax3(mx[t], x[e + 4], x[e + 5]);
        mx[t] = fmax3(mx[t], x[e + 6], x[e + 7]);
      }
      const float m_new = fmaxf(m, fmax3(mx[0], mx[1], fmaxf(mx[2], mx[3])));
      float corr = 1.0f;
      bool need = false;
      if (m == -INFINITY) {
        m = m_new;  // nothing accumulated yet (O holds zeros or nothing)
      } else if (m_new > m + kRescaleLog2) {
        need = true;
        corr = ex2(m - m_new);
        m = m_new;
      }
      if (__any_sync(0xffffffffu, need)) {
        // O is being accumulated by PV_{j-1}: wait for it, then rescale in TMEM.
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
      // p = 2^(s - m) (s is already scaled by scale*log2e through Q), truncated
      // to TF32 exactly as the tensor core reads it, so the row sum l matches
      // the P the PV MMA multiplies.  m is one of the row's scores, so the
      // row's maximum gives exactly 2^0 even at huge scores.
      const float neg_m = (m == -INFINITY) ? 0.0f : -m;
      // one add, one MUFU exponential, one mask and one add per score
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < BK / 32; c++) {
        uint32_t rr[32];
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          float pe[8];
#pragma unroll
          for (int u = 0; u < 8; u++) pe[u] = ex2(__fadd_rn(x[c * 32 + e + u], neg_m));
#pragma unroll
          for (int u = 0; u < 8; u++) {
            const uint32_t tb = __float_as_uint(pe[u]) & 0xFFFFE000u;
            rs[u & 3] += __uint_as_float(tb);
            rr[e + u] = tb;
          }
        }
        tmem_st32(t_s(b) + lane_off + c * 32, rr);
      }
      l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      tmem_wait_st();
      tc_fence_before();
      // (test hook: one thread of the first CTA withholds its arrive)
      if (!(p.test_skip == j && threadIdx.x == 128 && blockIdx.x == 0 && blockIdx.y == 0 &&
            blockIdx.z == 0))
        mbar_arrive(bar_p_full(b));
    }
    // epilogue: out = O / l, lse = ln(sum exp(s)) = (m + log2 l) * ln 2
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
            l > 0.0f ? (m + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
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
// 2-SM pair kernel (cta_group::2).  A cluster of two CTAs on two SMs computes
// 256 query rows (128 per CTA) of one (batch, head) slice.  The leader CTA
// (cluster rank 0) issues every MMA for the pair with M = 256: each SM's tensor
// core computes its own 128 rows, reading the B operand halves from both SMs'
// shared memory.  Each CTA therefore loads only half of every K tile (64 of
// its 128 keys) and half of every V tile (64 of the 128 head columns), which
// halves the L2->SM traffic per FLOP and doubles how many tiles the same
// shared memory can keep in flight.  Every load has one destination: each CTA's TMA
// writes only its own shared memory and signals the leader's barrier.
//
// Per CTA: TMEM columns Q [0, D), O [D, 2D), S/P buffers [2D, 2D + 2*BK);
// shared memory: K half-tiles [D/32 chunks][BK/2 keys][32], V half-tiles
// [D/64 chunks][BK keys][32] (the CTA's d range rank*D/2 .. +D/2).
// Barriers live at the same offsets in both CTAs.  q_full, k_full, v_full and
// p_full are waited on only in the leader (the peer arrives on them remotely);
// the MMA completions are committed to both CTAs' copies of k_empty, v_empty,
// s_full, o_done, o_final and drain.
template <int D, int BK, int NKS, int NVS, int NG>
struct PairCfg {
  static constexpr int kKHalf = BK / 2;                 // keys of a K tile held per CTA
  static constexpr int kDHalf = D / 2;                  // head columns of a V tile per CTA
  static constexpr int kKBytes = kKHalf * D * 4;        // per CTA
  static constexpr int kVBytes = BK * kDHalf * 4;       // per CTA
  static constexpr int kQBytes = kBM * D * 4;          // this CTA's 128 query rows
  static constexpr int kOffK = 0;
  static constexpr int kOffV = NKS * kKBytes;
  static constexpr int kOffQ = kOffV + NVS * kVBytes;   // D/32 swizzled [128 x 32] chunks
  static constexpr int kOffBar = kOffQ + kQBytes;
  static constexpr int kNumBars = 1 + 2 * NKS + 2 * NVS + 2 + 2 + 3 + 2 + 1;
  static constexpr int kOffRed = (kOffBar + kNumBars * 8 + 16 + 15) / 16 * 16;
  // softmax exchange: row maxima [2 blocks][NG][128], row sums [2 tiles][NG][128]
  static constexpr int kSmemBytes = kOffRed + 4 * NG * 128 * 4 + 1024;
  static constexpr int kTmemColsUsed = 2 * D + 2 * BK;
  static constexpr int kTmemCols = kTmemColsUsed <= 256 ? 256 : 512;
  static_assert(D % 64 == 0 && D <= 128, "pair kernel: D in {64, 128}");
  static_assert(BK % 64 == 0 && BK <= 256, "pair kernel: BK multiple of 64");
  static_assert(kTmemColsUsed <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared-memory budget");
};

// 4 + 4*NG warps: K producer, MMA, V producer, O store, then NG softmax warpgroups.
constexpr int pair_threads(int ng) { return 128 + 128 * ng; }

template <int D, int BK, int NKS, int NVS, int NG>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_threads(NG), 1)
    tc_fwd_tf32_pair(const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmO, FwdParams p, int n_pairs,
                     int n_split, float* split_lse) {
  // Persistent: cluster c computes work tiles w = c, c + C, ... (C clusters),
  // each tile = 256 query rows (a pair) of one slice, heaviest causal tiles
  // first.  Every ring and buffer index continues across tiles through the
  // global key-block counter G, so the producers run ahead into the next tile
  // while the current one finishes.  Each CTA's Q rows arrive by TMA in a
  // shared-memory buffer a tile ahead; at a tile change the softmax warps copy
  // them into TMEM (scaled, TF32-rounded), then write the finished tile's O
  // over them, and warp 3 stores that O by TMA and loads the next tile's Q
  // into the buffer.
  using C = PairCfg<D, BK, NKS, NVS, NG>;
  // (launched with launch_pdl: nothing below runs before the previous kernel on
  // the stream has completed; a CTA's set-up takes ~0.2 us, so little is lost)
  grid_dep_wait();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
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
  auto bar_p_full = [&](int b) { return bar0 + 8u * (kB2 + 2 + b); };
  // o_done(b) completes once per PV of the blocks G with G % 2 == b.
  auto bar_o_done = [&](int b) { return bar0 + 8u * (b == 0 ? kB2 + 4 : kB2 + 9); };
  // A K slot is free once the QK^T that read it has completed, and a V slot
  // once its PV has: with two slots, slot G % 2 frees exactly when S buffer
  // G % 2 fills (s_full) or PV(G) completes (o_done(G % 2)), so the producers
  // wait on those and the MMA warp commits no separate "empty" barriers.
  constexpr bool kKShare = NKS == 2, kVShare = NVS == 2;
  const uint32_t bar_drain = bar0 + 8u * (kB2 + 5);
  // o_final completes once per work tile (its last PV, or at once for a tile
  // that sees no key).  The next tile's first PV needs P of its first block,
  // which its softmax produces only after the previous tile's O was read out,
  // so no separate "O free" barrier is needed.
  const uint32_t bar_o_final = bar0 + 8u * (kB2 + 6);
  // Q staging buffer (this CTA's): q_smem_full completes when a tile's Q rows
  // have landed (TMA, issued by warp 3 once the buffer is free).
  const uint32_t bar_q_smem_full = bar0 + 8u * (kB2 + 7);
  // o_smem_full: the softmax warps are done with the buffer for one tile step
  // (this tile's Q copied into TMEM and the previous tile's O written over
  // it); warp 3 then stores that O out and loads the next tile's Q into it.
  const uint32_t bar_o_smem_full = bar0 + 8u * (kB2 + 8);
  const uint32_t sQ = sbase + C::kOffQ;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffBar + C::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto at_leader = [&](uint32_t bar) { return map_to_rank(bar, 0); };
  auto at_peer = [&](uint32_t bar) { return map_to_rank(bar, 1); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cid = (int)(blockIdx.x >> 1), n_clusters = (int)(gridDim.x >> 1);
  // With n_split > 1 each tile's key blocks are divided over n_split work
  // units, each writing its range-normalised O (through tmO, which then maps a
  // [n_split * bh, sq, d] workspace) and LSE (split_lse) for the LSE combine.
  const int n_work = n_pairs * p.bh * n_split;
  struct Tile {
    int bh, q0_pair, q0, q_rows, j0, n_kv, z;  // z: slice index in tmO's space
  };
  // Round k of the static schedule: tiles k*C .. k*C+C-1 (heaviest first),
  // dealt in snake order (reversed on odd rounds) so that every cluster's
  // total causal work comes out nearly equal.
  auto work_of = [&](int k) { return k * n_clusters + ((k & 1) ? n_clusters - 1 - cid : cid); };
  // (Integer division is a software routine on the GPU, and this runs on the
  // softmax warps' critical path at every tile change: one quotient per
  // divisor with the remainder by multiply-subtract, 32-bit arithmetic, and
  // the key-range split skipped when there is one part.  With two 64-bit
  // divisions the softmax warps took ~1100 cycles from a tile's last block to
  // the next tile's Q, now ~700; 256 x 1024 x 64: 180 -> 177 us, causal
  // 137 -> 133 us.)
  auto tile_of = [&](int w) {
    Tile t;
    int sp = 0;
    if (n_split > 1) {
      const int wq = w / n_split;
      sp = w - wq * n_split;
      w = wq;
    }
    // Causal: heaviest pairs first (pair-major), for the balance of the
    // persistent schedule.  Non-causal pairs cost the same, so they go
    // slice-major: the pairs of one slice run at the same time and share its
    // K/V through L2 (measured on one B200, 32 x 4096 x 128 non-causal:
    // 416 -> 377 us).
    int pair;
    if (p.causal) {
      const int wq = w / p.bh;
      pair = n_pairs - 1 - wq;
      t.bh = w - wq * p.bh;
    } else {
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
    if (n_split > 1) {  // (sp + 1) * nb < 17 * 2^24: no 32-bit overflow
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
    mbar_init(bar_q_full, 8 * NG);  // 4*NG softmax warps x 2 CTAs
    for (int s = 0; s < NKS; s++) {
      mbar_init(bar_k_full(s), 2);
      mbar_init(bar_k_empty(s), 1);
    }
    for (int s = 0; s < NVS; s++) {
      mbar_init(bar_v_full(s), 2);
      mbar_init(bar_v_empty(s), 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(bar_s_full(b), 1);
      mbar_init(bar_p_full(b), 8 * NG);
    }
    mbar_init(bar_o_done(0), 1);
    mbar_init(bar_o_done(1), 1);
    mbar_init(bar_drain, 1);
    mbar_init(bar_o_final, 1);
    mbar_init(bar_q_smem_full, 1);  // warp 3
    mbar_init(bar_o_smem_full, 4 * NG);  // the softmax warps of this CTA
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
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_q = tmem;
  const uint32_t t_o = tmem + (uint32_t)D;
  auto t_s = [&](int b) { return tmem + (uint32_t)(2 * D + b * BK); };
  const bool skip = *abort_flag != 0;

  if (warp == 0 || warp == 2) {
    // ------------------------------ TMA producers: warp 0 K halves, warp 2 V halves
    const bool is_k = warp == 0;
    const int NS = is_k ? NKS : NVS;
    if (lane == 0 && !skip) {
      int G = 0;   // global key-block counter
      bool ok = true;
      for (int k = 0; k * n_clusters < n_work && ok; k++) {
        const int w = work_of(k);
        if (w >= n_work) continue;
        const Tile t = tile_of(w);
        for (int j = 0; j < t.n_kv && ok; j++, G++) {
          const int s = G % NS;
          if (G >= NS) {
            const uint32_t empty = is_k ? (kKShare ? bar_s_full(G & 1) : bar_k_empty(s))
                                        : (kVShare ? bar_o_done(G & 1) : bar_v_empty(s));
            ok = mbar_wait(empty, ((G / NS) & 1) ^ 1, abort_flag, p.err, p.wait_ns);
          }
          if (!ok) break;
          const uint32_t full = at_leader(is_k ? bar_k_full(s) : bar_v_full(s));
          if (is_k) {
            mbar_expect_tx_cluster(full, C::kKBytes);
            for (int c = 0; c < D / 32; c++)
              tma_load_3d_pair(sK + s * C::kKBytes + c * C::kKHalf * 128, &tmK, full, 32 * c,
                               (t.j0 + j) * BK + (int)rank * C::kKHalf, t.bh);
          } else {
            mbar_expect_tx_cluster(full, C::kVBytes);
            for (int c = 0; c < C::kDHalf / 32; c++)
              tma_load_3d_pair(sV + s * C::kVBytes + c * BK * 128, &tmV, full,
                               (int)rank * C::kDHalf + 32 * c, (t.j0 + j) * BK, t.bh);
          }
        }
      }
      // Wait (bounded, ignoring the abort flag) for the last load of every slot
      // (the leader's barriers count both CTAs' bytes), so no TMA write can
      // land after the CTAs exit even when a consumer role aborted.
      volatile int no_abort = 0;
      if (leader)
        for (int g = max(0, G - NS); g < G; g++)
          mbar_wait(is_k ? bar_k_full(g % NS) : bar_v_full(g % NS), (g / NS) & 1, &no_abort,
                    p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (leader CTA only; warp-uniform, one
    // elected lane issues each tcgen05.mma / tcgen05.commit)
    if (leader && !skip) {
      constexpr uint32_t idesc_qk = instr_desc(2 * kBM, BK, false);
      constexpr uint32_t idesc_pv = instr_desc(2 * kBM, D, true);
      auto commit_both = [&](uint32_t bar) {
        tc_commit_pair_elect(bar);           // this CTA's copy
        tc_commit_pair_elect(at_peer(bar));  // the peer's copy
      };
      // PV of global block G (block j of its tile): O (+)= P(G) V(G)
      auto issue_pv = [&](int G, int j) -> bool {
        const int b = G & 1, sv = G % NVS;
        if (!__all_sync(0xffffffffu, mbar_wait(bar_p_full(b), (G >> 1) & 1, abort_flag, p.err, p.wait_ns)))
          return false;
        if (!__all_sync(0xffffffffu, mbar_wait(bar_v_full(sv), (G / NVS) & 1, abort_flag, p.err, p.wait_ns)))
          return false;
        tc_fence_after();
        // 8 keys per MMA = two 4-row groups (SBO = 512 B); 32-column chunks LBO apart
        const uint64_t vdesc = smem_desc(sV + sv * C::kVBytes, BK * 128, 512, kLayoutSw128Base32);
#pragma unroll
        for (int kk = 0; kk < BK / 8; kk++)
          mma_ts_pair_elect(t_o, t_s(b) + kk * 8, vdesc + (uint64_t)(kk * 64), idesc_pv,
                            (j > 0 || kk > 0) ? 1u : 0u);
        if (!kVShare) commit_both(bar_v_empty(sv));
        commit_both(bar_o_done(G & 1));
        return true;
      };
      bool ok = true;
      int G = 0, it = 0;
      for (int k = 0; k * n_clusters < n_work && ok; k++) {
        const int w = work_of(k);
        if (w >= n_work) continue;
        const Tile t = tile_of(w);
        ok = __all_sync(0xffffffffu, mbar_wait(bar_q_full, it & 1, abort_flag, p.err, p.wait_ns));
        if (!ok) break;
        tc_fence_after();
        for (int j = 0; j < t.n_kv && ok; j++) {
          const int Gj = G + j, s = Gj % NKS, b = Gj & 1;
          ok = __all_sync(0xffffffffu, mbar_wait(bar_k_full(s), (Gj / NKS) & 1, abort_flag, p.err, p.wait_ns));
          if (!ok) break;
          tc_fence_after();
          const uint64_t kdesc = smem_desc(sK + s * C::kKBytes, 16, 1024, kLayoutSw128);
#pragma unroll
          for (int kk = 0; kk < D / 8; kk++)
            mma_ts_pair_elect(t_s(b), t_q + kk * 8,
                              kdesc + (uint64_t)(((kk >> 2) * C::kKHalf * 128 + (kk & 3) * 32) >> 4),
                              idesc_qk, kk > 0 ? 1u : 0u);
          commit_both(bar_s_full(b));
          if (!kKShare) commit_both(bar_k_empty(s));
          if (j > 0) ok = issue_pv(Gj - 1, j - 1);
        }
        if (ok && t.n_kv > 0) ok = issue_pv(G + t.n_kv - 1, t.n_kv - 1);
        if (!ok) break;
        commit_both(bar_o_final);  // (at once for a tile with no key block)
        G += t.n_kv;
        it++;
      }
      commit_both(bar_drain);
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------ O store and Q load (one lane): after the
    // softmax warps are done with the buffer for a tile step, TMA-store the
    // previous tile's O from it (rows past the slice are clipped by the tensor
    // map), wait until the store has read it, and load the next tile's Q into
    // it at once, a whole tile ahead of its use.
    if (lane == 0 && !skip) {
      bool ok = true, have_prev = false;
      int it = 0, qit = 0;  // tile steps done, Q loads issued
      Tile pt{};
      auto store = [&](bool last) {
        if (pt.q_rows > 0)
          for (int c = 0; c < D / 32; c++)
            tma_store_3d(&tmO, sQ + c * (kBM * 128), 32 * c, pt.q0, pt.z);
        bulk_commit();
        if (last)
          bulk_wait_all();
        else
          bulk_wait_read_all();
      };
      // This CTA's 128 rows of a tile's Q, as D/32 swizzled [128 x 32] chunks
      // (rows past the slice read as zeros).
      auto load_q = [&](const Tile& q) {
        mbar_expect_tx(bar_q_smem_full, C::kQBytes);
        for (int c = 0; c < D / 32; c++)
          tma_load_3d(sQ + c * (kBM * 128), &tmQ, bar_q_smem_full, 32 * c, q.q0, q.bh);
        qit++;
      };
      auto next_work = [&](int k) {  // the round after k that has a tile, or -1
        for (int k2 = k + 1; k2 * n_clusters < n_work; k2++)
          if (work_of(k2) < n_work) return k2;
        return -1;
      };
      const int k0 = next_work(-1);
      if (k0 >= 0) load_q(tile_of(work_of(k0)));
      for (int k = k0; k >= 0 && ok; k = next_work(k)) {
        const Tile t = tile_of(work_of(k));
        ok = mbar_wait(bar_o_smem_full, it & 1, abort_flag, p.err, p.wait_ns);
        if (!ok) break;
        if (have_prev) store(false);
        const int kn = next_work(k);
        if (kn >= 0) load_q(tile_of(work_of(kn)));
        have_prev = true;
        pt = t;
        it++;
      }
      if (ok && have_prev && mbar_wait(bar_o_smem_full, it & 1, abort_flag, p.err, p.wait_ns)) store(true);
      // no Q load may land after exit, even when a consumer role aborted
      volatile int no_abort = 0;
      if (qit > 0) mbar_wait(bar_q_smem_full, (qit - 1) & 1, &no_abort, p.err);
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------ softmax: NG warpgroups, thread = (row, part)
    // Warpgroup g (warps 4+4g .. 7+4g) handles columns [g*BK/NG, (g+1)*BK/NG)
    // of every score row and O columns [g*D/NG, (g+1)*D/NG); the NG parts of a
    // row exchange partial maxima once per block through shared memory and
    // keep separate partial row sums until the epilogue.  The NG warps holding
    // the same 32 rows (warps 4+q, 8+q, ...) run on the same scheduler.
    constexpr int HC = BK / NG, HD = D / NG;
    constexpr int CW = HD >= 32 ? 32 : 16;  // O / Q columns per TMEM access
    static_assert(HC % 32 == 0 && HD % CW == 0, "softmax column split");
    const int g = (warp - kSoftmaxWarp0) >> 2;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter..
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float c_log2 = p.scale_log2;
    float* red = reinterpret_cast<float*>(smem + C::kOffRed);
    // the byte address of columns [col, col+CW) of row r in the swizzled
    // [128 x 32] chunks of the Q / O buffer: 16-byte unit u of row r sits at
    // unit u ^ (r & 7), so 32 threads touching one unit of 32 rows hit every bank
    auto buf_row = [&](int col) {
      return smem + C::kOffQ + (col >> 5) * (kBM * 128) + r * 128;
    };
    auto buf_unit = [&](int col, int e) { return ((((col & 31) >> 2) + e) ^ (r & 7)) << 4; };
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
    // state of the previous tile, written out after the next tile's Q is staged
    bool have_prev = false;
    Tile pt{};
    int pit = 0;
    float pm = -INFINITY, pl = 0.0f;
    // The previous tile's O (scaled by 1/l) into the Q buffer, in the same
    // swizzled layout, for a TMA store: returns false on a failure.  The Q rows
    // this thread wrote over were its own, already copied into TMEM.
    auto epilogue_smem = [&](bool go, float* l_out) -> bool {
      // all NG warps of the quarter reach this on every path
      bool w = go;
      if (w) w = __all_sync(0xffffffffu, mbar_wait(bar_o_final, pit & 1, abort_flag, p.err, p.wait_ns));
      if (*abort_flag) w = false;
      // row-sum exchange slot alternates by tile, so a slot is rewritten only
      // after every warp of the quarter has passed the next epilogue's barrier
      float* lslot = red + 2 * NG * 128 + (pit & 1) * (NG * 128);
      lslot[g * 128 + r] = pl;
      const bool fail = bar_any(1 + quarter, 32 * NG, !w);
      float l_row = 0.0f;
#pragma unroll
      for (int i = 0; i < NG; i++) l_row += lslot[i * 128 + r];
      *l_out = l_row;
      if (fail) return false;
      tc_fence_after();
      const float inv_l = l_row > 0.0f ? 1.0f / l_row : 0.0f;
#pragma unroll
      for (int c = 0; c < HD / CW; c++) {
        const int col = g * HD + c * CW;
        uint32_t rr[CW];
        if (pt.n_kv > 0) {
          tmem_ld_n<CW>(t_o + lane_off + col, rr);
          tmem_wait_ld_regs(rr);
        } else {
#pragma unroll
          for (int e = 0; e < CW; e++) rr[e] = 0u;
        }
        uint8_t* orow = buf_row(col);
#pragma unroll
        for (int e = 0; e < CW / 4; e++)
          *reinterpret_cast<float4*>(orow + buf_unit(col, e)) = make_float4(
              __uint_as_float(rr[4 * e]) * inv_l, __uint_as_float(rr[4 * e + 1]) * inv_l,
              __uint_as_float(rr[4 * e + 2]) * inv_l, __uint_as_float(rr[4 * e + 3]) * inv_l);
      }
      tc_fence_before();  // O reads done before this thread's next barrier arrive
      return true;
    };
    int G = 0, it = 0;
    // (a failure only skips the remaining work; the warps of a quarter still
    // meet at their per-block and epilogue barriers)
    for (int k = 0; k * n_clusters < n_work; k++) {
      const int w = work_of(k);
      if (w >= n_work) continue;
      const Tile t = tile_of(w);
      const long long qg = p.q_offset + t.q0 + r;
      // Stage this tile's Q from the shared-memory buffer.  The previous tile's
      // QK^T MMAs are complete: its last S was visible before its last P was
      // written.
      const bool okq =
          ok && __all_sync(0xffffffffu, mbar_wait(bar_q_smem_full, it & 1, abort_flag, p.err, p.wait_ns));
      if (okq) {
#pragma unroll
        for (int c = 0; c < HD / CW; c++) {
          const int col = g * HD + c * CW;
          const uint8_t* qrow = buf_row(col);
          uint32_t rr[CW];
#pragma unroll
          for (int e = 0; e < CW / 4; e++) {
            const float4 v4 = *reinterpret_cast<const float4*>(qrow + buf_unit(col, e));
            rr[4 * e + 0] = to_tf32_rna(v4.x * c_log2);
            rr[4 * e + 1] = to_tf32_rna(v4.y * c_log2);
            rr[4 * e + 2] = to_tf32_rna(v4.z * c_log2);
            rr[4 * e + 3] = to_tf32_rna(v4.w * c_log2);
          }
          tmem_st_n<CW>(t_q + lane_off + col, rr);
        }
        tmem_wait_st();
        tc_fence_before();
        warp_arrive_leader(bar_q_full);
      }
      float l_prev = 0.0f;
      const bool oke = have_prev ? epilogue_smem(okq, &l_prev) : okq;
      if (!oke) ok = false;
      if (ok) {
        // this warp's O rows (if any) reach the TMA store through warp 3
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_o_smem_full);
      }
      if (ok && have_prev && g == 0 && r < pt.q_rows && (p.lse || split_lse))
        (split_lse ? split_lse + (size_t)pt.z * p.sq : p.lse + (size_t)pt.bh * p.sq)[pt.q0 + r] =
            l_prev > 0.0f ? (pm + __log2f(l_prev)) * 0.69314718055994530942f : -INFINITY;
      float m = -INFINITY, l = 0.0f;  // l: this half's partial row sum
      for (int j = 0; j < t.n_kv && ok; j++) {
        const int Gj = G + j, b = Gj & 1;
        const bool wt =
            __all_sync(0xffffffffu, mbar_wait(bar_s_full(b), (Gj >> 1) & 1, abort_flag, p.err, p.wait_ns));
        tc_fence_after();
        float x[HC];
        if (wt) {
          uint32_t sr[HC];
#pragma unroll
          for (int c = 0; c < HC / 32; c++)
            tmem_ld32(t_s(b) + lane_off + g * HC + c * 32,
                      *reinterpret_cast<uint32_t(*)[32]>(sr + c * 32));
          tmem_wait_ld_regs(sr);
#pragma unroll
          for (int e = 0; e < HC; e++) x[e] = __uint_as_float(sr[e]);
        } else {
#pragma unroll
          for (int e = 0; e < HC; e++) x[e] = -INFINITY;
        }
        const int kbase = (t.j0 + j) * BK + g * HC;
        int lim = min(HC, p.sk - kbase);
        if (p.causal) lim = min(lim, causal_limit(qg, p.k_offset + kbase, HC));
        if (!__all_sync(0xffffffffu, lim == HC)) {
#pragma unroll
          for (int e = 0; e < HC; e++) x[e] = (e < lim) ? x[e] : -INFINITY;
        }
        float mx[4];
#pragma unroll
        for (int q = 0; q < 4; q++) mx[q] = -INFINITY;
#pragma unroll
        for (int e = 0; e < HC; e += 8) {
          const int q = (e >> 3) & 3;
          mx[q] = fmax3(mx[q], x[e], x[e + 1]);
          mx[q] = fmax3(mx[q], x[e + 2], x[e + 3]);
          mx[q] = fmax3(mx[q], x[e + 4], x[e + 5]);
          mx[q] = fmax3(mx[q], x[e + 6], x[e + 7]);
        }
        const float mx_half = fmax3(mx[0], mx[1], fmaxf(mx[2], mx[3]));
        float* slot = red + (Gj & 1) * (NG * 128);
        slot[g * 128 + r] = mx_half;
        // Only the NG warps holding the same 32 rows (on the same scheduler)
        // exchange parts, through named barrier 1+q; the OR makes all of them
        // leave the loop together on a failure.
        if (bar_any(1 + quarter, 32 * NG, !wt)) {
          ok = false;
          break;
        }
        float mx_row = mx_half;
#pragma unroll
        for (int i = 0; i < NG; i++) mx_row = fmaxf(mx_row, slot[i * 128 + r]);
        // All parts hold the same m and see the same mx_row, so they take
        // identical rescale decisions.
        const float m_new = fmaxf(m, mx_row);
        float corr = 1.0f;
        bool need = false;
        if (m == -INFINITY) {
          m = m_new;
        } else if (m_new > m + kRescaleLog2) {
          need = true;
          corr = ex2(m - m_new);
          m = m_new;
        }
        if (__any_sync(0xffffffffu, need) &&
            __all_sync(0xffffffffu, mbar_wait(bar_o_done((Gj - 1) & 1), ((Gj - 1) >> 1) & 1, abort_flag,
                                            p.err, p.wait_ns))) {
          // (a failed wait raises the abort flag; the loop then ends at the
          // next block's bar_any)
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < HD / CW; c++) {
            uint32_t rr[CW];
            tmem_ld_n<CW>(t_o + lane_off + g * HD + c * CW, rr);
            tmem_wait_ld_regs(rr);
#pragma unroll
            for (int e = 0; e < CW; e++) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * corr);
            tmem_st_n<CW>(t_o + lane_off + g * HD + c * CW, rr);
          }
          l *= corr;
        }
        // p = 2^(s - m): s is already scaled by scale*log2e through Q, and m is
        // one of the row's scores, so the row's maximum gives exactly 2^0.
        const float neg_m = (m == -INFINITY) ? 0.0f : -m;
        // One add, one MUFU exponential, one mask and one add per score: the
        // fewest issue slots (packed f32x2 forms and an FMA-pipe polynomial for
        // part of the exponentials measured slower here).
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < HC / 32; c++) {
          uint32_t rr[32];
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            float pe[8];
#pragma unroll
            for (int u = 0; u < 8; u++) pe[u] = ex2(__fadd_rn(x[c * 32 + e + u], neg_m));
#pragma unroll
            for (int u = 0; u < 8; u++) {
              const uint32_t tb = __float_as_uint(pe[u]) & 0xFFFFE000u;
              rs[u & 3] += __uint_as_float(tb);
              rr[e + u] = tb;
            }
          }
          tmem_st32(t_s(b) + lane_off + g * HC + c * 32, rr);
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
    if (have_prev) {
      float l_prev = 0.0f;
      if (epilogue_smem(ok, &l_prev)) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_o_smem_full);
        if (g == 0 && r < pt.q_rows && (p.lse || split_lse))
          (split_lse ? split_lse + (size_t)pt.z * p.sq : p.lse + (size_t)pt.bh * p.sq)[pt.q0 + r] =
              l_prev > 0.0f ? (pm + __log2f(l_prev)) * 0.69314718055994530942f : -INFINITY;
      }
    }
  }
  // Every MMA of the pair (which reads both CTAs' shared memory and writes both
  // CTAs' TMEM) completes before either CTA frees TMEM or exits.
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

// ---- host side -------------------------------------------------------------
template <int D, int BK, int VK, int NKS, int NVS>
cudaError_t launch_tf32(const FwdParams& p, cudaStream_t s, int n_split = 1, float* ws = nullptr) {
  using C = TcCfg<D, BK, VK, NKS, NVS>;
  CUtensorMap mk, mv;
  if (!make_map(&mk, p.k, D, p.sk, p.bh, BK, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mv, p.v, D, p.sk, p.bh, VK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(tc_fwd_tf32<D, BK, VK, NKS, NVS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  const int n_qt = (p.sq + kBM - 1) / kBM;
  const size_t rows = (size_t)p.bh * p.sq;
  float* split_lse = n_split > 1 ? ws + (size_t)n_split * rows * D : nullptr;
  dim3 grid(p.bh, n_qt, n_split);
  cudaError_t le = launch_pdl(tc_fwd_tf32<D, BK, VK, NKS, NVS>, grid, dim3(kThreads), C::kSmemBytes, s,
                              mk, mv, p, ws, split_lse);
  if (le != cudaSuccess) return le;
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || n_split == 1) return e;
  return launch_combine(ws, split_lse, n_split, (long long)rows, D, p.o, p.lse, s);
}

// n_split > 1: partials go to ws ([n_split][bh][sq][d] then [n_split][bh][sq])
// and are merged into p.o / p.lse by the LSE combine kernel.
template <int D, int BK, int NKS, int NVS, int NG>
cudaError_t launch_tf32_pair(const FwdParams& p, cudaStream_t s, int n_split = 1,
                             float* ws = nullptr) {
  using C = PairCfg<D, BK, NKS, NVS, NG>;
  CUtensorMap mk, mv;
  CUtensorMap mq, mo;
  const long long rows = (long long)p.bh * p.sq;
  float* ws_lse = n_split > 1 ? ws + (size_t)n_split * rows * D : nullptr;
  if (!make_map(&mk, p.k, D, p.sk, p.bh, BK / 2, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mv, p.v, D, p.sk, p.bh, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
      !make_map(&mq, p.q, D, p.sq, p.bh, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mo, n_split > 1 ? ws : p.o, D, p.sq, p.bh * n_split, kBM,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device
  static int sm_count[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(tc_fwd_tf32_pair<D, BK, NKS, NVS, NG>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&sm_count[dev & 63], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  const int n_pairs = (p.sq + 2 * kBM - 1) / (2 * kBM);
  const long long n_work = (long long)n_pairs * p.bh * n_split;
  // persistent: one cluster (2 SMs) per SM pair, at most one per work tile
  const int n_clusters = (int)(n_work < sm_count[dev & 63] / 2 ? n_work : sm_count[dev & 63] / 2);
  if (n_work > INT32_MAX) return cudaErrorInvalidValue;
  cudaError_t le = launch_pdl(tc_fwd_tf32_pair<D, BK, NKS, NVS, NG>, dim3(2 * n_clusters),
                              dim3(pair_threads(NG)), C::kSmemBytes, s, mk, mv, mq, mo, p, n_pairs,
                              n_split, ws_lse);
  if (le != cudaSuccess) return le;
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || n_split == 1) return e;
  return launch_combine(ws, ws_lse, n_split, rows, D, p.o, p.lse, s);
}

}  // namespace


// d = 64, 128: the CTA-pair kernel (more than 128 query rows) and the
// single-CTA kernel; d = 32, 96: the single-CTA kernel at every length (the
// pair kernel splits V's columns over two CTAs in 32-column TMA boxes, so it
// needs d % 64 == 0).
bool tc_supported(int d, int precision) {
  return precision == 0 && (d == 32 || d == 64 || d == 96 || d == 128);
}

// Key-range splits for the pair kernel: when the work tiles (256 rows of one
// slice) are at most half the SM pairs, each tile's key blocks are divided so
// that the units fill the pairs in one round, as long as the heaviest unit keeps
// enough blocks (8 at d = 128, 16 at d = 64) to outweigh the partials' extra
// traffic and the merge launch; at most 16 units per tile.  Measured on one
// B200: one 4096-row head 54 -> 35 us (4 units), one 8192-row causal head
// 98 -> 72 us (2 units); shorter slices (1 x 512, 4 x 2048 at d 64) got slower
// and are left whole.  Launches of at most 128 query rows (one CTA per slice in
// the single-CTA kernel, e.g. a chunk of a prefill against a long cache) split
// over blockIdx.z the same way when the slices are at most half the SMs.
// Longest per-cluster sum of work-unit costs under the pair kernels' static
// schedule (units in dispatch order, dealt to the clusters in snake rounds),
// in key blocks of `bk` keys; each unit also costs `tile_cost` blocks (its
// tile change).  Mirrors tile_of / work_of of the kernels.
double pair_schedule_makespan(const FwdParams& p, int n_split, int clusters, int bk,
                              double tile_cost) {
  const int n_pairs = (p.sq + 2 * kBM - 1) / (2 * kBM);
  const long long n_work = (long long)n_pairs * p.bh * n_split;
  if (n_work <= 0 || clusters <= 0) return 0.0;
  std::vector<double> load(clusters, 0.0);
  for (long long u = 0; u < n_work; u++) {
    const long long w = u / n_split;
    const int sp = (int)(u % n_split);
    const int pair = p.causal ? n_pairs - 1 - (int)(w / p.bh) : (int)(w % n_pairs);
    const int q0 = pair * 2 * kBM;
    const int rows = std::min(2 * kBM, p.sq - q0);
    int kend = p.sk;
    if (p.causal) kend = causal_limit(p.q_offset + q0 + rows - 1, p.k_offset, p.sk);
    const long long nb = (kend + bk - 1) / bk;
    const long long n_kv = (sp + 1) * nb / n_split - sp * nb / n_split;
    const long long k = u / clusters, i = u % clusters;
    load[(k & 1) ? clusters - 1 - i : i] += (double)n_kv + tile_cost;
  }
  return *std::max_element(load.begin(), load.end());
}

// Cost in microseconds of merging n_split partials per row: the extra partial
// outputs the kernel writes, and the LSE combine launch that reads them all.
double merge_cost_us(const FwdParams& p, int n_split) {
  const double rows = (double)p.bh * p.sq;
  const double bytes = rows * (p.d + 1) * 4.0 * (2.0 * n_split);
  return 4.0 + bytes / 5.0e6;  // ~5 TB/s, plus launch and tail
}

int tc_pick_splits(const FwdParams& p, int num_sms) {
  if (!(p.d == 32 || p.d == 64 || p.d == 96 || p.d == 128)) return 1;
  const bool pair = p.sq > kBM && (p.d == 64 || p.d == 128);
  if (!pair) {
    if (p.sq > kBM) return 1;
    // Single-CTA kernel, one CTA per slice.  Measured on one B200 (128 rows,
    // d 128): the split pays up to ~20 slices on 4096 keys (51 -> 32 us), is
    // neutral at 40 and slower at 74 (60 -> 78 us), so it needs 4 SMs per
    // slice; parts keep 4 blocks of 128 keys on caches up to 8k keys and 8 on
    // longer ones (1 x 100 x 32768: 320 -> 32 us with 32 parts), at most 64.
    if ((long long)p.bh * 4 > num_sms) return 1;
    int kend1 = p.sk;
    if (p.causal) kend1 = causal_limit(p.q_offset + p.sq - 1, p.k_offset, p.sk);
    const long long nb1 = (kend1 + 127) / 128;
    if (nb1 < 16) return 1;
    const long long min_blocks1 = nb1 >= 128 ? 8 : 4;
    long long split1 = num_sms / p.bh;
    if (split1 > nb1 / min_blocks1) split1 = nb1 / min_blocks1;
    if (split1 > 64) split1 = 64;
    return split1 < 1 ? 1 : (int)split1;
  }
  const long long n_pairs = (p.sq + 2 * kBM - 1) / (2 * kBM);
  const long long n_work = n_pairs * p.bh;
  const long long clusters = num_sms / 2;
  if (n_work > 2 * clusters) return 1;
  if (n_work * 2 > clusters) {
    // One or two rounds of tiles: the longest cluster sets the time.  Causal
    // tiles differ up to the whole key range, so a few heavy tiles can leave
    // most clusters idle (32 x 4096 x 128 over 8 GPUs: 64 tiles of 2..32 key
    // blocks on 74 clusters).  Split every tile's keys in two or three when
    // the schedule model says the shorter longest cluster pays for the merge.
    const double t_blk = p.d == 128 ? 1.35 : 0.75;  // us per 128-key block, one B200
    double best = 0.0;
    int best_s = 1;
    for (int sp = 1; sp <= 3; sp++) {
      const double t = pair_schedule_makespan(p, sp, (int)clusters, 128, 1.2) * t_blk +
                       (sp > 1 ? merge_cost_us(p, sp) : 0.0);
      if (sp == 1 || t < best) {
        best = t;
        best_s = sp;
      }
    }
    return best_s;
  }
  int kend = p.sk;
  if (p.causal) kend = causal_limit(p.q_offset + p.sq - 1, p.k_offset, p.sk);
  const long long max_nkv = (kend + 127) / 128;
  const long long min_blocks = p.d == 128 ? 8 : 16;
  long long split = clusters / n_work;
  if (split > max_nkv / min_blocks) split = max_nkv / min_blocks;
  if (split > 16) split = 16;
  return split < 1 ? 1 : (int)split;
}

size_t tc_scratch_floats(const FwdParams& p, int num_sms) {
  const int split = tc_pick_splits(p, num_sms);
  return split > 1 ? (size_t)split * p.bh * p.sq * (p.d + 1) : 0;
}

cudaError_t launch_tc(const FwdParams& p, int precision, float* scratch, size_t scratch_floats,
                      cudaStream_t s) {
  if (precision != 0) return cudaErrorInvalidValue;
  if (p.sq > 65535 * kBM) return cudaErrorInvalidValue;
  // split the key ranges when the scratch for it was provided
  int split = 1;
  if (scratch && scratch_floats > 0) {
    split = (int)(scratch_floats / ((size_t)p.bh * p.sq * (p.d + 1)));
    if (split < 1) split = 1;
  }
  // A pair covers 256 query rows; a single 128-row tile runs on one SM.  The
  // pair kernel runs two softmax warpgroups (four measured slower: the softmax
  // phases are bound by issue and latency, not by the number of warps).
  const bool single = p.sq <= kBM;
  if (p.d == 96) return launch_tf32<96, 128, 64, 2, 3>(p, s, split, scratch);
  if (p.d == 32) return launch_tf32<32, 128, 128, 3, 3>(p, s, split, scratch);
  if (p.d == 128)
    return single ? launch_tf32<128, 128, 64, 2, 3>(p, s, split, scratch)
                  : launch_tf32_pair<128, 128, 2, 2, 2>(p, s, split, scratch);
  if (p.d == 64)
    return single ? launch_tf32<64, 128, 128, 3, 3>(p, s, split, scratch)
                  : launch_tf32_pair<64, 128, 3, 3, 2>(p, s, split, scratch);
  return cudaErrorInvalidValue;
}

}  // namespace fa
