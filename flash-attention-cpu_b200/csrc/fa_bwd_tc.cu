// Tensor-core backward pass (TF32 precision): dQ, dK, dV on tcgen05 MMAs with
// the accumulators in tensor memory.  With c = scale * log2(e), Qs = c * Q and
// LSE2 = lse * log2(e), the forward's probabilities are P = 2^(Qs K^T - LSE2)
// (masked entries 0), and
//   D = rowsum(dO * O),  dV = P^T dO,  dP = dO V^T,  dS = P * (dP - D),
//   dK = scale dS^T Q,  dQ = scale dS K.
//
// Operand layouts.  Q and dO are contracted along the head dimension for the
// scores (K-major operands) and along the rows for the gradients (MN-major
// operands), and so is K in the dQ CTA.  A TF32 MN-major operand must use the
// "128-byte swizzle with 32-byte atoms" layout (layout type 1), and a K-major
// one reads the 16-byte-granule 128-byte swizzle (layout type 2), so each such
// tile is loaded twice by TMA, once per layout (tensor maps with
// CU_TENSOR_MAP_SWIZZLE_128B and CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B over the
// same row-major tensor).  Every tile is [D/32 chunks][rows][32 f32].  Each
// operand has its own single slot, freed by the commit of the MMA that reads it
// last, so the next block's copy of an early operand (the scores' K-major
// tiles) overlaps the current block's gradient MMAs.
//
// One launch runs two kinds of CTA (1 per SM: each allocates all 512 TMEM
// columns), interleaved, heaviest causal blocks first.  A small prepass
// writes LSE2 and D per query row (padded to a multiple of 128 rows: LSE2 =
// +inf, D = 0 there, so padded rows get P = 0).
//
// dK/dV CTA: 128 keys of one slice (MMA M = 128, thread = key row).
//   TMEM: K [0, D) (A operand of S^T, staged from registers), dV [D, 2D),
//   dK [2D, 3D), then NSB buffers of S^T (64 cols) and dP^T (64 cols); NSB = 2
//   when 3D + 256 <= 512, else 1.
//   shared memory: V [128 keys] (K-major A of dP^T); slots for the 64-row
//   query block's Q (K-major), dO (K-major), dO (MN-major), Q (MN-major) with
//   that block's LSE2 and D.
//   Per 64-row query block: S^T = K Qs^T (A from TMEM, Q scaled in the
//   softmax step), dP^T = V dO^T; the softmax warps overwrite S^T with P^T and
//   dP^T with dS^T in place; then dV += P^T dO and dK += dS^T Q (A from TMEM,
//   B MN-major).  With NSB = 1 the issue order dV_{i-1}, S^T_i, dK_{i-1},
//   dP^T_i keeps the tensor pipe busy while the softmax warps work.
//
// dQ CTA: 128 query rows of one slice (thread = query row).
//   TMEM: Qs [0, D) (scaled by c and rounded to TF32 while staged), dQ
//   [D, 2D), two buffers of S (64) and dP (64).
//   shared memory: dO [128 rows] (K-major A of dP); slots for the 64-key
//   block's K (K-major), V (K-major), K (MN-major).  Per key block: S = Qs K^T,
//   dP = dO V^T, dS written over S, then dQ += dS K.
//
// Warps: 0 TMA producer (one lane), 1 MMA issuer (one elected lane), 2..9
// "softmax" warps: warp w reads TMEM lanes 32*(w%4).., and warps w and w+4
// split each row's 64 columns.  All waits are bounded (kWaitLimitNs, or the
// limit a test sets); on expiry the CTA raises its abort flag and the device
// error word, every role leaves, in-flight copies and MMAs are drained and
// TMEM is freed.
#include "fa_tc_ptx.cuh"

namespace fa {
namespace {

constexpr int kTR = 128;      // rows of a CTA's own block (keys or query rows): MMA M
constexpr int kTB = 64;       // rows per streamed block (queries or keys): MMA N
constexpr int kTThreads = 320;
constexpr int kTWarp0 = 2;    // first softmax warp
constexpr int kTSoftThreads = 256;
constexpr float kLog2e = 1.44269504088896340736f;

struct BwdTcParams {
  const float* q;     // row-major inputs and outputs, as BwdParams
  const float* k;
  const float* lse2;  // [bh][sq_pad]: lse * log2(e) (+inf on padding and empty rows)
  const float* dvec;  // [bh][sq_pad]: rowsum(dO * O) (0 on padding)
  float* dq;
  float* dk;
  float* dv;
  int bh, sq, sk, sq_pad;
  long long q_offset, k_offset;
  int causal;
  float scale, scale_log2;
  int n_kv_cta, n_q_cta;  // bh * ceil(sk/128) and bh * ceil(sq/128)
  int* err;
  unsigned long long wait_ns;
};

// Tensor maps (3-D [bh][seq][d], boxes of 32 f32 x rows).  K-major maps use the
// 128-byte swizzle, MN-major ones the 32-byte-atom variant.
struct BwdMaps {
  CUtensorMap v128;  // V, 128-key box, K-major        (dK/dV)
  CUtensorMap qk;    // Q, 64-row box, K-major         (dK/dV)
  CUtensorMap qm;    // Q, 64-row box, MN-major        (dK/dV)
  CUtensorMap ok;    // dO, 64-row box, K-major        (dK/dV)
  CUtensorMap om;    // dO, 64-row box, MN-major       (dK/dV)
  CUtensorMap o128;  // dO, 128-row box, K-major       (dQ)
  CUtensorMap kk;    // K, 64-key box, K-major         (dQ)
  CUtensorMap km;    // K, 64-key box, MN-major        (dQ)
  CUtensorMap vk;    // V, 64-key box, K-major         (dQ)
};

template <int D>
struct BwdTcCfg {
  static constexpr int kNsbKV = (3 * D + 4 * kTB <= 512) ? 2 : 1;
  static constexpr int kTileB = kTB * D * 4;   // one 64-row tile
  static constexpr int kTileA = kTR * D * 4;   // one 128-row tile
  // dK/dV CTA: V | Q K-major | dO K-major | dO MN-major | Q MN-major | LSE2, D
  static constexpr int kKvV = 0;
  static constexpr int kKvQK = kTileA;
  static constexpr int kKvOK = kKvQK + kTileB;
  static constexpr int kKvOM = kKvOK + kTileB;
  static constexpr int kKvQM = kKvOM + kTileB;
  static constexpr int kKvVec = kKvQM + kTileB;
  static constexpr int kEndKV = kKvVec + 2 * kTB * 4;
  // dQ CTA: dO | K K-major | V K-major | K MN-major
  static constexpr int kQDO = 0;
  static constexpr int kQKK = kTileA;
  static constexpr int kQVK = kQKK + kTileB;
  static constexpr int kQKM = kQVK + kTileB;
  static constexpr int kEndQ = kQKM + kTileB;
  static constexpr int kOffBar = (kEndKV > kEndQ ? kEndKV : kEndQ);
  static constexpr int kNumBars = 20;
  // At least 116 KB, so that two CTAs never share an SM: each allocates all
  // 512 TMEM columns, and a second one would wait for the first to finish.
  static constexpr int kSmemUsed = kOffBar + kNumBars * 8 + 16 + 1024;
  static constexpr int kSmemBytes = kSmemUsed > 118784 ? kSmemUsed : 118784;
  static_assert(D % 32 == 0 && D <= 128, "D in {32, 64, 96, 128}");
  static_assert(2 * D + 4 * kTB <= 512, "dQ TMEM budget");
  static_assert(3 * D + 2 * kTB <= 512, "dK/dV TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared-memory budget");
};

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_ss_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
// Descriptors of a [D/32][R][32] tile; `kk` selects the kk-th group of 8
// elements along the inner product.  K-major (128-byte swizzle): the group
// sits in chunk kk/4 at byte 32*(kk%4) of each row.  MN-major (32-byte-atom
// swizzle): 8 rows = 1024 bytes per group, chunks R*128 bytes apart.
template <int R>
__device__ __forceinline__ uint64_t desc_k(uint32_t tile, int kk) {
  return smem_desc(tile + (uint32_t)((kk >> 2) * R * 128 + (kk & 3) * 32), 16, 1024, kLayoutSw128);
}
template <int R>
__device__ __forceinline__ uint64_t desc_mn(uint32_t tile, int kk) {
  return smem_desc(tile + (uint32_t)kk * 1024u, R * 128, 512, kLayoutSw128Base32);
}
template <int D, int R>
__device__ __forceinline__ void tma_tile(uint32_t dst, const CUtensorMap* map, uint32_t bar, int row,
                                         int bh) {
#pragma unroll
  for (int c = 0; c < D / 32; c++) tma_load_3d(dst + c * R * 128, map, bar, 32 * c, row, bh);
}

// Stages cols [c0, c0 + N) of a row-major row into TMEM, times `mul`, rounded
// to TF32 (zeros for a row past the end).
template <int N>
__device__ __forceinline__ void stage_row_to_tmem(const float* row, bool valid, float mul,
                                                  uint32_t taddr) {
#pragma unroll
  for (int c = 0; c < N; c += 16) {
    uint32_t r[16];
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 v = valid ? __ldg(reinterpret_cast<const float4*>(row + c + e))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      r[e] = to_tf32_rna(v.x * mul);
      r[e + 1] = to_tf32_rna(v.y * mul);
      r[e + 2] = to_tf32_rna(v.z * mul);
      r[e + 3] = to_tf32_rna(v.w * mul);
    }
    tmem_st16(taddr + c, r);
  }
}

// Writes this thread's row (N columns) of a TMEM accumulator, times `mul`, to a
// row-major output row.
template <int N>
__device__ __forceinline__ void tmem_row_out(uint32_t taddr, float* dst, float mul, bool store) {
#pragma unroll
  for (int c = 0; c < N; c += 16) {
    uint32_t r[16];
    tmem_ld16(taddr + c, r);
    tmem_wait_ld_regs(r);
    if (store) {
#pragma unroll
      for (int e = 0; e < 16; e += 4)
        *reinterpret_cast<float4*>(dst + c + e) =
            make_float4(__uint_as_float(r[e]) * mul, __uint_as_float(r[e + 1]) * mul,
                        __uint_as_float(r[e + 2]) * mul, __uint_as_float(r[e + 3]) * mul);
    }
  }
}
template <int N>
__device__ __forceinline__ void zero_row_out(float* dst) {
#pragma unroll
  for (int c = 0; c < N; c += 4) *reinterpret_cast<float4*>(dst + c) = make_float4(0.f, 0.f, 0.f, 0.f);
}

struct Bars {
  uint32_t b0;
  __device__ uint32_t operator()(int i) const { return b0 + 8u * (uint32_t)i; }
};
// Barrier indices.  Operand slots 0..3: dK/dV: Q K-major, dO K-major, dO
// MN-major, Q MN-major (+ LSE2, D); dQ: K K-major, V K-major, K MN-major.
constexpr int kBarStatic = 0;  // V (dK/dV) or dO (dQ) arrived
constexpr int kBarStaged = 1;  // K (dK/dV) or Qs (dQ) staged in TMEM by the 256 softmax threads
constexpr int kBarFull = 2;    // +slot: operand loaded
constexpr int kBarEmpty = 6;   // +slot: operand slot free again
constexpr int kBarS = 10;      // +buf: S (or S^T) complete
constexpr int kBarDP = 12;     // +buf: dP (or dP^T) complete
constexpr int kBarP = 14;      // +buf: P^T written (256 arrivals)
constexpr int kBarDS = 16;     // +buf: dS written (256 arrivals)
constexpr int kBarAcc = 18;    // the accumulators are final
constexpr int kBarDrain = 19;  // every MMA issued has completed

// The producer's loads of one operand slot: block i waits until the MMA that
// read block i-1 from the slot has completed.
struct SlotLoader {
  Bars bar;
  volatile int* abort_flag;
  int* err;
  unsigned long long wait_ns;
  __device__ bool acquire(int slot, int i) const {
    if (i == 0) return true;
    return mbar_wait(bar(kBarEmpty + slot), (i - 1) & 1, abort_flag, err, wait_ns);
  }
};

// ---------------------------------------------------------------- dK / dV CTA
template <int D>
__device__ void cta_dkdv(const BwdMaps& m, const BwdTcParams& p, int bh, int kb, uint32_t sbase,
                         Bars bar, uint32_t tmem, volatile int* abort_flag) {
  using C = BwdTcCfg<D>;
  constexpr int NSB = C::kNsbKV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = kb * kTR;
  int q_first = 0;
  if (p.causal) {
    const long long f = (long long)k0 + p.k_offset - p.q_offset;  // first row that sees key k0
    q_first = f <= 0 ? 0 : (f >= p.sq ? p.sq : (int)f);
  }
  const int qb0 = q_first / kTB;
  const int nqb = (p.sq + kTB - 1) / kTB - qb0;
  const uint32_t sV = sbase + C::kKvV, sQK = sbase + C::kKvQK, sOK = sbase + C::kKvOK;
  const uint32_t sOM = sbase + C::kKvOM, sQM = sbase + C::kKvQM, sVec = sbase + C::kKvVec;
  const uint32_t t_k = tmem, t_dv = tmem + D, t_dk = tmem + 2 * D;
  auto t_s = [&](int b) { return tmem + 3 * D + b * 2 * kTB; };
  auto t_dp = [&](int b) { return tmem + 3 * D + b * 2 * kTB + kTB; };
  const bool skip = *abort_flag != 0;

  if (warp == 0) {
    if (lane == 0 && !skip) {
      mbar_expect_tx(bar(kBarStatic), C::kTileA);
      tma_tile<D, kTR>(sV, &m.v128, bar(kBarStatic), k0, bh);
      const SlotLoader sl{bar, abort_flag, p.err, p.wait_ns};
      int loads[4] = {0, 0, 0, 0};  // loads issued per operand slot
      for (int i = 0; i < nqb; i++) {
        const int q0 = (qb0 + i) * kTB;
        const size_t r0 = (size_t)bh * p.sq_pad + q0;
        if (!sl.acquire(0, i)) break;
        mbar_expect_tx(bar(kBarFull + 0), C::kTileB);
        tma_tile<D, kTB>(sQK, &m.qk, bar(kBarFull + 0), q0, bh);
        loads[0]++;
        if (!sl.acquire(1, i)) break;
        mbar_expect_tx(bar(kBarFull + 1), C::kTileB);
        tma_tile<D, kTB>(sOK, &m.ok, bar(kBarFull + 1), q0, bh);
        loads[1]++;
        if (!sl.acquire(2, i)) break;
        mbar_expect_tx(bar(kBarFull + 2), C::kTileB);
        tma_tile<D, kTB>(sOM, &m.om, bar(kBarFull + 2), q0, bh);
        loads[2]++;
        if (!sl.acquire(3, i)) break;
        mbar_expect_tx(bar(kBarFull + 3), C::kTileB + 2 * kTB * 4);
        tma_tile<D, kTB>(sQM, &m.qm, bar(kBarFull + 3), q0, bh);
        bulk_load(sVec, p.lse2 + r0, kTB * 4, bar(kBarFull + 3));
        bulk_load(sVec + kTB * 4, p.dvec + r0, kTB * 4, bar(kBarFull + 3));
        loads[3]++;
      }
      // Wait (bounded, ignoring the abort flag) for the last load of every
      // slot, so no copy lands after the CTA exits even when a role aborted.
      volatile int no_abort = 0;
      mbar_wait(bar(kBarStatic), 0, &no_abort, p.err);
      for (int sl_i = 0; sl_i < 4; sl_i++)
        if (loads[sl_i] > 0) mbar_wait(bar(kBarFull + sl_i), (loads[sl_i] - 1) & 1, &no_abort, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (!skip) {
      constexpr uint32_t idesc_s = instr_desc(kTR, kTB, false);
      constexpr uint32_t idesc_g = instr_desc(kTR, D, true);
      bool ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarStatic), 0, abort_flag, p.err, p.wait_ns));
      ok = ok && __all_sync(0xffffffffu, mbar_wait(bar(kBarStaged), 0, abort_flag, p.err, p.wait_ns));
      tc_fence_after();
      auto wait_bar = [&](int b, int parity) {
        const bool w = mbar_wait(bar(b), parity, abort_flag, p.err, p.wait_ns);
        tc_fence_after();
        return __all_sync(0xffffffffu, w);
      };
      auto issue_s = [&](int i) {  // S^T = K Qs^T
        if (!wait_bar(kBarFull + 0, i & 1)) return false;
        const int b = i % NSB;
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++)
          mma_ts_elect(t_s(b), t_k + kk * 8, desc_k<kTB>(sQK, kk), idesc_s, kk > 0);
        tc_commit_elect(bar(kBarS + b));
        tc_commit_elect(bar(kBarEmpty + 0));
        return true;
      };
      auto issue_dp = [&](int i) {  // dP^T = V dO^T
        if (!wait_bar(kBarFull + 1, i & 1)) return false;
        const int b = i % NSB;
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++)
          mma_ss_elect(t_dp(b), desc_k<kTR>(sV, kk), desc_k<kTB>(sOK, kk), idesc_s, kk > 0);
        tc_commit_elect(bar(kBarDP + b));
        tc_commit_elect(bar(kBarEmpty + 1));
        return true;
      };
      auto issue_dv = [&](int i) {  // dV += P^T dO
        const int b = i % NSB;
        if (!wait_bar(kBarFull + 2, i & 1)) return false;
        if (!wait_bar(kBarP + b, (i / NSB) & 1)) return false;
#pragma unroll
        for (int kk = 0; kk < kTB / 8; kk++)
          mma_ts_elect(t_dv, t_s(b) + kk * 8, desc_mn<kTB>(sOM, kk), idesc_g,
                       (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit_elect(bar(kBarEmpty + 2));
        return true;
      };
      auto issue_dk = [&](int i) {  // dK += dS^T Q
        const int b = i % NSB;
        if (!wait_bar(kBarFull + 3, i & 1)) return false;
        if (!wait_bar(kBarDS + b, (i / NSB) & 1)) return false;
#pragma unroll
        for (int kk = 0; kk < kTB / 8; kk++)
          mma_ts_elect(t_dk, t_dp(b) + kk * 8, desc_mn<kTB>(sQM, kk), idesc_g,
                       (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit_elect(bar(kBarEmpty + 3));
        return true;
      };
      for (int i = 0; i < nqb && ok; i++) {
        if constexpr (NSB == 2) {
          ok = issue_s(i) && issue_dp(i);
          if (ok && i > 0) ok = issue_dv(i - 1) && issue_dk(i - 1);
        } else {
          if (i > 0) ok = issue_dv(i - 1);
          ok = ok && issue_s(i);
          if (ok && i > 0) ok = issue_dk(i - 1);
          ok = ok && issue_dp(i);
        }
      }
      if (ok && nqb > 0 && issue_dv(nqb - 1) && issue_dk(nqb - 1)) tc_commit_elect(bar(kBarAcc));
      // Drain: all MMAs issued by this warp complete before TMEM is freed.
      tc_commit_elect(bar(kBarDrain));
      volatile int no_abort = 0;
      mbar_wait(bar(kBarDrain), 0, &no_abort, p.err);
    }
    __syncwarp();
  } else {
    // softmax warps: thread = key row j, columns [32h, 32h + 32) of each block
    const int quarter = warp & 3, h = (warp - kTWarp0) >> 2;
    const int j = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = !skip;
    if (ok) {
      stage_row_to_tmem<D / 2>(p.k + ((size_t)bh * p.sk + k0 + j) * D + h * (D / 2),
                               k0 + j < p.sk, 1.0f, t_k + lane_off + h * (D / 2));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarStaged));
    }
    const long long kg = p.k_offset + k0 + j;
    const float* svec = reinterpret_cast<const float*>(__cvta_shared_to_generic(sVec));
    const float c = p.scale_log2;
    for (int i = 0; i < nqb && ok; i++) {
      const int b = i % NSB;
      const long long qg0 = p.q_offset + (long long)(qb0 + i) * kTB + 32 * h;
      // P of column e is nonzero only for e >= lo (causal)
      const long long lo = p.causal ? kg - qg0 : -1;
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar(kBarFull + 3), i & 1, abort_flag, p.err, p.wait_ns) &&
                          mbar_wait(bar(kBarS + b), (i / NSB) & 1, abort_flag, p.err, p.wait_ns));
      if (!ok) break;
      tc_fence_after();
      uint32_t x[32];
      tmem_ld32(t_s(b) + lane_off + 32 * h, x);
      tmem_wait_ld_regs(x);
      float pr[32];
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(svec + 32 * h + e);
        pr[e] = ex2(fmaf(__uint_as_float(x[e]), c, -l4.x));
        pr[e + 1] = ex2(fmaf(__uint_as_float(x[e + 1]), c, -l4.y));
        pr[e + 2] = ex2(fmaf(__uint_as_float(x[e + 2]), c, -l4.z));
        pr[e + 3] = ex2(fmaf(__uint_as_float(x[e + 3]), c, -l4.w));
      }
      if (__any_sync(0xffffffffu, lo > 0)) {
#pragma unroll
        for (int e = 0; e < 32; e++) pr[e] = (e >= lo) ? pr[e] : 0.0f;
      }
#pragma unroll
      for (int e = 0; e < 32; e++) x[e] = __float_as_uint(pr[e]);
      tmem_st32(t_s(b) + lane_off + 32 * h, x);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarP + b));
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar(kBarDP + b), (i / NSB) & 1, abort_flag, p.err, p.wait_ns));
      if (!ok) break;
      tc_fence_after();
      tmem_ld32(t_dp(b) + lane_off + 32 * h, x);
      tmem_wait_ld_regs(x);
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float4 d4 = *reinterpret_cast<const float4*>(svec + kTB + 32 * h + e);
        x[e] = __float_as_uint(pr[e] * (__uint_as_float(x[e]) - d4.x));
        x[e + 1] = __float_as_uint(pr[e + 1] * (__uint_as_float(x[e + 1]) - d4.y));
        x[e + 2] = __float_as_uint(pr[e + 2] * (__uint_as_float(x[e + 2]) - d4.z));
        x[e + 3] = __float_as_uint(pr[e + 3] * (__uint_as_float(x[e + 3]) - d4.w));
      }
      tmem_st32(t_dp(b) + lane_off + 32 * h, x);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarDS + b));
    }
    if (nqb > 0) {
      const bool w = ok ? mbar_wait(bar(kBarAcc), 0, abort_flag, p.err, p.wait_ns) : false;
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tc_fence_after();
      const bool row_ok = k0 + j < p.sk;
      const size_t ro = ((size_t)bh * p.sk + k0 + j) * D + h * (D / 2);
      if (nqb > 0) {
        tmem_row_out<D / 2>(t_dv + lane_off + h * (D / 2), p.dv + ro, 1.0f, row_ok);
        tmem_row_out<D / 2>(t_dk + lane_off + h * (D / 2), p.dk + ro, p.scale, row_ok);
      } else if (row_ok) {
        zero_row_out<D / 2>(p.dv + ro);
        zero_row_out<D / 2>(p.dk + ro);
      }
    }
    tc_fence_before();
  }
}

// ---------------------------------------------------------------- dQ CTA
template <int D>
__device__ void cta_dq(const BwdMaps& m, const BwdTcParams& p, int bh, int qb, uint32_t sbase,
                       Bars bar, uint32_t tmem, volatile int* abort_flag) {
  using C = BwdTcCfg<D>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * kTR;
  const int q_rows = min(kTR, p.sq - q0);
  int kend = p.sk;
  if (p.causal) kend = causal_limit(p.q_offset + q0 + q_rows - 1, p.k_offset, p.sk);
  const int nkb = (kend + kTB - 1) / kTB;
  const uint32_t sDO = sbase + C::kQDO, sKK = sbase + C::kQKK, sVK = sbase + C::kQVK;
  const uint32_t sKM = sbase + C::kQKM;
  const uint32_t t_q = tmem, t_dq = tmem + D;
  auto t_s = [&](int b) { return tmem + 2 * D + b * 2 * kTB; };
  auto t_dp = [&](int b) { return tmem + 2 * D + b * 2 * kTB + kTB; };
  const bool skip = *abort_flag != 0;

  if (warp == 0) {
    if (lane == 0 && !skip) {
      mbar_expect_tx(bar(kBarStatic), C::kTileA);
      tma_tile<D, kTR>(sDO, &m.o128, bar(kBarStatic), q0, bh);
      const SlotLoader sl{bar, abort_flag, p.err, p.wait_ns};
      int loads[3] = {0, 0, 0};
      for (int t = 0; t < nkb; t++) {
        const int kr = t * kTB;
        if (!sl.acquire(0, t)) break;
        mbar_expect_tx(bar(kBarFull + 0), C::kTileB);
        tma_tile<D, kTB>(sKK, &m.kk, bar(kBarFull + 0), kr, bh);
        loads[0]++;
        if (!sl.acquire(1, t)) break;
        mbar_expect_tx(bar(kBarFull + 1), C::kTileB);
        tma_tile<D, kTB>(sVK, &m.vk, bar(kBarFull + 1), kr, bh);
        loads[1]++;
        if (!sl.acquire(2, t)) break;
        mbar_expect_tx(bar(kBarFull + 2), C::kTileB);
        tma_tile<D, kTB>(sKM, &m.km, bar(kBarFull + 2), kr, bh);
        loads[2]++;
      }
      volatile int no_abort = 0;
      mbar_wait(bar(kBarStatic), 0, &no_abort, p.err);
      for (int sl_i = 0; sl_i < 3; sl_i++)
        if (loads[sl_i] > 0) mbar_wait(bar(kBarFull + sl_i), (loads[sl_i] - 1) & 1, &no_abort, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (!skip) {
      constexpr uint32_t idesc_s = instr_desc(kTR, kTB, false);
      constexpr uint32_t idesc_g = instr_desc(kTR, D, true);
      bool ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarStatic), 0, abort_flag, p.err, p.wait_ns));
      ok = ok && __all_sync(0xffffffffu, mbar_wait(bar(kBarStaged), 0, abort_flag, p.err, p.wait_ns));
      tc_fence_after();
      auto wait_bar = [&](int b, int parity) {
        const bool w = mbar_wait(bar(b), parity, abort_flag, p.err, p.wait_ns);
        tc_fence_after();
        return __all_sync(0xffffffffu, w);
      };
      auto issue_dq = [&](int t) {  // dQ += dS K
        const int b = t & 1;
        if (!wait_bar(kBarFull + 2, t & 1)) return false;
        if (!wait_bar(kBarDS + b, (t >> 1) & 1)) return false;
#pragma unroll
        for (int kk = 0; kk < kTB / 8; kk++)
          mma_ts_elect(t_dq, t_s(b) + kk * 8, desc_mn<kTB>(sKM, kk), idesc_g,
                       (t > 0 || kk > 0) ? 1u : 0u);
        tc_commit_elect(bar(kBarEmpty + 2));
        return true;
      };
      for (int t = 0; t < nkb && ok; t++) {
        const int b = t & 1;
        if (!(ok = wait_bar(kBarFull + 0, t & 1))) break;
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++)  // S = Qs K^T
          mma_ts_elect(t_s(b), t_q + kk * 8, desc_k<kTB>(sKK, kk), idesc_s, kk > 0);
        tc_commit_elect(bar(kBarS + b));
        tc_commit_elect(bar(kBarEmpty + 0));
        if (!(ok = wait_bar(kBarFull + 1, t & 1))) break;
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++)  // dP = dO V^T
          mma_ss_elect(t_dp(b), desc_k<kTR>(sDO, kk), desc_k<kTB>(sVK, kk), idesc_s, kk > 0);
        tc_commit_elect(bar(kBarDP + b));
        tc_commit_elect(bar(kBarEmpty + 1));
        if (t > 0) ok = issue_dq(t - 1);
      }
      if (ok && nkb > 0 && issue_dq(nkb - 1)) tc_commit_elect(bar(kBarAcc));
      tc_commit_elect(bar(kBarDrain));
      volatile int no_abort = 0;
      mbar_wait(bar(kBarDrain), 0, &no_abort, p.err);
    }
    __syncwarp();
  } else {
    // softmax warps: thread = query row r, key columns [32h, 32h + 32) of each block
    const int quarter = warp & 3, h = (warp - kTWarp0) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const size_t vrow = (size_t)bh * p.sq_pad + q0 + r;
    bool ok = !skip;
    float l2 = 0.f, dd = 0.f;
    if (ok) {
      l2 = __ldg(p.lse2 + vrow);
      dd = __ldg(p.dvec + vrow);
      stage_row_to_tmem<D / 2>(p.q + ((size_t)bh * p.sq + q0 + r) * D + h * (D / 2), r < q_rows,
                               p.scale_log2, t_q + lane_off + h * (D / 2));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarStaged));
    }
    const long long qg = p.q_offset + q0 + r;
    for (int t = 0; t < nkb && ok; t++) {
      const int b = t & 1;
      const int kc0 = t * kTB + 32 * h;  // first key of this thread's columns
      // visible columns [0, lim)
      int lim = min(32, p.sk - kc0);
      if (p.causal) lim = min(lim, causal_limit(qg, p.k_offset + kc0, 32));
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar(kBarS + b), (t >> 1) & 1, abort_flag, p.err, p.wait_ns));
      if (!ok) break;
      tc_fence_after();
      uint32_t x[32];
      tmem_ld32(t_s(b) + lane_off + 32 * h, x);
      tmem_wait_ld_regs(x);
      float pr[32];
#pragma unroll
      for (int e = 0; e < 32; e++) pr[e] = ex2(__uint_as_float(x[e]) - l2);
      if (!__all_sync(0xffffffffu, lim >= 32)) {
#pragma unroll
        for (int e = 0; e < 32; e++) pr[e] = (e < lim) ? pr[e] : 0.0f;
      }
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar(kBarDP + b), (t >> 1) & 1, abort_flag, p.err, p.wait_ns));
      if (!ok) break;
      tc_fence_after();
      tmem_ld32(t_dp(b) + lane_off + 32 * h, x);
      tmem_wait_ld_regs(x);
#pragma unroll
      for (int e = 0; e < 32; e++) x[e] = __float_as_uint(pr[e] * (__uint_as_float(x[e]) - dd));
      tmem_st32(t_s(b) + lane_off + 32 * h, x);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarDS + b));
    }
    if (nkb > 0) {
      const bool w = ok ? mbar_wait(bar(kBarAcc), 0, abort_flag, p.err, p.wait_ns) : false;
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tc_fence_after();
      const bool row_ok = r < q_rows;
      float* dst = p.dq + ((size_t)bh * p.sq + q0 + r) * D + h * (D / 2);
      if (nkb > 0)
        tmem_row_out<D / 2>(t_dq + lane_off + h * (D / 2), dst, p.scale, row_ok);
      else if (row_ok)
        zero_row_out<D / 2>(dst);
    }
    tc_fence_before();
  }
}

template <int D>
__global__ void __launch_bounds__(kTThreads, 1)
    tc_bwd_tf32(const __grid_constant__ BwdMaps m, BwdTcParams p) {
  using C = BwdTcCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const Bars bar{sbase + C::kOffBar};
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffBar + C::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5;

  // CTA i: the two kinds alternate while both last, heaviest causal blocks
  // first (low key blocks for dK/dV, high query blocks for dQ).
  const int i = blockIdx.x;
  const int both = 2 * min(p.n_kv_cta, p.n_q_cta);
  bool is_kv;
  int rank;
  if (i < both) {
    is_kv = (i & 1) == 0;
    rank = i >> 1;
  } else {
    is_kv = p.n_kv_cta > p.n_q_cta;
    rank = i - both / 2;
  }
  const int bh = rank % p.bh, blk = rank / p.bh;

  if (threadIdx.x == 0) {
    for (int b = 0; b < C::kNumBars; b++) {
      const bool many = b == kBarStaged || (b >= kBarP && b < kBarAcc);
      mbar_init(bar(b), many ? kTSoftThreads : 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // (launched with launch_pdl: the prepass's LSE2 and D are read below)
  grid_dep_wait();
  if (threadIdx.x == 0) *abort_flag = (*(volatile int*)p.err != 0) ? 1 : 0;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (is_kv)
    cta_dkdv<D>(m, p, bh, blk, sbase, bar, tmem, abort_flag);
  else
    cta_dq<D>(m, p, bh, (p.n_q_cta / p.bh) - 1 - blk, sbase, bar, tmem, abort_flag);
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u)
                 : "memory");
  }
}

// LSE2 = lse * log2(e) and D = rowsum(dO * O) per query row, padded to sq_pad
// rows (LSE2 = +inf, D = 0 on the padding and LSE2 = +inf on rows that see no
// key, so P = 0 there).  One warp per row.
__global__ void __launch_bounds__(256) bwd_rowvec(const float* __restrict__ o,
                                                  const float* __restrict__ dout,
                                                  const float* __restrict__ lse, float* lse2,
                                                  float* dvec, int bh, int sq, int sq_pad, int d) {
  const size_t w = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (size_t)bh * sq_pad) return;
  const int row = (int)(w % sq_pad);
  const size_t h = w / sq_pad;
  float acc = 0.0f, l2 = INFINITY;
  if (row < sq) {
    const size_t base = (h * sq + row) * d;
    for (int c = lane * 4; c < d; c += 128) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(o + base + c));
      const float4 b = __ldg(reinterpret_cast<const float4*>(dout + base + c));
      acc = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
    }
    acc = warp_sum(acc);
    const float l = lse[h * sq + row];
    if (l != -INFINITY) l2 = l * kLog2e;
  }
  if (lane == 0) {
    lse2[w] = l2;
    dvec[w] = acc;
  }
}

template <int D>
cudaError_t launch_tc_bwd_d(const BwdParams& bp, float* ws, cudaStream_t s) {
  using C = BwdTcCfg<D>;
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(tc_bwd_tf32<D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  BwdMaps m;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B, sw32 = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  if (!make_map(&m.v128, bp.v, D, bp.sk, bp.bh, kTR, sw) ||
      !make_map(&m.qk, bp.q, D, bp.sq, bp.bh, kTB, sw) ||
      !make_map(&m.qm, bp.q, D, bp.sq, bp.bh, kTB, sw32) ||
      !make_map(&m.ok, bp.dout, D, bp.sq, bp.bh, kTB, sw) ||
      !make_map(&m.om, bp.dout, D, bp.sq, bp.bh, kTB, sw32) ||
      !make_map(&m.o128, bp.dout, D, bp.sq, bp.bh, kTR, sw) ||
      !make_map(&m.kk, bp.k, D, bp.sk, bp.bh, kTB, sw) ||
      !make_map(&m.km, bp.k, D, bp.sk, bp.bh, kTB, sw32) ||
      !make_map(&m.vk, bp.v, D, bp.sk, bp.bh, kTB, sw))
    return cudaErrorNotSupported;
  const int sq_pad = (bp.sq + kTR - 1) / kTR * kTR;
  float* lse2 = ws;
  float* dvec = ws + (size_t)bp.bh * sq_pad;
  const size_t rows = (size_t)bp.bh * sq_pad;
  bwd_rowvec<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(bp.o, bp.dout, bp.lse, lse2, dvec, bp.bh,
                                                        bp.sq, sq_pad, D);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  BwdTcParams p{};
  p.q = bp.q; p.k = bp.k; p.lse2 = lse2; p.dvec = dvec;
  p.dq = bp.dq; p.dk = bp.dk; p.dv = bp.dv;
  p.bh = bp.bh; p.sq = bp.sq; p.sk = bp.sk; p.sq_pad = sq_pad;
  p.q_offset = bp.q_offset; p.k_offset = bp.k_offset; p.causal = bp.causal;
  p.scale = bp.scale;
  p.scale_log2 = bp.scale * kLog2e;
  p.n_kv_cta = bp.bh * ((bp.sk + kTR - 1) / kTR);
  p.n_q_cta = bp.bh * (sq_pad / kTR);
  p.err = bp.err;
  p.wait_ns = bp.wait_ns;
  e = launch_pdl(tc_bwd_tf32<D>, dim3(p.n_kv_cta + p.n_q_cta), dim3(kTThreads),
                 (size_t)C::kSmemBytes, s, m, p);
  count_launch();
  return e;
}

}  // namespace

bool tc_bwd_supported(int d) { return d == 32 || d == 64 || d == 96 || d == 128; }

size_t tc_bwd_workspace_floats(const BwdParams& p) {
  const size_t sq_pad = ((size_t)p.sq + kTR - 1) / kTR * kTR;
  return (size_t)p.bh * 2 * sq_pad;
}

cudaError_t launch_tc_bwd(const BwdParams& p, float* ws, cudaStream_t s) {
  switch (p.d) {
    case 32: return launch_tc_bwd_d<32>(p, ws, s);
    case 64: return launch_tc_bwd_d<64>(p, ws, s);
    case 96: return launch_tc_bwd_d<96>(p, ws, s);
    case 128: return launch_tc_bwd_d<128>(p, ws, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fa
