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
// operand streams through its own ring (one or two buffers, doubled in the
// order the operands are needed while shared memory allows); a buffer is
// freed by the commit of the MMA that reads it last, so the next block's copy
// of an early operand (the scores' K-major tiles) overlaps the current
// block's gradient MMAs.
//
// One launch runs two kinds of CTA (1 per SM: each allocates all 512 TMEM
// columns), interleaved, heaviest causal blocks first, slices in groups whose
// tiles fit in L2 together.  A small prepass writes LSE2 and D per query row
// (padded to a multiple of 128 rows: LSE2 = +inf, D = 0 there, so padded rows
// get P = 0).
//
// dK/dV CTA: 128 keys of one slice (MMA M = 128, thread = key row), query
//   blocks of QB rows: 128 at d <= 64, 64 above.
//   TMEM: K [0, D) (A operand of S^T, staged from registers), dV [D, 2D),
//   dK [2D, 3D), then NSB buffers of S^T (QB cols) and dP^T (QB cols); NSB = 2
//   when they fit twice, else 1 (every supported d today).
//   shared memory: V [128 keys] (K-major A of dP^T); rings for the query
//   block's Q (K-major), dO (K-major), dO (MN-major), Q (MN-major), and two
//   buffers for that block's LSE2 and D.
//   Per query block: S^T = K Qs^T (A from TMEM, Q scaled in the
//   softmax step), dP^T = V dO^T; the softmax warps overwrite S^T with P^T and
//   dP^T with dS^T in place; then dV += P^T dO and dK += dS^T Q (A from TMEM,
//   B MN-major).  With NSB = 1 the issue order dV_{i-1}, S^T_i, dK_{i-1},
//   dP^T_i keeps the tensor pipe busy while the softmax warps work.
//
// dQ CTA: 128 query rows of one slice (thread = query row).
//   TMEM: Qs [0, D) (scaled by c and rounded to TF32 while staged), dQ
//   [D, 2D), two buffers of S (64) and dP (64).
//   shared memory: dO [128 rows] (K-major A of dP); rings for the 64-key
//   block's K (K-major), V (K-major), K (MN-major).  Per key block: S = Qs K^T,
//   dP = dO V^T, dS written over S, then dQ += dS K.
//
// Warps: 0 and 10 TMA producers (one lane each: the operands of the scores,
// then those of the gradient MMAs), 1 MMA issuer (one elected lane), 2..9
// "softmax" warps: warp w reads TMEM lanes 32*(w%4).., and warps w and w+4
// split each row's 64 columns.  All waits are bounded (kWaitLimitNs, or the
// limit a test sets); on expiry the CTA raises its abort flag and the device
// error word, every role leaves, in-flight copies and MMAs are drained and
// TMEM is freed.
#include "fa_tc_ptx.cuh"

#include <algorithm>

namespace fa {
namespace {

constexpr int kTR = 128;      // rows of a CTA's own block (keys or query rows): MMA M
constexpr int kTB = 64;       // rows per streamed block (queries or keys): MMA N
constexpr int kTThreads = 352;
constexpr int kTWarp0 = 2;     // softmax warps 2..9
constexpr int kTWarpLate = 10;  // producer of the gradient MMAs' operands
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
  int nkb, nqb;       // key blocks (dK/dV CTAs) and query blocks (dQ CTAs) per slice
  int group;          // slices per scheduling group
  int* err;
  unsigned long long wait_ns;
  int test_skip;  // test hook: see the P arrive of the dK/dV CTA
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

// Depth of each operand ring: every ring starts single, then rings are
// doubled in the order given (earliest-needed operands first) while the
// shared memory allows.
constexpr int kSmemLimit = 232448 - 2048;  // room for barriers and alignment
constexpr int ring_depth(int fixed, int tile, int n_rings, int which) {
  int used = fixed + n_rings * tile;
  for (int r = 0; r < n_rings; r++) {
    if (used + tile > kSmemLimit) return 1;
    used += tile;
    if (r == which) return 2;
  }
  return 1;
}

template <int D>
struct BwdTcCfg {
  // Query rows per block of the dK/dV CTA (the N of its score MMAs): 128 while
  // TMEM holds K, dV, dK and one 128-column S^T / dP^T pair (d <= 64), so each
  // block carries twice the MMA work per fixed cost (barrier checks, commits);
  // else 64.
  static constexpr int kQB = (3 * D + 4 * kTB <= 512) ? 2 * kTB : kTB;
  static constexpr int kNsbKV = (3 * D + 4 * kQB <= 512) ? 2 : 1;
  static constexpr int kTileB = kTB * D * 4;   // one 64-row tile (dQ CTA)
  static constexpr int kTileQB = kQB * D * 4;  // one query-block tile (dK/dV CTA)
  static constexpr int kTileA = kTR * D * 4;   // one 128-row tile
  static constexpr int kVecBytes = 2 * kQB * 4;  // LSE2 and D of a query block
  // dK/dV CTA: V | rings Q K-major, dO K-major, dO MN-major, Q MN-major | two
  // buffers of LSE2 and D
  static constexpr int kKvFixed = kTileA + 2 * kVecBytes;
  static constexpr int kKvD0 = ring_depth(kKvFixed, kTileQB, 4, 0);
  static constexpr int kKvD1 = ring_depth(kKvFixed, kTileQB, 4, 1);
  static constexpr int kKvD2 = ring_depth(kKvFixed, kTileQB, 4, 2);
  static constexpr int kKvD3 = ring_depth(kKvFixed, kTileQB, 4, 3);
  static constexpr int kKvR0 = kTileA;
  static constexpr int kKvR1 = kKvR0 + kKvD0 * kTileQB;
  static constexpr int kKvR2 = kKvR1 + kKvD1 * kTileQB;
  static constexpr int kKvR3 = kKvR2 + kKvD2 * kTileQB;
  static constexpr int kKvVec = kKvR3 + kKvD3 * kTileQB;
  static constexpr int kEndKV = kKvVec + 2 * kVecBytes;
  // dQ CTA: dO | rings K K-major, V K-major, K MN-major
  static constexpr int kQD0 = ring_depth(kTileA, kTileB, 3, 0);
  static constexpr int kQD1 = ring_depth(kTileA, kTileB, 3, 1);
  static constexpr int kQD2 = ring_depth(kTileA, kTileB, 3, 2);
  static constexpr int kQR0 = kTileA;
  static constexpr int kQR1 = kQR0 + kQD0 * kTileB;
  static constexpr int kQR2 = kQR1 + kQD1 * kTileB;
  static constexpr int kEndQ = kQR2 + kQD2 * kTileB;
  static constexpr int kOffBar = (kEndKV > kEndQ ? kEndKV : kEndQ);
  static constexpr int kNumBars = 32;
  // At least 116 KB, so that two CTAs never share an SM: each allocates all
  // 512 TMEM columns, and a second one would wait for the first to finish.
  static constexpr int kSmemUsed = kOffBar + kNumBars * 8 + 16 + 1024;
  static constexpr int kSmemBytes = kSmemUsed > 118784 ? kSmemUsed : 118784;
  static_assert(D % 32 == 0 && D <= 128, "D in {32, 64, 96, 128}");
  static_assert(2 * D + 4 * kTB <= 512, "dQ TMEM budget");
  static_assert(3 * D + 2 * kQB * kNsbKV <= 512, "dK/dV TMEM budget");
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
// Descriptors of a [D/32][R][32] tile, built once per tile; `kk` (a
// compile-time loop index) selects the kk-th group of 8 elements along the
// inner product, added to the start-address field (16-byte units).  K-major
// (128-byte swizzle): the group sits in chunk kk/4 at byte 32*(kk%4) of each
// row.  MN-major (32-byte-atom swizzle): 8 rows = 1024 bytes per group, chunks
// R*128 bytes apart.
__device__ __forceinline__ uint64_t desc_k_base(uint32_t tile) {
  return smem_desc(tile, 16, 1024, kLayoutSw128);
}
template <int R>
__device__ __forceinline__ uint64_t desc_mn_base(uint32_t tile) {
  return smem_desc(tile, R * 128, 512, kLayoutSw128Base32);
}
template <int R>
constexpr uint64_t k_step(int kk) {
  return (uint64_t)(((kk >> 2) * R * 128 + (kk & 3) * 32) >> 4);
}
constexpr uint64_t mn_step(int kk) { return (uint64_t)(kk * 64); }

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
// Barrier indices.
constexpr int kBarStatic = 0;  // V (dK/dV) or dO (dQ) arrived
constexpr int kBarStaged = 1;  // K (dK/dV) or Qs (dQ) staged in TMEM by the 256 softmax threads
constexpr int kBarFull = 2;    // + 2 * ring + buffer: operand loaded
constexpr int kBarEmpty = 10;  // + 2 * ring + buffer: buffer free again
constexpr int kBarS = 18;      // +buf: S (or S^T) complete
constexpr int kBarDP = 20;     // +buf: dP (or dP^T) complete
constexpr int kBarP = 22;      // +buf: P^T written (256 arrivals)
constexpr int kBarDS = 24;     // +buf: dS written (256 arrivals)
constexpr int kBarAcc = 26;    // the accumulators are final
constexpr int kBarDrain = 27;  // every MMA issued has completed
constexpr int kBarVecFull = 28;   // +buf: LSE2 and D of a query block loaded (dK/dV CTA)
constexpr int kBarVecEmpty = 30;  // +buf: the softmax warps are done with them (256 arrivals)

// One operand stream: block i sits in buffer i % depth of the ring.  The
// producer reuses a buffer once the MMA that read it last has completed (its
// commit arrives on the buffer's empty barrier).
struct Ring {
  uint32_t base;
  int bytes, depth, idx;
  __device__ uint32_t buf(int i) const { return base + (uint32_t)((i % depth) * bytes); }
  __device__ int full(int i) const { return kBarFull + 2 * idx + i % depth; }
  __device__ int empty(int i) const { return kBarEmpty + 2 * idx + i % depth; }
  __device__ uint32_t phase(int i) const { return (uint32_t)(i / depth) & 1u; }
};
struct Ctl {
  Bars bar;
  volatile int* abort_flag;
  int* err;
  unsigned long long wait_ns;
  __device__ bool wait(int b, uint32_t parity) const {
    return mbar_wait(bar(b), parity, abort_flag, err, wait_ns);
  }
  // producer: buffer of block i is free
  __device__ bool acquire(const Ring& r, int i) const {
    return i < r.depth || wait(r.empty(i), ((uint32_t)(i / r.depth) - 1u) & 1u);
  }
  // warp-wide (MMA warp): block i of the ring has landed
  __device__ bool landed(const Ring& r, int i) const {
    const bool w = wait(r.full(i), r.phase(i));
    tc_fence_after();
    return __all_sync(0xffffffffu, w);
  }
  // Bounded wait, ignoring the abort flag, for the last `n` loads' landing, so
  // that no copy writes shared memory after the CTA exits.
  __device__ void drain(const Ring& r, int n) const {
    volatile int no_abort = 0;
    for (int i = n > r.depth ? n - r.depth : 0; i < n; i++)
      mbar_wait(bar(r.full(i)), r.phase(i), &no_abort, err);
  }
};

// ---------------------------------------------------------------- dK / dV CTA
template <int D>
__device__ void cta_dkdv(const BwdMaps& m, const BwdTcParams& p, int bh, int kb, uint32_t sbase,
                         const Ctl& ctl, uint32_t tmem) {
  using C = BwdTcCfg<D>;
  constexpr int NSB = C::kNsbKV;
  constexpr int QB = C::kQB;          // query rows per block
  constexpr int HALF = QB / 2;        // columns of a block per softmax thread
  const Bars bar = ctl.bar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = kb * kTR;
  int q_first = 0;
  if (p.causal) {
    const long long f = (long long)k0 + p.k_offset - p.q_offset;  // first row that sees key k0
    q_first = f <= 0 ? 0 : (f >= p.sq ? p.sq : (int)f);
  }
  const int qb0 = q_first / QB;
  const int nqb = (p.sq + QB - 1) / QB - qb0;
  const uint32_t sV = sbase;
  // rings: 0 Q K-major, 1 dO K-major, 2 dO MN-major, 3 Q MN-major (+ LSE2, D)
  const Ring rQK{sbase + C::kKvR0, C::kTileQB, C::kKvD0, 0};
  const Ring rOK{sbase + C::kKvR1, C::kTileQB, C::kKvD1, 1};
  const Ring rOM{sbase + C::kKvR2, C::kTileQB, C::kKvD2, 2};
  const Ring rQM{sbase + C::kKvR3, C::kTileQB, C::kKvD3, 3};
  // LSE2 and D of block i.  P needs LSE2 as soon as S^T is done.  With a
  // double-buffered Q MN-major ring they ride with that tile (it lands early
  // enough); with a single buffer (d = 96, 128) that tile waits for dK of the
  // previous block, so they get their own two-deep ring, loaded after the
  // scores' operands and released by the softmax warps after dS.
  constexpr bool kVecRing = C::kKvD3 < 2;
  auto vec = [&](int i) { return sbase + C::kKvVec + (i & 1) * C::kVecBytes; };
  const uint32_t t_k = tmem, t_dv = tmem + D, t_dk = tmem + 2 * D;
  auto t_s = [&](int b) { return tmem + 3 * D + b * 2 * QB; };
  auto t_dp = [&](int b) { return tmem + 3 * D + b * 2 * QB + QB; };
  const bool skip = *ctl.abort_flag != 0;

  if (warp == 0 || warp == kTWarpLate) {
    // producers: warp 0 V and the operands the scores read (needed first),
    // the late warp those of the gradient MMAs
    if (lane == 0 && !skip) {
      const bool early = warp == 0;
      if (early) {
        mbar_expect_tx(bar(kBarStatic), C::kTileA);
        tma_tile<D, kTR>(sV, &m.v128, bar(kBarStatic), k0, bh);
      }
      // one producer's two rings, block by block (inlined per producer so the
      // ring depths stay compile-time constants)
      auto stream = [&](const Ring& ra, const CUtensorMap* ma, const Ring& rb,
                        const CUtensorMap* mb, bool first) {
        int na = 0, nb = 0, nv = 0;
        for (int i = 0; i < nqb; i++) {
          const int q0 = (qb0 + i) * QB;
          if (!ctl.acquire(ra, i)) break;
          mbar_expect_tx(bar(ra.full(i)), C::kTileQB);
          tma_tile<D, QB>(ra.buf(i), ma, bar(ra.full(i)), q0, bh);
          na++;
          if (!ctl.acquire(rb, i)) break;
          const bool vec_here = first == kVecRing;  // this producer loads LSE2 and D
          mbar_expect_tx(bar(rb.full(i)), C::kTileQB + (vec_here && !kVecRing ? C::kVecBytes : 0));
          tma_tile<D, QB>(rb.buf(i), mb, bar(rb.full(i)), q0, bh);
          if (vec_here && !kVecRing) {
            const size_t r0 = (size_t)bh * p.sq_pad + q0;
            bulk_load(vec(i), p.lse2 + r0, QB * 4, bar(rb.full(i)));
            bulk_load(vec(i) + QB * 4, p.dvec + r0, QB * 4, bar(rb.full(i)));
          }
          nb++;
          if (vec_here && kVecRing) {
            if (i >= 2 && !ctl.wait(kBarVecEmpty + (i & 1), (uint32_t)((i >> 1) - 1) & 1u)) break;
            const size_t r0 = (size_t)bh * p.sq_pad + q0;
            mbar_expect_tx(bar(kBarVecFull + (i & 1)), C::kVecBytes);
            bulk_load(vec(i), p.lse2 + r0, QB * 4, bar(kBarVecFull + (i & 1)));
            bulk_load(vec(i) + QB * 4, p.dvec + r0, QB * 4, bar(kBarVecFull + (i & 1)));
            nv++;
          }
        }
        ctl.drain(ra, na);
        ctl.drain(rb, nb);
        volatile int no_abort = 0;
        for (int i = nv > 2 ? nv - 2 : 0; i < nv; i++)
          mbar_wait(bar(kBarVecFull + (i & 1)), (uint32_t)(i >> 1) & 1u, &no_abort, p.err);
      };
      if (early) {
        stream(rQK, &m.qk, rOK, &m.ok, true);
        volatile int no_abort = 0;
        mbar_wait(bar(kBarStatic), 0, &no_abort, p.err);
      } else {
        stream(rOM, &m.om, rQM, &m.qm, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (!skip) {
      constexpr uint32_t idesc_s = instr_desc(kTR, QB, false);
      constexpr uint32_t idesc_g = instr_desc(kTR, D, true);
      bool ok = __all_sync(0xffffffffu, ctl.wait(kBarStatic, 0));
      ok = ok && __all_sync(0xffffffffu, ctl.wait(kBarStaged, 0));
      tc_fence_after();
      auto issue_s = [&](int i) {  // S^T = K Q^T
        if (!ctl.landed(rQK, i)) return false;
        const int b = i % NSB;
        const uint64_t bd = desc_k_base(rQK.buf(i));
        const uint32_t ts = t_s(b);
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++)
          mma_ts_elect(ts, t_k + kk * 8, bd + k_step<QB>(kk), idesc_s, kk > 0);
        tc_commit_elect(bar(kBarS + b));
        tc_commit_elect(bar(rQK.empty(i)));
        return true;
      };
      auto issue_dp = [&](int i) {  // dP^T = V dO^T
        if (!ctl.landed(rOK, i)) return false;
        const int b = i % NSB;
        const uint64_t ad = desc_k_base(sV), bd = desc_k_base(rOK.buf(i));
        const uint32_t td = t_dp(b);
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++)
          mma_ss_elect(td, ad + k_step<kTR>(kk), bd + k_step<QB>(kk), idesc_s, kk > 0);
        tc_commit_elect(bar(kBarDP + b));
        tc_commit_elect(bar(rOK.empty(i)));
        return true;
      };
      auto issue_dv = [&](int i) {  // dV += P^T dO
        const int b = i % NSB;
        if (!ctl.landed(rOM, i)) return false;
        if (!__all_sync(0xffffffffu, ctl.wait(kBarP + b, (i / NSB) & 1))) return false;
        tc_fence_after();
        const uint64_t bd = desc_mn_base<QB>(rOM.buf(i));
        const uint32_t ta = t_s(b);
        const uint32_t acc0 = i > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < QB / 8; kk++)
          mma_ts_elect(t_dv, ta + kk * 8, bd + mn_step(kk), idesc_g, kk > 0 ? 1u : acc0);
        tc_commit_elect(bar(rOM.empty(i)));
        return true;
      };
      auto issue_dk = [&](int i) {  // dK += dS^T Q
        const int b = i % NSB;
        if (!ctl.landed(rQM, i)) return false;
        if (!__all_sync(0xffffffffu, ctl.wait(kBarDS + b, (i / NSB) & 1))) return false;
        tc_fence_after();
        const uint64_t bd = desc_mn_base<QB>(rQM.buf(i));
        const uint32_t ta = t_dp(b);
        const uint32_t acc0 = i > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < QB / 8; kk++)
          mma_ts_elect(t_dk, ta + kk * 8, bd + mn_step(kk), idesc_g, kk > 0 ? 1u : acc0);
        tc_commit_elect(bar(rQM.empty(i)));
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
    const float c = p.scale_log2;
    for (int i = 0; i < nqb && ok; i++) {
      const int b = i % NSB;
      const bool vec_in = kVecRing ? ctl.wait(kBarVecFull + (i & 1), (uint32_t)(i >> 1) & 1u)
                                   : ctl.wait(rQM.full(i), rQM.phase(i));
      ok = __all_sync(0xffffffffu, vec_in && ctl.wait(kBarS + b, (i / NSB) & 1));
      if (!ok) break;
      tc_fence_after();
      const float* svec = reinterpret_cast<const float*>(__cvta_shared_to_generic(vec(i)));
      float pr[HALF];
#pragma unroll
      for (int cc = 0; cc < HALF / 32; cc++) {  // 32 columns at a time
        const int col = HALF * h + 32 * cc;
        // P of column e is nonzero only for e >= lo (causal)
        const long long lo = p.causal ? kg - (p.q_offset + (long long)(qb0 + i) * QB + col) : -1;
        uint32_t x[32];
        tmem_ld32(t_s(b) + lane_off + col, x);
        tmem_wait_ld_regs(x);
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(svec + col + e);
          pr[32 * cc + e] = ex2(fmaf(__uint_as_float(x[e]), c, -l4.x));
          pr[32 * cc + e + 1] = ex2(fmaf(__uint_as_float(x[e + 1]), c, -l4.y));
          pr[32 * cc + e + 2] = ex2(fmaf(__uint_as_float(x[e + 2]), c, -l4.z));
          pr[32 * cc + e + 3] = ex2(fmaf(__uint_as_float(x[e + 3]), c, -l4.w));
        }
        if (__any_sync(0xffffffffu, lo > 0)) {
#pragma unroll
          for (int e = 0; e < 32; e++) pr[32 * cc + e] = (e >= lo) ? pr[32 * cc + e] : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 32; e++) x[e] = __float_as_uint(pr[32 * cc + e]);
        tmem_st32(t_s(b) + lane_off + col, x);
      }
      tmem_wait_st();
      tc_fence_before();
      // (test hook: one thread of the first CTA withholds its arrive)
      if (!(p.test_skip == i && threadIdx.x == 64 && blockIdx.x == 0)) mbar_arrive(bar(kBarP + b));
      ok = __all_sync(0xffffffffu, ctl.wait(kBarDP + b, (i / NSB) & 1));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < HALF / 32; cc++) {
        const int col = HALF * h + 32 * cc;
        uint32_t x[32];
        tmem_ld32(t_dp(b) + lane_off + col, x);
        tmem_wait_ld_regs(x);
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 d4 = *reinterpret_cast<const float4*>(svec + QB + col + e);
          x[e] = __float_as_uint(pr[32 * cc + e] * (__uint_as_float(x[e]) - d4.x));
          x[e + 1] = __float_as_uint(pr[32 * cc + e + 1] * (__uint_as_float(x[e + 1]) - d4.y));
          x[e + 2] = __float_as_uint(pr[32 * cc + e + 2] * (__uint_as_float(x[e + 2]) - d4.z));
          x[e + 3] = __float_as_uint(pr[32 * cc + e + 3] * (__uint_as_float(x[e + 3]) - d4.w));
        }
        tmem_st32(t_dp(b) + lane_off + col, x);
      }
      if (kVecRing) mbar_arrive(bar(kBarVecEmpty + (i & 1)));  // LSE2 and D are read
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarDS + b));
    }
    if (nqb > 0) {
      const bool w = ok ? ctl.wait(kBarAcc, 0) : false;
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
                       const Ctl& ctl, uint32_t tmem) {
  using C = BwdTcCfg<D>;
  const Bars bar = ctl.bar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * kTR;
  const int q_rows = min(kTR, p.sq - q0);
  int kend = p.sk;
  if (p.causal) kend = causal_limit(p.q_offset + q0 + q_rows - 1, p.k_offset, p.sk);
  const int nkb = (kend + kTB - 1) / kTB;
  const uint32_t sDO = sbase;
  // rings: 0 K K-major, 1 V K-major, 2 K MN-major
  const Ring rKK{sbase + C::kQR0, C::kTileB, C::kQD0, 0};
  const Ring rVK{sbase + C::kQR1, C::kTileB, C::kQD1, 1};
  const Ring rKM{sbase + C::kQR2, C::kTileB, C::kQD2, 2};
  const uint32_t t_q = tmem, t_dq = tmem + D;
  auto t_s = [&](int b) { return tmem + 2 * D + b * 2 * kTB; };
  auto t_dp = [&](int b) { return tmem + 2 * D + b * 2 * kTB + kTB; };
  const bool skip = *ctl.abort_flag != 0;

  if (warp == 0 || warp == kTWarpLate) {
    if (lane == 0 && !skip) {
      const bool early = warp == 0;
      int na = 0, nb = 0;
      if (early) {
        mbar_expect_tx(bar(kBarStatic), C::kTileA);
        tma_tile<D, kTR>(sDO, &m.o128, bar(kBarStatic), q0, bh);
        for (int t = 0; t < nkb; t++) {
          if (!ctl.acquire(rKK, t)) break;
          mbar_expect_tx(bar(rKK.full(t)), C::kTileB);
          tma_tile<D, kTB>(rKK.buf(t), &m.kk, bar(rKK.full(t)), t * kTB, bh);
          na++;
          if (!ctl.acquire(rVK, t)) break;
          mbar_expect_tx(bar(rVK.full(t)), C::kTileB);
          tma_tile<D, kTB>(rVK.buf(t), &m.vk, bar(rVK.full(t)), t * kTB, bh);
          nb++;
        }
        volatile int no_abort = 0;
        mbar_wait(bar(kBarStatic), 0, &no_abort, p.err);
        ctl.drain(rKK, na);
        ctl.drain(rVK, nb);
      } else {
        for (int t = 0; t < nkb; t++) {
          if (!ctl.acquire(rKM, t)) break;
          mbar_expect_tx(bar(rKM.full(t)), C::kTileB);
          tma_tile<D, kTB>(rKM.buf(t), &m.km, bar(rKM.full(t)), t * kTB, bh);
          na++;
        }
        ctl.drain(rKM, na);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (!skip) {
      constexpr uint32_t idesc_s = instr_desc(kTR, kTB, false);
      constexpr uint32_t idesc_g = instr_desc(kTR, D, true);
      bool ok = __all_sync(0xffffffffu, ctl.wait(kBarStatic, 0));
      ok = ok && __all_sync(0xffffffffu, ctl.wait(kBarStaged, 0));
      tc_fence_after();
      auto issue_dq = [&](int t) {  // dQ += dS K
        const int b = t & 1;
        if (!ctl.landed(rKM, t)) return false;
        if (!__all_sync(0xffffffffu, ctl.wait(kBarDS + b, (t >> 1) & 1))) return false;
        tc_fence_after();
        const uint64_t bd = desc_mn_base<kTB>(rKM.buf(t));
        const uint32_t ta = t_s(b);
        const uint32_t acc0 = t > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kTB / 8; kk++)
          mma_ts_elect(t_dq, ta + kk * 8, bd + mn_step(kk), idesc_g, kk > 0 ? 1u : acc0);
        tc_commit_elect(bar(rKM.empty(t)));
        return true;
      };
      for (int t = 0; t < nkb && ok; t++) {
        const int b = t & 1;
        if (!(ok = ctl.landed(rKK, t))) break;
        {
          const uint64_t bd = desc_k_base(rKK.buf(t));
          const uint32_t ts = t_s(b);
#pragma unroll
          for (int kk = 0; kk < D / 8; kk++)  // S = Qs K^T
            mma_ts_elect(ts, t_q + kk * 8, bd + k_step<kTB>(kk), idesc_s, kk > 0);
        }
        tc_commit_elect(bar(kBarS + b));
        tc_commit_elect(bar(rKK.empty(t)));
        if (!(ok = ctl.landed(rVK, t))) break;
        {
          const uint64_t ad = desc_k_base(sDO), bd = desc_k_base(rVK.buf(t));
          const uint32_t td = t_dp(b);
#pragma unroll
          for (int kk = 0; kk < D / 8; kk++)  // dP = dO V^T
            mma_ss_elect(td, ad + k_step<kTR>(kk), bd + k_step<kTB>(kk), idesc_s, kk > 0);
        }
        tc_commit_elect(bar(kBarDP + b));
        tc_commit_elect(bar(rVK.empty(t)));
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
      ok = __all_sync(0xffffffffu, ctl.wait(kBarS + b, (t >> 1) & 1));
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
      ok = __all_sync(0xffffffffu, ctl.wait(kBarDP + b, (t >> 1) & 1));
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
      const bool w = ok ? ctl.wait(kBarAcc, 0) : false;
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

  // CTA order: slices in groups of p.group (a group's Q, K, V and dO fit in
  // L2 together, so the CTAs of a slice find its tiles there); within a
  // group, the two kinds alternate while both last, heaviest causal blocks
  // first (low key blocks for dK/dV, high query blocks for dQ).
  const int per_group = p.group * (p.nkb + p.nqb);
  const int g = (int)blockIdx.x / per_group;
  const int h0 = g * p.group;
  const int gs = min(p.group, p.bh - h0);  // slices in this group
  const int i = (int)blockIdx.x - g * per_group;
  const int n_kv = gs * p.nkb, n_q = gs * p.nqb;
  const int both = 2 * min(n_kv, n_q);
  bool is_kv;
  int rank;
  if (i < both) {
    is_kv = (i & 1) == 0;
    rank = i >> 1;
  } else {
    is_kv = n_kv > n_q;
    rank = i - both / 2;
  }
  const int bh = h0 + rank % gs, blk = rank / gs;

  if (threadIdx.x == 0) {
    for (int b = 0; b < C::kNumBars; b++) {
      const bool many = b == kBarStaged || (b >= kBarP && b < kBarAcc) || b >= kBarVecEmpty;
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
  const Ctl ctl{bar, abort_flag, p.err, p.wait_ns};
  if (is_kv)
    cta_dkdv<D>(m, p, bh, blk, sbase, ctl, tmem);
  else
    cta_dq<D>(m, p, bh, p.nqb - 1 - blk, sbase, ctl, tmem);
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
      !make_map(&m.qk, bp.q, D, bp.sq, bp.bh, C::kQB, sw) ||
      !make_map(&m.qm, bp.q, D, bp.sq, bp.bh, C::kQB, sw32) ||
      !make_map(&m.ok, bp.dout, D, bp.sq, bp.bh, C::kQB, sw) ||
      !make_map(&m.om, bp.dout, D, bp.sq, bp.bh, C::kQB, sw32) ||
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
  p.nkb = (bp.sk + kTR - 1) / kTR;
  p.nqb = sq_pad / kTR;
  // Q, K, V and dO of `group` slices take at most ~48 MB (of the 126 MB L2).
  const double slice_bytes = 4.0 * D * (2.0 * bp.sq + 2.0 * bp.sk);
  p.group = (int)std::max(1.0, std::min((double)bp.bh, 48e6 / slice_bytes));
  p.err = bp.err;
  p.wait_ns = bp.wait_ns;
  p.test_skip = bp.test_skip;
  e = launch_pdl(tc_bwd_tf32<D>, dim3(bp.bh * (p.nkb + p.nqb)), dim3(kTThreads),
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
