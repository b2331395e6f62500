// CUDA-core kernels of the attention forward (exact f32 arithmetic):
//   simt_fwd     -- any d_head (<= 256), any lengths; the FA_PREC_FP32 path and
//                   the path for head sizes the tensor-core kernel does not tile.
//   decode_fwd   -- split-KV kernel for few query rows against long key
//                   ranges (decode / cross-attention shapes); HBM-bound, so it
//                   streams K/V with 16-byte loads, one warp per key.
//   lse_combine  -- merges split partials (o_p, lse_p) by log-sum-exp.
// Semantics follow the crate's v2 forward (src/v2.rs:160-385): score =
// dot(q,k) * (1/sqrt(d)), top-left causal mask, online softmax with a running
// max, out = acc * (l > 0 ? 1/l : 0).
#include "fa_common.cuh"

#include <atomic>

#include <math.h>

#include <mutex>

namespace fa {

namespace {

constexpr int kSimtBQ = 16;   // query rows per CTA (4 warps x 4 rows)
constexpr int kSimtBK = 32;   // keys per tile (one per lane in the score phase)
constexpr int kSimtRows = 4;  // rows per warp

template <int DCH>  // d <= 32 * DCH
__global__ void __launch_bounds__(128) simt_fwd(FwdParams p) {
  grid_dep_wait();  // (launched with launch_pdl)
  extern __shared__ float smem[];
  const int d = p.d;
  const int sk_stride = d | 1;  // odd row stride: lane-per-key reads are conflict-free
  float* sQ = smem;                       // [BQ][d]
  float* sK = sQ + kSimtBQ * d;           // [BK][sk_stride]
  float* sV = sK + kSimtBK * sk_stride;   // [BK][d]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.y;
  const int q0 = blockIdx.x * kSimtBQ;
  const float* Q = p.q + (size_t)bh * p.sq * d;
  const float* K = p.k + (size_t)bh * p.sk * d;
  const float* V = p.v + (size_t)bh * p.sk * d;

  const int q_rows = min(kSimtBQ, p.sq - q0);
  for (int x = tid; x < kSimtBQ * d; x += blockDim.x) {
    int r = x / d;
    sQ[x] = (r < q_rows) ? Q[(size_t)q0 * d + x] : 0.0f;
  }
  // Keys past the last one any row of this block can see are never loaded
  // (the crate's causal break, v2.rs:210-212).
  int kend = p.sk;
  if (p.causal) kend = causal_limit(p.q_offset + q0 + q_rows - 1, p.k_offset, p.sk);

  float m[kSimtRows], l[kSimtRows], acc[kSimtRows][DCH];
#pragma unroll
  for (int r = 0; r < kSimtRows; r++) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int t = 0; t < DCH; t++) acc[r][t] = 0.0f;
  }

  for (int kt = 0; kt < kend; kt += kSimtBK) {
    const int nk = min(kSimtBK, kend - kt);
    __syncthreads();
    for (int x = tid; x < kSimtBK * d; x += blockDim.x) {
      int j = x / d, c = x - j * d;
      float kv = 0.0f, vv = 0.0f;
      if (j < nk) {
        kv = K[(size_t)(kt + j) * d + c];
        vv = V[(size_t)(kt + j) * d + c];
      }
      sK[j * sk_stride + c] = kv;
      sV[x] = vv;
    }
    __syncthreads();
    float pr[kSimtRows];
#pragma unroll
    for (int r = 0; r < kSimtRows; r++) {
      const int i = warp * kSimtRows + r;
      const float* qr = sQ + i * d;
      const float* kr = sK + lane * sk_stride;
      float s = 0.0f;
      for (int c = 0; c < d; c++) s = fmaf(qr[c], kr[c], s);
      s *= p.scale;
      bool visible = lane < nk;
      if (p.causal) visible = visible && (p.k_offset + kt + lane <= p.q_offset + q0 + i);
      s = visible ? s : -INFINITY;
      float mx = warp_max(s);
      float m_new = fmaxf(m[r], mx);
      float pv, corr;
      if (m_new == -INFINITY) {  // nothing visible yet for this row
        pv = 0.0f;
        corr = 1.0f;
      } else {
        pv = expf(s - m_new);
        corr = expf(m[r] - m_new);
      }
      l[r] = l[r] * corr + warp_sum(pv);
#pragma unroll
      for (int t = 0; t < DCH; t++) acc[r][t] *= corr;
      m[r] = m_new;
      pr[r] = pv;
    }
    for (int j = 0; j < nk; j++) {
      const float* vr = sV + j * d;
      float vcol[DCH];
#pragma unroll
      for (int t = 0; t < DCH; t++) {
        int c = lane + 32 * t;
        vcol[t] = (c < d) ? vr[c] : 0.0f;
      }
#pragma unroll
      for (int r = 0; r < kSimtRows; r++) {
        float pj = __shfl_sync(0xffffffffu, pr[r], j);
#pragma unroll
        for (int t = 0; t < DCH; t++) acc[r][t] = fmaf(pj, vcol[t], acc[r][t]);
      }
    }
  }

#pragma unroll
  for (int r = 0; r < kSimtRows; r++) {
    const int i = warp * kSimtRows + r;
    if (i >= q_rows) continue;
    const size_t row = (size_t)bh * p.sq + q0 + i;
    const float inv_l = l[r] > 0.0f ? 1.0f / l[r] : 0.0f;
#pragma unroll
    for (int t = 0; t < DCH; t++) {
      int c = lane + 32 * t;
      if (c < d) p.o[row * d + c] = acc[r][t] * inv_l;
    }
    if (p.lse && lane == 0) p.lse[row] = l[r] > 0.0f ? m[r] + logf(l[r]) : -INFINITY;
  }
}

// ---------------------------------------------------------------------------
// Split-KV decode.  grid = (sq, bh, splits), 256 threads = 8 warps.  Each warp
// walks keys kb+warp, kb+warp+8, ... four at a time (16-byte K and V loads for
// four keys in flight per lane), keeping its own online-softmax state; the 8
// warp states are merged through shared memory at the end.
constexpr int kDecWarps = 8;
constexpr int kDecUnroll = 4;

template <int NV>  // float4 slots per lane: d <= 128 * NV, d % 4 == 0
__global__ void __launch_bounds__(256) decode_fwd(FwdParams p, int chunk, float* part_o,
                                                  float* part_lse) {
  grid_dep_wait();  // (launched with launch_pdl)
  __shared__ float s_m[kDecWarps], s_l[kDecWarps];
  extern __shared__ float s_acc[];  // [kDecWarps][d]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = blockIdx.x, bh = blockIdx.y, split = blockIdx.z;
  const int splits = gridDim.z;
  const int d = p.d, d4 = d >> 2;
  const float4* Q = reinterpret_cast<const float4*>(p.q + ((size_t)bh * p.sq + row) * d);
  const float4* K = reinterpret_cast<const float4*>(p.k + (size_t)bh * p.sk * d);
  const float4* V = reinterpret_cast<const float4*>(p.v + (size_t)bh * p.sk * d);

  int kb = split * chunk;
  int ke = min(p.sk, kb + chunk);
  if (p.causal) ke = min(ke, causal_limit(p.q_offset + row, p.k_offset, p.sk));

  float4 q4[NV];
#pragma unroll
  for (int t = 0; t < NV; t++) {
    int f = lane + 32 * t;
    q4[t] = (f < d4) ? Q[f] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float m = -INFINITY, l = 0.0f;
  float4 acc[NV];
#pragma unroll
  for (int t = 0; t < NV; t++) acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);

  for (int j0 = kb + warp; j0 < ke; j0 += kDecWarps * kDecUnroll) {
    float4 kv[kDecUnroll][NV], vv[kDecUnroll][NV];
#pragma unroll
    for (int u = 0; u < kDecUnroll; u++) {
      int j = j0 + u * kDecWarps;
#pragma unroll
      for (int t = 0; t < NV; t++) {
        int f = lane + 32 * t;
        bool ok = (j < ke) && (f < d4);
        kv[u][t] = ok ? __ldg(K + (size_t)j * d4 + f) : make_float4(0.f, 0.f, 0.f, 0.f);
        vv[u][t] = ok ? __ldg(V + (size_t)j * d4 + f) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float s[kDecUnroll];
#pragma unroll
    for (int u = 0; u < kDecUnroll; u++) {
      float a = 0.0f;
#pragma unroll
      for (int t = 0; t < NV; t++) {
        a = fmaf(q4[t].x, kv[u][t].x, a);
        a = fmaf(q4[t].y, kv[u][t].y, a);
        a = fmaf(q4[t].z, kv[u][t].z, a);
        a = fmaf(q4[t].w, kv[u][t].w, a);
      }
      s[u] = a;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < kDecUnroll; u++) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
    float mx = -INFINITY;
#pragma unroll
    for (int u = 0; u < kDecUnroll; u++) {
      s[u] = (j0 + u * kDecWarps < ke) ? s[u] * p.scale : -INFINITY;
      mx = fmaxf(mx, s[u]);
    }
    float m_new = fmaxf(m, mx);  // finite: key j0 < ke is always visible here
    float corr = expf(m - m_new);
    l *= corr;
#pragma unroll
    for (int t = 0; t < NV; t++) {
      acc[t].x *= corr; acc[t].y *= corr; acc[t].z *= corr; acc[t].w *= corr;
    }
#pragma unroll
    for (int u = 0; u < kDecUnroll; u++) {
      float pu = expf(s[u] - m_new);
      l += pu;
#pragma unroll
      for (int t = 0; t < NV; t++) {
        acc[t].x = fmaf(pu, vv[u][t].x, acc[t].x);
        acc[t].y = fmaf(pu, vv[u][t].y, acc[t].y);
        acc[t].z = fmaf(pu, vv[u][t].z, acc[t].z);
        acc[t].w = fmaf(pu, vv[u][t].w, acc[t].w);
      }
    }
    m = m_new;
  }

  if (lane == 0) { s_m[warp] = m; s_l[warp] = l; }
#pragma unroll
  for (int t = 0; t < NV; t++) {
    int f = lane + 32 * t;
    if (f < d4) reinterpret_cast<float4*>(s_acc + warp * d)[f] = acc[t];
  }
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kDecWarps; w++) M = fmaxf(M, s_m[w]);
  float L = 0.0f, wgt[kDecWarps];
#pragma unroll
  for (int w = 0; w < kDecWarps; w++) {
    wgt[w] = (s_m[w] == -INFINITY) ? 0.0f : expf(s_m[w] - M);
    L += s_l[w] * wgt[w];
  }
  const float inv_L = L > 0.0f ? 1.0f / L : 0.0f;
  const float lse_v = L > 0.0f ? M + logf(L) : -INFINITY;
  const size_t grow = (size_t)bh * p.sq + row;
  float* dst_o;
  float* dst_lse;
  if (splits == 1) {
    dst_o = p.o + grow * d;
    dst_lse = p.lse ? p.lse + grow : nullptr;
  } else {
    size_t rows = (size_t)p.bh * p.sq;
    dst_o = part_o + ((size_t)split * rows + grow) * d;
    dst_lse = part_lse + (size_t)split * rows + grow;
  }
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kDecWarps; w++) o = fmaf(s_acc[w * d + c], wgt[w], o);
    dst_o[c] = o * inv_L;
  }
  if (threadIdx.x == 0 && dst_lse) *dst_lse = lse_v;
}

// Log-sum-exp merge of n partials per row: one warp per row, 8 rows per CTA.
// The lanes reduce the row's max and sum over the parts, then each lane owns
// 4 (or 1) output columns and accumulates the parts with weights broadcast by
// shuffle, 32 parts at a time.  With at most 32 parts (every key-range split
// here) each lane loads its part's LSE once and keeps its weight, and the
// loads of all parts' columns are issued back to back, so a row costs two
// dependent memory round trips.
template <bool V4>
__global__ void __launch_bounds__(256) lse_combine(const float* __restrict__ o_parts,
                                                   const float* __restrict__ lse_parts,
                                                   int n, long long rows, int d,
                                                   float* __restrict__ out,
                                                   float* __restrict__ lse_out) {
  grid_dep_wait();  // (launched with launch_pdl: the partials come from the previous kernel)
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;  // (whole warps leave together)
  constexpr int W = V4 ? 4 : 1;
  const float* lrow = lse_parts + row;
  const size_t pstride = (size_t)rows;  // between parts, in the LSE planes
  const size_t ostride = (size_t)rows * d;
  const float* orow = o_parts + (size_t)row * d;
  float M, L, w_own = 0.0f;
  if (n <= 32) {
    const float lp = lane < n ? lrow[(size_t)lane * pstride] : -INFINITY;
    M = warp_max(lp);
    w_own = (M != -INFINITY && lp != -INFINITY) ? expf(lp - M) : 0.0f;
    L = warp_sum(w_own);
  } else {
    M = -INFINITY;
    for (int q = lane; q < n; q += 32) M = fmaxf(M, lrow[(size_t)q * pstride]);
    M = warp_max(M);
    L = 0.0f;
    if (M != -INFINITY)
      for (int q = lane; q < n; q += 32) {
        const float lp = lrow[(size_t)q * pstride];
        if (lp != -INFINITY) L += expf(lp - M);
      }
    L = warp_sum(L);
  }
  const float inv_L = L > 0.0f ? 1.0f / L : 0.0f;
  for (int c0 = 0; c0 < d; c0 += 32 * W) {
    const int c = c0 + lane * W;
    const bool active = c < d;
    float acc[W];
#pragma unroll
    for (int e = 0; e < W; e++) acc[e] = 0.0f;
    for (int p0 = 0; p0 < n && M != -INFINITY; p0 += 32) {
      float w = w_own;
      if (n > 32) {
        w = 0.0f;
        if (p0 + lane < n) {
          const float lp = lrow[(size_t)(p0 + lane) * pstride];
          if (lp != -INFINITY) w = expf(lp - M);
        }
      }
      const int cnt = min(32, n - p0);
#pragma unroll 4
      for (int i = 0; i < cnt; i++) {
        const float wi = __shfl_sync(0xffffffffu, w, i);
        if (!active) continue;
        const float* src = orow + (size_t)(p0 + i) * ostride + c;
        // a part with weight 0 contributes nothing, whatever its columns hold
        // (a select, not a branch, so the loads of all parts stay in flight)
        const bool use = wi != 0.0f;
        if constexpr (V4) {
          const float4 o = *reinterpret_cast<const float4*>(src);
          acc[0] = fmaf(wi, use ? o.x : 0.0f, acc[0]);
          acc[1] = fmaf(wi, use ? o.y : 0.0f, acc[1]);
          acc[2] = fmaf(wi, use ? o.z : 0.0f, acc[2]);
          acc[3] = fmaf(wi, use ? o.w : 0.0f, acc[3]);
        } else {
          acc[0] = fmaf(wi, use ? *src : 0.0f, acc[0]);
        }
      }
    }
    if (active) {
      float* dst = out + (size_t)row * d + c;
      if constexpr (V4)
        *reinterpret_cast<float4*>(dst) =
            make_float4(acc[0] * inv_L, acc[1] * inv_L, acc[2] * inv_L, acc[3] * inv_L);
      else
        *dst = acc[0] * inv_L;
    }
  }
  if (lane == 0 && lse_out) lse_out[row] = (L > 0.0f) ? M + logf(L) : -INFINITY;
}

template <int DCH>
cudaError_t launch_simt_t(const FwdParams& p, cudaStream_t s) {
  const int sk_stride = p.d | 1;
  size_t smem = sizeof(float) * ((size_t)kSimtBQ * p.d + (size_t)kSimtBK * sk_stride +
                                 (size_t)kSimtBK * p.d);
  // The attribute is set once per device, to the largest size this
  // instantiation can need (d up to DCH*32), so that concurrent calls with
  // other d never see it lowered under them.
  static std::atomic<unsigned long long> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    const int dmax = DCH * 32;
    const size_t smax = sizeof(float) * ((size_t)kSimtBQ * dmax + (size_t)kSimtBK * (dmax | 1) +
                                         (size_t)kSimtBK * dmax);
    cudaError_t e = cudaFuncSetAttribute(simt_fwd<DCH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smax);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  dim3 grid((p.sq + kSimtBQ - 1) / kSimtBQ, p.bh);
  cudaError_t le = launch_pdl(simt_fwd<DCH>, grid, dim3(128), smem, s, p);
  count_launch();
  return le != cudaSuccess ? le : cudaGetLastError();
}

}  // namespace

cudaError_t launch_simt(const FwdParams& p, cudaStream_t s) {
  const int dch = (p.d + 31) / 32;
  switch (dch) {
    case 1: return launch_simt_t<1>(p, s);
    case 2: return launch_simt_t<2>(p, s);
    case 3: return launch_simt_t<3>(p, s);
    case 4: return launch_simt_t<4>(p, s);
    case 5: return launch_simt_t<5>(p, s);
    case 6: return launch_simt_t<6>(p, s);
    case 7: return launch_simt_t<7>(p, s);
    case 8: return launch_simt_t<8>(p, s);
    default: return cudaErrorInvalidValue;
  }
}

bool decode_supported(int d) { return d > 0 && d % 4 == 0 && d <= 256; }

// 256-thread decode CTAs resident per SM on the current device (cached per
// device and instantiation).
static int decode_resident_per_sm(int d) {
  static std::atomic<int> cache[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 8;
  const int nv = d <= 128 ? 0 : 1;
  int r = cache[dev][nv].load();
  if (r > 0) return r;
  const size_t smem = sizeof(float) * kDecWarps * (nv ? 256 : 128);
  cudaError_t e = nv ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, decode_fwd<2>, 256, smem)
                     : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, decode_fwd<1>, 256, smem);
  if (e != cudaSuccess || r < 1) {
    cudaGetLastError();
    return 8;
  }
  cache[dev][nv].store(r);
  return r;
}

int decode_pick_splits(int bh, int sq, int sk, int num_sms, int d) {
  const long long ctas = (long long)bh * sq;
  // As many splits as keep every CTA in the first (only) wave: a second wave
  // of a few CTAs would run alone for a whole CTA's time.
  const long long slots = (long long)decode_resident_per_sm(d) * num_sms;
  long long splits = ctas >= slots ? 1 : slots / ctas;
  long long max_splits = (sk + 127) / 128;  // at least 128 keys per split
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  if (splits > 1024) splits = 1024;
  return (int)splits;
}

cudaError_t launch_decode(const FwdParams& p, int splits, float* scratch, cudaStream_t s) {
  int chunk = (p.sk + splits - 1) / splits;
  chunk = (chunk + 31) / 32 * 32;
  splits = (p.sk + chunk - 1) / chunk;
  if (splits < 1) splits = 1;
  const size_t rows = (size_t)p.bh * p.sq;
  float* part_o = scratch;
  float* part_lse = scratch ? scratch + (size_t)splits * rows * p.d : nullptr;
  dim3 grid(p.sq, p.bh, splits);
  size_t smem = sizeof(float) * kDecWarps * p.d;
  cudaError_t e = p.d <= 128
                      ? launch_pdl(decode_fwd<1>, grid, dim3(256), smem, s, p, chunk, part_o, part_lse)
                      : launch_pdl(decode_fwd<2>, grid, dim3(256), smem, s, p, chunk, part_o, part_lse);
  count_launch();
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  return launch_combine(part_o, part_lse, splits, (long long)rows, p.d, p.o, p.lse, s);
}

cudaError_t launch_combine(const float* o_parts, const float* lse_parts, int n_parts,
                           long long rows, int d, float* out, float* lse_out,
                           cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  const bool v4 = (d % 4) == 0 && (((uintptr_t)o_parts | (uintptr_t)out) & 15) == 0;
  cudaError_t e =
      v4 ? launch_pdl(lse_combine<true>, dim3(grid), dim3(256), 0, s, o_parts, lse_parts, n_parts,
                      rows, d, out, lse_out)
         : launch_pdl(lse_combine<false>, dim3(grid), dim3(256), 0, s, o_parts, lse_parts, n_parts,
                      rows, d, out, lse_out);
  count_launch();
  return e != cudaSuccess ? e : cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Fixed scratch for the allocation-free decode entry point.  Some callers of
// this library cannot allocate device memory at call time (for example code
// running under an allocator that forbids new device allocations, or an
// embedding runtime that owns all device memory and hands out only its own
// buffers).  For them the split partials of the decode kernel live in this
// file-scope array instead of a per-call allocation.  Every GPU that loads
// the library holds it (4 MiB) until the process exits.  All calls on a
// device share it, so calls whose kernels overlap on that GPU race; each call
// overwrites every partial it later reads, so nothing needs clearing.
constexpr size_t kStaticScratchFloats = size_t(1) << 20;
static __device__ __align__(256) float g_decode_scratch[kStaticScratchFloats];

size_t static_scratch_floats() { return kStaticScratchFloats; }

// Device address of the array on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device with that device current, and cached.
cudaError_t static_scratch_ptr(float** out) {
  constexpr int kMaxDev = 64;
  static std::mutex mu;
  static float* cache[kMaxDev] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    float* ptr = nullptr;
    e = cudaGetSymbolAddress((void**)&ptr, g_decode_scratch);
    if (e != cudaSuccess) return e;
    cache[dev] = ptr;
  }
  *out = cache[dev];
  return cudaSuccess;
}

}  // namespace fa
