// Backward pass of the forward in this library (the crate has none): given Q,
// K, V, the output O, its row LSE and dO, computes dQ, dK, dV in f32 on the
// CUDA cores, FlashAttention-2 style (the score matrix is recomputed block by
// block and never stored).  With P = exp(scale*Q K^T - lse) (masked entries 0):
//   Di = rowsum(dO_i * O_i)
//   dV = P^T dO,  dP = dO V^T,  dS = P * (dP - D),  dQ = scale dS K,  dK = scale dS^T Q
// Two kernels after the Di pass: one CTA per block of 64 keys accumulates dK and
// dV over the query rows that see those keys; one CTA per block of 64 query
// rows accumulates dQ over the keys its rows see.  Both tile their products
// over the threads (register micro-tiles) with operands in shared memory.
// Causal masking is top-left (row i sees keys j <= i), as in the forward.
#include "fa_common.cuh"

#include <atomic>

namespace fa {
namespace {

constexpr int kBwdThreads = 256;
constexpr int kBK = 64;  // keys per dK/dV CTA; keys per step of the dQ CTA
constexpr int kBQ = 32;  // query rows per step of the dK/dV CTA
constexpr int kBQ2 = 64;  // query rows per dQ CTA

__global__ void __launch_bounds__(256) bwd_dot_kernel(const float* __restrict__ o,
                                                      const float* __restrict__ dout,
                                                      float* __restrict__ dvec, size_t rows,
                                                      int d) {
  const size_t row = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* a = o + row * d;
  const float* b = dout + row * d;
  float s = 0.0f;
  for (int c = lane; c < d; c += 32) s = fmaf(a[c], b[c], s);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) dvec[row] = s;
}

// Column-major ("transposed") tile in shared memory: t[c * ld + r] = src[r][c]
// (rows past rows_valid and columns past d are zeros).  Consecutive threads
// take consecutive rows, so the shared-memory writes hit consecutive banks;
// each reads 16 bytes of its row when d and the base allow it.
template <int D>
__device__ __forceinline__ void load_tile_t(float* t, int ld, const float* src, int rows_valid,
                                            int rows, int d) {
  if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    for (int i = threadIdx.x; i < rows * (D / 4); i += kBwdThreads) {
      const int r = i % rows, c = (i / rows) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < rows_valid && c < d) v = *reinterpret_cast<const float4*>(src + (size_t)r * d + c);
      t[c * ld + r] = v.x;
      t[(c + 1) * ld + r] = v.y;
      t[(c + 2) * ld + r] = v.z;
      t[(c + 3) * ld + r] = v.w;
    }
  } else {
    for (int i = threadIdx.x; i < rows * D; i += kBwdThreads) {
      const int r = i % rows, c = i / rows;
      t[c * ld + r] = (r < rows_valid && c < d) ? src[(size_t)r * d + c] : 0.0f;
    }
  }
}
// Row-major tile: t[r * ld + c] = src[r][c] (ld a multiple of 4).
template <int D>
__device__ __forceinline__ void load_tile(float* t, int ld, const float* src, int rows_valid,
                                          int rows, int d) {
  if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    for (int i = threadIdx.x; i < rows * (D / 4); i += kBwdThreads) {
      const int r = i / (D / 4), c = (i % (D / 4)) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < rows_valid && c < d) v = *reinterpret_cast<const float4*>(src + (size_t)r * d + c);
      *reinterpret_cast<float4*>(t + r * ld + c) = v;
    }
  } else {
    for (int i = threadIdx.x; i < rows * D; i += kBwdThreads) {
      const int r = i / D, c = i % D;
      t[r * ld + c] = (r < rows_valid && c < d) ? src[(size_t)r * d + c] : 0.0f;
    }
  }
}

// dK, dV for 64 keys of one slice.  Threads: 16 x 16.  Score tiles (32 rows x
// 64 keys): thread (ty, tx) owns rows 2ty..2ty+1, keys 4tx..4tx+3.  dK / dV
// (64 keys x D): thread owns keys 4ty..4ty+3, columns tx + 16 i (i < D/16).
template <int D>
__global__ void __launch_bounds__(kBwdThreads) bwd_dkdv_kernel(BwdParams p) {
  extern __shared__ float sm[];
  float* kT = sm;                   // [D][kBK]
  float* vT = kT + D * kBK;         // [D][kBK]
  float* qT = vT + D * kBK;         // [D][kBQ]
  float* doT = qT + D * kBQ;        // [D][kBQ]
  float* qR = doT + D * kBQ;        // [kBQ][D]
  float* doR = qR + kBQ * D;        // [kBQ][D]
  float* pS = doR + kBQ * D;        // [kBQ][kBK]
  float* dsS = pS + kBQ * kBK;      // [kBQ][kBK]
  float* rowv = dsS + kBQ * kBK;    // lse [kBQ], D [kBQ]
  const int bh = blockIdx.y, k0 = blockIdx.x * kBK;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int nk = min(kBK, p.sk - k0);
  const float* kb = p.k + ((size_t)bh * p.sk + k0) * p.d;
  const float* vb = p.v + ((size_t)bh * p.sk + k0) * p.d;
  load_tile_t<D>(kT, kBK, kb, nk, kBK, p.d);
  load_tile_t<D>(vT, kBK, vb, nk, kBK, p.d);
  constexpr int NC = D / 16;
  float dk[4][NC], dv[4][NC];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int c = 0; c < NC; c++) dk[a][c] = dv[a][c] = 0.0f;
  // query rows that see any of these keys: all, or (causal) rows >= k0
  int q_begin = 0;
  if (p.causal) {
    const long long first = (long long)k0 - p.q_offset + p.k_offset;  // first row seeing key k0
    q_begin = first <= 0 ? 0 : (first >= p.sq ? p.sq : (int)first);
  }
  q_begin = q_begin / kBQ * kBQ;
  for (int q0 = q_begin; q0 < p.sq; q0 += kBQ) {
    const int nq = min(kBQ, p.sq - q0);
    __syncthreads();  // previous step's tiles are no longer read
    const size_t rbase = (size_t)bh * p.sq + q0;
    load_tile_t<D>(qT, kBQ, p.q + rbase * p.d, nq, kBQ, p.d);
    load_tile_t<D>(doT, kBQ, p.dout + rbase * p.d, nq, kBQ, p.d);
    load_tile<D>(qR, D, p.q + rbase * p.d, nq, kBQ, p.d);
    load_tile<D>(doR, D, p.dout + rbase * p.d, nq, kBQ, p.d);
    if (tid < kBQ) rowv[tid] = tid < nq ? p.lse[rbase + tid] : 0.0f;
    else if (tid < 2 * kBQ) rowv[tid] = tid - kBQ < nq ? p.dvec[rbase + tid - kBQ] : 0.0f;
    __syncthreads();
    // S and dP for rows 2ty.., keys 4tx..
    float s[2][4] = {}, dp[2][4] = {};
#pragma unroll 4
    for (int c = 0; c < D; c++) {
      const float2 qa = *reinterpret_cast<const float2*>(qT + c * kBQ + 2 * ty);
      const float2 da = *reinterpret_cast<const float2*>(doT + c * kBQ + 2 * ty);
      const float4 kk = *reinterpret_cast<const float4*>(kT + c * kBK + 4 * tx);
      const float4 vv = *reinterpret_cast<const float4*>(vT + c * kBK + 4 * tx);
      const float kq[4] = {kk.x, kk.y, kk.z, kk.w}, vq[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        s[0][j] = fmaf(qa.x, kq[j], s[0][j]);
        s[1][j] = fmaf(qa.y, kq[j], s[1][j]);
        dp[0][j] = fmaf(da.x, vq[j], dp[0][j]);
        dp[1][j] = fmaf(da.y, vq[j], dp[1][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int r = 2 * ty + i;
      const long long qg = p.q_offset + q0 + r;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int kc = 4 * tx + j;
        const bool live = r < nq && kc < nk && (!p.causal || p.k_offset + k0 + kc <= qg);
        const float pr = live ? expf(s[i][j] * p.scale - rowv[r]) : 0.0f;
        pS[r * kBK + kc] = pr;
        dsS[r * kBK + kc] = pr * (dp[i][j] - rowv[kBQ + r]);
      }
    }
    __syncthreads();
    // dV += P^T dO, dK += dS^T Q (scale applied at the end)
#pragma unroll 2
    for (int r = 0; r < kBQ; r++) {
      const float4 pp = *reinterpret_cast<const float4*>(pS + r * kBK + 4 * ty);
      const float4 ss = *reinterpret_cast<const float4*>(dsS + r * kBK + 4 * ty);
      const float pa[4] = {pp.x, pp.y, pp.z, pp.w}, sa[4] = {ss.x, ss.y, ss.z, ss.w};
#pragma unroll
      for (int c = 0; c < NC; c++) {
        const float od = doR[r * D + tx + 16 * c];
        const float oq = qR[r * D + tx + 16 * c];
#pragma unroll
        for (int a = 0; a < 4; a++) {
          dv[a][c] = fmaf(pa[a], od, dv[a][c]);
          dk[a][c] = fmaf(sa[a], oq, dk[a][c]);
        }
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const int kc = 4 * ty + a;
    if (kc >= nk) continue;
    float* dkr = p.dk + ((size_t)bh * p.sk + k0 + kc) * p.d;
    float* dvr = p.dv + ((size_t)bh * p.sk + k0 + kc) * p.d;
#pragma unroll
    for (int c = 0; c < NC; c++) {
      const int col = tx + 16 * c;
      if (col < p.d) {
        dkr[col] = dk[a][c] * p.scale;
        dvr[col] = dv[a][c];
      }
    }
  }
}

// dQ for 64 query rows of one slice.  Score tiles (64 rows x 64 keys): thread
// (ty, tx) owns rows 4ty..4ty+3, keys 4tx..4tx+3.  dQ (64 rows x D): thread
// owns rows 4ty..4ty+3, columns tx + 16 i.
template <int D>
__global__ void __launch_bounds__(kBwdThreads) bwd_dq_kernel(BwdParams p) {
  extern __shared__ float sm[];
  float* qT = sm;                    // [D][kBQ2]
  float* doT = qT + D * kBQ2;        // [D][kBQ2]
  float* kT = doT + D * kBQ2;        // [D][kBK]
  float* vT = kT + D * kBK;          // [D][kBK]
  float* kR = vT + D * kBK;          // [kBK][D]
  float* dsS = kR + kBK * D;         // [kBQ2][kBK + 4]
  float* rowv = dsS + kBQ2 * (kBK + 4);  // lse [kBQ2], D [kBQ2]
  constexpr int LDS = kBK + 4;
  const int bh = blockIdx.y, q0 = blockIdx.x * kBQ2;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int nq = min(kBQ2, p.sq - q0);
  const size_t rbase = (size_t)bh * p.sq + q0;
  load_tile_t<D>(qT, kBQ2, p.q + rbase * p.d, nq, kBQ2, p.d);
  load_tile_t<D>(doT, kBQ2, p.dout + rbase * p.d, nq, kBQ2, p.d);
  if (tid < kBQ2) rowv[tid] = tid < nq ? p.lse[rbase + tid] : 0.0f;
  else if (tid < 2 * kBQ2) rowv[tid] = tid - kBQ2 < nq ? p.dvec[rbase + tid - kBQ2] : 0.0f;
  constexpr int NC = D / 16;
  float dq[4][NC];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int c = 0; c < NC; c++) dq[a][c] = 0.0f;
  // keys any of these rows sees: all, or (causal) keys <= the last row
  int k_end = p.sk;
  if (p.causal) k_end = causal_limit(p.q_offset + q0 + nq - 1, p.k_offset, p.sk);
  for (int k0 = 0; k0 < k_end; k0 += kBK) {
    const int nk = min(kBK, p.sk - k0);
    __syncthreads();
    const float* kb = p.k + ((size_t)bh * p.sk + k0) * p.d;
    const float* vb = p.v + ((size_t)bh * p.sk + k0) * p.d;
    load_tile_t<D>(kT, kBK, kb, nk, kBK, p.d);
    load_tile_t<D>(vT, kBK, vb, nk, kBK, p.d);
    load_tile<D>(kR, D, kb, nk, kBK, p.d);
    __syncthreads();
    float s[4][4] = {}, dp[4][4] = {};
#pragma unroll 2
    for (int c = 0; c < D; c++) {
      const float4 qa = *reinterpret_cast<const float4*>(qT + c * kBQ2 + 4 * ty);
      const float4 da = *reinterpret_cast<const float4*>(doT + c * kBQ2 + 4 * ty);
      const float4 kk = *reinterpret_cast<const float4*>(kT + c * kBK + 4 * tx);
      const float4 vv = *reinterpret_cast<const float4*>(vT + c * kBK + 4 * tx);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, dv4[4] = {da.x, da.y, da.z, da.w};
      const float kq[4] = {kk.x, kk.y, kk.z, kk.w}, vq[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
          s[i][j] = fmaf(qv[i], kq[j], s[i][j]);
          dp[i][j] = fmaf(dv4[i], vq[j], dp[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int r = 4 * ty + i;
      const long long qg = p.q_offset + q0 + r;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int kc = 4 * tx + j;
        const bool live = r < nq && kc < nk && (!p.causal || p.k_offset + k0 + kc <= qg);
        const float pr = live ? expf(s[i][j] * p.scale - rowv[r]) : 0.0f;
        dsS[r * LDS + kc] = pr * (dp[i][j] - rowv[kBQ2 + r]);
      }
    }
    __syncthreads();
    // dQ += dS K (scale applied at the end)
#pragma unroll 2
    for (int kc = 0; kc < kBK; kc++) {
      float sa[4];
#pragma unroll
      for (int a = 0; a < 4; a++) sa[a] = dsS[(4 * ty + a) * LDS + kc];
#pragma unroll
      for (int c = 0; c < NC; c++) {
        const float kv = kR[kc * D + tx + 16 * c];
#pragma unroll
        for (int a = 0; a < 4; a++) dq[a][c] = fmaf(sa[a], kv, dq[a][c]);
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const int r = 4 * ty + a;
    if (r >= nq) continue;
    float* dqr = p.dq + (rbase + r) * p.d;
#pragma unroll
    for (int c = 0; c < NC; c++) {
      const int col = tx + 16 * c;
      if (col < p.d) dqr[col] = dq[a][c] * p.scale;
    }
  }
}

template <int D>
size_t dkdv_smem() {
  return sizeof(float) * (2 * D * kBK + 4 * D * kBQ + 2 * kBQ * kBK + 2 * kBQ);
}
template <int D>
size_t dq_smem() {
  return sizeof(float) * (2 * D * kBQ2 + 3 * D * kBK + kBQ2 * (kBK + 4) + 2 * kBQ2);
}

template <int D>
cudaError_t launch_bwd_d(const BwdParams& p, cudaStream_t s) {
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(bwd_dkdv_kernel<D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)dkdv_smem<D>());
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(bwd_dq_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)dq_smem<D>());
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  for (int b0 = 0; b0 < p.bh; b0 += 65535) {
    BwdParams q = p;
    q.bh = min(65535, p.bh - b0);
    const size_t qo = (size_t)b0 * p.sq * p.d, ko = (size_t)b0 * p.sk * p.d;
    q.q += qo; q.dout += qo; q.dq += qo;
    q.k += ko; q.v += ko; q.dk += ko; q.dv += ko;
    q.lse += (size_t)b0 * p.sq; q.dvec += (size_t)b0 * p.sq;
    bwd_dkdv_kernel<D><<<dim3((p.sk + kBK - 1) / kBK, q.bh), kBwdThreads, dkdv_smem<D>(), s>>>(q);
    count_launch();
    bwd_dq_kernel<D><<<dim3((p.sq + kBQ2 - 1) / kBQ2, q.bh), kBwdThreads, dq_smem<D>(), s>>>(q);
    count_launch();
  }
  return cudaGetLastError();
}

}  // namespace

size_t bwd_workspace_floats(const BwdParams& p) { return (size_t)p.bh * p.sq; }

cudaError_t launch_bwd(BwdParams p, float* dvec, cudaStream_t s) {
  p.dvec = dvec;
  const size_t rows = (size_t)p.bh * p.sq;
  bwd_dot_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(p.o, p.dout, dvec, rows, p.d);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.d <= 32) return launch_bwd_d<32>(p, s);
  if (p.d <= 64) return launch_bwd_d<64>(p, s);
  if (p.d <= 128) return launch_bwd_d<128>(p, s);
  return cudaErrorInvalidValue;
}

}  // namespace fa
