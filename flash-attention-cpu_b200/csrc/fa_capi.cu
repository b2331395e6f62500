// The C ABI (include/fa_b200.h): argument and shape validation with the
// crate's semantics, host<->device staging for the host-slice calls, kernel
// selection, and the error side channel.  Every compute step is a kernel of
// this library; there is no CPU path.
#include "fa_common.cuh"
#include "fa_host.h"
#include "../../include/fa_b200.h"

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>
#include <algorithm>

namespace fa {
namespace {
std::atomic<unsigned long long> g_launches{0};
}
void count_launch(int n) { g_launches.fetch_add((unsigned long long)n); }
unsigned long long launches_issued() { return g_launches.load(); }
}  // namespace fa

namespace {

thread_local std::string t_err;
thread_local const char* t_path = "";

std::atomic<int> g_precision{-1};
std::atomic<int> g_device{-1};
// test hook (fa_test_stall): the abortable-wait limit and the withheld arrive
std::atomic<unsigned long long> g_wait_ns{fa::kWaitLimitNs};
std::atomic<int> g_test_skip{-1};

constexpr int kMaxDevices = 64;
struct DeviceState {
  std::once_flag once;
  cudaError_t init_err = cudaSuccess;
  int* err_flag = nullptr;  // device word written by kernels on a bounded-wait timeout
  int num_sms = 148;
  int cc_major = 0, cc_minor = 0;
};
DeviceState g_dev[kMaxDevices];

int set_err(int code, const std::string& msg) {
  t_err = msg;
  return code;
}
int cuda_err(cudaError_t e, const char* what) {
  return set_err(FA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int env_precision() {
  const char* s = std::getenv("FA_B200_PRECISION");
  if (!s) return FA_PREC_3XTF32;
  if (!strcmp(s, "tf32") || !strcmp(s, "TF32")) return FA_PREC_TF32;
  if (!strcmp(s, "fp32") || !strcmp(s, "FP32")) return FA_PREC_FP32;
  return FA_PREC_3XTF32;
}
int precision() {
  int p = g_precision.load();
  if (p < 0) {
    int e = env_precision();
    g_precision.compare_exchange_strong(p, e);
    p = g_precision.load();
  }
  return p;
}

// Make `dev` current and initialise the library's state on it once.
int prepare_device_at(int dev) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return set_err(FA_ERR_NO_DEVICE, "no CUDA device available (this library has no CPU path)");
  }
  if (dev < 0 || dev >= n || dev >= kMaxDevices) return set_err(FA_ERR_ARG, "device index out of range");
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaSetDevice");
  DeviceState& st = g_dev[dev];
  std::call_once(st.once, [&] {
    cudaDeviceProp prop;
    st.init_err = cudaGetDeviceProperties(&prop, dev);
    if (st.init_err != cudaSuccess) return;
    st.num_sms = prop.multiProcessorCount;
    st.cc_major = prop.major;
    st.cc_minor = prop.minor;
    st.init_err = cudaMalloc(&st.err_flag, sizeof(int));
    if (st.init_err != cudaSuccess) return;
    st.init_err = cudaMemset(st.err_flag, 0, sizeof(int));
    if (st.init_err != cudaSuccess) return;
    // Keep freed stream-ordered allocations cached in the pool.
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
      uint64_t thr = ~0ull;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
  });
  if (st.init_err != cudaSuccess) return cuda_err(st.init_err, "device initialisation");
  if (st.cc_major != 10)
    return set_err(FA_ERR_NO_DEVICE, "this library is built for sm_100a (B200) only");
  return FA_OK;
}

// The library's device (fa_set_device, else the CUDA current device), made
// current and initialised.
int prepare_device(int* dev_out) {
  int dev = g_device.load();
  if (dev < 0) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
      cudaGetLastError();
      return set_err(FA_ERR_NO_DEVICE, "no CUDA device available (this library has no CPU path)");
    }
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  }
  int rc = prepare_device_at(dev);
  if (rc) return rc;
  *dev_out = dev;
  return FA_OK;
}

// Devices of the host-slice calls (fa_set_devices / FA_B200_DEVICES).  An
// empty list means the single device of prepare_device().
std::mutex g_devs_m;
bool g_devs_read = false;
std::vector<int> g_devs;

void read_devices_env() {  // under g_devs_m
  if (g_devs_read) return;
  g_devs_read = true;
  const char* s = std::getenv("FA_B200_DEVICES");
  if (!s || !*s) return;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  std::vector<int> v;
  if (!strcmp(s, "all")) {
    for (int i = 0; i < n && i < kMaxDevices; i++) v.push_back(i);
  } else {
    const char* c = s;
    while (*c) {
      char* end = nullptr;
      long x = strtol(c, &end, 10);
      if (end == c || x < 0 || x >= n || v.size() >= (size_t)kMaxDevices) return;  // ignored
      v.push_back((int)x);
      c = *end == ',' ? end + 1 : end;
      if (*end && *end != ',') return;
    }
  }
  if (v.size() > 1) g_devs = v;
}

std::vector<int> device_list() {
  std::lock_guard<std::mutex> lk(g_devs_m);
  read_devices_env();
  return g_devs;
}

bool mul_ok(size_t a, size_t b, size_t* r) {
  if (a != 0 && b > SIZE_MAX / a) return false;
  *r = a * b;
  return true;
}

// Kernel selection for one forward over bh slices.
int dispatch(fa::FwdParams p, int dev, cudaStream_t s) {
  const int prec = precision();
  DeviceState& st = g_dev[dev];
  p.err = st.err_flag;
  p.wait_ns = g_wait_ns.load();
  p.test_skip = g_test_skip.load();
  p.scale = 1.0f / sqrtf((float)p.d);
  p.scale_log2 = p.scale * 1.4426950408889634f;
  cudaError_t e = cudaSuccess;
  // The tensor-core kernels address Q/K/V/O through TMA tensor maps and the
  // decode kernel through 16-byte vector loads: both need 16-byte aligned
  // bases.  A device call on other pointers (a view at an odd float offset)
  // runs the CUDA-core f32 kernel, which reads floats one at a time.
  const bool a16 = (((uintptr_t)p.q | (uintptr_t)p.k | (uintptr_t)p.v | (uintptr_t)p.o) & 15) == 0;
  if (p.sq <= 16 && fa::decode_supported(p.d) && a16) {
    // Few query rows: split the key range so every SM streams K/V.
    t_path = "decode_splitkv";
    const int splits = fa::decode_pick_splits(p.bh, p.sq, p.sk, st.num_sms, p.d);
    float* scratch = nullptr;
    if (splits > 1) {
      size_t n = (size_t)splits * p.bh * p.sq * (p.d + 1);
      e = cudaMallocAsync((void**)&scratch, n * sizeof(float), s);
      if (e != cudaSuccess) return cuda_err(e, "cudaMallocAsync(split partials)");
    }
    // grid.y holds the slice index: at most 65535 slices per launch.
    for (int b0 = 0; b0 < p.bh && e == cudaSuccess; b0 += 65535) {
      fa::FwdParams q = p;
      q.bh = p.bh - b0 < 65535 ? p.bh - b0 : 65535;
      q.q += (size_t)b0 * p.sq * p.d;
      q.k += (size_t)b0 * p.sk * p.d;
      q.v += (size_t)b0 * p.sk * p.d;
      q.o += (size_t)b0 * p.sq * p.d;
      if (q.lse) q.lse += (size_t)b0 * p.sq;
      e = fa::launch_decode(q, splits, scratch, s);
    }
    if (scratch) cudaFreeAsync(scratch, s);
    if (e != cudaSuccess) return cuda_err(e, "decode launch");
    return FA_OK;
  }
  if (prec == FA_PREC_3XTF32 && (p.d == 32 || p.d == 64 || p.d == 96 || p.d == 128) && a16) {
    t_path = "tcgen05_3xtf32";
    float* ws = nullptr;
    e = cudaMallocAsync((void**)&ws, fa::tc3_workspace_floats(p, st.num_sms) * sizeof(float), s);
    if (e != cudaSuccess) return cuda_err(e, "cudaMallocAsync(3xTF32 split planes)");
    e = fa::launch_tc3(p, ws, st.num_sms, s);
    cudaFreeAsync(ws, s);
    if (e != cudaSuccess) return cuda_err(e, "tcgen05 3xTF32 launch");
    return FA_OK;
  }
  if (fa::tc_supported(p.d, prec) && a16) {
    t_path = prec == FA_PREC_TF32 ? "tcgen05_tf32" : "tcgen05_3xtf32";
    // a launch with few 256-row tiles splits the key range (partials + LSE merge)
    const size_t nws = fa::tc_scratch_floats(p, st.num_sms);
    float* ws = nullptr;
    if (nws) {
      e = cudaMallocAsync((void**)&ws, nws * sizeof(float), s);
      if (e != cudaSuccess) return cuda_err(e, "cudaMallocAsync(split partials)");
    }
    e = fa::launch_tc(p, prec, ws, nws, s);
    if (ws) cudaFreeAsync(ws, s);
    if (e != cudaSuccess) return cuda_err(e, "tcgen05 launch");
    return FA_OK;
  }
  if (p.d <= 256) {
    t_path = "simt_fp32";
    for (int b0 = 0; b0 < p.bh && e == cudaSuccess; b0 += 65535) {
      fa::FwdParams q = p;
      q.bh = p.bh - b0 < 65535 ? p.bh - b0 : 65535;
      q.q += (size_t)b0 * p.sq * p.d;
      q.k += (size_t)b0 * p.sk * p.d;
      q.v += (size_t)b0 * p.sk * p.d;
      q.o += (size_t)b0 * p.sq * p.d;
      if (q.lse) q.lse += (size_t)b0 * p.sq;
      e = fa::launch_simt(q, s);
    }
    if (e != cudaSuccess) return cuda_err(e, "simt launch");
    return FA_OK;
  }
  return set_err(FA_ERR_UNSUPPORTED, "d_head > 256 is not supported");
}

// Reads and clears the device error word after the stream has finished.
int check_err_flag(int dev, cudaStream_t s) {
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, g_dev[dev].err_flag, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_err(e, "kernel execution");
  if (h != 0) {
    cudaMemsetAsync(g_dev[dev].err_flag, 0, sizeof(int), s);
    cudaStreamSynchronize(s);
    return set_err(FA_ERR_TIMEOUT, "a bounded in-kernel wait expired (kernel aborted)");
  }
  return FA_OK;
}

// Three streams per (thread, device) for the host-slice calls: host-to-device
// copies, compute, device-to-host copies.  Large calls are cut into chunks of
// (batch, head) slices so that the copies of one chunk overlap the compute and
// the copies of the others (the two copy directions use separate engines).
struct HostCallStreams {
  cudaStream_t s[kMaxDevices][3] = {};
  // events of the chunked pipeline and a pinned word for the device error
  // flag, kept for the thread's next call
  cudaEvent_t ev[kMaxDevices][2 * 8 + 2] = {};
  int* err_host[kMaxDevices] = {};
};
thread_local HostCallStreams t_streams;

int host_streams(int dev, cudaStream_t** out) {
  for (int i = 0; i < 3; i++)
    if (!t_streams.s[dev][i]) {
      cudaError_t e = cudaStreamCreateWithFlags(&t_streams.s[dev][i], cudaStreamNonBlocking);
      if (e != cudaSuccess) return cuda_err(e, "cudaStreamCreate");
    }
  *out = t_streams.s[dev];
  return FA_OK;
}

// Host-slice forward with pageable buffers: every byte moves through the
// library's pinned rings (fa_host_stage.cu).  Per chunk of (batch, head)
// slices the host threads copy its Q, K, V pieces into free input slots and
// the copy engine moves each slot to HBM; the chunk's kernel runs once its
// inputs are in; its O (and LSE) pieces come back into output slots and the
// host threads copy them out once their event has completed.  So the host
// copies of one chunk overlap the transfers and the kernel of the others.
int host_forward_staged(const float* q, const float* k, const float* v, size_t bh, size_t sq,
                        size_t sk, size_t d, int causal, float* out, float* lse, int dev,
                        cudaStream_t s_in, cudaStream_t s_comp, cudaStream_t s_out) {
  fa::PinnedRing *rin = nullptr, *rout = nullptr;
  std::mutex* call = nullptr;
  cudaError_t e = fa::staging_acquire(dev, &rin, &rout, &call);
  if (e != cudaSuccess) return cuda_err(e, "pinned staging buffers");
  std::lock_guard<std::mutex> unlock(*call, std::adopt_lock);
  const size_t nq = bh * sq * d, nk = bh * sk * d, nl = bh * sq;
  const size_t bytes = (2 * nq + 2 * nk + nl) * sizeof(float);
  char* buf = nullptr;
  e = cudaMallocAsync((void**)&buf, bytes, s_in);
  if (e != cudaSuccess) return cuda_err(e, "cudaMallocAsync(staging)");
  float* dq = (float*)buf;
  float* dk = dq + nq;
  float* dv = dk + nk;
  float* dout = dv + nk;
  float* dlse = dout + nq;
  constexpr size_t kSlot = fa::PinnedRing::kSlotBytes;
  struct Piece {
    int slot;
    char* dst;
    size_t n;
  };
  std::vector<Piece> pend;  // output pieces in flight, oldest first
  size_t pend_head = 0;
  auto drain_one = [&]() -> cudaError_t {
    const Piece pc = pend[pend_head++];
    cudaError_t r = cudaEventSynchronize(rout->ev[pc.slot]);
    if (r == cudaSuccess) fa::parallel_copy(pc.dst, rout->buf[pc.slot], pc.n);
    rout->busy[pc.slot] = false;
    return r;
  };
  auto stage_in = [&](float* dst, const float* src, size_t n_bytes) -> cudaError_t {
    for (size_t off = 0; off < n_bytes; off += kSlot) {
      const size_t n = std::min(kSlot, n_bytes - off);
      const int sl = rin->next;
      rin->next = (sl + 1) % fa::PinnedRing::kSlots;
      if (rin->busy[sl]) {
        cudaError_t r = cudaEventSynchronize(rin->ev[sl]);
        if (r != cudaSuccess) return r;
      }
      fa::parallel_copy(rin->buf[sl], (const char*)src + off, n);
      cudaError_t r = cudaMemcpyAsync((char*)dst + off, rin->buf[sl], n, cudaMemcpyHostToDevice, s_in);
      if (r == cudaSuccess) r = cudaEventRecord(rin->ev[sl], s_in);
      if (r != cudaSuccess) return r;
      rin->busy[sl] = true;
    }
    return cudaSuccess;
  };
  auto stage_out = [&](float* dst, const float* src, size_t n_bytes) -> cudaError_t {
    for (size_t off = 0; off < n_bytes; off += kSlot) {
      const size_t n = std::min(kSlot, n_bytes - off);
      const int sl = rout->next;
      rout->next = (sl + 1) % fa::PinnedRing::kSlots;
      while (rout->busy[sl]) {
        cudaError_t r = drain_one();
        if (r != cudaSuccess) return r;
      }
      cudaError_t r = cudaMemcpyAsync(rout->buf[sl], (const char*)src + off, n, cudaMemcpyDeviceToHost, s_out);
      if (r == cudaSuccess) r = cudaEventRecord(rout->ev[sl], s_out);
      if (r != cudaSuccess) return r;
      rout->busy[sl] = true;
      pend.push_back({sl, (char*)dst + off, n});
    }
    return cudaSuccess;
  };
  // 8 chunks: the first inputs and the last outputs (which nothing overlaps)
  // stay short, and each piece is large enough that the copy pool's hand-off
  // per piece is small against the copy (config 2, pageable buffers, one B200:
  // 16 chunks 5.4-5.5 ms, 8 chunks 5.25-5.3 ms, 4 chunks 5.3-5.35 ms)
  const size_t n_chunks = bh < 8 ? bh : 8;
  const size_t per = (bh + n_chunks - 1) / n_chunks;
  cudaEvent_t ev_in = nullptr, ev_comp = nullptr;
  e = cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev_comp, cudaEventDisableTiming);
  int rc = FA_OK;
  for (size_t h0 = 0; h0 < bh && e == cudaSuccess && rc == FA_OK; h0 += per) {
    const size_t h1 = (h0 + per < bh) ? h0 + per : bh;
    const size_t oq = h0 * sq * d, ok_ = h0 * sk * d, cq = (h1 - h0) * sq * d,
                 ck = (h1 - h0) * sk * d;
    e = stage_in(dq + oq, q + oq, cq * sizeof(float));
    if (e == cudaSuccess) e = stage_in(dk + ok_, k + ok_, ck * sizeof(float));
    if (e == cudaSuccess) e = stage_in(dv + ok_, v + ok_, ck * sizeof(float));
    if (e == cudaSuccess) e = cudaEventRecord(ev_in, s_in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s_comp, ev_in, 0);
    if (e != cudaSuccess) break;
    fa::FwdParams p{};
    p.q = dq + oq; p.k = dk + ok_; p.v = dv + ok_; p.o = dout + oq;
    p.lse = lse ? dlse + h0 * sq : nullptr;
    p.bh = (int)(h1 - h0); p.sq = (int)sq; p.sk = (int)sk; p.d = (int)d;
    p.q_offset = 0; p.k_offset = 0; p.causal = causal ? 1 : 0;
    rc = dispatch(p, dev, s_comp);
    if (rc != FA_OK) break;
    e = cudaEventRecord(ev_comp, s_comp);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s_out, ev_comp, 0);
    if (e == cudaSuccess) e = stage_out(out + oq, dout + oq, cq * sizeof(float));
    if (e == cudaSuccess && lse)
      e = stage_out(lse + h0 * sq, dlse + h0 * sq, (h1 - h0) * sq * sizeof(float));
    // copy out whatever has already come back
    while (e == cudaSuccess && pend_head < pend.size() &&
           cudaEventQuery(rout->ev[pend[pend_head].slot]) == cudaSuccess)
      e = drain_one();
  }
  while (e == cudaSuccess && pend_head < pend.size()) e = drain_one();
  cudaStreamSynchronize(s_out);
  cudaStreamSynchronize(s_comp);
  cudaStreamSynchronize(s_in);
  for (size_t i = pend_head; i < pend.size(); i++) rout->busy[pend[i].slot] = false;
  if (rc == FA_OK && e != cudaSuccess) rc = cuda_err(e, "pinned staging");
  if (rc == FA_OK) rc = check_err_flag(dev, s_in);
  cudaFreeAsync(buf, s_in);
  cudaStreamSynchronize(s_in);
  if (ev_in) cudaEventDestroy(ev_in);
  if (ev_comp) cudaEventDestroy(ev_comp);
  return rc;
}

// Host-slice forward on one device: stage to HBM, run, copy back, check.
int host_forward_one(int dev, const float* q, const float* k, const float* v, size_t bh,
                     size_t sq, size_t sk, size_t d, int causal, float* out, float* lse) {
  int rc = prepare_device_at(dev);
  if (rc) return rc;
  cudaStream_t* st;
  if ((rc = host_streams(dev, &st))) return rc;
  cudaStream_t s_in = st[0], s_comp = st[1], s_out = st[2];
  const size_t nq = bh * sq * d, nk = bh * sk * d, nl = bh * sq;
  const size_t bytes = (2 * nq + 2 * nk + nl) * sizeof(float);
  // Pageable buffers of a large call go through the pinned rings.
  if (bytes >= (size_t(16) << 20) &&
      (fa::is_pageable(q) || fa::is_pageable(k) || fa::is_pageable(v) ||
       fa::is_pageable(out) || (lse && fa::is_pageable(lse))))
    return host_forward_staged(q, k, v, bh, sq, sk, d, causal, out, lse, dev, s_in, s_comp,
                               s_out);
  const size_t n_chunks = (bh >= 2 && bytes >= (size_t(32) << 20)) ? (bh < 8 ? bh : 8) : 1;
  const size_t per = (bh + n_chunks - 1) / n_chunks;
  cudaEvent_t* ev = t_streams.ev[dev];
  const int n_ev = (int)(2 * n_chunks + 2);
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < n_ev && e == cudaSuccess; i++)
    if (!ev[i]) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
  if (e == cudaSuccess && !t_streams.err_host[dev])
    e = cudaMallocHost((void**)&t_streams.err_host[dev], sizeof(int));
  if (e != cudaSuccess) return cuda_err(e, "host call events");
  int* err_h = t_streams.err_host[dev];
  char* buf = nullptr;
  e = cudaMallocAsync((void**)&buf, bytes, s_in);
  if (e != cudaSuccess) return cuda_err(e, "cudaMallocAsync(staging)");
  float* dq = (float*)buf;
  float* dk = dq + nq;
  float* dv = dk + nk;
  float* dout = dv + nk;
  float* dlse = dout + nq;
  for (size_t c = 0; c < n_chunks && e == cudaSuccess && rc == FA_OK; c++) {
    const size_t h0 = c * per, h1 = (h0 + per < bh) ? h0 + per : bh;
    if (h0 >= h1) break;
    const size_t oq = h0 * sq * d, ok_ = h0 * sk * d, cq = (h1 - h0) * sq * d,
                 ck = (h1 - h0) * sk * d;
    e = cudaMemcpyAsync(dq + oq, q + oq, cq * sizeof(float), cudaMemcpyHostToDevice, s_in);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dk + ok_, k + ok_, ck * sizeof(float), cudaMemcpyHostToDevice, s_in);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dv + ok_, v + ok_, ck * sizeof(float), cudaMemcpyHostToDevice, s_in);
    if (e == cudaSuccess) e = cudaEventRecord(ev[2 * c], s_in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s_comp, ev[2 * c], 0);
    if (e != cudaSuccess) break;
    fa::FwdParams p{};
    p.q = dq + oq; p.k = dk + ok_; p.v = dv + ok_; p.o = dout + oq;
    p.lse = lse ? dlse + h0 * sq : nullptr;
    p.bh = (int)(h1 - h0); p.sq = (int)sq; p.sk = (int)sk; p.d = (int)d;
    p.q_offset = 0; p.k_offset = 0; p.causal = causal ? 1 : 0;
    rc = dispatch(p, dev, s_comp);
    if (rc != FA_OK) break;
    e = cudaEventRecord(ev[2 * c + 1], s_comp);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s_out, ev[2 * c + 1], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(out + oq, dout + oq, cq * sizeof(float), cudaMemcpyDeviceToHost, s_out);
    if (e == cudaSuccess && lse)
      e = cudaMemcpyAsync(lse + h0 * sq, dlse + h0 * sq, (h1 - h0) * sq * sizeof(float),
                          cudaMemcpyDeviceToHost, s_out);
  }
  // The device error word comes back behind the outputs (s_out waited for the
  // last kernel), and one synchronisation covers both.  The staging buffer is
  // freed in stream order once s_out and s_comp are done with it.
  *err_h = 0;
  cudaError_t e2 = cudaMemcpyAsync(err_h, g_dev[dev].err_flag, sizeof(int),
                                   cudaMemcpyDeviceToHost, s_out);
  if (e2 == cudaSuccess) e2 = cudaEventRecord(ev[n_ev - 2], s_out);
  if (e2 == cudaSuccess) e2 = cudaEventRecord(ev[n_ev - 1], s_comp);
  if (e2 == cudaSuccess) e2 = cudaStreamWaitEvent(s_in, ev[n_ev - 2], 0);
  if (e2 == cudaSuccess) e2 = cudaStreamWaitEvent(s_in, ev[n_ev - 1], 0);
  cudaFreeAsync(buf, s_in);
  cudaError_t e3 = cudaStreamSynchronize(s_out);
  if (e2 != cudaSuccess) {  // (the ordering above failed: drain everything)
    cudaStreamSynchronize(s_comp);
    cudaStreamSynchronize(s_in);
  }
  if (e == cudaSuccess) e = e2 != cudaSuccess ? e2 : e3;
  if (rc == FA_OK && e != cudaSuccess) rc = cuda_err(e, "host staging");
  if (rc == FA_OK && *err_h != 0) {
    cudaMemsetAsync(g_dev[dev].err_flag, 0, sizeof(int), s_out);
    cudaStreamSynchronize(s_out);
    rc = set_err(FA_ERR_TIMEOUT, "a bounded in-kernel wait expired (kernel aborted)");
  }
  return rc;
}

// Host-slice forward: the device list (several GPUs), else one device.
int host_forward(const float* q, const float* k, const float* v, size_t bh, size_t sq,
                 size_t sk, size_t d, int causal, float* out, float* lse) {
  if (bh > (size_t)INT32_MAX || sq > (size_t)INT32_MAX || sk > (size_t)INT32_MAX || d > 256)
    return set_err(d > 256 ? FA_ERR_UNSUPPORTED : FA_ERR_ARG, "dimension too large");
  const std::vector<int> devs = device_list();
  if (devs.size() > 1)
    return fa::host_forward_devices(devs.data(), (int)devs.size(), q, k, v, bh, sq, sk, d, causal,
                                    out, lse);
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc) return rc;
  return host_forward_one(dev, q, k, v, bh, sq, sk, d, causal, out, lse);
}

int single_head(const float* q, size_t q_len, const float* k, size_t k_len, const float* v,
                size_t v_len, size_t sq, size_t sk, size_t d, const fa_config* cfg, float* out,
                size_t out_len) {
  t_err.clear();
  size_t nq, nk;
  if (!mul_ok(sq, d, &nq) || !mul_ok(sk, d, &nk)) return set_err(FA_ERR_ARG, "size overflow");
  // Same order and messages as src/common.rs:51-54.
  if (q_len != nq) return set_err(FA_ERR_SHAPE, "q shape mismatch");
  if (k_len != nk) return set_err(FA_ERR_SHAPE, "k shape mismatch");
  if (v_len != nk) return set_err(FA_ERR_SHAPE, "v shape mismatch");
  if (out_len != nq) return set_err(FA_ERR_SHAPE, "out shape mismatch");
  if (sq == 0 || sk == 0 || d == 0) return FA_OK;  // out untouched (common.rs:56)
  if (!q || !k || !v || !out) return set_err(FA_ERR_ARG, "null buffer pointer");
  const int causal = cfg ? (cfg->causal != 0) : 0;
  return host_forward(q, k, v, 1, sq, sk, d, causal, out, nullptr);
}

int multi_head(const float* q, size_t q_len, const float* k, size_t k_len, const float* v,
               size_t v_len, size_t batch, size_t heads, size_t sq, size_t sk, size_t d,
               const fa_config* cfg, float* out, size_t out_len) {
  t_err.clear();
  size_t bh, per_q, per_k, nq, nk;
  if (!mul_ok(batch, heads, &bh) || !mul_ok(sq, d, &per_q) || !mul_ok(sk, d, &per_k) ||
      !mul_ok(bh, per_q, &nq) || !mul_ok(bh, per_k, &nk))
    return set_err(FA_ERR_ARG, "size overflow");
  // src/common.rs:87-90 (the crate's multihead asserts carry no message).
  if (q_len != nq) return set_err(FA_ERR_SHAPE, "multihead q shape mismatch");
  if (k_len != nk) return set_err(FA_ERR_SHAPE, "multihead k shape mismatch");
  if (v_len != nk) return set_err(FA_ERR_SHAPE, "multihead v shape mismatch");
  if (out_len != nq) return set_err(FA_ERR_SHAPE, "multihead out shape mismatch");
  if (bh == 0 || sq == 0 || sk == 0 || d == 0) return FA_OK;
  if (!q || !k || !v || !out) return set_err(FA_ERR_ARG, "null buffer pointer");
  const int causal = cfg ? (cfg->causal != 0) : 0;
  return host_forward(q, k, v, bh, sq, sk, d, causal, out, nullptr);
}

int device_forward(const float* q, const float* k, const float* v, float* out, float* lse,
                   size_t bh, size_t sq, size_t sk, size_t d, int causal, size_t q_off,
                   size_t k_off, void* stream) {
  t_err.clear();
  if (bh == 0 || sq == 0 || sk == 0 || d == 0) return FA_OK;
  if (!q || !k || !v || !out) return set_err(FA_ERR_ARG, "null buffer pointer");
  if (bh > (size_t)INT32_MAX || sq > (size_t)INT32_MAX || sk > (size_t)INT32_MAX)
    return set_err(FA_ERR_ARG, "dimension too large");
  if (d > 256) return set_err(FA_ERR_UNSUPPORTED, "d_head > 256 is not supported");
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc) return rc;
  fa::FwdParams p{};
  p.q = q; p.k = k; p.v = v; p.o = out; p.lse = lse;
  p.bh = (int)bh; p.sq = (int)sq; p.sk = (int)sk; p.d = (int)d;
  p.q_offset = (long long)q_off; p.k_offset = (long long)k_off;
  p.causal = causal ? 1 : 0;
  return dispatch(p, dev, (cudaStream_t)stream);
}

}  // namespace

// Internal interface of the multi-device orchestration (fa_host.h).
namespace fa {
int status_error(int code, const std::string& msg) { return set_err(code, msg); }
int status_cuda(cudaError_t e, const char* what) { return cuda_err(e, what); }
std::string status_message() { return t_err; }
int prepare_device_on(int dev) { return prepare_device_at(dev); }
int device_sm_count(int dev) { return g_dev[dev].num_sms; }
int dispatch_on(FwdParams p, int dev, cudaStream_t s) { return dispatch(p, dev, s); }
int check_err_flag_on(int dev, cudaStream_t s) { return check_err_flag(dev, s); }
int host_forward_on(int dev, const float* q, const float* k, const float* v, size_t bh,
                    size_t sq, size_t sk, size_t d, int causal, float* out, float* lse) {
  return host_forward_one(dev, q, k, v, bh, sq, sk, d, causal, out, lse);
}
}  // namespace fa

extern "C" {

fa_config fa_config_default(void) {
  fa_config c;
  c.block_size_q = 64;
  c.block_size_kv = 128;
  c.causal = 0;
  return c;
}

#define FA_SINGLE(name)                                                                       \
  int name(const float* q, size_t q_len, const float* k, size_t k_len, const float* v,       \
           size_t v_len, size_t sq, size_t sk, size_t d, const fa_config* cfg, float* out,    \
           size_t out_len) {                                                                  \
    return single_head(q, q_len, k, k_len, v, v_len, sq, sk, d, cfg, out, out_len);           \
  }
FA_SINGLE(fa_flash_attention_v1)
FA_SINGLE(fa_flash_attention_v2)
FA_SINGLE(fa_flash_attention_v3)
FA_SINGLE(fa_flash_attention)
#undef FA_SINGLE

#define FA_MULTI(name)                                                                        \
  int name(const float* q, size_t q_len, const float* k, size_t k_len, const float* v,       \
           size_t v_len, size_t batch, size_t heads, size_t sq, size_t sk, size_t d,          \
           const fa_config* cfg, float* out, size_t out_len) {                                \
    return multi_head(q, q_len, k, k_len, v, v_len, batch, heads, sq, sk, d, cfg, out,        \
                      out_len);                                                               \
  }
FA_MULTI(fa_flash_attention_multihead_v1)
FA_MULTI(fa_flash_attention_multihead_v2)
FA_MULTI(fa_flash_attention_multihead_v3)
FA_MULTI(fa_flash_attention_multihead)
#undef FA_MULTI

int fa_flash_attention_multihead_lse(const float* q, const float* k, const float* v,
                                     size_t batch_heads, size_t sq, size_t sk, size_t d,
                                     int causal, float* out, float* lse) {
  t_err.clear();
  if (batch_heads == 0 || sq == 0 || sk == 0 || d == 0) return FA_OK;
  if (!q || !k || !v || !out) return set_err(FA_ERR_ARG, "null buffer pointer");
  return host_forward(q, k, v, batch_heads, sq, sk, d, causal, out, lse);
}

int fa_forward_device(const float* q, const float* k, const float* v, float* out, float* lse,
                      size_t bh, size_t sq, size_t sk, size_t d, int causal, void* stream) {
  return device_forward(q, k, v, out, lse, bh, sq, sk, d, causal, 0, 0, stream);
}

int fa_forward_partial_device(const float* q, const float* k, const float* v, float* out,
                              float* lse, size_t bh, size_t sq, size_t sk, size_t d, int causal,
                              size_t q_offset, size_t k_offset, void* stream) {
  return device_forward(q, k, v, out, lse, bh, sq, sk, d, causal, q_offset, k_offset, stream);
}

int fa_backward_device(const float* q, const float* k, const float* v, const float* out,
                       const float* lse, const float* dout, float* dq, float* dk, float* dv,
                       size_t bh, size_t sq, size_t sk, size_t d, int causal, void* stream) {
  t_err.clear();
  if (bh == 0 || sq == 0 || sk == 0 || d == 0) return FA_OK;
  if (!q || !k || !v || !out || !lse || !dout || !dq || !dk || !dv)
    return set_err(FA_ERR_ARG, "null buffer pointer");
  if (d > 128) return set_err(FA_ERR_UNSUPPORTED, "backward: d_head > 128 is not supported");
  if (bh > (size_t)INT32_MAX || sq > (size_t)INT32_MAX || sk > (size_t)INT32_MAX)
    return set_err(FA_ERR_ARG, "dimension too large");
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  fa::BwdParams p{};
  p.q = q; p.k = k; p.v = v; p.o = out; p.lse = lse; p.dout = dout;
  p.dq = dq; p.dk = dk; p.dv = dv;
  p.bh = (int)bh; p.sq = (int)sq; p.sk = (int)sk; p.d = (int)d;
  p.causal = causal ? 1 : 0;
  p.scale = 1.0f / sqrtf((float)d);
  p.err = g_dev[dev].err_flag;
  p.wait_ns = g_wait_ns.load();
  p.test_skip = g_test_skip.load();
  // TF32 precision on 16-byte aligned buffers with a supported head size runs
  // the tensor-core kernels; everything else the exact f32 CUDA-core kernels.
  bool aligned = true;
  for (const void* ptr : {(const void*)q, (const void*)k, (const void*)v, (const void*)out,
                          (const void*)dout, (const void*)dq, (const void*)dk, (const void*)dv})
    aligned = aligned && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0;
  const bool tc = precision() == FA_PREC_TF32 && aligned && fa::tc_bwd_supported((int)d);
  float* ws = nullptr;
  const size_t ws_floats = tc ? fa::tc_bwd_workspace_floats(p) : fa::bwd_workspace_floats(p);
  cudaError_t e = cudaMallocAsync((void**)&ws, ws_floats * sizeof(float), s);
  if (e != cudaSuccess) return cuda_err(e, "cudaMallocAsync(backward workspace)");
  e = tc ? fa::launch_tc_bwd(p, ws, s) : fa::launch_bwd(p, ws, s);
  cudaFreeAsync(ws, s);
  if (e != cudaSuccess) return cuda_err(e, "backward launch");
  t_path = tc ? "tc_tf32_backward" : "simt_backward";
  return FA_OK;
}

int fa_flash_attention_backward(const float* q, const float* k, const float* v, const float* out,
                                const float* lse, const float* dout, float* dq, float* dk,
                                float* dv, size_t bh, size_t sq, size_t sk, size_t d,
                                int causal) {
  t_err.clear();
  if (bh == 0 || sq == 0 || sk == 0 || d == 0) return FA_OK;
  if (!q || !k || !v || !out || !lse || !dout || !dq || !dk || !dv)
    return set_err(FA_ERR_ARG, "null buffer pointer");
  size_t nq, nk;
  if (!mul_ok(bh, sq, &nq) || !mul_ok(nq, d, &nq) || !mul_ok(bh, sk, &nk) || !mul_ok(nk, d, &nk))
    return set_err(FA_ERR_ARG, "size overflow");
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc) return rc;
  cudaStream_t* st;
  if ((rc = host_streams(dev, &st))) return rc;
  cudaStream_t s = st[1];
  const size_t nl = bh * sq;
  const size_t floats = 4 * nq + 4 * nk + nl;  // q o do dq, k v dk dv, lse
  float* buf = nullptr;
  cudaError_t e = cudaMallocAsync((void**)&buf, floats * sizeof(float), s);
  if (e != cudaSuccess) return cuda_err(e, "cudaMallocAsync(backward buffers)");
  float *dq_ = buf, *dO = dq_ + nq, *dout_ = dO + nq, *dqo = dout_ + nq;
  float *dk_ = dqo + nq, *dv_ = dk_ + nk, *dko = dv_ + nk, *dvo = dko + nk, *dl = dvo + nk;
  const struct {
    float* dst;
    const float* src;
    size_t n;
  } ins[] = {{dq_, q, nq}, {dO, out, nq}, {dout_, dout, nq}, {dk_, k, nk}, {dv_, v, nk},
             {dl, lse, nl}};
  for (const auto& c : ins)
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(c.dst, c.src, c.n * sizeof(float), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) {
    rc = fa_backward_device(dq_, dk_, dv_, dO, dl, dout_, dqo, dko, dvo, bh, sq, sk, d, causal,
                            s);
    if (rc == FA_OK) {
      e = cudaMemcpyAsync(dq, dqo, nq * sizeof(float), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(dk, dko, nk * sizeof(float), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(dv, dvo, nk * sizeof(float), cudaMemcpyDeviceToHost, s);
    }
  }
  cudaError_t e2 = cudaStreamSynchronize(s);
  cudaFreeAsync(buf, s);
  cudaStreamSynchronize(s);
  if (rc != FA_OK) return rc;
  if (e == cudaSuccess) e = e2;
  if (e != cudaSuccess) return cuda_err(e, "backward copies");
  return check_err_flag(dev, s);  // a bounded wait that ran out (FA_ERR_TIMEOUT)
}

int fa_lse_combine_device(const float* o_parts, const float* lse_parts, size_t n_parts,
                          size_t rows, size_t d, float* out, float* lse_out, void* stream) {
  t_err.clear();
  if (rows == 0 || d == 0) return FA_OK;
  if (n_parts == 0 || !o_parts || !lse_parts || !out)
    return set_err(FA_ERR_ARG, "null buffer pointer or zero parts");
  if (rows > (size_t)INT32_MAX || n_parts > (size_t)INT32_MAX || d > 4096)
    return set_err(FA_ERR_ARG, "dimension too large");
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc) return rc;
  t_path = "lse_combine";
  cudaError_t e = fa::launch_combine(o_parts, lse_parts, (int)n_parts, (long long)rows, (int)d,
                                     out, lse_out, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_err(e, "combine launch");
  return FA_OK;
}

int fa_forward_decode_noalloc(const float* q, const float* k, const float* v, float* out,
                              float* lse, size_t bh, size_t sq, size_t sk, size_t d, int causal,
                              void* stream) {
  t_err.clear();
  if (bh == 0 || sq == 0 || sk == 0 || d == 0) return FA_OK;
  if (!q || !k || !v || !out) return set_err(FA_ERR_ARG, "null buffer pointer");
  // Sizes are checked on their size_t values, before any narrowing cast.
  if (sq > 16 || d > 256 || !fa::decode_supported((int)d))
    return set_err(FA_ERR_UNSUPPORTED,
                   "fa_forward_decode_noalloc handles seq_len_q <= 16 and d_head % 4 == 0, "
                   "d_head <= 256");
  if (bh > 65535) return set_err(FA_ERR_UNSUPPORTED, "fa_forward_decode_noalloc: batch_heads > 65535");
  if (sk > (size_t)INT32_MAX)
    return set_err(FA_ERR_UNSUPPORTED, "fa_forward_decode_noalloc: seq_len_k > 2147483647");
  // The decode kernel reads Q, K and V with 16-byte vector loads; the regular
  // entry point sends other pointers to the scalar kernel, this one refuses
  // them before any device call.
  if ((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15) != 0 ||
      ((uintptr_t)lse & 3) != 0)
    return set_err(FA_ERR_UNSUPPORTED,
                   "fa_forward_decode_noalloc: q, k, v and out must be 16-byte aligned");
  // Device checks without the library's lazy set-up (which allocates).  The
  // device chosen by fa_set_device applies here as in every other call.
  int dev = g_device.load(), major = 0, sms = 0;
  cudaError_t e = dev >= 0 ? cudaSetDevice(dev) : cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(FA_ERR_NO_DEVICE, std::string("no usable CUDA device: ") + cudaGetErrorString(e));
  }
  if (major != 10) return set_err(FA_ERR_NO_DEVICE, "this library is built for sm_100a (B200) only");
  const int splits = fa::decode_pick_splits((int)bh, (int)sq, (int)sk, sms, (int)d);
  const size_t need = splits > 1 ? (size_t)splits * bh * sq * (d + 1) : 0;
  if (need > fa::static_scratch_floats())
    return set_err(FA_ERR_UNSUPPORTED,
                   "fa_forward_decode_noalloc: needs " + std::to_string(need) +
                       " floats of scratch, the fixed limit is " +
                       std::to_string(fa::static_scratch_floats()));
  float* scratch = nullptr;
  e = fa::static_scratch_ptr(&scratch);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetSymbolAddress(decode scratch)");
  fa::FwdParams p{};
  p.q = q; p.k = k; p.v = v; p.o = out; p.lse = lse;
  p.bh = (int)bh; p.sq = (int)sq; p.sk = (int)sk; p.d = (int)d;
  p.causal = causal ? 1 : 0;
  p.scale = 1.0f / sqrtf((float)p.d);
  p.scale_log2 = p.scale * 1.4426950408889634f;
  p.err = nullptr;  // the decode kernels have no bounded waits
  e = fa::launch_decode(p, splits, scratch, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_err(e, "decode launch");
  t_path = "decode_splitkv_noalloc";
  return FA_OK;
}

int fa_sync_status(void* stream) {
  t_err.clear();
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc) return rc;
  return check_err_flag(dev, (cudaStream_t)stream);
}

int fa_test_stall(int skip_block, unsigned long long wait_ns) {
  g_wait_ns.store(wait_ns ? wait_ns : fa::kWaitLimitNs);
  g_test_skip.store(skip_block < 0 ? -1 : skip_block);
  return FA_OK;
}

int fa_set_precision(int p) {
  if (p < FA_PREC_TF32 || p > FA_PREC_FP32) return set_err(FA_ERR_ARG, "unknown precision");
  g_precision.store(p);
  return FA_OK;
}
int fa_get_precision(void) { return precision(); }

int fa_set_device(int device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return set_err(FA_ERR_NO_DEVICE, "no CUDA device available");
  }
  if (device < 0 || device >= n) return set_err(FA_ERR_ARG, "device index out of range");
  g_device.store(device);
  return FA_OK;
}

int fa_set_devices(const int* devices, int n) {
  t_err.clear();
  if (n < 0 || n > kMaxDevices || (n > 0 && !devices))
    return set_err(FA_ERR_ARG, "device list: bad pointer or length");
  int count = 0;
  if (n > 0 && (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)) {
    cudaGetLastError();
    return set_err(FA_ERR_NO_DEVICE, "no CUDA device available");
  }
  for (int i = 0; i < n; i++)
    if (devices[i] < 0 || devices[i] >= count) return set_err(FA_ERR_ARG, "device index out of range");
  std::lock_guard<std::mutex> lk(g_devs_m);
  g_devs_read = true;  // an explicit list overrides FA_B200_DEVICES
  g_devs.clear();
  if (n > 1) g_devs.assign(devices, devices + n);
  else if (n == 1) g_device.store(devices[0]);
  return FA_OK;
}

int fa_get_devices(int* devices, int capacity) {
  const std::vector<int> v = device_list();
  if (devices)
    for (int i = 0; i < (int)v.size() && i < capacity; i++) devices[i] = v[i];
  return (int)v.size();
}

int fa_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

const char* fa_last_error(void) { return t_err.c_str(); }
uint64_t fa_launch_count(void) { return fa::launches_issued(); }
const char* fa_last_path(void) { return t_path; }

int fa_pin_host(void* ptr, size_t bytes) {
  t_err.clear();
  if (!ptr || bytes == 0) return set_err(FA_ERR_ARG, "null or empty host range");
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc) return rc;
  cudaError_t e = cudaHostRegister(ptr, bytes, cudaHostRegisterDefault);
  if (e == cudaErrorHostMemoryAlreadyRegistered) {
    cudaGetLastError();
    return FA_OK;
  }
  if (e != cudaSuccess) return cuda_err(e, "cudaHostRegister");
  return FA_OK;
}

int fa_unpin_host(void* ptr) {
  t_err.clear();
  if (!ptr) return set_err(FA_ERR_ARG, "null host pointer");
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc) return rc;
  cudaError_t e = cudaHostUnregister(ptr);
  if (e != cudaSuccess) return cuda_err(e, "cudaHostUnregister");
  return FA_OK;
}

void fa_shutdown(void) {
  int cur = 0;
  const bool have_cur = cudaGetDevice(&cur) == cudaSuccess;
  fa::staging_release_all();
  fa::devices_release();
  // the calling thread's streams, pipeline events and pinned error word
  for (int d = 0; d < kMaxDevices; d++) {
    bool set = false;
    for (int i = 0; i < 3; i++)
      if (t_streams.s[d][i]) {
        if (!set) cudaSetDevice(d);
        set = true;
        cudaStreamSynchronize(t_streams.s[d][i]);
        cudaStreamDestroy(t_streams.s[d][i]);
        t_streams.s[d][i] = nullptr;
      }
    for (cudaEvent_t& e : t_streams.ev[d])
      if (e) {
        if (!set) cudaSetDevice(d);
        set = true;
        cudaEventDestroy(e);
        e = nullptr;
      }
    if (t_streams.err_host[d]) {
      cudaFreeHost(t_streams.err_host[d]);
      t_streams.err_host[d] = nullptr;
    }
  }
  if (have_cur) cudaSetDevice(cur);  // the caller's device, as it was
}

}  // extern "C"
