// Host-side staging for the host-slice calls made with pageable buffers (the
// crate's `&[f32]` / `&mut [f32]` are ordinary heap memory).  A copy engine
// reads pageable memory only through the driver's own bounce buffers, which
// runs at a fraction of the PCIe rate, so such a call instead goes through
// rings of pinned slots that the library owns: host threads copy a piece of
// the input into a slot while the copy engine moves the previous slot to the
// device, and outputs come back the same way in reverse.
#include "fa_common.cuh"

#include <algorithm>
#include <cstdlib>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include <immintrin.h>

namespace fa {
namespace {

// Copy with non-temporal (streaming) stores: the destination lines are written
// without being read first, which saves a third of the memory traffic of an
// ordinary copy when many threads copy at once (the staged calls are bound by
// host memory bandwidth).  AVX2 when the CPU has it, else memcpy.
__attribute__((target("avx2"))) void copy_stream_avx2(char* dst, const char* src, size_t n) {
  const size_t head = std::min(n, (size_t)((32 - ((uintptr_t)dst & 31)) & 31));
  std::memcpy(dst, src, head);
  dst += head;
  src += head;
  n -= head;
  size_t i = 0;
  for (; i + 128 <= n; i += 128) {
    const __m256i a = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i));
    const __m256i b = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i + 32));
    const __m256i c = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i + 64));
    const __m256i d = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i + 96));
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i), a);
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i + 32), b);
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i + 64), c);
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i + 96), d);
  }
  std::memcpy(dst + i, src + i, n - i);
  _mm_sfence();  // the streamed stores are complete before the copy counts as done
}

void copy_stream(char* dst, const char* src, size_t n) {
  static const bool avx2 = __builtin_cpu_supports("avx2");
  if (avx2 && n >= 4096)
    copy_stream_avx2(dst, src, n);
  else
    std::memcpy(dst, src, n);
}

// A fixed pool of worker threads for one large memcpy at a time: the caller
// takes the first part, each worker one of the others.  Up to 16 threads, one
// per hardware thread; FA_B200_COPY_THREADS (read once) sets the count, for
// processes that share a host (one process per GPU: divide the cores).
class CopyPool {
 public:
  CopyPool() {
    const unsigned hw = std::thread::hardware_concurrency();
    n_ = (int)std::min(16u, std::max(1u, hw));
    if (const char* e = std::getenv("FA_B200_COPY_THREADS")) {
      const int v = std::atoi(e);
      if (v >= 1 && v <= 64) n_ = v;
    }
    for (int i = 1; i < n_; i++) workers_.emplace_back([this, i] { run(i); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  void copy(char* dst, const char* src, size_t bytes) {
    if (n_ == 1 || bytes < (size_t(1) << 20)) {  // (a hand-off costs ~10-50 us)
      copy_stream(dst, src, bytes);
      return;
    }
    std::lock_guard<std::mutex> call(call_m_);  // one parallel copy at a time
    {
      std::lock_guard<std::mutex> lk(m_);
      dst_ = dst;
      src_ = src;
      bytes_ = bytes;
      pending_ = n_ - 1;
      gen_++;
    }
    cv_.notify_all();
    part(0);
    std::unique_lock<std::mutex> lk(m_);
    done_cv_.wait(lk, [this] { return pending_ == 0; });
  }

 private:
  void part(int i) {
    // 64-byte aligned split points
    const size_t per = ((bytes_ + n_ - 1) / n_ + 63) & ~size_t(63);
    const size_t a = std::min(bytes_, per * i), b = std::min(bytes_, a + per);
    if (b > a) copy_stream(dst_ + a, src_ + a, b - a);
  }
  void run(int i) {
    unsigned long long seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(m_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
      }
      part(i);
      {
        std::lock_guard<std::mutex> lk(m_);
        if (--pending_ == 0) done_cv_.notify_one();
      }
    }
  }
  int n_ = 1;
  std::vector<std::thread> workers_;
  std::mutex m_, call_m_;
  std::condition_variable cv_, done_cv_;
  bool stop_ = false;
  unsigned long long gen_ = 0;
  int pending_ = 0;
  char* dst_ = nullptr;
  const char* src_ = nullptr;
  size_t bytes_ = 0;
};

CopyPool& copy_pool() {
  static CopyPool pool;
  return pool;
}

struct Rings {
  std::mutex call;  // one staged call per device at a time
  bool ready = false;
  PinnedRing in, out;
};
Rings g_rings[64];

}  // namespace

void parallel_copy(void* dst, const void* src, size_t bytes) {
  copy_pool().copy(static_cast<char*>(dst), static_cast<const char*>(src), bytes);
}

bool is_pageable(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type == cudaMemoryTypeUnregistered;
}

// Frees whatever a ring holds (slots and events created so far).
static void ring_free(PinnedRing& r) {
  for (int i = 0; i < PinnedRing::kSlots; i++) {
    if (r.ev[i]) {
      cudaEventSynchronize(r.ev[i]);
      cudaEventDestroy(r.ev[i]);
      r.ev[i] = nullptr;
    }
    if (r.buf[i]) {
      cudaFreeHost(r.buf[i]);
      r.buf[i] = nullptr;
    }
    r.busy[i] = false;
  }
  r.next = 0;
}

// All slots of a ring, or none: on a failure the slots and events already
// created are freed again, so a later call starts from an empty ring.
static cudaError_t ring_init(PinnedRing& r) {
  for (int i = 0; i < PinnedRing::kSlots; i++) {
    cudaError_t e = cudaMallocHost((void**)&r.buf[i], PinnedRing::kSlotBytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r.ev[i], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      cudaGetLastError();  // clear the (non-sticky) error of the failed call
      ring_free(r);
      return e;
    }
    r.busy[i] = false;
  }
  r.next = 0;
  return cudaSuccess;
}

cudaError_t staging_acquire(int dev, PinnedRing** in, PinnedRing** out, std::mutex** call) {
  Rings& g = g_rings[dev & 63];
  *call = &g.call;
  g.call.lock();
  if (!g.ready) {
    cudaError_t e = ring_init(g.in);
    if (e == cudaSuccess) {
      e = ring_init(g.out);
      if (e != cudaSuccess) ring_free(g.in);
    }
    if (e != cudaSuccess) {
      g.call.unlock();
      return e;
    }
    g.ready = true;
  }
  *in = &g.in;
  *out = &g.out;
  return cudaSuccess;
}

cudaError_t staged_copy_h2d(int dev, void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (!is_pageable(src)) return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s);
  PinnedRing *rin = nullptr, *rout = nullptr;
  std::mutex* call = nullptr;
  cudaError_t e = staging_acquire(dev, &rin, &rout, &call);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> unlock(*call, std::adopt_lock);
  constexpr size_t kSlot = PinnedRing::kSlotBytes;
  for (size_t off = 0; off < bytes && e == cudaSuccess; off += kSlot) {
    const size_t n = std::min(kSlot, bytes - off);
    const int sl = rin->next;
    rin->next = (sl + 1) % PinnedRing::kSlots;
    if (rin->busy[sl] && (e = cudaEventSynchronize(rin->ev[sl])) != cudaSuccess) break;
    parallel_copy(rin->buf[sl], static_cast<const char*>(src) + off, n);
    e = cudaMemcpyAsync(static_cast<char*>(dst) + off, rin->buf[sl], n, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaEventRecord(rin->ev[sl], s);
    rin->busy[sl] = e == cudaSuccess;
  }
  return e;
}

cudaError_t staged_copy_d2h(int dev, void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (!is_pageable(dst)) {
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s);
    return e == cudaSuccess ? cudaStreamSynchronize(s) : e;
  }
  PinnedRing *rin = nullptr, *rout = nullptr;
  std::mutex* call = nullptr;
  cudaError_t e = staging_acquire(dev, &rin, &rout, &call);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> unlock(*call, std::adopt_lock);
  constexpr size_t kSlot = PinnedRing::kSlotBytes;
  struct Piece {
    int slot;
    size_t off, n;
  };
  std::vector<Piece> pend;  // pieces in flight, oldest first
  size_t head = 0;
  auto drain_one = [&]() -> cudaError_t {
    const Piece pc = pend[head++];
    cudaError_t r = cudaEventSynchronize(rout->ev[pc.slot]);
    if (r == cudaSuccess) parallel_copy(static_cast<char*>(dst) + pc.off, rout->buf[pc.slot], pc.n);
    rout->busy[pc.slot] = false;
    return r;
  };
  for (size_t off = 0; off < bytes && e == cudaSuccess; off += kSlot) {
    const size_t n = std::min(kSlot, bytes - off);
    const int sl = rout->next;
    rout->next = (sl + 1) % PinnedRing::kSlots;
    while (e == cudaSuccess && rout->busy[sl]) {
      if (head < pend.size()) {
        e = drain_one();
      } else {  // (a slot left busy by an earlier call: wait for its copy)
        e = cudaEventSynchronize(rout->ev[sl]);
        rout->busy[sl] = false;
      }
    }
    if (e != cudaSuccess) break;
    e = cudaMemcpyAsync(rout->buf[sl], static_cast<const char*>(src) + off, n,
                        cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaEventRecord(rout->ev[sl], s);
    if (e != cudaSuccess) break;
    rout->busy[sl] = true;
    pend.push_back({sl, off, n});
  }
  while (head < pend.size()) {
    cudaError_t r = drain_one();
    if (e == cudaSuccess) e = r;
  }
  return e;
}

void staging_release_all() {
  for (int d = 0; d < 64; d++) {
    Rings& g = g_rings[d];
    std::lock_guard<std::mutex> lk(g.call);
    if (!g.ready) continue;
    cudaSetDevice(d);
    ring_free(g.in);
    ring_free(g.out);
    g.ready = false;
  }
}

}  // namespace fa
