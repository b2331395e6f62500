// The host-slice forward over several GPUs of one process (fa_set_devices /
// FA_B200_DEVICES).  The crate fans its (batch, head) slices out over every
// core (src/common.rs:72-101); here they fan out over GPUs:
//
//   Several slices: contiguous slice ranges, one per device, each running the
//   whole single-device call (its own copies in over its own host link, its
//   own kernels, its own copies out) on a persistent host thread per device.
//   There is no collective: the slices are independent.
//
//   Fewer slices than devices, long sequences (the crate's single-head
//   flash_attention_v2 on a long head, src/v2.rs:49-121): each slice's keys
//   are split into 2G chunks dealt zig-zag (device g gets chunks g and
//   2G-1-g, which balances the causal work).  Each device computes, for each
//   of its chunks, the range-normalised partial output and LSE of every query
//   row that sees the chunk; the partial rows go to the device that owns
//   them (query rows are cut into 2G row chunks dealt the same way) by peer
//   copies (copy engines over NVLink; no kernel reads another GPU's memory),
//   and each owner merges its rows' partials with the LSE combine kernel and
//   copies them to the host.
//
// A device may appear more than once in the list: its entries then share the
// GPU, which runs the same partial kernels, copies and merges (this is how the
// logic is tested on one GPU).
#include <algorithm>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/fa_b200.h"
#include "fa_host.h"

namespace fa {
namespace {

constexpr int kMaxSlots = 64;

// Persistent host threads: run(n, fn) calls fn(i) for i in [0, n), i = 0 on
// the calling thread and i > 0 on worker i, and returns when all are done.
// The workers keep their per-thread streams and events across calls.
class Pool {
 public:
  static Pool& get() {
    static Pool* p = new Pool();  // never destroyed: workers may outlive static teardown
    return *p;
  }
  void run(int n, const std::function<void(int)>& fn) {
    std::lock_guard<std::mutex> call(call_m_);
    {
      std::lock_guard<std::mutex> lk(m_);
      while ((int)workers_ + 1 < n) {
        const int i = ++workers_;
        const unsigned long long g = gen_;
        std::thread([this, i, g] { loop(i, g); }).detach();
      }
      fn_ = &fn;
      n_ = n;
      pending_ = n - 1;
      gen_++;
    }
    cv_.notify_all();
    fn(0);
    std::unique_lock<std::mutex> lk(m_);
    done_cv_.wait(lk, [this] { return pending_ == 0; });
    fn_ = nullptr;
  }

 private:
  void loop(int i, unsigned long long seen) {
    for (;;) {
      const std::function<void(int)>* fn = nullptr;
      {
        std::unique_lock<std::mutex> lk(m_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        if (i >= n_) continue;
        fn = fn_;
      }
      (*fn)(i);
      std::lock_guard<std::mutex> lk(m_);
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }
  std::mutex call_m_, m_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int)>* fn_ = nullptr;
  int n_ = 0, pending_ = 0, workers_ = 0;
  unsigned long long gen_ = 0;
};

struct Result {
  int rc = FA_OK;
  std::string msg;
};
int first_error(const std::vector<Result>& r) {
  for (const Result& x : r)
    if (x.rc != FA_OK) return status_error(x.rc, x.msg);
  return FA_OK;
}

// ---- several slices: contiguous ranges per device -------------------------
int shard_slices(const int* devs, int n, const float* q, const float* k, const float* v,
                 size_t bh, size_t sq, size_t sk, size_t d, int causal, float* out, float* lse) {
  std::vector<Result> res(n);
  Pool::get().run(n, [&](int i) {
    const size_t h0 = bh * i / n, h1 = bh * (i + 1) / n;
    if (h1 <= h0) return;
    res[i].rc = host_forward_on(devs[i], q + h0 * sq * d, k + h0 * sk * d, v + h0 * sk * d,
                                h1 - h0, sq, sk, d, causal, out + h0 * sq * d,
                                lse ? lse + h0 * sq : nullptr);
    if (res[i].rc != FA_OK) res[i].msg = status_message();
  });
  return first_error(res);
}

// ---- one long slice: key-range split with peer exchange --------------------
struct KvSlot {  // cached per position in the device list
  int dev = -1;
  cudaStream_t s = nullptr;
  cudaEvent_t sent = nullptr;
  float* ws = nullptr;
  size_t ws_floats = 0;
};
std::mutex g_kv_m;  // one key-range-split call at a time
KvSlot g_kv[kMaxSlots];
unsigned long long g_peer_on[kMaxSlots] = {};  // bit j of [i]: i reaches j's memory

void slot_free(KvSlot& k) {
  if (k.dev < 0) return;
  cudaSetDevice(k.dev);
  if (k.s) cudaStreamSynchronize(k.s);
  if (k.ws) cudaFree(k.ws);
  if (k.sent) cudaEventDestroy(k.sent);
  if (k.s) cudaStreamDestroy(k.s);
  k = KvSlot{};
}

// Slot resources on `dev` with at least `floats` of workspace (dev current).
cudaError_t slot_ready(KvSlot& k, int dev, size_t floats) {
  if (k.dev != dev) {
    slot_free(k);
    cudaSetDevice(dev);
    k.dev = dev;
    cudaError_t e = cudaStreamCreateWithFlags(&k.s, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&k.sent, cudaEventDisableTiming);
    if (e != cudaSuccess) return e;
  }
  if (k.ws_floats < floats) {
    if (k.ws) {
      cudaStreamSynchronize(k.s);
      cudaFree(k.ws);
      k.ws = nullptr;
      k.ws_floats = 0;
    }
    cudaError_t e = cudaMalloc((void**)&k.ws, floats * sizeof(float));
    if (e != cudaSuccess) return e;
    k.ws_floats = floats;
  }
  return cudaSuccess;
}

void enable_peers(const int* devs, int n) {
  for (int i = 0; i < n; i++)
    for (int j = 0; j < n; j++) {
      const int a = devs[i], b = devs[j];
      if (a == b || a >= kMaxSlots || b >= kMaxSlots || (g_peer_on[a] >> b & 1)) continue;
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, a, b) == cudaSuccess && can) {
        cudaSetDevice(a);
        cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) e = cudaSuccess;
        cudaGetLastError();
        if (e != cudaSuccess) continue;  // peer copies then stage through the host
      }
      g_peer_on[a] |= 1ull << b;
    }
}

size_t up16(size_t x) { return (x + 15) & ~size_t(15); }  // 64-byte aligned regions

// The plan of one split: key chunks, row chunks and each slot's workspace layout.
struct Plan {
  int n = 0, nch = 0;  // devices, chunks (2n)
  size_t sq = 0, sk = 0, d = 0;
  bool causal = false;
  size_t kc = 0, rc = 0;  // keys per key chunk, rows per row chunk
  struct Chunk {
    size_t k0 = 0, k1 = 0;   // key range
    int slot = 0;            // the device-list position that computes it
    bool used = false;       // some row sees it
    size_t rfirst = 0;       // first row chunk that sees it
    size_t kv_off = 0;       // its K (and V) rows in the slot's K/V regions
    size_t po = 0, pl = 0;   // its partial output / LSE in the slot's workspace
  };
  struct Rows {
    size_t r0 = 0, r1 = 0;   // row range
    int owner = 0;
    std::vector<int> parts;  // chunks contributing, in order
    size_t recv = 0;         // [parts][len][d] then [parts][len] in the owner's workspace
    size_t out = 0, lse = 0; // merged rows (owner's workspace)
  };
  std::vector<Chunk> ch;
  std::vector<Rows> rows;
  struct Slot {
    size_t qrow0 = 0;        // first query row held
    size_t q = 0, k = 0, v = 0, kv_len = 0, total = 0;
    bool any = false;
  };
  std::vector<Slot> slot;

  static int owner_of(int x, int n) { return x < n ? x : 2 * n - 1 - x; }

  void build(int n_, size_t sq_, size_t sk_, size_t d_, bool causal_) {
    n = n_; nch = 2 * n; sq = sq_; sk = sk_; d = d_; causal = causal_;
    kc = ((sk + nch - 1) / nch + 127) / 128 * 128;
    rc = ((sq + nch - 1) / nch + 127) / 128 * 128;
    ch.assign(nch, Chunk{});
    rows.assign(nch, Rows{});
    slot.assign(n, Slot{});
    for (int c = 0; c < nch; c++) {
      Chunk& x = ch[c];
      x.k0 = std::min(sk, c * kc);
      x.k1 = std::min(sk, (c + 1) * kc);
      x.slot = owner_of(c, n);
      x.used = x.k1 > x.k0 && (!causal || x.k0 < sq);  // top-left: row i sees key j <= i
      x.rfirst = causal ? x.k0 / rc : 0;
    }
    for (int r = 0; r < nch; r++) {
      Rows& y = rows[r];
      y.r0 = std::min(sq, r * rc);
      y.r1 = std::min(sq, (r + 1) * rc);
      y.owner = owner_of(r, n);
      if (y.r1 > y.r0)
        for (int c = 0; c < nch; c++)
          if (ch[c].used && ch[c].rfirst <= (size_t)r) y.parts.push_back(c);
    }
    for (int s = 0; s < n; s++) {
      Slot& z = slot[s];
      z.qrow0 = sq;
      for (int c = 0; c < nch; c++)
        if (ch[c].used && ch[c].slot == s) {
          z.any = true;
          z.qrow0 = std::min(z.qrow0, ch[c].rfirst * rc);
          ch[c].kv_off = z.kv_len;
          z.kv_len += up16((ch[c].k1 - ch[c].k0) * d);
        }
      size_t off = 0;
      if (z.any) {
        z.q = off;
        off += up16((sq - z.qrow0) * d);
        z.k = off;
        off += z.kv_len;
        z.v = off;
        off += z.kv_len;
        for (int c = 0; c < nch; c++)
          if (ch[c].used && ch[c].slot == s) {
            const size_t prow = sq - ch[c].rfirst * rc;
            ch[c].po = off;
            off += up16(prow * d);
            ch[c].pl = off;
            off += up16(prow);
          }
      }
      for (int r = 0; r < nch; r++)
        if (rows[r].owner == s && rows[r].r1 > rows[r].r0) {
          const size_t len = rows[r].r1 - rows[r].r0, np = rows[r].parts.size();
          rows[r].recv = off;
          off += up16(np * len * d) + up16(np * len);
          rows[r].out = off;
          off += up16(len * d);
          rows[r].lse = off;
          off += up16(len);
        }
      z.total = off;
    }
  }
};

int kv_split_slice(const int* devs, int n, const float* q, const float* k, const float* v,
                   size_t sq, size_t sk, size_t d, int causal, float* out, float* lse) {
  std::lock_guard<std::mutex> lk(g_kv_m);
  Plan P;
  P.build(n, sq, sk, d, causal != 0);
  // set-up on the calling thread: library state, peer access, workspaces
  for (int s = 0; s < n; s++) {
    int rc = prepare_device_on(devs[s]);
    if (rc) return rc;
  }
  enable_peers(devs, n);
  for (int s = 0; s < n; s++) {
    cudaSetDevice(devs[s]);
    cudaError_t e = slot_ready(g_kv[s], devs[s], P.slot[s].total ? P.slot[s].total : 16);
    if (e != cudaSuccess) return status_cuda(e, "key-range split workspace");
  }
  std::vector<Result> res(n);
  auto fail = [&](int s, int rc) {
    res[s].rc = rc;
    res[s].msg = status_message();
  };
  // Phase 1 (per device, in parallel): inputs in, partials, peer copies out.
  Pool::get().run(n, [&](int s) {
    KvSlot& K = g_kv[s];
    const Plan::Slot& z = P.slot[s];
    const int dev = devs[s];
    int rc = prepare_device_on(dev);
    if (rc) return fail(s, rc);
    float* ws = K.ws;
    cudaError_t e = cudaSuccess;
    if (z.any) {
      // (pageable host memory goes through the device's pinned rings)
      e = staged_copy_h2d(dev, ws + z.q, q + z.qrow0 * d, (sq - z.qrow0) * d * sizeof(float), K.s);
      for (int c = 0; c < P.nch && e == cudaSuccess; c++) {
        const Plan::Chunk& x = P.ch[c];
        if (!x.used || x.slot != s) continue;
        const size_t nb = (x.k1 - x.k0) * d * sizeof(float);
        e = staged_copy_h2d(dev, ws + z.k + x.kv_off, k + x.k0 * d, nb, K.s);
        if (e == cudaSuccess) e = staged_copy_h2d(dev, ws + z.v + x.kv_off, v + x.k0 * d, nb, K.s);
      }
      if (e != cudaSuccess) return fail(s, status_cuda(e, "key-range split inputs"));
      for (int c = 0; c < P.nch; c++) {
        const Plan::Chunk& x = P.ch[c];
        if (!x.used || x.slot != s) continue;
        const size_t row0 = x.rfirst * P.rc;
        FwdParams p{};
        p.q = ws + z.q + (row0 - z.qrow0) * d;
        p.k = ws + z.k + x.kv_off;
        p.v = ws + z.v + x.kv_off;
        p.o = ws + x.po;
        p.lse = ws + x.pl;
        p.bh = 1;
        p.sq = (int)(sq - row0);
        p.sk = (int)(x.k1 - x.k0);
        p.d = (int)d;
        p.q_offset = (long long)row0;
        p.k_offset = (long long)x.k0;
        p.causal = causal ? 1 : 0;
        rc = dispatch_on(p, dev, K.s);
        if (rc) return fail(s, rc);
      }
      // every partial row block to its owner's receive slots
      for (int r = 0; r < P.nch && e == cudaSuccess; r++) {
        const Plan::Rows& y = P.rows[r];
        const size_t len = y.r1 - y.r0, np = y.parts.size();
        for (size_t i = 0; i < np && e == cudaSuccess; i++) {
          const Plan::Chunk& x = P.ch[y.parts[i]];
          if (x.slot != s) continue;
          const size_t off = y.r0 - x.rfirst * P.rc;  // row offset inside the partial
          float* dst = g_kv[y.owner].ws + y.recv;
          const int ddev = devs[y.owner];
          e = cudaMemcpyPeerAsync(dst + i * len * d, ddev, ws + x.po + off * d, dev,
                                  len * d * sizeof(float), K.s);
          if (e == cudaSuccess)
            e = cudaMemcpyPeerAsync(dst + up16(np * len * d) + i * len, ddev, ws + x.pl + off, dev,
                                    len * sizeof(float), K.s);
        }
      }
      if (e != cudaSuccess) return fail(s, status_cuda(e, "key-range split exchange"));
    }
    e = cudaEventRecord(K.sent, K.s);
    if (e != cudaSuccess) return fail(s, status_cuda(e, "key-range split event"));
  });
  int rc = first_error(res);
  if (rc != FA_OK) {
    for (int s = 0; s < n; s++) {
      cudaSetDevice(devs[s]);
      cudaStreamSynchronize(g_kv[s].s);
    }
    return rc;
  }
  // Phase 2 (per device, in parallel): wait for every device's copies, merge
  // the owned row chunks, copy them out, check the bounded-wait flag.
  Pool::get().run(n, [&](int s) {
    KvSlot& K = g_kv[s];
    const int dev = devs[s];
    int rc2 = prepare_device_on(dev);
    if (rc2) return fail(s, rc2);
    cudaError_t e = cudaSuccess;
    for (int t = 0; t < n && e == cudaSuccess; t++)
      if (t != s) e = cudaStreamWaitEvent(K.s, g_kv[t].sent, 0);
    for (int r = 0; r < P.nch && e == cudaSuccess; r++) {
      const Plan::Rows& y = P.rows[r];
      if (y.owner != s || y.r1 <= y.r0) continue;
      const size_t len = y.r1 - y.r0, np = y.parts.size();
      e = launch_combine(K.ws + y.recv, K.ws + y.recv + up16(np * len * d), (int)np,
                         (long long)len, (int)d, K.ws + y.out, K.ws + y.lse, K.s);
      if (e == cudaSuccess)
        e = staged_copy_d2h(dev, out + y.r0 * d, K.ws + y.out, len * d * sizeof(float), K.s);
      if (e == cudaSuccess && lse)
        e = staged_copy_d2h(dev, lse + y.r0, K.ws + y.lse, len * sizeof(float), K.s);
    }
    if (e != cudaSuccess) {
      cudaStreamSynchronize(K.s);
      return fail(s, status_cuda(e, "key-range split merge"));
    }
    rc2 = check_err_flag_on(dev, K.s);  // (synchronises the stream)
    if (rc2) return fail(s, rc2);
  });
  return first_error(res);
}

// A split pays when the slices cannot fill the devices and a slice is long.
bool use_kv_split(size_t bh, size_t sq, size_t sk, size_t d, int n) {
  return bh < (size_t)n && sq > 16 && sk >= (size_t)n * 2 * 1024 &&
         (double)sq * (double)sk * (double)d >= 8.0e9;
}

}  // namespace

int host_forward_devices(const int* devs, int n, const float* q, const float* k, const float* v,
                         size_t bh, size_t sq, size_t sk, size_t d, int causal, float* out,
                         float* lse) {
  if (n > kMaxSlots) n = kMaxSlots;
  if (use_kv_split(bh, sq, sk, d, n)) {
    for (size_t h = 0; h < bh; h++) {
      int rc = kv_split_slice(devs, n, q + h * sq * d, k + h * sk * d, v + h * sk * d, sq, sk, d,
                              causal, out + h * sq * d, lse ? lse + h * sq : nullptr);
      if (rc) return rc;
    }
    return FA_OK;
  }
  // Small calls stay on one device: the copies of a few MB do not gain from
  // more host links, and every device adds a fixed cost.
  const size_t bytes = 4 * bh * (2 * sq * d + 2 * sk * d);
  int use = bh < (size_t)n ? (int)bh : n;
  if (bytes < (size_t(8) << 20)) use = 1;
  if (use <= 1) return host_forward_on(devs[0], q, k, v, bh, sq, sk, d, causal, out, lse);
  return shard_slices(devs, use, q, k, v, bh, sq, sk, d, causal, out, lse);
}

void devices_release() {
  std::lock_guard<std::mutex> lk(g_kv_m);
  for (int s = 0; s < kMaxSlots; s++) slot_free(g_kv[s]);
}

}  // namespace fa
