// Shared definitions of the B200 attention-forward kernels.
#pragma once
#include <cuda_runtime.h>
#include <mutex>
#include <stdint.h>

namespace fa {

// One forward launch over `bh` independent (batch, head) slices.
// Q/OUT slice stride = sq*d elements, K/V slice stride = sk*d, LSE stride = sq.
// Causal masking compares global positions: query row i sits at q_offset + i,
// key j at k_offset + j; key visible iff k_offset + j <= q_offset + i.
struct FwdParams {
  const float* q;
  const float* k;
  const float* v;
  float* o;    // normalised output, [bh, sq, d]
  float* lse;  // nullable, [bh, sq], natural log of the scaled-score row sums
  int bh, sq, sk, d;
  long long q_offset, k_offset;
  int causal;
  float scale;       // 1/sqrt(d), computed in f32 as the crate does (v2.rs:171)
  float scale_log2;  // scale * log2(e): scores go straight into exp2
  int* err;          // device error word (0 = ok), see ErrCode
  // Limit of the tensor-core kernels' abortable waits (kWaitLimitNs unless a
  // test shortens it), and the test hook: with test_skip >= 0, one softmax
  // warp of the first CTA (pair) does not announce P of key block test_skip,
  // so the MMA issuer's wait for it runs out and the abort path is taken.
  unsigned long long wait_ns;
  int test_skip;
};

// Backward pass (fa_bwd.cu): gradients of the forward above.
struct BwdParams {
  const float* q;
  const float* k;
  const float* v;
  const float* o;     // forward output
  const float* lse;   // forward row LSE (natural log, scaled scores)
  const float* dout;  // gradient of the output
  float* dq;
  float* dk;
  float* dv;
  float* dvec;        // workspace [bh, sq]: rowsum(dO * O)
  int bh, sq, sk, d;
  long long q_offset, k_offset;
  int causal;
  float scale;
  int* err;                    // device error word (the tensor-core kernels' bounded waits)
  unsigned long long wait_ns;  // limit of those waits
  int test_skip;               // test hook, as FwdParams::test_skip (P of query block test_skip)
};

enum ErrCode : int {
  kErrNone = 0,
  kErrTimeout = 1,  // a bounded mbarrier wait expired
};

// Upper bound on any single in-kernel wait.  No legitimate wait in these
// kernels lasts more than a few milliseconds.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch: kernels launched with launch_pdl may start
// while the previous kernel on the stream is finishing.  Each such kernel does
// its set-up (barrier init, tensor-memory allocation) and then calls
// grid_dep_wait() before it touches global memory, which waits until the
// previous grid has completed and its writes are visible.  grid_dep_launch()
// lets the next kernel be scheduled early (it still waits in grid_dep_wait).
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Visible-key count for query global position qg against keys starting at
// global position kg0 with n keys: keys [kg0, kg0+n) ∩ (-inf, qg].
__host__ __device__ __forceinline__ int causal_limit(long long qg, long long kg0, int n) {
  long long lim = qg - kg0 + 1;
  return lim < 0 ? 0 : (lim > n ? n : (int)lim);
}

// Launch with the programmatic-stream-serialization attribute (see
// grid_dep_wait): the kernel must call grid_dep_wait() before it reads or
// writes global memory that earlier work on the stream produces or uses.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace fa

// Launchers implemented in the .cu files; return cudaError_t of the launch.
namespace fa {
cudaError_t launch_simt(const FwdParams& p, cudaStream_t s);
// Split-KV decode family: partial buffers are caller-provided scratch of
// `splits * bh * sq * (d + 1)` floats (ignored when splits == 1).
int decode_pick_splits(int bh, int sq, int sk, int num_sms, int d);
cudaError_t launch_decode(const FwdParams& p, int splits, float* scratch, cudaStream_t s);
cudaError_t launch_combine(const float* o_parts, const float* lse_parts, int n_parts,
                           long long rows, int d, float* out, float* lse_out,
                           cudaStream_t s);
bool decode_supported(int d);
// Fixed device array used by the allocation-free decode entry point.
size_t static_scratch_floats();
cudaError_t static_scratch_ptr(float** out);
// tcgen05 family.  tc_supported() says whether a tensor-core kernel exists for d.
bool tc_supported(int d, int precision);
cudaError_t launch_tc(const FwdParams& p, int precision, float* scratch,
                      size_t scratch_floats, cudaStream_t s);
// Workspace (floats) for the key-range split of small launches; 0 = no split.
size_t tc_scratch_floats(const FwdParams& p, int num_sms);
// 3xTF32 family (d = 64, 128): workspace of tc3_workspace_floats() floats
// (hi/lo planes of K and V, then the key-range partials of small launches).
size_t tc3_workspace_floats(const FwdParams& p, int num_sms);
cudaError_t launch_tc3(const FwdParams& p, float* ws, int num_sms, cudaStream_t s);
// Schedule model of the persistent CTA-pair kernels (fa_tc.cu): the longest
// per-cluster work in key blocks of `bk` keys, and the cost of merging
// n_split partials per row (microseconds).
double pair_schedule_makespan(const FwdParams& p, int n_split, int clusters, int bk,
                              double tile_cost);
double merge_cost_us(const FwdParams& p, int n_split);
unsigned long long launches_issued();
void count_launch(int n = 1);

// Host staging for host-slice calls with pageable buffers (fa_host_stage.cu).
// A ring of pinned slots: a slot is reused after its event (recorded after the
// copy that reads or writes it) has completed.
struct PinnedRing {
  static constexpr int kSlots = 4;
  static constexpr size_t kSlotBytes = size_t(16) << 20;
  char* buf[kSlots] = {};
  cudaEvent_t ev[kSlots] = {};
  bool busy[kSlots] = {};
  int next = 0;
};
// memcpy split over a fixed pool of host threads (single-threaded below 1 MB).
void parallel_copy(void* dst, const void* src, size_t bytes);
// true for memory the copy engines cannot read directly (not pinned or registered)
bool is_pageable(const void* p);
// Locks the device's staging rings (allocated on first use) for one call; the
// caller unlocks *call when done.
size_t bwd_workspace_floats(const BwdParams& p);
// Enqueues the three backward kernels (d_head <= 128); `dvec` is workspace of
// bwd_workspace_floats(p) floats.
cudaError_t launch_bwd(BwdParams p, float* dvec, cudaStream_t s);
// Tensor-core backward, TF32 (fa_bwd_tc.cu): d in {32, 64, 96, 128}, 16-byte
// aligned buffers; `ws` is workspace of tc_bwd_workspace_floats(p) floats.
bool tc_bwd_supported(int d);
size_t tc_bwd_workspace_floats(const BwdParams& p);
cudaError_t launch_tc_bwd(const BwdParams& p, float* ws, cudaStream_t s);
cudaError_t staging_acquire(int dev, PinnedRing** in, PinnedRing** out, std::mutex** call);
// One copy between host memory and device `dev` (current), enqueued on `s`.
// Pageable host memory goes through the device's pinned rings with the copy
// pool; page-locked memory is copied directly.  staged_copy_h2d returns once
// every piece is handed to the copy engine (the source may then be reused);
// staged_copy_d2h returns once `dst` holds the data.
cudaError_t staged_copy_h2d(int dev, void* dst, const void* src, size_t bytes, cudaStream_t s);
cudaError_t staged_copy_d2h(int dev, void* dst, const void* src, size_t bytes, cudaStream_t s);
void staging_release_all();
}  // namespace fa
