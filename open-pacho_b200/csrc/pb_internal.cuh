// Internal declarations shared by the libpacho_b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda.h>
#include <stdint.h>
#include <stdio.h>
#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <utility>
#include <string>
#include <vector>

#include "../../include/pacho_b200.h"

namespace pb {

// ---------------------------------------------------------------- errors --

void set_error(const char* fmt, ...);

#define PB_FAIL(code, ...)        \
  do {                            \
    ::pb::set_error(__VA_ARGS__); \
    return (code);                \
  } while (0)

#define PB_CUDA(call)                                                                  \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess) {                                                           \
      ::pb::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                      __LINE__);                                                       \
      return e_ == cudaErrorMemoryAllocation ? PB_ERR_OOM : PB_ERR_CUDA;               \
    }                                                                                  \
  } while (0)

#define PB_CHECK(expr)     \
  do {                     \
    int s_ = (expr);       \
    if (s_ != PB_OK) return s_; \
  } while (0)

// Launch-error check after a kernel launch; counts the launch.
#define PB_LAUNCHED(st)                                                                   \
  do {                                                                                    \
    cudaError_t e_ = cudaGetLastError();                                                  \
    if (e_ != cudaSuccess) {                                                              \
      ::pb::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(e_), __FILE__, \
                      __LINE__);                                                          \
      return PB_ERR_CUDA;                                                                 \
    }                                                                                     \
    (st)->launches.fetch_add(1, std::memory_order_relaxed);                               \
  } while (0)

// Kernel-side error codes written to the device error word.
enum : int {
  KERR_NONE = 0,
  KERR_WAIT_TIMEOUT = 1,  // a bounded mbarrier wait gave up
  KERR_BAD_ARGUMENT = 2,
};

// --------------------------------------------------------------- context --

struct Device {
  int ordinal = -1;
  cudaStream_t stream = nullptr;
  // Copy streams of pb_gemm_host (host -> device, device -> host) and the
  // events that order its chunks; created on first use.
  cudaStream_t up = nullptr, down = nullptr;
  std::vector<cudaEvent_t> host_events;
  cudaMemPool_t pool = nullptr;
  int sm_count = 0;
  // Scratch memory for multi-block reductions and GEMM operand splits.  Grown
  // on demand, stream-ordered, so consecutive operations may reuse it.
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  // Zero-initialised arrival counters for "last block finishes" reductions.
  // Every kernel that uses them leaves them at zero again.
  unsigned int* counters = nullptr;
  size_t counters_n = 0;
  // Operand tags of the 3xTF32 GEMM: a word per row of A / column group of B
  // holding the generation of the last launch that found a tiny value there.
  // Generations only grow, so the tags never need clearing.
  unsigned int* tags = nullptr;
  size_t tags_n = 0;
  unsigned int tag_gen = 0;
  // Kernel error word in mapped, pinned host memory (no copy needed to read it).
  int* err_host = nullptr;
  int* err_dev = nullptr;
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  // Marks this stream's position for another device's stream to wait on
  // (pb_copy_peer, pb_stream_wait); no timing.
  cudaEvent_t order_ev = nullptr;
  std::atomic<uint64_t> launches{0};
  // Per-kernel timer (pb_ktimer_*): event pairs around main kernels while on
  // (1), or on with the pairs kept across reads (2: events inside a graph).
  int kt_on = 0;
  size_t kt_used = 0;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> kt_events;
  // Device address of the fixed DOT scratch of pb_dot_noalloc, looked up when
  // the context is created (with the device current).
  void* dot_static = nullptr;
  // NCCL communicator (ncclComm_t) when joined.
  void* comm = nullptr;
  int nranks = 1, rank = 0;
  // Peer mailboxes (pb_peer_export/import): every rank's slot array mapped
  // into this device's address space (own first allocated here), the call
  // sequence number of the next exchange.
  struct MailSlot* box[8] = {};
  int box_ranks = 0, box_rank = 0;
  unsigned long long box_seq = 0;
  unsigned long long box_wait_ns = 10ull * 1000 * 1000 * 1000;  // mailbox wait limit
  // A stream capture (pb_capture_begin) is in progress: nothing may allocate.
  int capturing = 0;
  // Instantiated graphs not yet destroyed.  While any lives, a buffer that
  // grows is retired (kept) instead of freed: a graph may still use it.
  int graphs_live = 0;
  std::vector<void*> retired;
};

}  // namespace pb

struct pb_ctx {
  int ndev = 0;
  pb::Device* devs = nullptr;
  std::recursive_mutex mu;
};

namespace pb {

// pb_gemm / pb_gemm_ex with an explicit kernel choice (pb_gemm.cu).
int gemm_dispatch(pb_ctx* ctx, int dev, int dtype, int batch_ndim, const int64_t* batch_shape,
                  const int64_t* a_bstride, const int64_t* b_bstride, int64_t M, int64_t N,
                  int64_t K, const void* A, const void* B, void* C, int algo);

// Validates (ctx, dev), makes the device current and returns its state.
int enter(pb_ctx* ctx, int dev, Device** out);
// Reads and clears the device's kernel error word (after a synchronisation):
// PB_ERR_DEVICE with the kernel's reason if a kernel raised it.
int check_kernel_error(Device* d);
// Ensure at least `bytes` of scratch; returns the pointer.
int scratch(Device* d, size_t bytes, void** out);
// Ensure at least `n` zeroed counters; returns the pointer.
int counters(Device* d, size_t n, unsigned int** out);
// Raise `kernel`'s dynamic shared-memory limit to `bytes` on d's device, once
// per (kernel, device): the attribute is per device, so a context over
// several devices sets it on each.  The device must be current (enter()).
inline int allow_smem(Device* d, const void* kernel, size_t bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> g(mu);
  const auto key = std::make_pair(kernel, d->ordinal);
  if (done.count(key)) return PB_OK;
  PB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  done.insert(key);
  return PB_OK;
}
// Blocks of `threads` threads of `kernel` resident on d's device at once (one
// wave), from the occupancy API, cached per (kernel, device).  Grids sized to
// it avoid a partial second wave.
inline int64_t resident_blocks(Device* d, const void* kernel, int threads) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int64_t> known;
  std::lock_guard<std::mutex> g(mu);
  const auto key = std::make_pair(kernel, d->ordinal);
  auto it = known.find(key);
  if (it != known.end()) return it->second;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t n = (int64_t)per_sm * d->sm_count;
  known[key] = n;
  return n;
}
// Per-kernel timer: bracket the main kernel of an entry point (no-ops while
// the timer is off).  kt_begin records the start event, kt_end the end event.
int kt_begin(Device* d);
int kt_end(Device* d);
// Resolve the fixed DOT scratch of pb_dot_noalloc on d's device and load the
// kernels it launches (pb_blas1.cu); called by pb_init with the device current.
int dot_static_prepare(Device* d);
// Fill `count` elements of dtype PB_F32 / PB_F64 / PB_BOOL with `value`.
int fill_device(Device* d, int dtype, void* dst, size_t count, double value);
// Ensure at least `n` operand tag words; returns them and a fresh generation.
int operand_tags(Device* d, size_t n, unsigned int** out, unsigned int* gen);
// Driver entry point for cuTensorMapEncodeTiled (resolved once).
int tensor_map_encoder(void** fn);

// Entry points implemented per translation unit, all on an entered device.
// push: write the pair into every rank's mailbox instead of pair_out.
int norm_pair_global(Device* d, int dtype, int64_t n, const void* x, void* pair_out,
                     const struct PushArgs* push = nullptr);
// Unmap the peers' mailboxes and free this one (pb_peer.cu).
int peer_close(Device* d);
// Stream wait bounded in time that also watches the NCCL communicator.
int comm_stream_wait(Device* d);

// ---- peer mailboxes: NVLink exchange of one small result per rank --------
//
// Rank r's mailbox holds two 32-byte slots per writer rank (one per parity of
// the call sequence number): slot [w * 2 + seq % 2] is written only by rank w,
// over NVLink, with the payload first and the sequence number last (release,
// system scope); the owner reads the sequence number with acquire loads.  Two
// parities suffice: rank w can start call s+2 only after its own call s+1,
// whose merge needed every rank's value of s+1, which each rank pushes only
// after its merge of call s (stream order).
constexpr int kMaxRanks = 8;
struct MailSlot {
  double a;                // norm: ssq; DOT: partial sum
  int e, cls;              // norm: scale exponent and class
  double unused;
  unsigned long long seq;  // call sequence number, stored last
};
static_assert(sizeof(MailSlot) == 32, "mailbox slot size");

struct PushArgs {
  MailSlot* box[kMaxRanks];  // every rank's mailbox, own included
  int nranks, rank, parity;
  unsigned long long seq;
};

// Wait (one thread) until `slot` carries sequence number `seq`; false, with
// the kernel error flag set, after `limit_ns` (the context's limit, 10 s
// unless pb_peer_set_wait changed it).  The acquire load orders the payload
// reads after it.
constexpr unsigned long long kMailboxWaitNs = 10ull * 1000 * 1000 * 1000;
__device__ __forceinline__ bool mailbox_wait(const MailSlot* slot, unsigned long long seq, int* err,
                                             unsigned long long limit_ns) {
  unsigned long long t0, t, v;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(&slot->seq) : "memory");
    if (v == seq) return true;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > limit_ns) {
      atomicExch(err, KERR_WAIT_TIMEOUT);
      return false;
    }
    __nanosleep(256);
  }
}

// Push this rank's value into every mailbox (one thread).
__device__ __forceinline__ void push_slot(const PushArgs& a, double value, int e, int cls) {
  for (int r = 0; r < a.nranks; ++r) {
    MailSlot* s = a.box[r] + (a.rank * 2 + a.parity);
    s->a = value;
    s->e = e;
    s->cls = cls;
  }
  __threadfence_system();
  for (int r = 0; r < a.nranks; ++r) {
    unsigned long long* q = &(a.box[r] + (a.rank * 2 + a.parity))->seq;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(q), "l"(a.seq) : "memory");
  }
}

// Batch-offset table (up to 8 broadcast dims), passed by value to kernels.
// ---------------------------------------- division by launch constants --
//
// Quotients by a divisor fixed for a launch (batch extents, tile counts, the
// K split) as a multiply-high and a shift instead of a 64-bit division
// routine, which costs a single-thread pipeline stage (the TMA producer
// between two tiles) about a microsecond per tile.  Granlund and Montgomery,
// "Division by invariant integers using multiplication" (PLDI 1994), section
// 4: with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// floor(n / d) = (mulhi(m, n) + n) >> l for every 32-bit n for which the sum
// does not overflow, so for all n < 2^31 when 1 <= d <= 2^31.  Other operands
// take the plain division.
struct FastDiv {
  int64_t d;
  uint32_t m, s;
  uint32_t lim;  // operands below lim take the multiply (0: none do)
};

inline FastDiv make_fastdiv(int64_t d) {
  FastDiv f{d, 0u, 0u, 0u};
  if (d < 1 || d > (int64_t(1) << 31)) return f;
  uint32_t l = 0;
  while ((int64_t(1) << l) < d) ++l;
  f.m = (uint32_t)((((uint64_t(1) << l) - (uint64_t)d) << 32) / (uint64_t)d + 1);
  f.s = l;
  f.lim = 0x80000000u;
  return f;
}

__host__ __device__ __forceinline__ uint32_t mulhi32(uint32_t a, uint32_t b) {
#ifdef __CUDA_ARCH__
  return __umulhi(a, b);
#else
  return (uint32_t)(((uint64_t)a * b) >> 32);
#endif
}

__host__ __device__ __forceinline__ int64_t fdiv(int64_t n, const FastDiv& f) {
  if ((uint64_t)n < f.lim) {
    const uint32_t x = (uint32_t)n;
    return (int64_t)((mulhi32(x, f.m) + x) >> f.s);
  }
  return n / f.d;
}

struct BatchMap {
  int ndim;
  int64_t shape[8];
  int64_t a_stride[8];
  int64_t b_stride[8];
  FastDiv div[8];  // make_fastdiv(shape[i])
};

__host__ __device__ inline void batch_offsets(const BatchMap& m, int64_t b, int64_t* ao,
                                              int64_t* bo) {
  int64_t a = 0, c = 0;
  for (int i = m.ndim - 1; i >= 0; --i) {
    const int64_t q = fdiv(b, m.div[i]);
    const int64_t idx = b - q * m.shape[i];
    b = q;
    a += idx * m.a_stride[i];
    c += idx * m.b_stride[i];
  }
  *ao = a;
  *bo = c;
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ------------------------------------------- non-finite GEMM outputs --
//
// The 3xTF32 split gives a non-finite value x the parts hi = x, lo = 0, so a
// cross term lo * (+-Inf) is 0 * Inf = NaN where IEEE arithmetic (and the
// reference's float32 GEMM) yields +-Inf; a magnitude within 2^-12 of
// FLT_MAX can also round its hi part up to Inf.  Every such output is
// non-finite, so the tcgen05 epilogues mark the kNonFiniteTile-square tile
// of each non-finite output in a zeroed counter array laid out as
//   nf[0]      any tile marked
//   nf[1]      arrival counter of the repair kernel
//   nf[2 + t]  tile t = (batch * tiles_m + m / kNonFiniteTile) * tiles_n + n / kNonFiniteTile
// and a repair launch recomputes the marked tiles with float32 FMA from the
// original operands, then returns every word to zero.
constexpr int kNonFiniteTile = 128;

__device__ __forceinline__ void mark_nonfinite(unsigned int* nf, int64_t bz, int64_t row,
                                               int64_t col, int64_t tiles_m, int64_t tiles_n) {
  nf[2 + (bz * tiles_m + row / kNonFiniteTile) * tiles_n + col / kNonFiniteTile] = 1u;
  nf[0] = 1u;
}

// Launched right after the kernels that mark (programmatic dependent launch:
// it waits for them on the device); returns at once when nothing is marked.
int gemm_nonfinite_repair_f32(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N,
                              int64_t K, const float* A, const float* B, float* C,
                              unsigned int* nf);

// ------------------------------------------------------- device helpers --

// Merge-friendly (scale exponent, sum of squares, class) triple for the
// scaled norm: value^2 = ssq * 2^(2*e); cls 0 finite, 1 saw +-Inf, 2 saw NaN.
struct NormPair {
  double ssq;
  int e;
  int cls;
};

}  // namespace pb
