// Internal declarations shared by the libpacho_b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda.h>
#include <stdint.h>
#include <stdio.h>
#include <atomic>
#include <mutex>
#include <string>

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
  // Kernel error word in mapped, pinned host memory (no copy needed to read it).
  int* err_host = nullptr;
  int* err_dev = nullptr;
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  std::atomic<uint64_t> launches{0};
  // NCCL communicator (ncclComm_t) when joined.
  void* comm = nullptr;
  int nranks = 1, rank = 0;
};

}  // namespace pb

struct pb_ctx {
  int ndev = 0;
  pb::Device* devs = nullptr;
  std::recursive_mutex mu;
};

namespace pb {

// Validates (ctx, dev), makes the device current and returns its state.
int enter(pb_ctx* ctx, int dev, Device** out);
// Ensure at least `bytes` of scratch; returns the pointer.
int scratch(Device* d, size_t bytes, void** out);
// Ensure at least `n` zeroed counters; returns the pointer.
int counters(Device* d, size_t n, unsigned int** out);
// Driver entry point for cuTensorMapEncodeTiled (resolved once).
int tensor_map_encoder(void** fn);

// Entry points implemented per translation unit, all on an entered device.
int norm_pair_global(Device* d, int dtype, int64_t n, const void* x, void* pair_out);
// Stream wait bounded in time that also watches the NCCL communicator.
int comm_stream_wait(Device* d);

// Batch-offset table (up to 8 broadcast dims), passed by value to kernels.
struct BatchMap {
  int ndim;
  int64_t shape[8];
  int64_t a_stride[8];
  int64_t b_stride[8];
};

__host__ __device__ inline void batch_offsets(const BatchMap& m, int64_t b, int64_t* ao,
                                              int64_t* bo) {
  int64_t a = 0, c = 0;
  for (int i = m.ndim - 1; i >= 0; --i) {
    int64_t idx = b % m.shape[i];
    b /= m.shape[i];
    a += idx * m.a_stride[i];
    c += idx * m.b_stride[i];
  }
  *ao = a;
  *bo = c;
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ------------------------------------------------------- device helpers --

// Merge-friendly (scale exponent, sum of squares, class) triple for the
// scaled norm: value^2 = ssq * 2^(2*e); cls 0 finite, 1 saw +-Inf, 2 saw NaN.
struct NormPair {
  double ssq;
  int e;
  int cls;
};

}  // namespace pb
