// GEMV, DOT and fill kernels of libpacho_b200 (HBM-bound).
//
// Reference behaviour: matvec_data (src/openpacho/_cuda_gemv.py:47-95) flattens
// every leading dimension of A into independent rows and computes y = A @ x;
// DOT is the one-row case.  The reference launches one 128-thread block per row
// (or per 1024-term DOT chunk) with scalar strided loads and a shared-memory
// tree, then a second reduction launch (_cuda_gemv.py:67-84).
//
// This design: 256-thread blocks, 128-bit non-caching loads of the streamed
// operand (A, or both DOT vectors), the reused vector x through the read-only
// L1 path, a warp-shuffle tree, and -- when a row is split across blocks to
// fill 148 SMs -- per-block partials in scratch merged by the last block to
// arrive (one launch, fixed merge order, hence deterministic results).
#include "pb_internal.cuh"

namespace pb {
namespace {

// Plan parameters (compile-time so variants can be built and measured):
// PB_GEMV_WAVES  -- block-chunks of a split row = WAVES x resident blocks;
// PB_GEMV_ROW_KB -- row bytes one warp streams before more warps share a row;
// PB_GEMV_PERSIST -- whole-row grids capped at PERSIST x resident blocks.
#ifndef PB_GEMV_WAVES
#define PB_GEMV_WAVES 1
#endif
#ifndef PB_GEMV_ROW_KB
#define PB_GEMV_ROW_KB 8
#endif
#ifndef PB_GEMV_PERSIST
#define PB_GEMV_PERSIST 1
#endif
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <typename T> struct V16;
template <> struct V16<float> { using type = float4; static constexpr int n = 4; };
template <> struct V16<double> { using type = double2; static constexpr int n = 2; };

// Streaming 16-byte load that does not allocate in L1 (the matrix is read once).
__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ double2 ld_stream(const double2* p) {
  double2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.f64 {%0,%1}, [%2];"
               : "=d"(v.x), "=d"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float dotv(float4 a, float4 b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}
__device__ __forceinline__ double dotv(double2 a, double2 b, double acc) {
  acc = fma(a.x, b.x, acc);
  return fma(a.y, b.y, acc);
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum of A[row, k0:k1] * x[k0:k1] by the `nthr` threads of one row group.
// STREAM_X: x is itself streamed once (DOT) instead of reused (GEMV).
// Offsets inside the chunk are 32-bit (chunks are < 2^31 elements) and the
// pointers advance incrementally, which keeps the loop at few registers.
template <typename T, bool ALIGNED, bool STREAM_X>
__device__ __forceinline__ T row_partial(const T* __restrict__ a, const T* __restrict__ x,
                                         int64_t k0, int64_t k1, int tid, int nthr) {
  using V = typename V16<T>::type;
  constexpr int VN = V16<T>::n;
  T acc0 = T(0), acc1 = T(0), acc2 = T(0), acc3 = T(0);
  a += k0;
  x += k0;
  const int len = (int)(k1 - k0);
  int body = 0;
  if (ALIGNED) {
    // k0 is a multiple of VN and the row start is 16-byte aligned.
    const int nv = len / VN;
    const V* av = reinterpret_cast<const V*>(a) + tid;
    const V* xv = reinterpret_cast<const V*>(x) + tid;
    int v = tid;
#pragma unroll 1
    for (; v + 3 * nthr < nv; v += 4 * nthr, av += 4 * nthr, xv += 4 * nthr) {
      const V r0 = ld_stream(av), r1 = ld_stream(av + nthr), r2 = ld_stream(av + 2 * nthr),
              r3 = ld_stream(av + 3 * nthr);
      V x0, x1, x2, x3;
      if (STREAM_X) {
        x0 = ld_stream(xv); x1 = ld_stream(xv + nthr); x2 = ld_stream(xv + 2 * nthr);
        x3 = ld_stream(xv + 3 * nthr);
      } else {
        x0 = __ldg(xv); x1 = __ldg(xv + nthr); x2 = __ldg(xv + 2 * nthr); x3 = __ldg(xv + 3 * nthr);
      }
      acc0 = dotv(r0, x0, acc0);
      acc1 = dotv(r1, x1, acc1);
      acc2 = dotv(r2, x2, acc2);
      acc3 = dotv(r3, x3, acc3);
    }
#pragma unroll 1
    for (; v < nv; v += nthr, av += nthr, xv += nthr)
      acc0 = dotv(ld_stream(av), STREAM_X ? ld_stream(xv) : __ldg(xv), acc0);
    body = nv * VN;
  }
  for (int k = body + tid; k < len; k += nthr) acc1 = fma(__ldg(a + k), __ldg(x + k), acc1);
  return (acc0 + acc1) + (acc2 + acc3);
}

// Block = kWarps warps; G = kWarps / rows_per_block warps per row.  Block b
// covers row group b / nchunks and K-chunk b % nchunks.
template <typename T, bool ALIGNED, bool STREAM_X>
__global__ void __launch_bounds__(kThreads)
    gemv_kernel(const T* __restrict__ A, const T* __restrict__ x, T* __restrict__ y,
                int64_t rows, int64_t K, int64_t lda, int rows_per_block, int64_t chunk,
                int nchunks, T* __restrict__ partial, unsigned int* __restrict__ counters,
                const T* __restrict__ resid) {
  __shared__ T red[kWarps];
  __shared__ bool last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = kWarps / rows_per_block;
  const int64_t group = blockIdx.x / nchunks;
  const int c = blockIdx.x % nchunks;
  const int sub = warp / G;
  const int64_t row = group * rows_per_block + sub;
  const int tid = (warp % G) * 32 + lane;
  T v = T(0);
  if (row < rows) {
    const int64_t k0 = (int64_t)c * chunk;
    const int64_t k1 = min(K, k0 + chunk);
    v = row_partial<T, ALIGNED, STREAM_X>(A + row * lda, x, k0, k1, tid, G * 32);
  }
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (nchunks == 1) {
    if (threadIdx.x < rows_per_block) {
      const int64_t r = group * rows_per_block + threadIdx.x;
      if (r < rows) {
        T s = T(0);
        for (int w = 0; w < G; ++w) s += red[threadIdx.x * G + w];
        y[r] = resid ? resid[r] - s : s;
      }
    }
    return;
  }
  // Split row (rows_per_block == 1): publish this chunk's partial, and let the
  // last block to arrive merge all of them in chunk order.
  if (threadIdx.x == 0) {
    T s = T(0);
    for (int w = 0; w < kWarps; ++w) s += red[w];
    partial[row * nchunks + c] = s;
    __threadfence();
    unsigned int prev = atomicAdd(&counters[row], 1u);
    last = (prev == (unsigned int)(nchunks - 1));
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  T s = T(0);
  for (int i = threadIdx.x; i < nchunks; i += kThreads) s += __ldcg(partial + row * nchunks + i);
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    T t = T(0);
    for (int w = 0; w < kWarps; ++w) t += red[w];
    y[row] = resid ? resid[row] - t : t;
    counters[row] = 0u;  // leave the counter ready for the next launch
  }
}

// Whole rows (no split): G = kWarps / rows_per_block warps per row; blocks
// stride over row groups, so with the grid capped at the resident block count
// the imbalance at the end is one group in many instead of a partial last
// wave.  In-row offsets are 32-bit (the launcher guarantees K < 2^31).
template <typename T, bool ALIGNED>
__global__ void __launch_bounds__(kThreads, 4)
    gemv_rows_kernel(const T* __restrict__ A, const T* __restrict__ x, T* __restrict__ y,
                     int64_t rows, int K, int rows_per_block, const T* __restrict__ resid) {
  using V = typename V16<T>::type;
  constexpr int VN = V16<T>::n;
  __shared__ T red[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = kWarps / rows_per_block;
  const int sub = warp / G;
  const int tid = (warp % G) * 32 + lane;
  const int nthr = G * 32;
  const int64_t groups = (rows + rows_per_block - 1) / rows_per_block;
#pragma unroll 1
  for (int64_t group = blockIdx.x; group < groups; group += gridDim.x) {
    const int64_t row = group * rows_per_block + sub;
    T acc0 = T(0), acc1 = T(0), acc2 = T(0), acc3 = T(0);
    if (row < rows) {
      const T* a = A + row * (int64_t)K;
      int body = 0;
      if (ALIGNED) {
        const int nv = K / VN;
        const V* av = reinterpret_cast<const V*>(a) + tid;
        const V* xv = reinterpret_cast<const V*>(x) + tid;
        int v = tid;
#pragma unroll 1
        for (; v + 3 * nthr < nv; v += 4 * nthr, av += 4 * nthr, xv += 4 * nthr) {
          const V r0 = ld_stream(av), r1 = ld_stream(av + nthr), r2 = ld_stream(av + 2 * nthr),
                  r3 = ld_stream(av + 3 * nthr);
          const V x0 = __ldg(xv), x1 = __ldg(xv + nthr), x2 = __ldg(xv + 2 * nthr),
                  x3 = __ldg(xv + 3 * nthr);
          acc0 = dotv(r0, x0, acc0);
          acc1 = dotv(r1, x1, acc1);
          acc2 = dotv(r2, x2, acc2);
          acc3 = dotv(r3, x3, acc3);
        }
#pragma unroll 1
        for (; v < nv; v += nthr, av += nthr, xv += nthr) acc0 = dotv(ld_stream(av), __ldg(xv), acc0);
        body = nv * VN;
      }
      for (int k = body + tid; k < K; k += nthr) acc1 = fma(__ldg(a + k), __ldg(x + k), acc1);
    }
    const T v = warp_sum((acc0 + acc1) + (acc2 + acc3));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x < rows_per_block) {
      const int64_t r = group * rows_per_block + threadIdx.x;
      if (r < rows) {
        T s = T(0);
        for (int w = 0; w < G; ++w) s += red[threadIdx.x * G + w];
        y[r] = resid ? resid[r] - s : s;
      }
    }
    __syncthreads();
  }
}

template <typename T>
__global__ void fill_kernel(T* __restrict__ out, size_t n, T value) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = value;
}

struct GemvPlan {
  int rows_per_block;
  int nchunks;
  int64_t chunk;
  int64_t blocks;
};

// `resident`: blocks of the split kernel that fit at once (one wave).
GemvPlan plan_gemv(int64_t rows, int64_t K, int64_t elem, int64_t resident) {
  GemvPlan p;
  if (rows >= 2 * resident || K * elem <= 16384) {
    // Whole rows per block: one warp per row up to 32 KiB rows (warp-only
    // reduction), more warps per row beyond that.
    p.nchunks = 1;
    p.chunk = K;
    const int64_t bytes = K * elem;
    constexpr int64_t R = (int64_t)PB_GEMV_ROW_KB << 10;
    int G = bytes > 4 * R ? 8 : bytes > 2 * R ? 4 : bytes > R ? 2 : 1;
    p.rows_per_block = kWarps / G;
  } else {
    p.rows_per_block = 1;
    // Equal block-chunks, PB_GEMV_WAVES waves of resident blocks.
    int64_t want = ceil_div(PB_GEMV_WAVES * resident, rows);
    int64_t most = ceil_div(K, 2048);
    int64_t n = want < most ? want : most;
    if (n < 1) n = 1;
    p.chunk = ceil_div(ceil_div(K, n), 64) * 64;
    p.nchunks = (int)ceil_div(K, p.chunk);
  }
  p.blocks = ceil_div(rows, p.rows_per_block) * p.nchunks;
  return p;
}

// Grid of the whole-row kernel: persistent (capped at PB_GEMV_PERSIST waves
// of its resident blocks).
int64_t rows_grid(const GemvPlan& p, int64_t resident) {
  const int64_t cap = (int64_t)PB_GEMV_PERSIST * resident;
  return p.blocks < cap ? p.blocks : cap;
}

// resid: nullptr for y = A x; else the residual epilogue y = resid - A x, with
// A x rounded to T before the subtraction (one rounding each, as the eager
// product followed by an elementwise subtract).
template <typename T, bool STREAM_X>
int launch_gemv(Device* d, const T* A, const T* x, T* y, int64_t rows, int64_t K, int64_t lda,
                const T* resid = nullptr) {
  GemvPlan p = plan_gemv(rows, K, sizeof(T),
                         resident_blocks(d, (const void*)gemv_kernel<T, true, STREAM_X>, kThreads));
  if (p.blocks > INT32_MAX) PB_FAIL(PB_ERR_UNSUPPORTED, "GEMV grid too large");
  T* partial = nullptr;
  unsigned int* cnt = nullptr;
  if (p.nchunks > 1) {
    void* s;
    PB_CHECK(scratch(d, (size_t)rows * p.nchunks * sizeof(T), &s));
    partial = (T*)s;
    PB_CHECK(counters(d, (size_t)rows, &cnt));
  }
  constexpr int VN = V16<T>::n;
  bool aligned = ((uintptr_t)A % 16 == 0) && ((uintptr_t)x % 16 == 0) &&
                 (rows == 1 || lda % VN == 0) && (p.chunk % VN == 0);
  if (p.nchunks == 1 && !STREAM_X && lda == K && K < INT32_MAX) {
    const unsigned grid =
        (unsigned)rows_grid(p, resident_blocks(d, (const void*)gemv_rows_kernel<T, true>, kThreads));
    PB_CHECK(kt_begin(d));
    if (aligned)
      gemv_rows_kernel<T, true><<<grid, kThreads, 0, d->stream>>>(A, x, y, rows, (int)K,
                                                                   p.rows_per_block, resid);
    else
      gemv_rows_kernel<T, false><<<grid, kThreads, 0, d->stream>>>(A, x, y, rows, (int)K,
                                                                    p.rows_per_block, resid);
    PB_LAUNCHED(d);
    return kt_end(d);
  }
  PB_CHECK(kt_begin(d));
  if (aligned)
    gemv_kernel<T, true, STREAM_X><<<(unsigned)p.blocks, kThreads, 0, d->stream>>>(
        A, x, y, rows, K, lda, p.rows_per_block, p.chunk, p.nchunks, partial, cnt, resid);
  else
    gemv_kernel<T, false, STREAM_X><<<(unsigned)p.blocks, kThreads, 0, d->stream>>>(
        A, x, y, rows, K, lda, p.rows_per_block, p.chunk, p.nchunks, partial, cnt, resid);
  PB_LAUNCHED(d);
  return kt_end(d);
}

// ---- DOT for callers that cannot allocate ------------------------------
// pb_dot_noalloc runs the same DOT kernel as pb_dot, but its per-block partial
// sums and arrival counter live in this fixed file-scope device array instead
// of the context's scratch, so the call never allocates.  The array is part of
// the library image: every GPU that loads the library holds it (33 KiB) until
// the process exits.
constexpr int kStaticDotPartials = 4096;
constexpr size_t kStaticDotCounterOffset = kStaticDotPartials * sizeof(double);
static __device__ __align__(256) unsigned char g_dot_scratch[kStaticDotCounterOffset + 256];

// In host code `g_dot_scratch` is only a host-side stand-in for the device
// array.  pb_init calls dot_static_prepare with each device current: it looks
// the array's device address up for that device (kept in the context) and
// loads the DOT kernels and their occupancy figures, so that with lazy module
// loading no pb_dot_noalloc call is the one that loads code or data onto the
// device.
template <typename T>
static int prepare_dot_kernels(Device* d) {
  cudaFuncAttributes attr;
  PB_CUDA(cudaFuncGetAttributes(&attr, gemv_kernel<T, true, true>));
  PB_CUDA(cudaFuncGetAttributes(&attr, gemv_kernel<T, false, true>));
  resident_blocks(d, (const void*)gemv_kernel<T, true, true>, kThreads);
  return PB_OK;
}


template <typename T>
int launch_dot_static(Device* d, const T* x, const T* y, T* out, int64_t n) {
  GemvPlan p = plan_gemv(1, n, sizeof(T),
                         resident_blocks(d, (const void*)gemv_kernel<T, true, true>, kThreads));
  if (p.nchunks > kStaticDotPartials)
    PB_FAIL(PB_ERR_UNSUPPORTED,
            "pb_dot_noalloc: this DOT needs %d partial sums but the static scratch holds %d",
            p.nchunks, kStaticDotPartials);
  T* partial = nullptr;
  unsigned int* cnt = nullptr;
  if (p.nchunks > 1) {
    void* base = d->dot_static;
    if (!base) PB_FAIL(PB_ERR_UNAVAILABLE, "static DOT scratch not resolved for this device");
    partial = (T*)base;
    cnt = (unsigned int*)((char*)base + kStaticDotCounterOffset);
    // The array keeps whatever the previous call left; the arrival counter must
    // start at zero.  (A memset of existing memory allocates nothing.)
    PB_CUDA(cudaMemsetAsync(cnt, 0, sizeof(unsigned int), d->stream));
  }
  constexpr int VN = V16<T>::n;
  const bool aligned =
      ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) && (p.chunk % VN == 0);
  if (aligned)
    gemv_kernel<T, true, true><<<(unsigned)p.blocks, kThreads, 0, d->stream>>>(
        x, y, out, 1, n, n, p.rows_per_block, p.chunk, p.nchunks, partial, cnt, nullptr);
  else
    gemv_kernel<T, false, true><<<(unsigned)p.blocks, kThreads, 0, d->stream>>>(
        x, y, out, 1, n, n, p.rows_per_block, p.chunk, p.nchunks, partial, cnt, nullptr);
  PB_LAUNCHED(d);
  return PB_OK;
}

template <typename T>
int launch_fill(Device* d, T* out, size_t n, T value) {
  if (!n) return PB_OK;
  size_t blocks = (n + 255) / 256;
  size_t cap = (size_t)d->sm_count * 32;
  if (blocks > cap) blocks = cap;
  fill_kernel<T><<<(unsigned)blocks, 256, 0, d->stream>>>(out, n, value);
  PB_LAUNCHED(d);
  return PB_OK;
}

}  // namespace

int dot_static_prepare(Device* d) {
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_dot_scratch);
  if (e != cudaSuccess || !ptr)
    PB_FAIL(PB_ERR_CUDA, "cudaGetSymbolAddress(static DOT scratch) failed: %s",
            cudaGetErrorString(e));
  d->dot_static = ptr;
  PB_CHECK(prepare_dot_kernels<float>(d));
  PB_CHECK(prepare_dot_kernels<double>(d));
  return PB_OK;
}

// DOT into device memory (the local partial of the sharded DOT).
int dot_device(Device* d, int dtype, int64_t n, const void* x, const void* y, void* out) {
  if (!n) return fill_device(d, dtype, out, 1, 0.0);
  if (!x || !y) PB_FAIL(PB_ERR_INVALID, "null input");
  if (dtype == PB_F32)
    return launch_gemv<float, true>(d, (const float*)x, (const float*)y, (float*)out, 1, n, n);
  return launch_gemv<double, true>(d, (const double*)x, (const double*)y, (double*)out, 1, n, n);
}

int fill_device(Device* d, int dtype, void* dst, size_t count, double value) {
  if (dtype == PB_F32) return launch_fill<float>(d, (float*)dst, count, (float)value);
  if (dtype == PB_F64) return launch_fill<double>(d, (double*)dst, count, value);
  if (dtype == PB_BOOL)
    return launch_fill<unsigned char>(d, (unsigned char*)dst, count, value != 0.0 ? 1 : 0);
  PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
}

}  // namespace pb

using namespace pb;

extern "C" {

int pb_fill(pb_ctx* ctx, int dev, int dtype, void* dst, size_t count, double value) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (!count) return PB_OK;
  if (!dst) PB_FAIL(PB_ERR_INVALID, "null destination");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  return fill_device(d, dtype, dst, count, value);
}

int pb_gemv(pb_ctx* ctx, int dev, int dtype, int64_t rows, int64_t K, const void* A,
            const void* x, void* y) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (rows < 0 || K < 0) PB_FAIL(PB_ERR_INVALID, "negative GEMV extent");
  if (!rows) return PB_OK;
  if (!y) PB_FAIL(PB_ERR_INVALID, "null output");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!K) return fill_device(d, dtype, y, (size_t)rows, 0.0);
  if (!A || !x) PB_FAIL(PB_ERR_INVALID, "null input");
  if (dtype == PB_F32)
    return launch_gemv<float, false>(d, (const float*)A, (const float*)x, (float*)y, rows, K, K);
  if (dtype == PB_F64)
    return launch_gemv<double, false>(d, (const double*)A, (const double*)x, (double*)y, rows, K,
                                      K);
  PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
}

int pb_gemv_residual(pb_ctx* ctx, int dev, int dtype, int64_t rows, int64_t K, const void* A,
                     const void* x, const void* b, void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (rows < 0 || K < 0) PB_FAIL(PB_ERR_INVALID, "negative GEMV extent");
  if (!rows) return PB_OK;
  if (!out || !b) PB_FAIL(PB_ERR_INVALID, "null residual operand or output");
  if (dtype != PB_F32 && dtype != PB_F64) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  const size_t bytes = (size_t)rows * (dtype == PB_F32 ? 4 : 8);
  // K == 0: A x is zero, so the result is b - 0 = b (the reference casts b).
  if (!K) {
    if (out != b) PB_CUDA(cudaMemcpyAsync(out, b, bytes, cudaMemcpyDeviceToDevice, d->stream));
    return PB_OK;
  }
  if (!A || !x) PB_FAIL(PB_ERR_INVALID, "null input");
  if (dtype == PB_F32)
    return launch_gemv<float, false>(d, (const float*)A, (const float*)x, (float*)out, rows, K, K,
                                     (const float*)b);
  return launch_gemv<double, false>(d, (const double*)A, (const double*)x, (double*)out, rows, K,
                                    K, (const double*)b);
}

int pb_dot(pb_ctx* ctx, int dev, int dtype, int64_t n, const void* x, const void* y, void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (n < 0) PB_FAIL(PB_ERR_INVALID, "negative DOT length");
  if (!out) PB_FAIL(PB_ERR_INVALID, "null output");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!n) return fill_device(d, dtype, out, 1, 0.0);
  if (!x || !y) PB_FAIL(PB_ERR_INVALID, "null input");
  if (dtype == PB_F32)
    return launch_gemv<float, true>(d, (const float*)x, (const float*)y, (float*)out, 1, n, n);
  if (dtype == PB_F64)
    return launch_gemv<double, true>(d, (const double*)x, (const double*)y, (double*)out, 1, n,
                                     n);
  PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
}

int pb_dot_noalloc(pb_ctx* ctx, int dev, int dtype, int64_t n, const void* x, const void* y,
                   void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (n < 0) PB_FAIL(PB_ERR_INVALID, "negative DOT length");
  if (!out) PB_FAIL(PB_ERR_INVALID, "null output");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!n) return fill_device(d, dtype, out, 1, 0.0);
  if (!x || !y) PB_FAIL(PB_ERR_INVALID, "null input");
  if (dtype == PB_F32)
    return launch_dot_static<float>(d, (const float*)x, (const float*)y, (float*)out, n);
  if (dtype == PB_F64)
    return launch_dot_static<double>(d, (const double*)x, (const double*)y, (double*)out, n);
  PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
}

}  // extern "C"
