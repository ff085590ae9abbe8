// Overflow/underflow-safe Euclidean / Frobenius norm (HBM-bound).
//
// Reference: norm_data (src/openpacho/_norm.py:39-118).  The NumPy branch
// (:44-52) divides by s = max|x| and returns s * sqrt(sum((x/s)^2)), with
// Inf passed through and NaN winning; the GPU branch keeps a (scale, ssq)
// pair per lane, merges pairs with one division per element (_merge, :28-36)
// and needs one launch per 4096x reduction of the partial count (:62-118).
//
// This design keeps the pair idea but makes every step exact and cheap:
//  * float32 input: squares are accumulated in float64.  Any float32 square
//    lies in [2^-298, 2^256], far inside float64's range, so no scaling is
//    needed at all and Inf/NaN propagate through the sum with the required
//    precedence (NaN + Inf = NaN).
//  * float64 input: the pair is (E, ssq) meaning sum(x^2) = ssq * 2^(2E) with
//    E an integer exponent clamped to [-1000, 1000].  Each thread rescales by
//    the power of two 2^-E (exact) once per batch of 8 elements, so there is
//    no division; non-finite inputs only set a class flag (1 Inf, 2 NaN).
//  * one launch: blocks that share a row publish pairs to scratch and the last
//    block to arrive merges them in a fixed order (deterministic).
#include <math.h>

#include <type_traits>

#include "pb_internal.cuh"

namespace pb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kEmin = -1000, kEmax = 1000;

__device__ __forceinline__ double pow2(int e) {  // 2^e for e in [-1022, 1023]
  return __hiloint2double((e + 1023) << 20, 0);
}

// Pair merge: a <- a (+) b.  Equal exponents (always the case for float32
// input, whose pairs all carry e = 0) need no rescaling.
__device__ __forceinline__ void merge(NormPair& a, const NormPair& b) {
  if (a.e == b.e) {
    a.ssq += b.ssq;
  } else {
    const int E = max(a.e, b.e);
    double s = 0.0;
    if (a.ssq != 0.0) s += ldexp(a.ssq, 2 * (a.e - E));
    if (b.ssq != 0.0) s += ldexp(b.ssq, 2 * (b.e - E));
    a.ssq = s;
    a.e = E;
  }
  a.cls = max(a.cls, b.cls);
}

__device__ __forceinline__ NormPair shfl_pair(const NormPair& p, int off) {
  NormPair q;
  q.ssq = __shfl_xor_sync(0xffffffffu, p.ssq, off);
  q.e = __shfl_xor_sync(0xffffffffu, p.e, off);
  q.cls = __shfl_xor_sync(0xffffffffu, p.cls, off);
  return q;
}

__device__ __forceinline__ NormPair warp_merge(NormPair p) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    NormPair q = shfl_pair(p, o);
    merge(p, q);
  }
  return p;
}

// ---- float32 accumulation: exact squares in float64 -------------------
struct AccF32 {
  double s[4];
  __device__ void init() { s[0] = s[1] = s[2] = s[3] = 0.0; }
  __device__ __forceinline__ void add4(float4 v, int u) {
    double a = v.x, b = v.y, c = v.z, d = v.w;
    s[u] = fma(a, a, s[u]);
    s[u] = fma(b, b, s[u]);
    s[u] = fma(c, c, s[u]);
    s[u] = fma(d, d, s[u]);
  }
  __device__ __forceinline__ void add1(float v) {
    double a = v;
    s[1] = fma(a, a, s[1]);
  }
  __device__ NormPair pair() const {
    NormPair p;
    p.ssq = (s[0] + s[1]) + (s[2] + s[3]);
    p.e = 0;
    p.cls = 0;
    return p;
  }
};

// ---- float64 accumulation: power-of-two scaled pair --------------------
struct AccF64 {
  double s[2];
  int E;
  int cls;
  __device__ void init() {
    s[0] = s[1] = 0.0;
    E = kEmin;
    cls = 0;
  }
  __device__ __forceinline__ static int bexp(double v) {
    return (__double2hiint(v) >> 20) & 0x7ff;
  }
  // Accumulate a batch of n values (n <= 8).
  template <int N>
  __device__ __forceinline__ void batch(double (&v)[N]) {
    int eb = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) eb = max(eb, bexp(v[i]));
    if (eb == 0x7ff) {  // a NaN or Inf in this batch: record its class, drop it
      eb = 0;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if (bexp(v[i]) == 0x7ff) {
          cls = max(cls, isnan(v[i]) ? 2 : 1);
          v[i] = 0.0;
        }
        eb = max(eb, bexp(v[i]));
      }
    }
    int e = min(max(eb - 1023, kEmin), kEmax);
    if (e > E) {
      int sh = 2 * (E - e);
      s[0] = ldexp(s[0], sh);
      s[1] = ldexp(s[1], sh);
      E = e;
    }
    const double S = pow2(-E);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      double y = v[i] * S;
      s[i & 1] = fma(y, y, s[i & 1]);
    }
  }
  __device__ __forceinline__ void add1(double x) {
    double v[1] = {x};
    batch<1>(v);
  }
  __device__ NormPair pair() const {
    NormPair p;
    p.ssq = s[0] + s[1];
    p.e = E;
    p.cls = cls;
    return p;
  }
};

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

// Partial pair of x[k0:k1] for one row group of `nthr` threads.  Offsets
// inside the chunk are 32-bit (chunks are < 2^31 elements) and pointers
// advance incrementally, keeping the streaming loop at few registers.
template <bool ALIGNED>
__device__ NormPair row_pair(const float* __restrict__ x, int64_t k0, int64_t k1, int tid,
                             int nthr) {
  AccF32 acc;
  acc.init();
  x += k0;
  const int len = (int)(k1 - k0);
  int body = 0;
  if (ALIGNED) {
    const int nv = len / 4;
    const float4* xv = reinterpret_cast<const float4*>(x) + tid;
    int v = tid;
    // Eight 16-byte loads in flight per thread (four left this kernel near
    // 0.91 of the copy bandwidth at four resident blocks per SM); element
    // 4*nthr*j + 4*tid + c still lands in lane j % 4, as in the four-load step.
#pragma unroll 1
    for (; v + 7 * nthr < nv; v += 8 * nthr, xv += 8 * nthr) {
      float4 r[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = ld_stream(xv + i * nthr);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc.add4(r[i], i & 3);
    }
    if (v + 3 * nthr < nv) {
      const float4 r0 = ld_stream(xv), r1 = ld_stream(xv + nthr), r2 = ld_stream(xv + 2 * nthr),
                   r3 = ld_stream(xv + 3 * nthr);
      acc.add4(r0, 0);
      acc.add4(r1, 1);
      acc.add4(r2, 2);
      acc.add4(r3, 3);
      v += 4 * nthr;
      xv += 4 * nthr;
    }
#pragma unroll 1
    for (; v < nv; v += nthr, xv += nthr) acc.add4(ld_stream(xv), 0);
    body = nv * 4;
  }
  for (int k = body + tid; k < len; k += nthr) acc.add1(__ldg(x + k));
  return acc.pair();
}

template <bool ALIGNED>
__device__ NormPair row_pair(const double* __restrict__ x, int64_t k0, int64_t k1, int tid,
                             int nthr) {
  AccF64 acc;
  acc.init();
  x += k0;
  const int len = (int)(k1 - k0);
  int body = 0;
  if (ALIGNED) {
    const int nv = len / 2;
    const double2* xv = reinterpret_cast<const double2*>(x) + tid;
    int v = tid;
#pragma unroll 1
    for (; v + 3 * nthr < nv; v += 4 * nthr, xv += 4 * nthr) {
      const double2 t0 = ld_stream(xv), t1 = ld_stream(xv + nthr), t2 = ld_stream(xv + 2 * nthr),
                    t3 = ld_stream(xv + 3 * nthr);
      double r[8] = {t0.x, t0.y, t1.x, t1.y, t2.x, t2.y, t3.x, t3.y};
      acc.batch<8>(r);
    }
#pragma unroll 1
    for (; v < nv; v += nthr, xv += nthr) {
      const double2 t = ld_stream(xv);
      double r[2] = {t.x, t.y};
      acc.batch<2>(r);
    }
    body = nv * 2;
  }
  for (int k = body + tid; k < len; k += nthr) acc.add1(__ldg(x + k));
  return acc.pair();
}

template <typename T>
__device__ __forceinline__ T finalize(const NormPair& p) {
  if (p.cls == 2) return T(NAN);
  if (p.cls == 1) return T(INFINITY);
  double r = sqrt(p.ssq);
  if (p.e != 0) r *= pow2(p.e);
  return T(r);
}

// Block-wide merge of one pair per thread group; result valid in thread 0 of
// each group of `G` warps (written to red[group]).
__device__ __forceinline__ void store_warp_pair(NormPair* red, NormPair p) {
  p = warp_merge(p);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = p;
}

// Rows of length K (inner == 1).  Same decomposition as the GEMV kernel.
// PAIR_OUT: write the merged pair of the single row instead of the norm
// (used by the multi-GPU combine): to pair_out, or, when push.nranks > 0,
// straight into every rank's mailbox over NVLink (the compute and the
// exchange of the sharded norm in one kernel).
template <typename T, bool ALIGNED, bool PAIR_OUT>
__global__ void __launch_bounds__(kThreads)
    norm_rows_kernel(const T* __restrict__ x, T* __restrict__ out, NormPair* __restrict__ pair_out,
                     int64_t rows, int64_t K, int rows_per_block, int64_t chunk, int nchunks,
                     NormPair* __restrict__ partial, unsigned int* __restrict__ counters,
                     const PushArgs push) {
  __shared__ NormPair red[kWarps];
  __shared__ bool last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = kWarps / rows_per_block;
  const int64_t group = blockIdx.x / nchunks;
  const int c = blockIdx.x % nchunks;
  const int64_t row = group * rows_per_block + warp / G;
  NormPair p;
  p.ssq = 0.0;
  p.e = (sizeof(T) == 8) ? kEmin : 0;
  p.cls = 0;
  if (row < rows) {
    const int64_t k0 = (int64_t)c * chunk;
    const int64_t k1 = min(K, k0 + chunk);
    p = row_pair<ALIGNED>(x + row * K, k0, k1, (warp % G) * 32 + lane, G * 32);
  }
  store_warp_pair(red, p);
  __syncthreads();
  if (nchunks == 1) {
    if (threadIdx.x < rows_per_block) {
      const int64_t r = group * rows_per_block + threadIdx.x;
      if (r < rows) {
        NormPair s = red[threadIdx.x * G];
        for (int w = 1; w < G; ++w) merge(s, red[threadIdx.x * G + w]);
        if (PAIR_OUT && push.nranks) push_slot(push, s.ssq, s.e, s.cls);
        else if (PAIR_OUT) pair_out[r] = s;
        else out[r] = finalize<T>(s);
      }
    }
    return;
  }
  if (threadIdx.x == 0) {
    NormPair s = red[0];
    for (int w = 1; w < kWarps; ++w) merge(s, red[w]);
    partial[row * nchunks + c] = s;
    __threadfence();
    unsigned int prev = atomicAdd(&counters[row], 1u);
    last = (prev == (unsigned int)(nchunks - 1));
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  NormPair s;
  s.ssq = 0.0;
  s.e = kEmin;
  s.cls = 0;
  for (int i = threadIdx.x; i < nchunks; i += kThreads) {
    NormPair q;
    const NormPair* src = partial + row * nchunks + i;
    q.ssq = __ldcg(&src->ssq);
    q.e = __ldcg(&src->e);
    q.cls = __ldcg(&src->cls);
    merge(s, q);
  }
  store_warp_pair(red, s);
  __syncthreads();
  if (threadIdx.x == 0) {
    NormPair t = red[0];
    for (int w = 1; w < kWarps; ++w) merge(t, red[w]);
    if (PAIR_OUT && push.nranks) push_slot(push, t.ssq, t.e, t.cls);
    else if (PAIR_OUT) pair_out[row] = t;
    else out[row] = finalize<T>(t);
    counters[row] = 0u;
  }
}

// Reduced axis in the middle: out[o, i] = norm(x[o, :, i]).  Thread per
// (o, i), coalesced along i; the reduced axis may be split into `nchunks`
// block-chunks merged by the last block per (o, i-tile).
template <typename T>
__global__ void __launch_bounds__(kThreads)
    norm_cols_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t outer, int64_t R,
                     int64_t inner, int64_t itiles, int64_t chunk, int nchunks,
                     NormPair* __restrict__ partial, unsigned int* __restrict__ counters) {
  __shared__ bool last;
  const int64_t tile = blockIdx.x / nchunks;  // (o, itile)
  const int c = blockIdx.x % nchunks;
  const int64_t o = tile / itiles;
  const int64_t i = (tile % itiles) * kThreads + threadIdx.x;
  const bool live = i < inner;
  using Acc = typename std::conditional<sizeof(T) == 4, AccF32, AccF64>::type;
  Acc acc;
  acc.init();
  if (live) {
    const int64_t r0 = (int64_t)c * chunk, r1 = min(R, r0 + chunk);
    const T* base = x + o * R * inner + i;
    for (int64_t r = r0; r < r1; ++r) acc.add1(__ldg(base + r * inner));
  }
  NormPair p = acc.pair();
  if (nchunks == 1) {
    if (live) out[o * inner + i] = finalize<T>(p);
    return;
  }
  const int64_t slot = o * inner + i;
  if (live) partial[slot * nchunks + c] = p;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int prev = atomicAdd(&counters[tile], 1u);
    last = (prev == (unsigned int)(nchunks - 1));
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (live) {
    NormPair s;
    s.ssq = 0.0;
    s.e = kEmin;
    s.cls = 0;
    for (int j = 0; j < nchunks; ++j) {
      NormPair q;
      const NormPair* src = partial + slot * nchunks + j;
      q.ssq = __ldcg(&src->ssq);
      q.e = __ldcg(&src->e);
      q.cls = __ldcg(&src->cls);
      merge(s, q);
    }
    out[slot] = finalize<T>(s);
  }
  if (threadIdx.x == 0) counters[tile] = 0u;
}

struct Strided {
  int on, rn;
  int64_t oshape[8], ostride[8], rshape[8], rstride[8];
};

// General axis sets: one block per output element.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    norm_strided_kernel(const T* __restrict__ x, T* __restrict__ out, Strided s, int64_t R) {
  __shared__ NormPair red[kWarps];
  int64_t o = blockIdx.x, base = 0;
  for (int d = s.on - 1; d >= 0; --d) {
    base += (o % s.oshape[d]) * s.ostride[d];
    o /= s.oshape[d];
  }
  using Acc = typename std::conditional<sizeof(T) == 4, AccF32, AccF64>::type;
  Acc acc;
  acc.init();
  for (int64_t r = threadIdx.x; r < R; r += kThreads) {
    int64_t rr = r, off = base;
    for (int d = s.rn - 1; d >= 0; --d) {
      off += (rr % s.rshape[d]) * s.rstride[d];
      rr /= s.rshape[d];
    }
    acc.add1(__ldg(x + off));
  }
  store_warp_pair(red, acc.pair());
  __syncthreads();
  if (threadIdx.x == 0) {
    NormPair t = red[0];
    for (int w = 1; w < kWarps; ++w) merge(t, red[w]);
    out[blockIdx.x] = finalize<T>(t);
  }
}

// Merge `n` pairs in index order (rank order for the multi-GPU combine, so
// every rank computes the identical result) and write the norm.
template <typename T>
__global__ void norm_pairs_finalize_kernel(const NormPair* __restrict__ p, int n,
                                           T* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    NormPair s = p[0];
    for (int i = 1; i < n; ++i) merge(s, p[i]);
    *out = finalize<T>(s);
  }
}

__global__ void norm_pair_zero_kernel(NormPair* __restrict__ p, int e0) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    p->ssq = 0.0;
    p->e = e0;
    p->cls = 0;
  }
}

struct Plan {
  int rows_per_block;
  int nchunks;
  int64_t chunk;
  int64_t blocks;
};

// `resident`: blocks of the row kernel that fit at once (one wave).
Plan plan_rows(int64_t rows, int64_t K, int64_t elem, int64_t resident) {
  Plan p;
  if (rows >= 2 * resident || K * elem <= 16384) {
    // Whole rows per block: a warp per row up to 32 KiB rows (warp-only
    // reduction), more warps per row beyond that.
    p.nchunks = 1;
    p.chunk = K;
    const int64_t bytes = K * elem;
    int G = bytes > (128 << 10) ? 8 : bytes > (64 << 10) ? 4 : bytes > (32 << 10) ? 2 : 1;
    p.rows_per_block = kWarps / G;
  } else {
    p.rows_per_block = 1;
    int64_t want = ceil_div(resident, rows);  // one wave of equal block-chunks
    int64_t most = ceil_div(K, 2048);
    int64_t n = want < most ? want : most;
    if (n < 1) n = 1;
    p.chunk = ceil_div(ceil_div(K, n), 64) * 64;
    p.nchunks = (int)ceil_div(K, p.chunk);
  }
  p.blocks = ceil_div(rows, p.rows_per_block) * p.nchunks;
  return p;
}

template <typename T, bool PAIR_OUT>
int launch_rows(Device* d, const T* x, T* out, NormPair* pair_out, int64_t rows, int64_t K,
                const PushArgs& push = PushArgs{}) {
  Plan p = plan_rows(rows, K, sizeof(T),
                     resident_blocks(d, (const void*)norm_rows_kernel<T, true, PAIR_OUT>, kThreads));
  if (p.blocks > INT32_MAX) PB_FAIL(PB_ERR_UNSUPPORTED, "norm grid too large");
  NormPair* partial = nullptr;
  unsigned int* cnt = nullptr;
  if (p.nchunks > 1) {
    void* s;
    PB_CHECK(scratch(d, (size_t)rows * p.nchunks * sizeof(NormPair), &s));
    partial = (NormPair*)s;
    PB_CHECK(counters(d, (size_t)rows, &cnt));
  }
  constexpr int VN = 16 / sizeof(T);
  bool aligned = ((uintptr_t)x % 16 == 0) && (rows == 1 || K % VN == 0) && (p.chunk % VN == 0);
  PB_CHECK(kt_begin(d));
  if (aligned)
    norm_rows_kernel<T, true, PAIR_OUT><<<(unsigned)p.blocks, kThreads, 0, d->stream>>>(
        x, out, pair_out, rows, K, p.rows_per_block, p.chunk, p.nchunks, partial, cnt, push);
  else
    norm_rows_kernel<T, false, PAIR_OUT><<<(unsigned)p.blocks, kThreads, 0, d->stream>>>(
        x, out, pair_out, rows, K, p.rows_per_block, p.chunk, p.nchunks, partial, cnt, push);
  PB_LAUNCHED(d);
  return kt_end(d);
}

template <typename T>
int launch_cols(Device* d, const T* x, T* out, int64_t outer, int64_t R, int64_t inner) {
  const int64_t itiles = ceil_div(inner, kThreads);
  const int64_t tiles = outer * itiles;
  const int64_t resident = (int64_t)d->sm_count * (2048 / kThreads);
  int64_t n = 1;
  if (tiles < 2 * resident) {
    n = ceil_div(2 * resident, tiles);
    int64_t most = ceil_div(R, 64);
    if (n > most) n = most;
    if (n < 1) n = 1;
  }
  const int64_t chunk = ceil_div(R, n);
  const int nchunks = (int)ceil_div(R, chunk);
  if (tiles * nchunks > INT32_MAX) PB_FAIL(PB_ERR_UNSUPPORTED, "norm grid too large");
  NormPair* partial = nullptr;
  unsigned int* cnt = nullptr;
  if (nchunks > 1) {
    void* s;
    PB_CHECK(scratch(d, (size_t)outer * inner * nchunks * sizeof(NormPair), &s));
    partial = (NormPair*)s;
    PB_CHECK(counters(d, (size_t)tiles, &cnt));
  }
  PB_CHECK(kt_begin(d));
  norm_cols_kernel<T><<<(unsigned)(tiles * nchunks), kThreads, 0, d->stream>>>(
      x, out, outer, R, inner, itiles, chunk, nchunks, partial, cnt);
  PB_LAUNCHED(d);
  return kt_end(d);
}

}  // namespace

int norm_pair_global(Device* d, int dtype, int64_t n, const void* x, void* pair_out,
                     const PushArgs* push) {
  const PushArgs none{};
  const PushArgs& p = push ? *push : none;
  if (dtype == PB_F32)
    return launch_rows<float, true>(d, (const float*)x, nullptr, (NormPair*)pair_out, 1, n, p);
  if (dtype == PB_F64)
    return launch_rows<double, true>(d, (const double*)x, nullptr, (NormPair*)pair_out, 1, n, p);
  PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
}

// Merge the pairs of every rank from this rank's mailbox, in rank order, and
// write the norm: one thread, each wait bounded (the context's limit, 10 s by
// default) with the kernel error flag set when it runs out.
template <typename T>
__global__ void mailbox_norm_kernel(const MailSlot* box, int nranks, int parity,
                                    unsigned long long seq, T* out, int* err,
                                    unsigned long long wait_ns) {
  if (threadIdx.x != 0) return;
  NormPair s;
  for (int r = 0; r < nranks; ++r) {
    const MailSlot* slot = box + r * 2 + parity;
    if (!mailbox_wait(slot, seq, err, wait_ns)) return;
    NormPair q;
    q.ssq = *(volatile const double*)&slot->a;
    q.e = *(volatile const int*)&slot->e;
    q.cls = *(volatile const int*)&slot->cls;
    if (r == 0) s = q;
    else merge(s, q);
  }
  *out = finalize<T>(s);
}

__global__ void push_empty_kernel(const PushArgs a, int e0) {
  if (threadIdx.x == 0) push_slot(a, 0.0, e0, 0);
}

// The neutral pair of an empty slice, pushed to every rank.
int norm_push_empty(Device* d, int dtype, const PushArgs& a) {
  push_empty_kernel<<<1, 32, 0, d->stream>>>(a, dtype == PB_F64 ? kEmin : 0);
  PB_LAUNCHED(d);
  return PB_OK;
}

int mailbox_norm(Device* d, int dtype, int parity, unsigned long long seq, void* out) {
  if (dtype == PB_F32)
    mailbox_norm_kernel<float><<<1, 32, 0, d->stream>>>(d->box[d->box_rank], d->box_ranks, parity,
                                                        seq, (float*)out, d->err_dev, d->box_wait_ns);
  else
    mailbox_norm_kernel<double><<<1, 32, 0, d->stream>>>(d->box[d->box_rank], d->box_ranks, parity,
                                                         seq, (double*)out, d->err_dev, d->box_wait_ns);
  PB_LAUNCHED(d);
  return PB_OK;
}

int norm_pairs_finalize(Device* d, int dtype, const void* pairs, int n, void* out) {
  if (dtype == PB_F32)
    norm_pairs_finalize_kernel<float><<<1, 32, 0, d->stream>>>((const NormPair*)pairs, n, (float*)out);
  else
    norm_pairs_finalize_kernel<double><<<1, 32, 0, d->stream>>>((const NormPair*)pairs, n,
                                                                (double*)out);
  PB_LAUNCHED(d);
  return PB_OK;
}

int norm_pair_zero(Device* d, int dtype, void* pair) {
  norm_pair_zero_kernel<<<1, 32, 0, d->stream>>>((NormPair*)pair, dtype == PB_F64 ? kEmin : 0);
  PB_LAUNCHED(d);
  return PB_OK;
}

int fill_device(Device* d, int dtype, void* dst, size_t count, double value);

}  // namespace pb

using namespace pb;

extern "C" {

int pb_norm(pb_ctx* ctx, int dev, int dtype, int64_t outer, int64_t reduced, int64_t inner,
            const void* x, void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (outer < 0 || reduced < 0 || inner < 0) PB_FAIL(PB_ERR_INVALID, "negative norm extent");
  if (dtype != PB_F32 && dtype != PB_F64) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  const int64_t count = outer * inner;
  if (!count) return PB_OK;
  if (!out) PB_FAIL(PB_ERR_INVALID, "null output");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  // _norm.py:42-43: an empty reduction gives 0.
  if (!reduced) return fill_device(d, dtype, out, (size_t)count, 0.0);
  if (!x) PB_FAIL(PB_ERR_INVALID, "null input");
  if (inner == 1) {
    if (dtype == PB_F32)
      return launch_rows<float, false>(d, (const float*)x, (float*)out, nullptr, outer, reduced);
    return launch_rows<double, false>(d, (const double*)x, (double*)out, nullptr, outer, reduced);
  }
  if (dtype == PB_F32)
    return launch_cols<float>(d, (const float*)x, (float*)out, outer, reduced, inner);
  return launch_cols<double>(d, (const double*)x, (double*)out, outer, reduced, inner);
}

int pb_norm_strided(pb_ctx* ctx, int dev, int dtype, int out_ndim, const int64_t* out_shape,
                    const int64_t* out_strides, int red_ndim, const int64_t* red_shape,
                    const int64_t* red_strides, const void* x, void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (dtype != PB_F32 && dtype != PB_F64) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  if (out_ndim < 0 || out_ndim > 8 || red_ndim < 0 || red_ndim > 8)
    PB_FAIL(PB_ERR_UNSUPPORTED, "norm supports at most 8 output and 8 reduced dims");
  Strided s;
  s.on = out_ndim;
  s.rn = red_ndim;
  int64_t count = 1, R = 1;
  for (int i = 0; i < out_ndim; ++i) {
    if (out_shape[i] < 0) PB_FAIL(PB_ERR_INVALID, "negative extent");
    s.oshape[i] = out_shape[i];
    s.ostride[i] = out_strides[i];
    count *= out_shape[i];
  }
  for (int i = 0; i < red_ndim; ++i) {
    if (red_shape[i] < 0) PB_FAIL(PB_ERR_INVALID, "negative extent");
    s.rshape[i] = red_shape[i];
    s.rstride[i] = red_strides[i];
    R *= red_shape[i];
  }
  if (!count) return PB_OK;
  if (!out) PB_FAIL(PB_ERR_INVALID, "null output");
  if (count > INT32_MAX) PB_FAIL(PB_ERR_UNSUPPORTED, "too many outputs for strided norm");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!R) return fill_device(d, dtype, out, (size_t)count, 0.0);
  if (!x) PB_FAIL(PB_ERR_INVALID, "null input");
  PB_CHECK(kt_begin(d));
  if (dtype == PB_F32)
    norm_strided_kernel<float><<<(unsigned)count, kThreads, 0, d->stream>>>((const float*)x,
                                                                            (float*)out, s, R);
  else
    norm_strided_kernel<double><<<(unsigned)count, kThreads, 0, d->stream>>>(
        (const double*)x, (double*)out, s, R);
  PB_LAUNCHED(d);
  return kt_end(d);
}

}  // extern "C"
