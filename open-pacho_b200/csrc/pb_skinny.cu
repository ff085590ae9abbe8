// Skinny products: C[b] = A[a(b)] @ B[b(b)] with M <= 8 rows, which covers
// vector @ matrix (M = 1, the a.ndim == 1 case of the matmul contract) and
// its batched, shared-vector form.
//
// Reference: CUDABackend.matmul sends these to cuBLAS ?gemv with
// Operation.N per batch entry (src/openpacho/_cuda_blas.py:43-61) or, for an
// unbatched vector @ matrix, to a GEMM with m = 1 (src/openpacho/_cuda.py:
// 496-498, 527-551).  Both read B once; so does this kernel.
//
// The work is one pass over B (HBM bound): lanes run along N with 16-byte
// loads, each holding MR x V accumulators (V = 4 floats or 2 doubles); the
// block's TY thread groups take interleaved rows of its K range; blocks split
// K further so the grid is one wave (SMs x resident blocks).  Partials are
// combined in a fixed order: over the groups in shared memory, then over the
// K ranges by the block that finishes a column strip last (an arrival
// counter), so the result is deterministic and one launch does everything.
#include "pb_internal.cuh"

namespace pb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxRows = 8;

template <typename T> struct Vec16;
template <> struct Vec16<float> { using type = float4; static constexpr int n = 4; };
template <> struct Vec16<double> { using type = double2; static constexpr int n = 2; };

template <typename T>
struct SkinnyParams {
  const T* A;       // batch of M x K
  const T* B;       // batch of K x N
  T* C;             // batch x M x N
  T* partial;       // ksplit x batch x M x N (ksplit > 1)
  unsigned int* arrivals;  // batch x strips, zero on entry and on exit
  int64_t M, N, K;
  int64_t batch;
  int64_t strips;   // column strips of tx * V columns
  int64_t kchunk;   // K range per split
  int ksplit;
  int tx, ty;       // lanes along N, thread groups along K (tx * ty = kThreads)
  BatchMap map;
};

// Rows of A staged per pass, transposed to [k][MR] in shared memory.
constexpr int kStageK = 512;

// Four resident blocks (64 registers) for up to two rows, two above that.
template <typename T, int MR, bool ALIGNED>
__global__ void __launch_bounds__(kThreads, MR <= 2 ? 4 : 2) skinny_kernel(const SkinnyParams<T> p) {
  constexpr int V = Vec16<T>::n;
  using VT = typename Vec16<T>::type;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* red = reinterpret_cast<T*>(smem_raw);        // [ty][MR][tx * V]
  T* as = red + (size_t)kThreads * MR * V;        // [kStageK][MR]
  __shared__ bool last;
  const int lx = threadIdx.x % p.tx, ly = threadIdx.x / p.tx;
  const int width = p.tx * V;                // columns per strip
  const int64_t strip = blockIdx.x, split = blockIdx.y;
  const int64_t n0 = strip * width + (int64_t)lx * V;
  const int64_t k0 = split * p.kchunk, k1 = min(p.K, k0 + p.kchunk);

  for (int64_t bz = blockIdx.z; bz < p.batch; bz += gridDim.z) {
    int64_t ao, bo;
    batch_offsets(p.map, bz, &ao, &bo);
    const T* A = p.A + ao * p.M * p.K;
    const T* B = p.B + bo * p.K * p.N;
    T acc[MR][V];
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < V; ++j) acc[m][j] = T(0);

    auto step = [&](int64_t k, int kl) {
      T b[V];
      if (ALIGNED) {
        if (n0 < p.N) {
          const VT q = __ldg(reinterpret_cast<const VT*>(B + k * p.N + n0));
          const T* qs = reinterpret_cast<const T*>(&q);
#pragma unroll
          for (int j = 0; j < V; ++j) b[j] = qs[j];
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j) b[j] = T(0);
        }
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) b[j] = n0 + j < p.N ? __ldg(B + k * p.N + n0 + j) : T(0);
      }
      const T* a = as + kl * MR;  // the same address across the group: a broadcast
#pragma unroll
      for (int m = 0; m < MR; ++m)
#pragma unroll
        for (int j = 0; j < V; ++j) acc[m][j] = fma(a[m], b[j], acc[m][j]);
    };
    for (int64_t kc = k0; kc < k1; kc += kStageK) {
      const int kn = (int)min((int64_t)kStageK, k1 - kc);
      __syncthreads();  // the previous pass is done with `as`
      for (int i = threadIdx.x; i < kStageK * MR; i += kThreads) {
        const int m = i / kStageK, kl = i % kStageK;  // coalesced along k
        as[kl * MR + m] = (m < p.M && kl < kn) ? __ldg(A + m * p.K + kc + kl) : T(0);
      }
      __syncthreads();
      // Interleaved rows; four in flight per thread.
      int kl = ly;
      for (; kl + 3 * p.ty < kn; kl += 4 * p.ty) {
        step(kc + kl, kl);
        step(kc + kl + p.ty, kl + p.ty);
        step(kc + kl + 2 * p.ty, kl + 2 * p.ty);
        step(kc + kl + 3 * p.ty, kl + 3 * p.ty);
      }
      for (; kl < kn; kl += p.ty) step(kc + kl, kl);
    }

    // Sum the thread groups in order.
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < V; ++j) red[((int64_t)ly * MR + m) * width + lx * V + j] = acc[m][j];
    __syncthreads();
    const int outs = MR * width;
    for (int o = threadIdx.x; o < outs; o += kThreads) {
      T s = red[o];
      for (int g = 1; g < p.ty; ++g) s += red[(int64_t)g * outs + o];
      red[o] = s;
    }
    __syncthreads();

    const int64_t col0 = strip * width;
    if (p.ksplit == 1) {
      for (int o = threadIdx.x; o < outs; o += kThreads) {
        const int m = o / width, c = o % width;
        if (m < p.M && col0 + c < p.N) p.C[(bz * p.M + m) * p.N + col0 + c] = red[o];
      }
    } else {
      const int64_t plane = p.batch * p.M * p.N;
      for (int o = threadIdx.x; o < outs; o += kThreads) {
        const int m = o / width, c = o % width;
        if (m < p.M && col0 + c < p.N)
          p.partial[split * plane + (bz * p.M + m) * p.N + col0 + c] = red[o];
      }
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        unsigned int* count = p.arrivals + bz * p.strips + strip;
        last = atomicAdd(count, 1u) == (unsigned int)(p.ksplit - 1);
        if (last) *count = 0u;
      }
      __syncthreads();
      if (last) {
        __threadfence();
        for (int o = threadIdx.x; o < outs; o += kThreads) {
          const int m = o / width, c = o % width;
          if (m >= p.M || col0 + c >= p.N) continue;
          const T* src = p.partial + (bz * p.M + m) * p.N + col0 + c;
          T s = __ldcg(src);
#pragma unroll 4
          for (int sp = 1; sp < p.ksplit; ++sp) s += __ldcg(src + sp * plane);
          p.C[(bz * p.M + m) * p.N + col0 + c] = s;
        }
      }
    }
    __syncthreads();  // red and `last` are reused by the next batch entry
  }
}

template <typename T, int MR>
int launch_rows(Device* d, SkinnyParams<T>& p, bool aligned) {
  constexpr int V = Vec16<T>::n;
  const size_t smem = ((size_t)kThreads * V + kStageK) * MR * sizeof(T);
  auto kernel = aligned ? skinny_kernel<T, MR, true> : skinny_kernel<T, MR, false>;
  PB_CHECK(allow_smem(d, (const void*)kernel, smem));
  const unsigned gz = (unsigned)(p.batch < 65535 ? p.batch : 65535);
  PB_CHECK(kt_begin(d));
  kernel<<<dim3((unsigned)p.strips, (unsigned)p.ksplit, gz), kThreads, smem, d->stream>>>(p);
  PB_LAUNCHED(d);
  return kt_end(d);
}

template <typename T>
int skinny(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
           const T* A, const T* B, T* C) {
  constexpr int V = Vec16<T>::n;
  SkinnyParams<T> p;
  p.A = A;
  p.B = B;
  p.C = C;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = batch;
  p.map = map;
  // Lanes along N: enough for the row (at least a warp), the rest along K.
  const int64_t lanes = ceil_div(N, (int64_t)V);
  int tx = 32;
  while (tx < kThreads && tx < lanes) tx *= 2;
  p.tx = tx;
  p.ty = kThreads / tx;
  p.strips = ceil_div(N, (int64_t)tx * V);
  if (p.strips > INT32_MAX) PB_FAIL(PB_ERR_UNSUPPORTED, "skinny product too wide");
  // Split K so that the grid stays within one wave of resident blocks, with
  // at least 64 rows per thread group (the final merge reads every split).
  const int64_t base = p.strips * batch;
  const int64_t want = (int64_t)d->sm_count * (M <= 2 ? 4 : 2);
  int64_t ksplit = base >= want ? 1 : want / base;
  const int64_t most = ceil_div(K, (int64_t)p.ty * 64);
  if (ksplit > most) ksplit = most;
  if (ksplit > 65535) ksplit = 65535;
  if (ksplit < 1) ksplit = 1;
  p.kchunk = ceil_div(K, ksplit);
  p.ksplit = (int)ceil_div(K, p.kchunk);
  p.partial = nullptr;
  p.arrivals = nullptr;
  if (p.ksplit > 1) {
    void* ws;
    PB_CHECK(scratch(d, (size_t)p.ksplit * batch * M * N * sizeof(T), &ws));
    p.partial = (T*)ws;
    PB_CHECK(counters(d, (size_t)(batch * p.strips), &p.arrivals));
  }
  const bool aligned = N % V == 0 && ((uintptr_t)B & 15) == 0;
  if (M == 1) return launch_rows<T, 1>(d, p, aligned);
  if (M == 2) return launch_rows<T, 2>(d, p, aligned);
  if (M <= 4) return launch_rows<T, 4>(d, p, aligned);
  return launch_rows<T, kMaxRows>(d, p, aligned);
}

}  // namespace

int gemm_skinny(Device* d, int dtype, const BatchMap& map, int64_t batch, int64_t M, int64_t N,
                int64_t K, const void* A, const void* B, void* C) {
  if (M > kMaxRows) PB_FAIL(PB_ERR_INVALID, "skinny product with %lld rows", (long long)M);
  if (dtype == PB_F32)
    return skinny<float>(d, map, batch, M, N, K, (const float*)A, (const float*)B, (float*)C);
  return skinny<double>(d, map, batch, M, N, K, (const double*)A, (const double*)B, (double*)C);
}

}  // namespace pb
