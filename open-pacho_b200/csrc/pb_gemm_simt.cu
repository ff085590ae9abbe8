// Register-tiled SIMT GEMM: the float64 path (DFMA) and the float32 path for
// shapes too small or skinny for a 128-row tcgen05 tile.
//
// Reference: the fp64 GEMM of the custom CUDA provider is one thread per
// output with a serial K loop (src/openpacho/_cuda.py:619-636); the fp32
// register GEMM uses 64 threads per 32x32 tile with 4x4 accumulators
// (src/openpacho/_gemm.py:24-99) and broadcast batch offsets (_gemm.py:13-21).
//
// This kernel: 128x128 output tile per 256-thread CTA, 8x8 accumulators per
// thread split into four 4x4 quadrants (rows ty*4 and 64+ty*4, columns tx*4
// and 64+tx*4) so shared-memory reads are conflict-free 16-byte vectors; K
// advances in 16-wide slices, double-buffered in shared memory with the next
// slice prefetched into registers while the current one is multiplied.
#include "pb_internal.cuh"

namespace pb {
namespace {

constexpr int BM = 128, BN = 128, BK = 16, NT = 256;

template <typename T>
struct SimtParams {
  const T* A;
  const T* B;
  T* C;
  int64_t M, N, K;
  int64_t batch;
  BatchMap map;
  // Repair mode (non-null): only the tiles marked in nf are computed, by a
  // persistent grid, and the marks are cleared (layout in pb_internal.cuh).
  unsigned int* nf;
};

static_assert(BM == kNonFiniteTile && BN == kNonFiniteTile, "repair tiles are SIMT tiles");

// One BM x BN output tile of batch entry bz at (m0, n0).
template <typename T>
__device__ __forceinline__ void simt_tile(const SimtParams<T>& p, int64_t bz, int64_t m0,
                                          int64_t n0, T* As, T* Bs) {
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t M = p.M, N = p.N, K = p.K;

  // Global->register staging coordinates.
  const int a_row = tid >> 1, a_k = (tid & 1) * 8;  // A: 128 rows x 16 k
  const int b_k = tid >> 4, b_col = (tid & 15) * 8;  // B: 16 k x 128 cols

  int64_t ao, bo;
  batch_offsets(p.map, bz, &ao, &bo);
  const T* A = p.A + ao * M * K;
  const T* B = p.B + bo * K * N;
  T* C = p.C + bz * M * N;

  T acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = T(0);

  T ra[8], rb[8];
  auto load = [&](int64_t k0) {
    const int64_t gr = m0 + a_row;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t gk = k0 + a_k + j;
      ra[j] = (gr < M && gk < K) ? __ldg(A + gr * K + gk) : T(0);
    }
    const int64_t gk = k0 + b_k;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t gc = n0 + b_col + j;
      rb[j] = (gk < K && gc < N) ? __ldg(B + gk * N + gc) : T(0);
    }
  };
  auto store = [&](int buf) {
    T* as = As + buf * BK * BM;
    T* bs = Bs + buf * BK * BN;
#pragma unroll
    for (int j = 0; j < 8; ++j) as[(a_k + j) * BM + a_row] = ra[j];
#pragma unroll
    for (int j = 0; j < 8; ++j) bs[b_k * BN + b_col + j] = rb[j];
  };

  const int64_t ktiles = ceil_div(K, (int64_t)BK);
  load(0);
  store(0);
  __syncthreads();
  for (int64_t kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load((kt + 1) * BK);
    const T* as = As + buf * BK * BM;
    const T* bs = Bs + buf * BK * BN;
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      T a[8], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = as[kk * BM + ty * 4 + i];
        a[4 + i] = as[kk * BM + 64 + ty * 4 + i];
        b[i] = bs[kk * BN + tx * 4 + i];
        b[4 + i] = bs[kk * BN + 64 + tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) store(buf ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t r = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t c = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (c < N) C[r * N + c] = acc[i][j];
    }
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(NT, 1) simt_gemm_kernel(SimtParams<T> p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* As = reinterpret_cast<T*>(smem_raw);  // [2][BK][BM], transposed A slice
  T* Bs = As + 2 * BK * BM;                // [2][BK][BN]
  if (p.nf == nullptr) {
    const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
    for (int64_t bz = blockIdx.z; bz < p.batch; bz += gridDim.z) simt_tile(p, bz, m0, n0, As, Bs);
    return;
  }
  // Repair mode: wait for the marking kernels, then recompute marked tiles.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  volatile unsigned int* nf = p.nf;
  if (nf[0] == 0u) return;
  const int64_t tiles_m = ceil_div(p.M, (int64_t)BM), tiles_n = ceil_div(p.N, (int64_t)BN);
  const int64_t per_batch = tiles_m * tiles_n, total = p.batch * per_batch;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    if (nf[2 + t] == 0u) continue;
    const int64_t bz = t / per_batch, r = t % per_batch;
    simt_tile(p, bz, (r / tiles_n) * BM, (r % tiles_n) * BN, As, Bs);
    if (threadIdx.x == 0) nf[2 + t] = 0u;
  }
  // The last block to finish clears the summary word and the counter.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.nf + 1, 1u) == gridDim.x - 1) {
      nf[0] = 0u;
      nf[1] = 0u;
    }
  }
}

template <typename T>
int launch_simt(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                const T* A, const T* B, T* C) {
  SimtParams<T> p{A, B, C, M, N, K, batch, map, nullptr};
  const int64_t gx = ceil_div(N, (int64_t)BN), gy = ceil_div(M, (int64_t)BM);
  if (gx > INT32_MAX || gy > 65535) PB_FAIL(PB_ERR_UNSUPPORTED, "GEMM grid too large");
  const unsigned gz = (unsigned)(batch < 65535 ? batch : 65535);
  const size_t smem = 2 * BK * (BM + BN) * sizeof(T);
  PB_CHECK(allow_smem(d, (const void*)simt_gemm_kernel<T>, smem));
  PB_CHECK(kt_begin(d));
  simt_gemm_kernel<T><<<dim3((unsigned)gx, (unsigned)gy, gz), NT, smem, d->stream>>>(p);
  PB_LAUNCHED(d);
  return kt_end(d);
}

}  // namespace

int gemm_nonfinite_repair_f32(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N,
                              int64_t K, const float* A, const float* B, float* C,
                              unsigned int* nf) {
  SimtParams<float> p{A, B, C, M, N, K, batch, map, nf};
  const int64_t tiles = batch * ceil_div(M, (int64_t)BM) * ceil_div(N, (int64_t)BN);
  const unsigned grid = (unsigned)(tiles < d->sm_count ? tiles : d->sm_count);
  const size_t smem = 2 * BK * (BM + BN) * sizeof(float);
  PB_CHECK(allow_smem(d, (const void*)simt_gemm_kernel<float>, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = d->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PB_CUDA(cudaLaunchKernelEx(&cfg, simt_gemm_kernel<float>, p));
  PB_LAUNCHED(d);
  return PB_OK;
}

int gemm_simt_f32(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const float* A, const float* B, float* C) {
  return launch_simt<float>(d, map, batch, M, N, K, A, B, C);
}

int gemm_simt_f64(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const double* A, const double* B, double* C) {
  return launch_simt<double>(d, map, batch, M, N, K, A, B, C);
}

}  // namespace pb
