// float32 GEMM as error-compensated 3xTF32 on the sm_100a tensor cores.
//
// Reference: CUDABackend.matmul routes float32 products to the register GEMM
// (src/openpacho/_cuda.py:506-518, src/openpacho/_gemm.py:24-137) and the
// reference forbids silent TF32 (cuBLAS PEDANTIC_MATH, _cuda.py:194).  This
// path keeps float32 accuracy on TF32 tensor cores by splitting every operand
// x = hi + lo with hi = rn_tf32(x) and lo = rn_tf32(x - hi) and summing
// hi*hi + hi*lo + lo*hi (the lo*lo term is below float32 resolution).
//
// Structure
//  1. split pass (HBM-bound): A (rows x K) -> A' (rows x 3Kp) = [lo | hi | hi]
//     and B (K x N) -> B't (N x 3Kp) = [hi | lo | hi] (transposed to K-major),
//     Kp = K rounded up to 32, zero padded.  Then sum_k' A'[m,k'] B't[n,k'] is
//     the three-product sum, small terms first.
//  2. GEMM C = A' B't^T on tcgen05: 128 x BN output tile per CTA (BN 128 or
//     256), K' in 32-element (128-byte) slices moved by TMA with 128-byte
//     swizzle into a 4-stage shared-memory ring (no multicast), one thread
//     issuing tcgen05.mma.kind::tf32 into a TMEM accumulator, and all four
//     warps draining TMEM with tcgen05.ld into C.
//  Every mbarrier wait is bounded in wall time (%globaltimer); on expiry the
//  kernel raises the device error word, stops issuing, waits (bounded) for
//  its own copies, frees TMEM and returns.
#include <cudaTypedefs.h>

#include "pb_internal.cuh"

namespace pb {

int gemm_simt_f32(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const float* A, const float* B, float* C);

namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per 128-byte swizzled row
constexpr int STAGES = 4;
constexpr int THREADS = 128;
constexpr uint64_t kTimeoutNs = 4ull * 1000 * 1000 * 1000;

// ------------------------------------------------------------ split pass --

__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi and lo parts; non-finite values keep hi = x and lo = 0.
__device__ __forceinline__ void split(float x, float& hi, float& lo) {
  hi = tf32_rn(x);
  lo = isfinite(x) ? tf32_rn(x - hi) : 0.0f;
}

// A (rows x K) -> A' (rows x 3Kp): [lo | hi | hi].
__global__ void split_a_kernel(const float* __restrict__ A, float* __restrict__ Ap, int64_t rows,
                               int64_t K, int64_t Kp) {
  const int64_t total = rows * Kp;
  const int64_t K3 = 3 * Kp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / Kp, k = i % Kp;
    const float x = k < K ? __ldg(A + r * K + k) : 0.0f;
    float hi, lo;
    split(x, hi, lo);
    float* o = Ap + r * K3 + k;
    o[0] = lo;
    o[Kp] = hi;
    o[2 * Kp] = hi;
  }
}

// B (nmat x K x N) -> B't (nmat*N x 3Kp): [hi | lo | hi], transposed via a
// 32x32 shared tile so both the read (along N) and write (along K) coalesce.
__global__ void split_bt_kernel(const float* __restrict__ B, float* __restrict__ Bt, int64_t K,
                                int64_t N, int64_t Kp) {
  __shared__ float tile[32][33];
  const int64_t mat = blockIdx.z;
  const int64_t k0 = (int64_t)blockIdx.y * 32, n0 = (int64_t)blockIdx.x * 32;
  const float* src = B + mat * K * N;
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int64_t k = k0 + j, n = n0 + threadIdx.x;
    tile[j][threadIdx.x] = (k < K && n < N) ? __ldg(src + k * N + n) : 0.0f;
  }
  __syncthreads();
  const int64_t K3 = 3 * Kp;
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int64_t n = n0 + j, k = k0 + threadIdx.x;
    if (n < N && k < Kp) {
      float hi, lo;
      split(tile[threadIdx.x][j], hi, lo);
      float* o = Bt + (mat * N + n) * K3 + k;
      o[0] = hi;
      o[Kp] = lo;
      o[2 * Kp] = hi;
    }
  }
}

// --------------------------------------------------------- PTX wrappers --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: false if the wait expired or another role already gave up.
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                       int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicExch(err, (int)KERR_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), leading offset unused (1), sm_100 version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t instr_desc(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------ GEMM kernel --

struct Tf32Params {
  float* C;
  int64_t M, N;
  int kblocks;  // K' / 32
  int tiles_m, tiles_n;
  int64_t batch;
  BatchMap map;
  int* err;
};

template <int BN>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int TOTAL = STAGES * STAGE + 1024 /*align slack*/ + 256 /*barriers*/;
};

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    tf32x3_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, Tf32Params p) {
  extern __shared__ unsigned char smem_raw[];
  // Swizzled tiles need 1024-byte alignment.
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + STAGES * Smem<BN>::STAGE;
  uint64_t* bar_ptr = reinterpret_cast<uint64_t*>(gbase + STAGES * Smem<BN>::STAGE);
  // Layout after the stages: full[STAGES], empty[STAGES], done, tmem slot, abort.
  const uint32_t full0 = bars, empty0 = bars + 8 * STAGES, done = bars + 16 * STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ptr + 2 * STAGES + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Tile coordinates: grouped raster (16 M-tiles per group) for L2 reuse.
  const int64_t t = blockIdx.x;
  constexpr int GM = 16;
  const int64_t per_group = (int64_t)GM * p.tiles_n;
  const int64_t group = t / per_group;
  const int64_t first_m = group * GM;
  const int64_t gm = min((int64_t)GM, (int64_t)p.tiles_m - first_m);
  const int64_t in_group = t % per_group;
  const int64_t m_tile = first_m + in_group % gm;
  const int64_t n_tile = in_group / gm;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  for (int64_t bz = blockIdx.y; bz < p.batch; bz += gridDim.y) {
    int64_t ao, bo;
    batch_offsets(p.map, bz, &ao, &bo);
    const int32_t a_row = (int32_t)(ao * p.M + m_tile * BM);
    const int32_t b_row = (int32_t)(bo * p.N + n_tile * BN);
    const int64_t iter = (bz - blockIdx.y) / gridDim.y;  // phase offset across batch loops
    const int nk = p.kblocks;
    const int64_t kbase = iter * nk;

    if (warp == 0) {
      if (lane == 0) {
        int issued = 0;
        for (int kb = 0; kb < nk; ++kb) {
          const int64_t g = kbase + kb;
          const int s = (int)(g % STAGES);
          const uint32_t ph = (uint32_t)((g / STAGES) & 1);
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag, p.err)) break;
          const uint32_t sa = base + s * Smem<BN>::STAGE;
          const uint32_t sb = sa + Smem<BN>::A_BYTES;
          mbar_expect_tx(full0 + 8 * s, Smem<BN>::STAGE);
          tma_load_2d(sa, &map_a, kb * BK, a_row, full0 + 8 * s);
          tma_load_2d(sb, &map_b, kb * BK, b_row, full0 + 8 * s);
          ++issued;
        }
        if (*abort_flag) {
          // Drain: wait (bounded) for the copies this thread issued.
          for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb) {
            const int64_t g = kbase + kb;
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(full0 + 8 * (int)(g % STAGES), (uint32_t)((g / STAGES) & 1)) &&
                   globaltimer() - t0 < kTimeoutNs) {
            }
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        const uint32_t idesc = instr_desc(BN);
        for (int kb = 0; kb < nk; ++kb) {
          const int64_t g = kbase + kb;
          const int s = (int)(g % STAGES);
          const uint32_t ph = (uint32_t)((g / STAGES) & 1);
          if (!mbar_wait(full0 + 8 * s, ph, abort_flag, p.err)) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = base + s * Smem<BN>::STAGE;
          const uint32_t sb = sa + Smem<BN>::A_BYTES;
          const uint64_t da = smem_desc(sa), db = smem_desc(sb);
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            // +32 bytes per 8-element K step inside the swizzled row.
            umma_tf32(tmem, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(empty0 + 8 * s);
        }
        umma_commit(done);  // arrives once every issued MMA has completed
      }
    }
    __syncwarp();

    // Epilogue: all four warps; warp w owns TMEM lanes (tile rows) 32w..32w+31.
    const bool ok = mbar_wait(done, (uint32_t)(iter & 1), abort_flag, p.err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // tcgen05.ld is warp-collective: take the decision once per warp.
    if (__all_sync(0xffffffffu, ok && !*abort_flag)) {
      const int64_t row = m_tile * BM + warp * 32 + lane;
      float* crow = p.C + bz * p.M * p.N + row * p.N;
      const bool vec = (p.N % 4) == 0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), r);
        const int64_t col0 = n_tile * BN + c * 32;
        if (row < p.M) {
          if (vec && col0 + 32 <= p.N) {
            float4* dst = reinterpret_cast<float4*>(crow + col0);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) crow[col0 + j] = __uint_as_float(r[j]);
          }
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (*abort_flag) break;
  }

  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)BN));
  }
}

int encode_kmajor(CUtensorMap* map, const float* ptr, int64_t rows, int64_t cols, int box_rows) {
  void* fn;
  PB_CHECK(tensor_map_encoder(&fn));
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(float)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)ptr, dims, strides, box,
                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) PB_FAIL(PB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PB_OK;
}

template <int BN>
int launch_tf32(Device* d, const CUtensorMap& ma, const CUtensorMap& mb, const Tf32Params& p) {
  const int smem = Smem<BN>::TOTAL;
  static bool configured = false;
  if (!configured) {
    PB_CUDA(cudaFuncSetAttribute(tf32x3_gemm_kernel<BN>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  const int64_t tiles = (int64_t)p.tiles_m * p.tiles_n;
  if (tiles > INT32_MAX) PB_FAIL(PB_ERR_UNSUPPORTED, "GEMM grid too large");
  const unsigned gy = (unsigned)(p.batch < 65535 ? p.batch : 65535);
  tf32x3_gemm_kernel<BN><<<dim3((unsigned)tiles, gy), THREADS, smem, d->stream>>>(ma, mb, p);
  PB_LAUNCHED(d);
  return PB_OK;
}

int64_t matrices_used(const BatchMap& m, bool a) {
  int64_t last = 0;
  for (int i = 0; i < m.ndim; ++i) last += (m.shape[i] - 1) * (a ? m.a_stride[i] : m.b_stride[i]);
  return last + 1;
}

}  // namespace

// algo: 0 auto, 1 SIMT, 2 3xTF32 tcgen05.
int gemm_f32_algo(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const float* A, const float* B, float* C, int algo) {
  if (algo == 0) algo = (M >= 64 && N >= 64 && K >= 32) ? 2 : 1;
  if (algo == 1) return gemm_simt_f32(d, map, batch, M, N, K, A, B, C);
  if (algo != 2) PB_FAIL(PB_ERR_INVALID, "unknown GEMM algorithm %d", algo);

  const int64_t Kp = ceil_div(K, (int64_t)BK) * BK;
  const int64_t K3 = 3 * Kp;
  const int64_t nA = matrices_used(map, true), nB = matrices_used(map, false);
  const int64_t rows_a = nA * M, rows_b = nB * N;
  if (rows_a > INT32_MAX || rows_b > INT32_MAX || K3 / BK > INT32_MAX)
    PB_FAIL(PB_ERR_UNSUPPORTED, "GEMM operand too large for 32-bit TMA coordinates");
  const size_t bytes_a = (size_t)rows_a * K3 * sizeof(float);
  const size_t bytes_b = (size_t)rows_b * K3 * sizeof(float);
  void* ws;
  PB_CHECK(scratch(d, bytes_a + bytes_b, &ws));
  float* Ap = (float*)ws;
  float* Bt = (float*)((char*)ws + bytes_a);

  {
    const int64_t total = rows_a * Kp;
    int64_t blocks = ceil_div(total, (int64_t)256);
    const int64_t cap = (int64_t)d->sm_count * 16;
    if (blocks > cap) blocks = cap;
    split_a_kernel<<<(unsigned)blocks, 256, 0, d->stream>>>(A, Ap, rows_a, K, Kp);
    PB_LAUNCHED(d);
    const int64_t gx = ceil_div(N, (int64_t)32), gy = ceil_div(Kp, (int64_t)32);
    if (gx > INT32_MAX || gy > 65535 || nB > 65535)
      PB_FAIL(PB_ERR_UNSUPPORTED, "B operand too large for the split grid");
    split_bt_kernel<<<dim3((unsigned)gx, (unsigned)gy, (unsigned)nB), dim3(32, 8), 0, d->stream>>>(
        B, Bt, K, N, Kp);
    PB_LAUNCHED(d);
  }

  const int tiles_m = (int)ceil_div(M, (int64_t)BM);
  const bool wide = ceil_div(N, (int64_t)256) * tiles_m * batch >= d->sm_count && N > 128;
  const int BN = wide ? 256 : 128;
  CUtensorMap ma, mb;
  PB_CHECK(encode_kmajor(&ma, Ap, rows_a, K3, BM));
  PB_CHECK(encode_kmajor(&mb, Bt, rows_b, K3, BN));
  Tf32Params p;
  p.C = C;
  p.M = M;
  p.N = N;
  p.kblocks = (int)(K3 / BK);
  p.tiles_m = tiles_m;
  p.tiles_n = (int)ceil_div(N, (int64_t)BN);
  p.batch = batch;
  p.map = map;
  p.err = d->err_dev;
  if (BN == 256) return launch_tf32<256>(d, ma, mb, p);
  return launch_tf32<128>(d, ma, mb, p);
}

}  // namespace pb
