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
//     swizzle into a 4-stage shared-memory ring (each CTA loads its own tiles), one thread
//     issuing tcgen05.mma.kind::tf32 into a TMEM accumulator, and all four
//     warps draining TMEM with tcgen05.ld into C.
//  Every mbarrier wait is bounded in wall time (%globaltimer); on expiry the
//  kernel raises the device error word, stops issuing, waits (bounded) for
//  its own copies, frees TMEM and returns.
#include <cfloat>
#include <cstring>
#include <utility>
#include <cudaTypedefs.h>

#include "pb_internal.cuh"

// Build parameters of the 3xTF32 kernels (each measured on and off).
#ifndef PB_TF32_SPLIT_EARLY
#define PB_TF32_SPLIT_EARLY 1  // split A into registers before waiting for its TMEM buffer
#endif
#ifndef PB_TF32_WARM
#define PB_TF32_WARM 0  // 1: warm the launch parameters and prefetch the tensor maps at entry
#endif
#ifndef PB_TF32_PROMOTE_BATCH
#define PB_TF32_PROMOTE_BATCH 1  // several accumulator loads per wait; 16 warps at FBN = 128
#endif

namespace pb {

int gemm_simt_f32(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const float* A, const float* B, float* C);

namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per 128-byte swizzled row
constexpr int STAGES = 4;
constexpr uint64_t kTimeoutNs = 4ull * 1000 * 1000 * 1000;

// ------------------------------------------------------------ split pass --

__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Operand magnitudes the split cannot carry at float32 accuracy: nonzero
// |x| < 2^-57.  A product with such a factor can fall below 2^-115, where the
// lo*hi cross terms (or the whole product) become subnormal and the tensor
// core flushes them.  Rows of A and kTagCols-column groups of B holding one
// are tagged by the split passes, and the epilogue recomputes the outputs
// they touch with float32 FMA.
constexpr uint32_t kTinyExp = 127 - 57;  // biased exponent of 2^-57
constexpr float kTinyMag = 0x1p-57f;     // 2^-57: below it (zero included) the exact check runs
constexpr int kTagCols = 64;

__device__ __forceinline__ bool tiny(float x) {
  return (__float_as_uint(x) & 0x7fffffffu) - 1u < (kTinyExp << 23) - 1u;
}

// hi and lo parts; non-finite values keep hi = x and lo = 0.  Returns tiny(x).
__device__ __forceinline__ bool split(float x, float& hi, float& lo) {
  hi = tf32_rn(x);
  lo = isfinite(x) ? tf32_rn(x - hi) : 0.0f;
  return tiny(x);
}

// A (rows x K) -> A' (rows x 3Kp): [lo | hi | hi].
__global__ void split_a_kernel(const float* __restrict__ A, float* __restrict__ Ap, int64_t rows,
                               int64_t K, int64_t Kp, unsigned int* rowtag, unsigned int* tagany,
                               unsigned int gen) {
  const int64_t total = rows * Kp;
  const int64_t K3 = 3 * Kp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / Kp, k = i % Kp;
    const float x = k < K ? __ldg(A + r * K + k) : 0.0f;
    float hi, lo;
    if (split(x, hi, lo)) {
      rowtag[r] = gen;
      tagany[0] = gen;
    }
    float* o = Ap + r * K3 + k;
    o[0] = lo;
    o[Kp] = hi;
    o[2 * Kp] = hi;
  }
}

// The same split with 16-byte accesses (K % 4 == 0, A 16-byte aligned): a
// thread per 4 consecutive k of a row, the row found by a multiply-shift
// division by Kp / 4 (a launch constant) instead of a 64-bit division per
// element, which made the scalar pass issue-bound (16384^2: ~6 ms).
__global__ void __launch_bounds__(256) split_a4_kernel(const float* __restrict__ A,
                                                       float* __restrict__ Ap, int64_t rows,
                                                       int64_t K, int64_t Kp, FastDiv fd_q,
                                                       unsigned int* rowtag, unsigned int* tagany,
                                                       unsigned int gen) {
  const int64_t q = Kp / 4;
  const int64_t total = rows * q;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = fdiv(i, fd_q);
    const int64_t k = (i - r * q) * 4;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (k < K) v = __ldg(reinterpret_cast<const float4*>(A + r * K + k));
    float4 h, l;
    bool t = split(v.x, h.x, l.x);
    t |= split(v.y, h.y, l.y);
    t |= split(v.z, h.z, l.z);
    t |= split(v.w, h.w, l.w);
    if (t) {
      rowtag[r] = gen;
      tagany[0] = gen;
    }
    float4* o = reinterpret_cast<float4*>(Ap + r * 3 * Kp + k);
    o[0] = l;
    o[Kp / 4] = h;
    o[Kp / 2] = h;
  }
}

// B (nmat x K x N) -> B't, transposed to K-major through shared memory.
// SEGS = 3 writes [hi | lo | hi] (nmat*N x 3Kp, for the pre-split GEMM),
// SEGS = 2 writes [hi | lo] (nmat*N x 2Kp, for the GEMM that splits A in
// tensor memory).  A 256-thread block moves a 32 (k) x 64 (n) tile: float4
// loads along n, and float4 stores along k, eight lanes per 128-byte row
// segment, so both sides coalesce; the transposing shared-memory reads are
// conflict-free (row pitch 65 words).  Grid: (ceil(N/64), Kp/32, nmat).
constexpr int SPLIT_TK = 32, SPLIT_TN = 64;

template <int SEGS>
__global__ void __launch_bounds__(256) split_bt_kernel(const float* __restrict__ B, float* __restrict__ Bt,
                                                       int64_t K, int64_t N, int64_t Kp,
                                                       unsigned int* coltag, int64_t groups,
                                                       unsigned int* tagany, unsigned int gen) {
  __shared__ float tile[SPLIT_TK][SPLIT_TN + 1];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the GEMM may start its prologue
  const int64_t mat = blockIdx.z;
  const int64_t k0 = (int64_t)blockIdx.y * SPLIT_TK, n0 = (int64_t)blockIdx.x * SPLIT_TN;
  const float* src = B + mat * K * N;
  const int t = threadIdx.x;
  const bool vec = (N % 4) == 0 && n0 + SPLIT_TN <= N && ((uintptr_t)src & 15) == 0;
  bool tiny_seen = false;
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int r = pass * 16 + (t >> 4), c = (t & 15) * 4;  // 16 float4 per 64-wide row
    const int64_t k = k0 + r;
    float v[4];
    if (k < K && vec) {
      const float4 q = __ldg(reinterpret_cast<const float4*>(src + k * N + n0 + c));
      v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (k < K && n0 + c + j < N) ? __ldg(src + k * N + n0 + c + j) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      tile[r][c + j] = v[j];
      tiny_seen |= tiny(v[j]);
    }
  }
  if (tiny_seen) {
    // Column group of each tiny value (rare: re-read the four values).
    for (int pass = 0; pass < 2; ++pass) {
      const int r = pass * 16 + (t >> 4), c = (t & 15) * 4;
      for (int j = 0; j < 4; ++j)
        if (tiny(tile[r][c + j])) {
          coltag[mat * groups + (n0 + c + j) / kTagCols] = gen;
          tagany[0] = gen;
        }
    }
  }
  __syncthreads();
  const int64_t KS = SEGS * Kp;
  const int kq = t & 7;  // float4 along k: k = 4*kq .. 4*kq+3
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int nl = pass * 32 + (t >> 3);
    const int64_t n = n0 + nl;
    if (n >= N) continue;
    float4 h, l;
    float* hp = &h.x;
    float* lp = &l.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float hi, lo;
      split(tile[4 * kq + j][nl], hi, lo);
      hp[j] = hi;
      lp[j] = lo;
    }
    float* o = Bt + (mat * N + n) * KS + k0 + 4 * kq;
    *reinterpret_cast<float4*>(o) = h;
    *reinterpret_cast<float4*>(o + Kp) = l;
    if (SEGS == 3) *reinterpret_cast<float4*>(o + 2 * Kp) = h;
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
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
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

// Bulk tensor store of a box from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int32_t x,
                                             int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(x), "r"(y), "r"(z)
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// The source buffers of this thread's bulk stores may be overwritten.
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// This thread's bulk stores have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

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

// TMEM -> registers, 32 lanes x 32 columns of 32-bit values.  The wait is part
// of the same asm statement so no use of the outputs can precede it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]),"=r"(r[1]),"=r"(r[2]),"=r"(r[3]),"=r"(r[4]),"=r"(r[5]),"=r"(r[6]),"=r"(r[7]),"=r"(r[8]),"=r"(r[9]),"=r"(r[10]),"=r"(r[11]),"=r"(r[12]),"=r"(r[13]),"=r"(r[14]),"=r"(r[15]),"=r"(r[16]),"=r"(r[17]),"=r"(r[18]),"=r"(r[19]),"=r"(r[20]),"=r"(r[21]),"=r"(r[22]),"=r"(r[23]),"=r"(r[24]),"=r"(r[25]),"=r"(r[26]),"=r"(r[27]),"=r"(r[28]),"=r"(r[29]),"=r"(r[30]),"=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// TMEM -> registers, 32 lanes x 16 columns (load and wait in one statement).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]),"=r"(r[1]),"=r"(r[2]),"=r"(r[3]),"=r"(r[4]),"=r"(r[5]),"=r"(r[6]),"=r"(r[7]),"=r"(r[8]),"=r"(r[9]),"=r"(r[10]),"=r"(r[11]),"=r"(r[12]),"=r"(r[13]),"=r"(r[14]),"=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Three 16-column loads in flight before one wait.
__device__ __forceinline__ void tmem_ld16x3(uint32_t ta, uint32_t (&a)[48]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%48];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%49];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47}, [%50];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(a[0]),"=r"(a[1]),"=r"(a[2]),"=r"(a[3]),"=r"(a[4]),"=r"(a[5]),"=r"(a[6]),"=r"(a[7]),"=r"(a[8]),"=r"(a[9]),"=r"(a[10]),"=r"(a[11]),"=r"(a[12]),"=r"(a[13]),"=r"(a[14]),"=r"(a[15]),
        "=r"(a[16]),"=r"(a[17]),"=r"(a[18]),"=r"(a[19]),"=r"(a[20]),"=r"(a[21]),"=r"(a[22]),"=r"(a[23]),"=r"(a[24]),"=r"(a[25]),"=r"(a[26]),"=r"(a[27]),"=r"(a[28]),"=r"(a[29]),"=r"(a[30]),"=r"(a[31]),
        "=r"(a[32]),"=r"(a[33]),"=r"(a[34]),"=r"(a[35]),"=r"(a[36]),"=r"(a[37]),"=r"(a[38]),"=r"(a[39]),"=r"(a[40]),"=r"(a[41]),"=r"(a[42]),"=r"(a[43]),"=r"(a[44]),"=r"(a[45]),"=r"(a[46]),"=r"(a[47])
      : "r"(ta), "r"(ta + 16u), "r"(ta + 32u)
      : "memory");
}

// Two 32-column loads in flight before one wait.
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, uint32_t tb, uint32_t (&a)[32],
                                            uint32_t (&b)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(a[0]),"=r"(a[1]),"=r"(a[2]),"=r"(a[3]),"=r"(a[4]),"=r"(a[5]),"=r"(a[6]),"=r"(a[7]),"=r"(a[8]),"=r"(a[9]),"=r"(a[10]),"=r"(a[11]),"=r"(a[12]),"=r"(a[13]),"=r"(a[14]),"=r"(a[15]),"=r"(a[16]),"=r"(a[17]),"=r"(a[18]),"=r"(a[19]),"=r"(a[20]),"=r"(a[21]),"=r"(a[22]),"=r"(a[23]),"=r"(a[24]),"=r"(a[25]),"=r"(a[26]),"=r"(a[27]),"=r"(a[28]),"=r"(a[29]),"=r"(a[30]),"=r"(a[31]),"=r"(b[0]),"=r"(b[1]),"=r"(b[2]),"=r"(b[3]),"=r"(b[4]),"=r"(b[5]),"=r"(b[6]),"=r"(b[7]),"=r"(b[8]),"=r"(b[9]),"=r"(b[10]),"=r"(b[11]),"=r"(b[12]),"=r"(b[13]),"=r"(b[14]),"=r"(b[15]),"=r"(b[16]),"=r"(b[17]),"=r"(b[18]),"=r"(b[19]),"=r"(b[20]),"=r"(b[21]),"=r"(b[22]),"=r"(b[23]),"=r"(b[24]),"=r"(b[25]),"=r"(b[26]),"=r"(b[27]),"=r"(b[28]),"=r"(b[29]),"=r"(b[30]),"=r"(b[31])
      : "r"(ta), "r"(tb)
      : "memory");
}

// ------------------------------------------------------------ GEMM kernel --
//
// Persistent kernel, one CTA per SM, 10 warps:
//   warp 0      TMA producer (one elected lane) for the 4-stage A/B ring;
//   warp 1      TMEM allocator and MMA issuer (one elected lane);
//   warps 2..9  accumulator warps.  The MMA thread accumulates CHUNK = 8
//               K-slices (32 tcgen05.mma steps) into one of two TMEM buffers,
//               then commits it; the accumulator warps add that chunk into
//               float32 registers with round-to-nearest and release the
//               buffer.  The tensor core's own accumulation truncates (~0.3 ulp
//               of bias per step, so the error grew linearly with K: 1.9e-5 at
//               K=8192 without promotion); promoting every 32 steps keeps
//               3xTF32 at float32-class accuracy (6.5e-7 at K=8192, flat in K).
//               Measured on B200: CHUNK 4/8 cost 216.5/226.6 TFLOP/s at 8192^3
//               for 3.7e-7/6.5e-7 relative error.  With two buffers the
//               promotion of chunk c overlaps the MMAs of chunk c+1, and the
//               store of one tile overlaps the next tile's first chunks.
// Warp w (2..9) reads TMEM lane quadrant w % 4 (rows 32*(w%4) .. +31 of the
// tile) and column half (w - 2) / 4 of the BN columns.

#ifndef PB_TF32_CHUNK
#define PB_TF32_CHUNK 8
#endif
#ifndef PB_TF32_LD_PAIR
#define PB_TF32_LD_PAIR 1
#endif
constexpr int CHUNK = PB_TF32_CHUNK;     // K-slices per promotion
constexpr int ACC_WARPS = 8;
constexpr int GEMM_THREADS = 32 * (2 + ACC_WARPS);

struct Tf32Params {
  float* C;
  float* partial;  // ksplit > 1: per-split fp32 tiles, [ksplit][batch][M][N]
  const float* A;  // the caller's operands (non-finite repair)
  const float* B;
  int64_t M, N, K;
  int kblocks;  // K' / 32
  int tiles_m, tiles_n;
  int64_t tiles;  // tiles_m * tiles_n * batch
  int ksplit;     // K-slice ranges per tile (work items = tiles * ksplit)
  BatchMap map;
  int* err;
  unsigned int* nf;          // non-finite tile marks (pb_internal.cuh)
  int64_t nf_tm, nf_tn;      // kNonFiniteTile tiles along M and N
  int repair_inline;         // recompute flagged outputs where they are written
  int tma_store;             // epilogue stores through the output tensor map
  unsigned int* tagany;      // generation if any operand of this launch is tagged
  unsigned int* rowtag;      // per row of A (all matrices): generation if tiny
  unsigned int* coltag;      // per kTagCols columns of each B matrix
  int64_t cgroups;           // ceil(N / kTagCols)
  unsigned int gen;          // this launch's generation
  int64_t batch;             // matrices in the product
  // Launch-constant divisors of the tile schedule: the K split, tiles per
  // matrix, tiles per group of GM M-tiles, and the last group's height.
  FastDiv fd_ksplit, fd_tiles, fd_group, fd_gm_last;
};

constexpr int GM = 16;  // M-tiles per raster group (a power of two)

// Work item w -> (tile, K split).
__device__ __forceinline__ void item_of(const Tf32Params& p, int64_t w, int64_t& tile, int& split) {
  tile = fdiv(w, p.fd_ksplit);
  split = (int)(w - tile * p.ksplit);
}

// K-slice range [kb0, kb1) of split `s`.
__device__ __forceinline__ void split_range(const Tf32Params& p, int s, int& kb0, int& kb1) {
  kb0 = (int)fdiv((int64_t)s * p.kblocks, p.fd_ksplit);
  kb1 = (int)fdiv((int64_t)(s + 1) * p.kblocks, p.fd_ksplit);
}

template <int BN>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  // barriers: full[S], empty[S], accf[2], acce[2]; then tmem slot and abort flag
  static constexpr int TOTAL = STAGES * STAGE + 1024 /*align slack*/ + 256;
};

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

struct TileCoord {
  int64_t bz, m_tile, n_tile;
};

// Tile t -> (batch, m, n): batches in order; inside a batch a grouped raster
// of 16 M-tiles so CTAs running together share A and B tiles in L2.
__device__ __forceinline__ TileCoord tile_coord(const Tf32Params& p, int64_t t) {
  TileCoord c;
  c.bz = fdiv(t, p.fd_tiles);
  const int64_t r = t - c.bz * p.fd_tiles.d;
  const int64_t group = fdiv(r, p.fd_group);
  const int64_t first_m = group * GM;
  const int64_t in_group = r - group * p.fd_group.d;
  if (first_m + GM <= p.tiles_m) {  // a full group of GM M-tiles
    c.m_tile = first_m + (in_group & (GM - 1));
    c.n_tile = in_group / GM;
  } else {  // the last, shorter group: tiles_m % GM M-tiles
    c.n_tile = fdiv(in_group, p.fd_gm_last);
    c.m_tile = first_m + (in_group - c.n_tile * p.fd_gm_last.d);
  }
  return c;
}

// First reads of the launch parameters miss the constant cache in a chain of
// dependent loads (~1.8 us before the first TMA when measured with
// %globaltimer stamps).  One otherwise idle lane computes its CTA's first work
// item during set-up -- before the programmatic-launch wait, so under a
// preceding kernel's tail -- which brings those lines into the cache for every
// warp; the tensor maps are prefetched likewise.  The result is only kept
// alive through a shared-memory word.
__device__ __forceinline__ void warm_params(const Tf32Params& p, volatile int* sink) {
  int64_t tile;
  int split;
  item_of(p, blockIdx.x, tile, split);
  const TileCoord tc = tile_coord(p, tile);
  int kb0, kb1;
  split_range(p, split, kb0, kb1);
  int64_t ao, bo;
  batch_offsets(p.map, tc.bz, &ao, &bo);
  *sink = (int)(ao + bo + kb0 + kb1 + tc.m_tile + tc.n_tile + p.gen + (int)p.M + (int)p.N);
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Above these K a flagged output is not recomputed where it is written but
// its tile is marked for the tiled repair launch: in the epilogue the
// pipeline waits for the recomputation (bounded by kTimeoutNs); in the
// split reduction each flagged element is a strided dot product of its own.
constexpr int64_t kInlineRepairMaxK = 1 << 18;
constexpr int64_t kReduceRepairMaxK = 1 << 13;

// Row segment of COLS values from col0: plain stores, float4 when aligned.
template <int COLS>
__device__ __forceinline__ void store_row(float* dst, const float (&v)[COLS], int64_t col0,
                                          int64_t N) {
  if ((N % 4) == 0 && col0 + COLS <= N && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int j = 0; j < COLS / 4; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < COLS; ++j)
      if (col0 + j < N) dst[j] = v[j];
  }
}

__device__ __forceinline__ bool nonfinite(float x) { return !(fabsf(x) <= FLT_MAX); }

// Recomputes C[row, col0 .. col0+ncols) with sequential float32 FMA over the
// caller's operands: the IEEE classes of +-Inf and NaN results.  Kept out of
// line so the accumulator registers of the hot loop are not affected.
__device__ __noinline__ void repair_row(const float* arow, const float* bcol, float* crow,
                                        int64_t N, int64_t K, int ncols) {
  for (int j = 0; j < ncols; ++j) {
    float s = 0.0f;
    for (int64_t k = 0; k < K; ++k) s = fmaf(arow[k], bcol[k * N + j], s);
    crow[j] = s;
  }
}

// The row segment (row, col0 ..) of batch entry bz was written with a
// non-finite value or from a tiny operand: recompute it now, or mark its tile
// for the repair launch.
__device__ __forceinline__ void handle_nonfinite(const Tf32Params& p, int64_t bz, int64_t row,
                                                 int64_t col0, int cols) {
  if (!p.repair_inline) {
    mark_nonfinite(p.nf, bz, row, col0, p.nf_tm, p.nf_tn);
    return;
  }
  int64_t ao, bo;
  batch_offsets(p.map, bz, &ao, &bo);
  repair_row(p.A + (ao * p.M + row) * p.K, p.B + bo * p.K * p.N + col0,
             p.C + (bz * p.M + row) * p.N + col0, p.N, p.K, (int)min((int64_t)cols, p.N - col0));
}

// True if row `row` of batch entry bz or one of the columns col0 .. +COLS
// touches an operand tagged as tiny in this launch.
template <int COLS>
__device__ __forceinline__ bool tagged(const Tf32Params& p, int64_t bz, int64_t row, int64_t col0) {
  int64_t ao, bo;
  batch_offsets(p.map, bz, &ao, &bo);
  bool t = __ldcg(p.rowtag + ao * p.M + row) == p.gen;
  const unsigned int* ct = p.coltag + bo * p.cgroups + col0 / kTagCols;
  const int64_t last = min(col0 + COLS, p.N) - 1;
  for (int64_t g = 0; g <= last / kTagCols - col0 / kTagCols; ++g) t |= __ldcg(ct + g) == p.gen;
  return t;
}

// Epilogue of one work item: this thread's row segment (row, col0 ..
// col0+COLS) of the tile.  With K split, the split's partial tile is stored
// for splitk_reduce_kernel; otherwise the values are final.
template <int COLS>
__device__ __forceinline__ void finish_item(const Tf32Params& p, const TileCoord& tc, int split,
                                            int64_t row, int64_t col0, const float (&acc)[COLS]) {
  if (row >= p.M) return;
  if (p.ksplit > 1) {
    const int64_t batch = p.batch;
    store_row<COLS>(p.partial + split * batch * p.M * p.N + (tc.bz * p.M + row) * p.N + col0, acc,
                    col0, p.N);
    return;
  }
  bool bad = false;
#pragma unroll
  for (int j = 0; j < COLS; ++j) bad |= nonfinite(acc[j]);
  store_row<COLS>(p.C + (tc.bz * p.M + row) * p.N + col0, acc, col0, p.N);
  if (__ldcg(p.tagany) == p.gen) bad |= tagged<COLS>(p, tc.bz, row, col0);
  if (bad) handle_nonfinite(p, tc.bz, row, col0, COLS);
}

template <int BN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    tf32x3_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, Tf32Params p) {
  extern __shared__ unsigned char smem_raw[];
  // Swizzled tiles need 1024-byte alignment.
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + STAGES * Smem<BN>::STAGE;
  uint64_t* bar_ptr = reinterpret_cast<uint64_t*>(gbase + STAGES * Smem<BN>::STAGE);
  const uint32_t full0 = bars, empty0 = bars + 8 * STAGES;
  const uint32_t accf0 = bars + 16 * STAGES, acce0 = accf0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ptr + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulator buffers

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, ACC_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (PB_TF32_WARM) {
      prefetch_map(&map_a);
      prefetch_map(&map_b);
    }
  }
  if (PB_TF32_WARM && warp == 2 && lane == 0) warm_params(p, abort_flag + 1);
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int64_t items = p.tiles * p.ksplit;
  // Launched as a programmatic dependent of the split pass: the prologue above
  // overlapped its tail; nothing it wrote is read before this wait.  The next
  // launch (split reduction or repair) may be scheduled from now on; it waits
  // for this grid in turn.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int64_t g = 0;  // k-slices issued by this CTA (ring position)
      for (int64_t w = blockIdx.x; w < items && !*abort_flag; w += gridDim.x) {
        int64_t tile;
        int split;
        item_of(p, w, tile, split);
        const TileCoord tc = tile_coord(p, tile);
        int kb0, kb1;
        split_range(p, split, kb0, kb1);
        int64_t ao, bo;
        batch_offsets(p.map, tc.bz, &ao, &bo);
        const int32_t a_row = (int32_t)(ao * p.M + tc.m_tile * BM);
        const int32_t b_row = (int32_t)(bo * p.N + tc.n_tile * BN);
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = (int)(g % STAGES);
          if (!mbar_wait(empty0 + 8 * s, (uint32_t)(((g / STAGES) & 1) ^ 1), abort_flag, p.err))
            break;
          const uint32_t sa = base + s * Smem<BN>::STAGE;
          mbar_expect_tx(full0 + 8 * s, Smem<BN>::STAGE);
          tma_load_2d(sa, &map_a, kb * BK, a_row, full0 + 8 * s);
          tma_load_2d(sa + Smem<BN>::A_BYTES, &map_b, kb * BK, b_row, full0 + 8 * s);
        }
      }
      if (*abort_flag) {
        // Drain (bounded): the last STAGES copies this thread may have issued.
        for (int64_t q = (g > STAGES ? g - STAGES : 0); q < g; ++q) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(full0 + 8 * (int)(q % STAGES), (uint32_t)((q / STAGES) & 1)) &&
                 globaltimer() - t0 < kTimeoutNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = instr_desc(BN);
      int64_t g = 0, gc = 0;  // k-slices consumed / chunks produced by this CTA
      bool ok = true;
      for (int64_t w = blockIdx.x; w < items && ok; w += gridDim.x) {
        int64_t tile;
        int split;
        item_of(p, w, tile, split);
        int kb0, kb1;
        split_range(p, split, kb0, kb1);
        const int nchunks = (kb1 - kb0 + CHUNK - 1) / CHUNK;
        for (int c = 0; c < nchunks && ok; ++c, ++gc) {
          const int buf = (int)(gc & 1);
          ok = mbar_wait(acce0 + 8 * buf, (uint32_t)(((gc >> 1) & 1) ^ 1), abort_flag, p.err);
          if (!ok) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t d = tmem + (uint32_t)(buf * BN);
          const int kb_start = kb0 + c * CHUNK;
          const int kb_end = min(kb1, kb_start + CHUNK);
          for (int kb = kb_start; kb < kb_end; ++kb, ++g) {
            const int s = (int)(g % STAGES);
            ok = mbar_wait(full0 + 8 * s, (uint32_t)((g / STAGES) & 1), abort_flag, p.err);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = base + s * Smem<BN>::STAGE;
            const uint64_t da = smem_desc(sa), db = smem_desc(sa + Smem<BN>::A_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 8; ++k)  // +32 bytes per 8-element K step
              umma_tf32(d, da + 2 * k, db + 2 * k, idesc, (kb > kb_start || k > 0) ? 1u : 0u);
            umma_commit(empty0 + 8 * s);
          }
          umma_commit(accf0 + 8 * buf);  // chunk complete -> accumulator warps
        }
      }
    }
  } else {
    // -------------------------------------------------- accumulator warps
    constexpr int COLS = BN / 2;
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(half * COLS);
    int64_t gc = 0;
    for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
      int64_t tile;
      int split;
      item_of(p, w, tile, split);
      const TileCoord tc = tile_coord(p, tile);
      int kb0, kb1;
      split_range(p, split, kb0, kb1);
      const int nchunks = (kb1 - kb0 + CHUNK - 1) / CHUNK;
      float acc[COLS];
#pragma unroll
      for (int i = 0; i < COLS; ++i) acc[i] = 0.0f;
      bool ok = true;
      for (int c = 0; c < nchunks; ++c, ++gc) {
        const int buf = (int)(gc & 1);
        ok = mbar_wait(accf0 + 8 * buf, (uint32_t)((gc >> 1) & 1), abort_flag, p.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
#if PB_TF32_LD_PAIR
        // Two 32-column loads in flight per wait.
#pragma unroll
        for (int piece = 0; piece < COLS / 32; piece += 2) {
          uint32_t r0[32], r1[32];
          tmem_ld32x2(lane_base + (uint32_t)(buf * BN + piece * 32),
                      lane_base + (uint32_t)(buf * BN + piece * 32 + 32), r0, r1);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            acc[piece * 32 + i] += __uint_as_float(r0[i]);
            acc[piece * 32 + 32 + i] += __uint_as_float(r1[i]);
          }
        }
#else
#pragma unroll
        for (int piece = 0; piece < COLS / 32; ++piece) {
          uint32_t r[32];
          tmem_ld32(lane_base + (uint32_t)(buf * BN + piece * 32), r);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[piece * 32 + i] += __uint_as_float(r[i]);
        }
#endif
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(acce0 + 8 * buf);
      }
      if (!ok || *abort_flag) break;
      finish_item<COLS>(p, tc, split, tc.m_tile * BM + quad * 32 + lane,
                        tc.n_tile * BN + half * COLS, acc);
    }
  }

  // Every issued MMA has been consumed by an accumulator warp (or the run was
  // aborted); make sure the MMAs have landed before TMEM is released.
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (*abort_flag) {
      // Bounded wait for the last committed chunk of each buffer.
      const uint64_t t0 = globaltimer();
      while (globaltimer() - t0 < 1000000ull) {
      }
    }
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS));
  }
}

// ------------------------------------------ GEMM with A split into TMEM --
//
// Variant used when A's rows are 16-byte aligned (K % 4 == 0): A is loaded
// raw by TMA, and each 128 x 32 slice is split into hi/lo by the eight
// accumulator warps straight into tensor memory, from where the MMAs read it
// (A operand in TMEM, B in shared memory).  A's bytes cross HBM and L2 once;
// shared memory holds only what TMA delivers (raw A and the pre-split B
// [hi | lo], K-major), so FBN = 128 fits 4 stages and FBN = 64 fits 6.
// Per slice the MMA thread issues lo*hi, hi*lo, hi*hi (small terms first)
// into the TMEM accumulator, promoted to fp32 registers every FCHUNK slices
// (36 MMA steps).
// Warps: 0 TMA producer, 1 MMA issuer, 2..5 split A (warp w owns the 32 rows
// at TMEM lanes 32*(w%4).. of every slice), 6..13 promote and store (warp w
// owns the same lanes and column half (w-6)/4 of the accumulator).  With
// the epilogue on warps of its own, the split never waits for a tile's
// stores, so the tensor pipe keeps a full queue across tile boundaries.
// TMEM columns: accumulators [0, 2*FBN), then for stage s A hi at
// 2*FBN + 64*s and A lo 32 columns further.  A stage's A columns are free
// once its full barrier fires: the TMA for slice g is only issued after the
// MMAs of slice g - STAGES (the previous user of the columns) completed.

#ifndef PB_TF32_WIDE
#define PB_TF32_WIDE 1  // 0: no 128 x 192 tiles (measurement builds)
#endif
#ifndef PB_TF32_FCHUNK
#define PB_TF32_FCHUNK 3
#endif
constexpr int FCHUNK = PB_TF32_FCHUNK;
constexpr int T_SPLIT_WARPS = 4, T_ACC_WARPS = 8;

// Warp roles by tile width.  FBN = 64: 14 warps (TMA, MMA, split 2..5,
// promote/store 6..13) at the 128 registers a thread that 14 warps leave (the
// register file is split over the SM's four sub-partitions).  FBN = 128 / 192:
// the promote warps hold 64 / 96 running sums each plus the accumulator
// columns in flight, so 16 warps are launched at 128 registers as four warp
// groups -- {TMA, MMA, two idle}, {split x4}, {promote/store x4} x 2 -- and
// after set-up the first two groups give registers up for the last two
// (setmaxnreg): 64 + 96 + 176 + 176 = 512 = 4 x 128, so the increase is
// always available.
template <int FBN>
struct TRoles {
  static constexpr bool kRegs = PB_TF32_PROMOTE_BATCH ? FBN >= 128 : FBN == 192;
  static constexpr int SPLIT0 = kRegs ? 4 : 2;        // first A-split warp
  static constexpr int ACC0 = SPLIT0 + T_SPLIT_WARPS;  // first promote/store warp
  static constexpr int THREADS = 32 * (ACC0 + T_ACC_WARPS);
  static constexpr int REG_CTRL = 64, REG_SPLIT = 96, REG_ACC = 176;
  static_assert(!kRegs || (THREADS == 512 && REG_CTRL + REG_SPLIT + 2 * REG_ACC <= 4 * 128),
                "register reallocation must fit the launch's 512 x 128 registers");
};

template <int FBN>
struct TSmem {
  static constexpr int A_BYTES = BM * BK * 4;   // 16 KiB raw A slice
  static constexpr int B_BYTES = FBN * BK * 4;  // B hi or B lo slice
  static constexpr int A = 0, BHI = A_BYTES, BLO = A_BYTES + B_BYTES;
  static constexpr int STAGE = A_BYTES + 2 * B_BYTES;
  static constexpr int STAGES = FBN == 192 ? 3 : FBN == 128 ? 4 : 6;
  // A hi/lo buffers in tensor memory.  At FBN = 192 the two accumulators take
  // 384 of the 512 columns, so only two slices' A parts fit: those buffers
  // cycle on their own (the split of slice g waits for the MMAs of slice
  // g - TST), decoupled from the shared-memory ring.
  static constexpr int TST = FBN == 192 ? 2 : STAGES;
  // Epilogue staging: a 32 x 32 fp32 box (4 KiB, 128-byte swizzle) per warp.
  static constexpr int OUT = STAGES * STAGE, OUT_BYTES = T_ACC_WARPS * 4096;
  static constexpr int TOTAL = OUT + OUT_BYTES + 1024 + 256;
  static constexpr uint32_t ACOL = 2 * FBN;     // first A column in TMEM
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(ACOL + 64 * TST <= TMEM_COLS, "TMEM columns");
  static_assert(8 * (3 * STAGES + 6) + 8 <= 256, "barrier area");
};

// hi = round-to-nearest tf32 of x (ties away), lo = tf32(x - hi), in
// integer arithmetic (off the slower conversion pipe) and without branches.
// A non-finite x gives hi = x and lo = NaN, and a magnitude within 2^-12 of
// FLT_MAX rounds hi up to Inf: both make every output they touch non-finite,
// and the epilogue recomputes those.
__device__ __forceinline__ void split_bits(float x, uint32_t& hi, uint32_t& lo) {
  const uint32_t b = __float_as_uint(x);
  hi = (b + 0x1000u) & 0xffffe000u;
  lo = (__float_as_uint(x - __uint_as_float(hi)) + 0x1000u) & 0xffffe000u;
}

// Warp-group register reallocation (every warp of the group executes it).
template <int N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// D (TMEM) += A (TMEM, 128 lanes x 8 columns at tmem_a) * B (smem descriptor).
__device__ __forceinline__ void umma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate));
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// Epilogue of one work item through the output tensor map: the warp's 32
// rows x COLS columns go out as COLS/32 boxes of 32 x 32, staged in the warp's
// 4 KiB buffer with the 128-byte swizzle (16-byte chunk j of row r at j ^ r%8)
// and stored by lane 0 with cp.async.bulk.tensor; rows past M and columns
// past N are clipped by the map.  With K split, the box goes to the split's
// partial plane (z = split * batch + bz).  Flagged outputs are recomputed after
// the warp's stores complete.
template <int COLS>
// `boxes_room`: staging buffers of 4 KiB at `stage` (1, or COLS/32 when the
// CTA's operand ring is idle -- its last work item): with one, each box
// waits for the previous one to leave the buffer; with one per box, all
// boxes are staged first and stored back to back.
__device__ __forceinline__ void store_tma(const Tf32Params& p, const CUtensorMap* map_c,
                                          const TileCoord& tc, int split, int quad, int64_t col0,
                                          const float (&acc)[COLS], float4* stage,
                                          uint32_t stage_u32, bool boxes_room = false) {
  const int lane = threadIdx.x & 31;
  const int64_t row = tc.m_tile * BM + quad * 32 + lane;
  const int64_t batch = p.batch;
  const int32_t z = (int32_t)(p.ksplit > 1 ? split * batch + tc.bz : tc.bz);
  // The launch's tag word, read before the staging work so its L2 round trip
  // overlaps it.
  const unsigned int any = p.ksplit == 1 ? __ldcg(p.tagany) : 0u;
  bool bad = false;
  if (p.ksplit == 1 && row < p.M) {
#pragma unroll
    for (int j = 0; j < COLS; ++j) bad |= nonfinite(acc[j]);
  }
#pragma unroll
  for (int c = 0; c < COLS / 32; ++c) {
    float4* box = boxes_room ? stage + c * 256 : stage;  // 256 float4 = 4 KiB
    const uint32_t box_u32 = boxes_room ? stage_u32 + c * 4096u : stage_u32;
    if (!boxes_room) {
      if (lane == 0) bulk_wait_read();  // the previous box has left the buffer
      __syncwarp();
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      box[lane * 8 + (j ^ (lane & 7))] =
          make_float4(acc[c * 32 + 4 * j], acc[c * 32 + 4 * j + 1], acc[c * 32 + 4 * j + 2],
                      acc[c * 32 + 4 * j + 3]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0)
      tma_store_3d(map_c, box_u32, (int32_t)(col0 + c * 32), (int32_t)(tc.m_tile * BM + quad * 32),
                   z);
  }
  if (p.ksplit > 1) return;
  if (row < p.M && any == p.gen) bad |= tagged<COLS>(p, tc.bz, row, col0);
  if (__any_sync(0xffffffffu, bad)) {
    if (lane == 0) bulk_wait_all();
    __syncwarp();
    if (bad) handle_nonfinite(p, tc.bz, row, col0, COLS);
  }
}

template <int FBN>
__global__ void __launch_bounds__(TRoles<FBN>::THREADS, 1)
    tf32x3_tmem_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_c, Tf32Params p, int Kp) {
  using L = TSmem<FBN>;
  using R = TRoles<FBN>;
  constexpr int S = L::STAGES;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + L::OUT + L::OUT_BYTES;
  uint64_t* bar_ptr = reinterpret_cast<uint64_t*>(gbase + L::OUT + L::OUT_BYTES);
  // full[S] (TMA landed), ready[S] (A split into TMEM), empty[S] (MMAs done), accf[2], acce[2]
  const uint32_t full0 = bars, ready0 = bars + 8 * S, empty0 = bars + 16 * S;
  const uint32_t accf0 = bars + 24 * S, acce0 = accf0 + 16;
  // tfree[TST] (MMAs of the slice done with a TMEM A buffer; used when TST < S)
  constexpr int TS = L::TST;
  constexpr bool kTfree = TS < S;
  const uint32_t tfree0 = acce0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ptr + 3 * S + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(ready0 + 8 * s, T_SPLIT_WARPS);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, T_ACC_WARPS);
    }
    if (kTfree)
      for (int t = 0; t < TS; ++t) mbar_init(tfree0 + 8 * t, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (PB_TF32_WARM) {
      prefetch_map(&map_a);
      prefetch_map(&map_b);
      if (p.tma_store) prefetch_map(&map_c);
    }
  }
  if (PB_TF32_WARM && warp == 2 && lane == 0) warm_params(p, abort_flag + 1);
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(L::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int64_t items = p.tiles * p.ksplit;
  // Launched as a programmatic dependent of the split pass.  Each role waits
  // for the preceding grid (griddepcontrol.wait) only right before its first
  // access to memory that grid may write -- the producer before its first TMA
  // load, the promote/store warps before their first global access, the split
  // warps before writing a tag -- so the set-up and the first work item's
  // bookkeeping (about 2 us when cold) overlap the preceding grid's tail.  The
  // next launch (split reduction or repair) may be scheduled from now on; it
  // waits for this grid in turn.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if constexpr (R::kRegs) reg_dealloc<R::REG_CTRL>();
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int64_t g = 0;
      for (int64_t w = blockIdx.x; w < items && !*abort_flag; w += gridDim.x) {
        int64_t tile;
        int split;
        item_of(p, w, tile, split);
        const TileCoord tc = tile_coord(p, tile);
        int kb0, kb1;
        split_range(p, split, kb0, kb1);
        int64_t ao, bo;
        batch_offsets(p.map, tc.bz, &ao, &bo);
        const int32_t a_row = (int32_t)(ao * p.M + tc.m_tile * BM);
        const int32_t b_row = (int32_t)(bo * p.N + tc.n_tile * FBN);
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = (int)(g % S);
          if (!mbar_wait(empty0 + 8 * s, (uint32_t)(((g / S) & 1) ^ 1), abort_flag, p.err)) break;
          const uint32_t st = base + s * L::STAGE;
          if (g == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
          mbar_expect_tx(full0 + 8 * s, L::STAGE);
          tma_load_2d(st + L::A, &map_a, kb * BK, a_row, full0 + 8 * s);
          tma_load_2d(st + L::BHI, &map_b, kb * BK, b_row, full0 + 8 * s);
          tma_load_2d(st + L::BLO, &map_b, Kp + kb * BK, b_row, full0 + 8 * s);
        }
      }
      if (*abort_flag) {
        for (int64_t q = (g > S ? g - S : 0); q < g; ++q) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(full0 + 8 * (int)(q % S), (uint32_t)((q / S) & 1)) &&
                 globaltimer() - t0 < kTimeoutNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if constexpr (R::kRegs) reg_dealloc<R::REG_CTRL>();
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = instr_desc(FBN);
      int64_t g = 0, gc = 0;
      bool ok = true;
      for (int64_t w = blockIdx.x; w < items && ok; w += gridDim.x) {
        int64_t tile;
        int split;
        item_of(p, w, tile, split);
        int kb0, kb1;
        split_range(p, split, kb0, kb1);
        const int nchunks = (kb1 - kb0 + FCHUNK - 1) / FCHUNK;
        for (int c = 0; c < nchunks && ok; ++c, ++gc) {
          const int buf = (int)(gc & 1);
          ok = mbar_wait(acce0 + 8 * buf, (uint32_t)(((gc >> 1) & 1) ^ 1), abort_flag, p.err);
          if (!ok) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t d = tmem + (uint32_t)(buf * FBN);
          const int kb_start = kb0 + c * FCHUNK;
          const int kb_end = min(kb1, kb_start + FCHUNK);
          for (int kb = kb_start; kb < kb_end; ++kb, ++g) {
            const int s = (int)(g % S);
            ok = mbar_wait(ready0 + 8 * s, (uint32_t)((g / S) & 1), abort_flag, p.err);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t st = base + s * L::STAGE;
            const uint32_t ahi = tmem + L::ACOL + 64u * (uint32_t)(g % TS), alo = ahi + 32u;
            const uint64_t bhi = smem_desc(st + L::BHI), blo = smem_desc(st + L::BLO);
            const bool first = kb == kb_start;
#pragma unroll
            for (int k = 0; k < BK / 8; ++k)
              umma_tf32_ts(d, alo + 8 * k, bhi + 2 * k, idesc, (!first || k > 0) ? 1u : 0u);
#pragma unroll
            for (int k = 0; k < BK / 8; ++k) umma_tf32_ts(d, ahi + 8 * k, blo + 2 * k, idesc, 1u);
#pragma unroll
            for (int k = 0; k < BK / 8; ++k) umma_tf32_ts(d, ahi + 8 * k, bhi + 2 * k, idesc, 1u);
            umma_commit(empty0 + 8 * s);
            if (kTfree) umma_commit(tfree0 + 8 * (int)(g % TS));
          }
          umma_commit(accf0 + 8 * buf);
        }
      }
    }
  } else if (warp >= R::SPLIT0 && warp < R::ACC0) {
    // ----------------------------------- split A (warps 2..5, or 4..7)
    if constexpr (R::kRegs) reg_dealloc<R::REG_SPLIT>();
    // Each lane splits its row of every landed A slice (32 values) into the
    // stage's hi and lo columns of its TMEM lane.
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // row of the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    int64_t g = 0;
    bool ok = true;
    for (int64_t w = blockIdx.x; w < items && ok; w += gridDim.x) {
      int64_t tile;
      int split;
      item_of(p, w, tile, split);
      const TileCoord tc = tile_coord(p, tile);
      int kb0, kb1;
      split_range(p, split, kb0, kb1);
      int64_t ao, bo;
      batch_offsets(p.map, tc.bz, &ao, &bo);
      const int64_t arow = ao * p.M + tc.m_tile * BM + row;  // row of A over all matrices
      for (int kb = kb0; kb < kb1; ++kb, ++g) {
        const int s = (int)(g % S);
        bool got = mbar_wait(full0 + 8 * s, (uint32_t)((g / S) & 1), abort_flag, p.err);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        // Split the landed slice into registers first: only the TMEM stores
        // wait for the buffer, so the loads and arithmetic stay out of the
        // chain "MMAs of slice g - TS done -> split g -> MMAs of g".
        // This lane's row is 128 bytes; the 128-byte swizzle stores its 16-byte
        // chunk j at position j ^ (row % 8).
        const float4* src = reinterpret_cast<const float4*>(gbase + s * L::STAGE + L::A + row * 128);
        const int t = (int)(g % TS);
        if (kTfree && !PB_TF32_SPLIT_EARLY) {
          got = mbar_wait(tfree0 + 8 * t, (uint32_t)(((g / TS) & 1) ^ 1), abort_flag, p.err);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
        }
        float amin = FLT_MAX;  // smallest magnitude of the row's 32 values (NaN ignored)
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 v = src[q ^ (row & 7)];
          split_bits(v.x, hi[4 * q], lo[4 * q]);
          split_bits(v.y, hi[4 * q + 1], lo[4 * q + 1]);
          split_bits(v.z, hi[4 * q + 2], lo[4 * q + 2]);
          split_bits(v.w, hi[4 * q + 3], lo[4 * q + 3]);
          amin = fminf(amin, fminf(fminf(fabsf(v.x), fabsf(v.y)), fminf(fabsf(v.z), fabsf(v.w))));
        }
        // The TMEM buffer of this slice was last read by the MMAs of slice
        // g - TS (with TS == S the full barrier above already implies it).
        if (kTfree && PB_TF32_SPLIT_EARLY) {
          got = mbar_wait(tfree0 + 8 * t, (uint32_t)(((g / TS) & 1) ^ 1), abort_flag, p.err);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acol = tmem + lane_off + L::ACOL + 64u * (uint32_t)t;
        __syncwarp();  // converged for the .aligned TMEM stores
        tmem_st32(acol, hi);
        tmem_st32(acol + 32u, lo);
        if (amin < kTinyMag) {
          // A zero or tiny value: tag the row if one of the 32 is tiny.
          bool tagged_row = false;
#pragma unroll
          for (int t8 = 0; t8 < 8; ++t8) {
            const float4 v = src[t8 ^ (row & 7)];
            tagged_row |= tiny(v.x) | tiny(v.y) | tiny(v.z) | tiny(v.w);
          }
          if (tagged_row) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            p.rowtag[arow] = p.gen;
            p.tagany[0] = p.gen;
            __threadfence();
          }
        }
        __syncwarp();
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(ready0 + 8 * s);
      }
    }
  } else if (warp >= R::ACC0) {
    // ------------------- promote and store (warps 6..13, or 8..15)
    if constexpr (R::kRegs) reg_alloc<R::REG_ACC>();
    asm volatile("griddepcontrol.wait;" ::: "memory");  // before any global access
    // Every FCHUNK slices the MMA thread commits a chunk of the tile into one
    // of the two TMEM accumulators; these warps add it into fp32 registers,
    // free the accumulator, and at the end of the work item store the tile.
    constexpr int COLS = FBN / 2;
    const int quad = warp & 3;
    const int half = (warp - R::ACC0) >> 2;
    const int row = quad * 32 + lane;  // row of the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t acc_base = tmem + lane_off + (uint32_t)(half * COLS);
    int64_t gc = 0;
    bool ok = true;
    float acc[COLS];

    auto promote = [&](bool first) {
      const int buf = (int)(gc & 1);
      const bool got = mbar_wait(accf0 + 8 * buf, (uint32_t)((gc >> 1) & 1), abort_flag, p.err);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        return;
      }
      // Several loads in flight per wait: each wait is a full round trip
      // through tensor memory, slowed by the MMAs' own traffic there, and the
      // next chunk's MMAs wait for this buffer.  With the registers moved to
      // these warps (TRoles::kRegs): 64 columns per wait (two 32-column
      // loads) for 64 running sums, 48 (three 16-column loads) for 96; else
      // one 32-column load per wait.
      constexpr int PIECE = !PB_TF32_PROMOTE_BATCH ? (COLS > 64 ? 16 : 32)
                            : COLS == 96 ? 48 : (COLS == 64 && R::kRegs) ? 64 : 32;
#pragma unroll
      for (int piece = 0; piece < COLS / PIECE; ++piece) {
        uint32_t r[PIECE];
        const uint32_t ta = acc_base + (uint32_t)(buf * FBN + piece * PIECE);
        if constexpr (PIECE == 16) {
          tmem_ld16(ta, r);
        } else if constexpr (PIECE == 48) {
          tmem_ld16x3(ta, r);
        } else if constexpr (PIECE == 64) {
          uint32_t (&lo32)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
          uint32_t (&hi32)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
          tmem_ld32x2(ta, ta + 32u, lo32, hi32);
        } else {
          tmem_ld32(ta, r);
        }
#pragma unroll
        for (int i = 0; i < PIECE; ++i)
          acc[piece * PIECE + i] =
              first ? __uint_as_float(r[i]) : acc[piece * PIECE + i] + __uint_as_float(r[i]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * buf);
      ++gc;
    };

    for (int64_t w = blockIdx.x; w < items && ok; w += gridDim.x) {
      int64_t tile;
      int split;
      item_of(p, w, tile, split);
      int kb0, kb1;
      split_range(p, split, kb0, kb1);
      const int nchunks = (kb1 - kb0 + FCHUNK - 1) / FCHUNK;
      for (int c = 0; c < nchunks && ok; ++c) promote(c == 0);
      if (!ok || *abort_flag) break;
      const TileCoord tc = tile_coord(p, tile);
      const int64_t col0 = tc.n_tile * FBN + half * COLS;
      if (p.tma_store)
      {
        // The CTA's last work item: no TMA load is outstanding and every MMA
        // has completed (the last chunk's commit covers them all), so the
        // operand ring can stage all of this warp's boxes.
        const bool last = w + (int64_t)gridDim.x >= items;
        const uint32_t off = last ? (uint32_t)((warp - R::ACC0) * (COLS / 32) * 4096)
                                  : (uint32_t)(L::OUT + (warp - R::ACC0) * 4096);
        static_assert(T_ACC_WARPS * (COLS / 32) * 4096 <= L::OUT, "ring holds every box");
        store_tma<COLS>(p, &map_c, tc, split, quad, col0, acc,
                        reinterpret_cast<float4*>(gbase + off), base + off, last);
      }
      else
        finish_item<COLS>(p, tc, split, tc.m_tile * BM + row, col0, acc);
    }
    if (lane == 0) bulk_wait_all();  // staging buffers are read before the CTA exits
  } else {
    // Warps 2 and 3 of the first warp group (FBN = 192) have no role; they
    // give their registers up with the group.
    if constexpr (R::kRegs) reg_dealloc<R::REG_CTRL>();
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (*abort_flag) {
      const uint64_t t0 = globaltimer();
      while (globaltimer() - t0 < 1000000ull) {
      }
    }
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(L::TMEM_COLS));
  }
}

// C = sum over splits of the partial tiles, in split order (deterministic);
// flagged outputs (non-finite, or touching a tagged operand) are recomputed.
__global__ void splitk_reduce_kernel(const Tf32Params p, int64_t count) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the GEMM's partial tiles
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const bool tags = __ldcg(p.tagany) == p.gen;
  auto check = [&](int64_t i, float v) {
    const int64_t bz = i / (p.M * p.N), r = i % (p.M * p.N);
    if (nonfinite(v) || (tags && tagged<1>(p, bz, r / p.N, r % p.N)))
      handle_nonfinite(p, bz, r / p.N, r % p.N, 1);
  };
  if ((count & 3) == 0) {
    const int64_t n4 = count / 4;
    const float4* p4 = reinterpret_cast<const float4*>(p.partial);
    float4* c4 = reinterpret_cast<float4*>(p.C);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
      float4 s = p4[i];
      for (int k = 1; k < p.ksplit; ++k) {
        const float4 v = p4[k * n4 + i];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      c4[i] = s;
      if (tags || nonfinite(s.x) || nonfinite(s.y) || nonfinite(s.z) || nonfinite(s.w)) {
        check(4 * i, s.x);
        check(4 * i + 1, s.y);
        check(4 * i + 2, s.z);
        check(4 * i + 3, s.w);
      }
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
      float s = p.partial[i];
      for (int k = 1; k < p.ksplit; ++k) s += p.partial[k * count + i];
      p.C[i] = s;
      check(i, s);
    }
  }
}

// Launch as a programmatic dependent of the previous kernel on the stream: it
// may be scheduled before that kernel finishes and must execute
// griddepcontrol.wait before reading anything the previous kernel wrote.
template <typename... Params, typename... Args>
int launch_dependent(Device* d, void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = d->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PB_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  PB_LAUNCHED(d);
  return PB_OK;
}

int launch_reduce(Device* d, const Tf32Params& p, int64_t count) {
  int64_t blocks = ceil_div(count / 4 + 1, (int64_t)256);
  const int64_t cap = (int64_t)d->sm_count * 8;
  if (blocks > cap) blocks = cap;
  return launch_dependent(d, splitk_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, p, count);
}

// Output planes (z x rows x cols, row-major) stored in 32 x 32 boxes with the
// 128-byte swizzle.  Needs cols % 4 == 0 (16-byte row pitch) and a 16-byte
// aligned base.
int encode_out(CUtensorMap* map, float* ptr, int64_t z, int64_t rows, int64_t cols) {
  void* fn;
  PB_CHECK(tensor_map_encoder(&fn));
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)z};
  cuuint64_t strides[2] = {(cuuint64_t)cols * sizeof(float), (cuuint64_t)(rows * cols) * sizeof(float)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)ptr, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) PB_FAIL(PB_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return PB_OK;
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
  PB_CHECK(allow_smem(d, (const void*)tf32x3_gemm_kernel<BN>, smem));
  // Persistent: one CTA per SM (shared memory allows no more), work items strided.
  const int64_t items = p.tiles * p.ksplit;
  const int64_t grid = items < d->sm_count ? items : d->sm_count;
  PB_CHECK(kt_begin(d));
  PB_CHECK(launch_dependent(d, tf32x3_gemm_kernel<BN>, dim3((unsigned)grid), dim3(GEMM_THREADS),
                            (size_t)smem, ma, mb, p));
  return kt_end(d);
}

// Operands and non-finite handling of a launch (after p.ksplit is set); the
// tile marks of the repair launch live in the zeroed counter words.
int finish_setup(Device* d, Tf32Params& p, int64_t batch, int64_t M, int64_t N, int64_t K,
                 const float* A, const float* B) {
  p.A = A;
  p.B = B;
  p.K = K;
  p.batch = batch;
  p.fd_ksplit = make_fastdiv(p.ksplit);
  p.fd_tiles = make_fastdiv((int64_t)p.tiles_m * p.tiles_n);
  p.fd_group = make_fastdiv((int64_t)GM * p.tiles_n);
  p.fd_gm_last = make_fastdiv(p.tiles_m % GM ? p.tiles_m % GM : GM);
  p.repair_inline = K <= (p.ksplit > 1 ? kReduceRepairMaxK : kInlineRepairMaxK);
  p.nf_tm = ceil_div(M, (int64_t)kNonFiniteTile);
  p.nf_tn = ceil_div(N, (int64_t)kNonFiniteTile);
  PB_CHECK(counters(d, 2 + (size_t)(batch * p.nf_tm * p.nf_tn), &p.nf));
  return PB_OK;
}

// Operand tag words of a launch: the any word, rows of A, then column groups
// of each B.
int tag_setup(Device* d, Tf32Params& p, int64_t rows_a, int64_t nB, int64_t N) {
  p.cgroups = ceil_div(N, (int64_t)kTagCols);
  unsigned int* tags;
  PB_CHECK(operand_tags(d, (size_t)(1 + rows_a + nB * p.cgroups), &tags, &p.gen));
  p.tagany = tags;
  p.rowtag = tags + 1;
  p.coltag = tags + 1 + rows_a;
  return PB_OK;
}

int64_t matrices_used(const BatchMap& m, bool a) {
  int64_t last = 0;
  for (int i = 0; i < m.ndim; ++i) last += (m.shape[i] - 1) * (a ? m.a_stride[i] : m.b_stride[i]);
  return last + 1;
}

template <int FBN>
int launch_tmem(Device* d, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                const Tf32Params& p, int64_t Kp) {
  const int smem = TSmem<FBN>::TOTAL;
  PB_CHECK(allow_smem(d, (const void*)tf32x3_tmem_kernel<FBN>, smem));
  const int64_t items = p.tiles * p.ksplit;
  const int64_t grid = items < d->sm_count ? items : d->sm_count;
  PB_CHECK(kt_begin(d));
  PB_CHECK(launch_dependent(d, tf32x3_tmem_kernel<FBN>, dim3((unsigned)grid), dim3(TRoles<FBN>::THREADS),
                            (size_t)smem, ma, mb, mc, p, (int)Kp));
  return kt_end(d);
}

}  // namespace

// 3xTF32 with A split into tensor memory (K % 4 == 0): B -> [hi | lo]
// K-major once, then the TMEM-split kernel (and the split reduction when K
// is split).
int gemm_f32_fused(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                   int64_t Kp, int64_t nA, int64_t nB, const float* A, const float* B, float* C) {
  const int64_t rows_a = nA * M, rows_b = nB * N;
  const size_t bytes_b = (size_t)rows_b * 2 * Kp * sizeof(float);
  const int tiles_m = (int)ceil_div(M, (int64_t)BM);
  // 128-wide tiles (split K when they are few): at 128 x 64 the A split per
  // slice costs as much as the slice's MMAs (1024^3 on B200: 57.0 TFLOP/s
  // against 59.7 with 128 x 128 and a 2-way split).
  // 128 x 192 where it pads N no more than 128 x 128 does (config 3: N = 384
  // = 2 x 192): a third less A splitting per flop and the wider MMA's higher
  // rate (measured back to back: 2806 flop/clk/SM at N = 128, 3799 at 256).
  const int64_t waste128 = ceil_div(N, (int64_t)128) * 128 - N;
  const int64_t waste192 = ceil_div(N, (int64_t)192) * 192 - N;
  const int fbn = N <= 64 ? 64 : (N >= 192 && waste192 <= waste128 && PB_TF32_WIDE) ? 192 : 128;
  const int tiles_n = (int)ceil_div(N, (int64_t)fbn);
  const int64_t tiles = (int64_t)tiles_m * tiles_n * batch;
  const int kblocks = (int)(Kp / BK);
  int ksplit = 1;
  if (tiles < d->sm_count) {
    ksplit = (int)(d->sm_count / tiles);
    const int most = kblocks / (2 * FCHUNK);
    if (ksplit > most) ksplit = most;
    if (ksplit < 1) ksplit = 1;
  }
  const size_t bytes_p = ksplit > 1 ? (size_t)ksplit * batch * M * N * sizeof(float) : 0;
  void* ws;
  PB_CHECK(scratch(d, bytes_b + bytes_p, &ws));
  float* Bt = (float*)ws;
  Tf32Params p;
  p.C = C;
  p.partial = ksplit > 1 ? (float*)((char*)ws + bytes_b) : nullptr;
  p.M = M;
  p.N = N;
  p.kblocks = kblocks;
  p.tiles_m = tiles_m;
  p.tiles_n = tiles_n;
  p.tiles = tiles;
  p.ksplit = ksplit;
  p.map = map;
  p.err = d->err_dev;
  // Everything that may enqueue a memset goes first: the GEMM launch has to
  // follow the split kernel directly (it is that kernel's programmatic
  // dependent).
  PB_CHECK(tag_setup(d, p, rows_a, nB, N));
  PB_CHECK(finish_setup(d, p, batch, M, N, K, A, B));
  CUtensorMap ma, mb, mc;
  PB_CHECK(encode_kmajor(&ma, A, rows_a, K, BM));
  PB_CHECK(encode_kmajor(&mb, Bt, rows_b, 2 * Kp, fbn));
  float* out = ksplit > 1 ? p.partial : C;
  p.tma_store = N % 4 == 0 && ((uintptr_t)out & 15) == 0;
  memset(&mc, 0, sizeof(mc));
  if (p.tma_store) PB_CHECK(encode_out(&mc, out, ksplit * batch, M, N));
  const int64_t gx = ceil_div(N, (int64_t)SPLIT_TN), gy = Kp / SPLIT_TK;
  if (gx > INT32_MAX || gy > 65535 || nB > 65535)
    PB_FAIL(PB_ERR_UNSUPPORTED, "B operand too large for the split grid");
  split_bt_kernel<2><<<dim3((unsigned)gx, (unsigned)gy, (unsigned)nB), 256, 0, d->stream>>>(
      B, Bt, K, N, Kp, p.coltag, p.cgroups, p.tagany, p.gen);
  PB_LAUNCHED(d);
  PB_CHECK(fbn == 192   ? launch_tmem<192>(d, ma, mb, mc, p, Kp)
           : fbn == 128 ? launch_tmem<128>(d, ma, mb, mc, p, Kp)
                        : launch_tmem<64>(d, ma, mb, mc, p, Kp));
  if (ksplit > 1) PB_CHECK(launch_reduce(d, p, batch * M * N));
  if (p.repair_inline) return PB_OK;
  return gemm_nonfinite_repair_f32(d, map, batch, M, N, K, A, B, C, p.nf);
}

// Products with at most this many columns take the kernel that splits A in
// tensor memory.  The pre-split kernel's extra pass over A costs about
// 12*M*K bytes, a share of the GEMM that shrinks as 1/N, while its 256-wide
// tiles (TMEM holds no A slices there) need half the A work per MMA.
// Measured on B200 (effective TFLOP/s, pre-split vs TMEM split): 1024^3 51
// vs 57-60, (8,16)x512x384x256 52 vs 70, 16384x1024x4096 148 vs 199, 2048^3
// 137 vs 141, 4096^3 177 vs 187, 6144^3 210 vs 193, 8192^3 218 vs 195.
#ifndef PB_TF32_FUSED_MAX_N
#define PB_TF32_FUSED_MAX_N 4096
#endif

// algo: 0 auto, 1 SIMT, 2 3xTF32 (kernel by size), 4 pre-split, 5 A split in TMEM.
int gemm_f32_algo(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const float* A, const float* B, float* C, int algo) {
  if (algo == 0) algo = (M >= 64 && N >= 64 && K >= 32) ? 2 : 1;
  if (algo == 1) return gemm_simt_f32(d, map, batch, M, N, K, A, B, C);
  if (algo != PB_GEMM_TF32X3 && algo != PB_GEMM_TF32X3_FUSED && algo != PB_GEMM_TF32X3_PRESPLIT)
    PB_FAIL(PB_ERR_INVALID, "unknown GEMM algorithm %d", algo);

  const int64_t Kp = ceil_div(K, (int64_t)BK) * BK;
  const int64_t K3 = 3 * Kp;
  const int64_t nA = matrices_used(map, true), nB = matrices_used(map, false);
  // Two 3xTF32 kernels: A split in tensor memory (TMA needs 16-byte aligned
  // rows of A: K % 4 == 0) or both operands split in HBM first.
  const bool can_fuse = K % 4 == 0 && (uintptr_t)A % 16 == 0 && nA * M <= INT32_MAX &&
                        nB * N <= INT32_MAX && Kp / BK <= INT32_MAX;
  if (algo == PB_GEMM_TF32X3_FUSED && !can_fuse)
    PB_FAIL(PB_ERR_UNSUPPORTED, "the in-kernel A split needs K %% 4 == 0 and aligned A");
  if (algo == PB_GEMM_TF32X3_FUSED || (algo == PB_GEMM_TF32X3 && can_fuse && N <= PB_TF32_FUSED_MAX_N))
    return gemm_f32_fused(d, map, batch, M, N, K, Kp, nA, nB, A, B, C);
  const int64_t rows_a = nA * M, rows_b = nB * N;
  if (rows_a > INT32_MAX || rows_b > INT32_MAX || K3 / BK > INT32_MAX)
    PB_FAIL(PB_ERR_UNSUPPORTED, "GEMM operand too large for 32-bit TMA coordinates");
  const size_t bytes_a = (size_t)rows_a * K3 * sizeof(float);
  const size_t bytes_b = (size_t)rows_b * K3 * sizeof(float);
  // Tile width: 256 unless 128-wide tiles pad N less (config 3: N = 384).
  const int64_t waste256 = ceil_div(N, (int64_t)256) * 256 - N;
  const int64_t waste128 = ceil_div(N, (int64_t)128) * 128 - N;
  const int BN = (N > 128 && waste256 <= waste128) ? 256 : 128;
  const int tiles_m = (int)ceil_div(M, (int64_t)BM);
  const int64_t tiles = (int64_t)tiles_m * ceil_div(N, (int64_t)BN) * batch;
  const int kblocks = (int)(K3 / BK);
  // Too few tiles to occupy every SM: split K' into ranges of at least two
  // promotion chunks each; fp32 partial tiles summed by a second kernel.
  int ksplit = 1;
  if (tiles < d->sm_count) {
    ksplit = (int)(d->sm_count / tiles);
    const int most = kblocks / (2 * CHUNK);
    if (ksplit > most) ksplit = most;
    if (ksplit < 1) ksplit = 1;
  }
  const size_t bytes_p = ksplit > 1 ? (size_t)ksplit * batch * M * N * sizeof(float) : 0;
  void* ws;
  PB_CHECK(scratch(d, bytes_a + bytes_b + bytes_p, &ws));
  float* Ap = (float*)ws;
  float* Bt = (float*)((char*)ws + bytes_a);
  Tf32Params p;
  p.C = C;
  p.partial = ksplit > 1 ? (float*)((char*)ws + bytes_a + bytes_b) : nullptr;
  p.M = M;
  p.N = N;
  p.kblocks = kblocks;
  p.tiles_m = tiles_m;
  p.tiles_n = (int)ceil_div(N, (int64_t)BN);
  p.tiles = tiles;
  p.ksplit = ksplit;
  p.map = map;
  p.err = d->err_dev;
  p.tma_store = 0;
  // Memsets first: the GEMM is the split kernel's programmatic dependent.
  PB_CHECK(tag_setup(d, p, rows_a, nB, N));
  PB_CHECK(finish_setup(d, p, batch, M, N, K, A, B));
  CUtensorMap ma, mb;
  PB_CHECK(encode_kmajor(&ma, Ap, rows_a, K3, BM));
  PB_CHECK(encode_kmajor(&mb, Bt, rows_b, K3, BN));

  {
    const int64_t total = rows_a * Kp;
    int64_t blocks = ceil_div(total, (int64_t)256);
    const int64_t cap = (int64_t)d->sm_count * 16;
    if (blocks > cap) blocks = cap;
    if (K % 4 == 0 && (uintptr_t)A % 16 == 0 && rows_a * (Kp / 4) < (int64_t(1) << 31)) {
      int64_t b4 = ceil_div(rows_a * (Kp / 4), (int64_t)256);
      if (b4 > cap) b4 = cap;
      split_a4_kernel<<<(unsigned)b4, 256, 0, d->stream>>>(A, Ap, rows_a, K, Kp,
                                                           make_fastdiv(Kp / 4), p.rowtag,
                                                           p.tagany, p.gen);
    } else {
      split_a_kernel<<<(unsigned)blocks, 256, 0, d->stream>>>(A, Ap, rows_a, K, Kp, p.rowtag,
                                                              p.tagany, p.gen);
    }
    PB_LAUNCHED(d);
    const int64_t gx = ceil_div(N, (int64_t)SPLIT_TN), gy = Kp / SPLIT_TK;
    if (gx > INT32_MAX || gy > 65535 || nB > 65535)
      PB_FAIL(PB_ERR_UNSUPPORTED, "B operand too large for the split grid");
    split_bt_kernel<3><<<dim3((unsigned)gx, (unsigned)gy, (unsigned)nB), 256, 0, d->stream>>>(
        B, Bt, K, N, Kp, p.coltag, p.cgroups, p.tagany, p.gen);
    PB_LAUNCHED(d);
  }
  PB_CHECK(BN == 256 ? launch_tf32<256>(d, ma, mb, p) : launch_tf32<128>(d, ma, mb, p));
  if (ksplit > 1) PB_CHECK(launch_reduce(d, p, batch * M * N));
  if (p.repair_inline) return PB_OK;
  return gemm_nonfinite_repair_f32(d, map, batch, M, N, K, A, B, C, p.nf);
}

}  // namespace pb
