// float64 GEMM on the FP64 tensor path (DMMA, mma.sync m16n8k4 .f64; m16n8k8 selectable).
//
// Reference: the custom CUDA provider computes every float64 product with one
// thread per output and a serial K loop (src/openpacho/_cuda.py:619-636); the
// reference's 16x16 shared-tile candidate (benchmarks/cuda_fp64_tile.py:46-97)
// was never promoted (docs/cuda-fp64-gemm-results.md:172-177).
//
// This kernel: 128x128 output tile per 256-thread CTA; 8 warps in a 2 (M) x 4
// (N) grid, each owning 64x32 = 4x4 tiles of m16n8, i.e. 16 DMMA per K-step of
// 4 with 64 float64 accumulators per thread.  K advances in slices of 16 through
// a 4-stage cp.async ring.  Both operands keep their global layout in shared
// memory, so every copy reads consecutive addresses (16-byte copies when K and
// N are even and the bases aligned, else 8-byte): A as [m][k] with a 160-byte
// row pitch, B as [k][n] with a 1056-byte pitch; with those pitches a
// half-warp's fragment load of 16 doubles covers all 32 banks once.  Tails in
// M, N, K are zero-filled by the copies (src-size 0) and masked at the store.
#include "pb_internal.cuh"

namespace pb {
namespace {

// Measured on B200 (8192^3, TFLOP/s, one run each): m16n8k4, TK 16, 4 stages
// 31.9; 5 or 6 stages 31.6; TK 32 with 3 stages 32.4; m16n8k8 31.3 (with B
// transposed in shared memory, before 16-byte copies: 28.5 / 27.9 / 22.2).
#ifndef PB_DMMA_K
#define PB_DMMA_K 4  // DMMA shape m16n8k4 or m16n8k8
#endif
#ifndef PB_DMMA_TK
#define PB_DMMA_TK 16  // K per shared-memory stage
#endif
#ifndef PB_DMMA_STAGES
#define PB_DMMA_STAGES 4
#endif
constexpr int TM = 128, TN = 128, TK = PB_DMMA_TK, PITCH = TK + 4, NSTAGE = PB_DMMA_STAGES, NT = 256;
constexpr int PITCHB = TN + 4;  // B rows [k][n]
static_assert(TK % PB_DMMA_K == 0 && (TM * TK) % (2 * NT) == 0 && (TN * TK) % (2 * NT) == 0,
              "stage shape");
constexpr int STAGE_DOUBLES = TM * PITCH + TK * PITCHB;

struct DmmaParams {
  const double* A;
  const double* B;
  double* C;
  int64_t M, N, K;
  int64_t batch;
  BatchMap map;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// 8-byte asynchronous copy; `bytes` = 0 writes zeros.
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
// 16-byte asynchronous copy (L2 only); `bytes` = 0 writes zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void dmma(double (&c)[4], double a0, double a1, double b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%0,%1,%2,%3};"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a0), "d"(a1), "d"(b0));
}

#if PB_DMMA_K == 8
// m16n8k8: a = (g, t), (g+8, t), (g, t+4), (g+8, t+4); b = (t, g), (t+4, g).
__device__ __forceinline__ void dmma8(double (&c)[4], const double (&a)[4], const double (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}
#endif

template <bool VEC>
__global__ void __launch_bounds__(NT, 1) dmma_gemm_kernel(DmmaParams p) {
  extern __shared__ __align__(16) double smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wm = warp >> 2, wn = warp & 3;  // warp tile origin: (wm*64, wn*32)
  const int64_t m0 = (int64_t)blockIdx.y * TM, n0 = (int64_t)blockIdx.x * TN;
  const int64_t M = p.M, N = p.N, K = p.K;
  const int64_t ktiles = (K + TK - 1) / TK;

  for (int64_t bz = blockIdx.z; bz < p.batch; bz += gridDim.z) {
    int64_t ao, bo;
    batch_offsets(p.map, bz, &ao, &bo);
    const double* A = p.A + ao * M * K;
    const double* B = p.B + bo * K * N;
    double* C = p.C + bz * M * N;

    // Stage loader: A rows of TK doubles (K-contiguous), B rows of TN doubles
    // (N-contiguous); consecutive threads copy consecutive addresses.  With
    // VEC, K and N are even, so a pair never straddles the K or N edge.
    auto load = [&](int64_t kt, int stage) {
      double* sa = smem + stage * STAGE_DOUBLES;
      double* sb = sa + TM * PITCH;
      const int64_t k0 = kt * TK;
      if constexpr (VEC) {
#pragma unroll
        for (int i = 0; i < TM * TK / (2 * NT); ++i) {
          const int idx = i * NT + tid, r = idx / (TK / 2), kk = 2 * (idx % (TK / 2));
          const int64_t gr = m0 + r, gk = k0 + kk;
          const bool ok = gr < M && gk < K;
          cp_async16(smem_u32(sa + r * PITCH + kk), ok ? (const void*)(A + gr * K + gk) : (const void*)A,
                     ok ? 16 : 0);
        }
#pragma unroll
        for (int i = 0; i < TN * TK / (2 * NT); ++i) {
          const int idx = i * NT + tid, kk = idx / (TN / 2), nn = 2 * (idx % (TN / 2));
          const int64_t gk = k0 + kk, gn = n0 + nn;
          const bool ok = gk < K && gn < N;
          cp_async16(smem_u32(sb + kk * PITCHB + nn), ok ? (const void*)(B + gk * N + gn) : (const void*)B,
                     ok ? 16 : 0);
        }
      } else {
#pragma unroll
        for (int i = 0; i < TM * TK / NT; ++i) {
          const int idx = i * NT + tid, r = idx / TK, kk = idx % TK;
          const int64_t gr = m0 + r, gk = k0 + kk;
          const bool ok = gr < M && gk < K;
          cp_async8(smem_u32(sa + r * PITCH + kk), ok ? (const void*)(A + gr * K + gk) : (const void*)A,
                    ok ? 8 : 0);
        }
#pragma unroll
        for (int i = 0; i < TN * TK / NT; ++i) {
          const int idx = i * NT + tid, kk = idx / TN, nn = idx % TN;
          const int64_t gk = k0 + kk, gn = n0 + nn;
          const bool ok = gk < K && gn < N;
          cp_async8(smem_u32(sb + kk * PITCHB + nn), ok ? (const void*)(B + gk * N + gn) : (const void*)B,
                    ok ? 8 : 0);
        }
      }
    };

    double acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.0;

#pragma unroll
    for (int s = 0; s < NSTAGE - 1; ++s) {
      if (s < ktiles) load(s, s);
      cp_async_commit();
    }
    for (int64_t kt = 0; kt < ktiles; ++kt) {
      cp_async_wait<NSTAGE - 2>();
      __syncthreads();
      const int64_t next = kt + NSTAGE - 1;
      if (next < ktiles) load(next, (int)(next % NSTAGE));
      cp_async_commit();
      const double* sa = smem + (kt % NSTAGE) * STAGE_DOUBLES + (wm * 64) * PITCH;
      const double* sb = smem + (kt % NSTAGE) * STAGE_DOUBLES + TM * PITCH + wn * 32;
#if PB_DMMA_K == 8
#pragma unroll
      for (int k8 = 0; k8 < TK; k8 += 8) {
        double a[4][4], b[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[i][0] = sa[(i * 16 + g) * PITCH + k8 + t];
          a[i][1] = sa[(i * 16 + g + 8) * PITCH + k8 + t];
          a[i][2] = sa[(i * 16 + g) * PITCH + k8 + t + 4];
          a[i][3] = sa[(i * 16 + g + 8) * PITCH + k8 + t + 4];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          b[j][0] = sb[(k8 + t) * PITCHB + j * 8 + g];
          b[j][1] = sb[(k8 + t + 4) * PITCHB + j * 8 + g];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) dmma8(acc[i][j], a[i], b[j]);
      }
#else
#pragma unroll
      for (int k4 = 0; k4 < TK; k4 += 4) {
        double a[4][2], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[i][0] = sa[(i * 16 + g) * PITCH + k4 + t];
          a[i][1] = sa[(i * 16 + g + 8) * PITCH + k4 + t];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = sb[(k4 + t) * PITCHB + j * 8 + g];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) dmma(acc[i][j], a[i][0], a[i][1], b[j]);
      }
#endif
    }
    cp_async_wait<0>();
    __syncthreads();

    // Epilogue: fragment element c of tile (i, j) sits at row i*16 + g (+8 for
    // c >= 2), column j*8 + 2t + (c & 1) of the warp tile.
    const bool pairs = (N % 2) == 0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t r = m0 + wm * 64 + i * 16 + g + h * 8;
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t c = n0 + wn * 32 + j * 8 + 2 * t;
          double* dst = C + r * N + c;
          if (pairs && c + 1 < N) {
            *reinterpret_cast<double2*>(dst) = make_double2(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
          } else {
            if (c < N) dst[0] = acc[i][j][2 * h];
            if (c + 1 < N) dst[1] = acc[i][j][2 * h + 1];
          }
        }
      }
  }
}

}  // namespace

int gemm_dmma_f64(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const double* A, const double* B, double* C) {
  DmmaParams p{A, B, C, M, N, K, batch, map};
  const int64_t gx = ceil_div(N, (int64_t)TN), gy = ceil_div(M, (int64_t)TM);
  if (gx > INT32_MAX || gy > 65535) PB_FAIL(PB_ERR_UNSUPPORTED, "GEMM grid too large");
  const unsigned gz = (unsigned)(batch < 65535 ? batch : 65535);
  const int smem = NSTAGE * STAGE_DOUBLES * (int)sizeof(double);
  // 16-byte copies need even K and N (rows of 16-byte multiples) and aligned bases.
  const bool vec = K % 2 == 0 && N % 2 == 0 && ((uintptr_t)A & 15) == 0 && ((uintptr_t)B & 15) == 0;
  auto kernel = vec ? dmma_gemm_kernel<true> : dmma_gemm_kernel<false>;
  PB_CHECK(allow_smem(d, (const void*)kernel, smem));
  PB_CHECK(kt_begin(d));
  kernel<<<dim3((unsigned)gx, (unsigned)gy, gz), NT, smem, d->stream>>>(p);
  PB_LAUNCHED(d);
  return kt_end(d);
}

}  // namespace pb
