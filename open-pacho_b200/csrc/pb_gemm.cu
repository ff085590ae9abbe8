// pb_gemm: validation, broadcast batch map and kernel selection by dtype/shape.
//
// Reference routing: CUDABackend.matmul (src/openpacho/_cuda.py:493-637):
// K == 0 -> zeros; float32 tiles -> register GEMM; everything else a direct
// kernel or cuBLAS.  Here: K == 0 -> zeros; at most 8 rows (vector @ matrix
// and the like) -> the skinny kernel, one pass over B; float64 -> DMMA
// tensor-core tiles; float32 -> 3xTF32 tcgen05 when the output has at least
// one 64x64 block and K >= 32, else the float32 SIMT tile kernel.
#include "pb_internal.cuh"

namespace pb {

int gemm_f32_algo(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const float* A, const float* B, float* C, int algo);
int gemm_simt_f64(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const double* A, const double* B, double* C);
int gemm_dmma_f64(Device* d, const BatchMap& map, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const double* A, const double* B, double* C);
int gemm_skinny(Device* d, int dtype, const BatchMap& map, int64_t batch, int64_t M, int64_t N,
                int64_t K, const void* A, const void* B, void* C);

static int build_map(int batch_ndim, const int64_t* shape, const int64_t* as, const int64_t* bs,
                     BatchMap* map, int64_t* batch) {
  if (batch_ndim < 0 || batch_ndim > 8) PB_FAIL(PB_ERR_UNSUPPORTED, "at most 8 batch dimensions");
  if (batch_ndim && (!shape || !as || !bs)) PB_FAIL(PB_ERR_INVALID, "null batch description");
  map->ndim = batch_ndim;
  int64_t b = 1;
  for (int i = 0; i < batch_ndim; ++i) {
    if (shape[i] < 0 || as[i] < 0 || bs[i] < 0) PB_FAIL(PB_ERR_INVALID, "negative batch extent");
    map->shape[i] = shape[i];
    map->a_stride[i] = as[i];
    map->b_stride[i] = bs[i];
    map->div[i] = make_fastdiv(shape[i]);
    b *= shape[i];
  }
  *batch = b;
  return PB_OK;
}

int gemm_dispatch(pb_ctx* ctx, int dev, int dtype, int batch_ndim, const int64_t* batch_shape,
                  const int64_t* a_bstride, const int64_t* b_bstride, int64_t M, int64_t N,
                  int64_t K, const void* A, const void* B, void* C, int algo) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (dtype != PB_F32 && dtype != PB_F64) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  if (M < 0 || N < 0 || K < 0) PB_FAIL(PB_ERR_INVALID, "negative GEMM extent");
  BatchMap map;
  int64_t batch;
  PB_CHECK(build_map(batch_ndim, batch_shape, a_bstride, b_bstride, &map, &batch));
  const int64_t count = batch * M * N;
  if (!count) return PB_OK;
  if (!C) PB_FAIL(PB_ERR_INVALID, "null output");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!K) return fill_device(d, dtype, C, (size_t)count, 0.0);
  if (!A || !B) PB_FAIL(PB_ERR_INVALID, "null input");
  if (algo == PB_GEMM_SKINNY || (algo == PB_GEMM_AUTO && M <= 8)) {
    if (M > 8) PB_FAIL(PB_ERR_UNSUPPORTED, "the skinny kernel takes at most 8 rows");
    return gemm_skinny(d, dtype, map, batch, M, N, K, A, B, C);
  }
  if (dtype == PB_F64) {
    if (algo == PB_GEMM_SIMT)
      return gemm_simt_f64(d, map, batch, M, N, K, (const double*)A, (const double*)B, (double*)C);
    if (algo == PB_GEMM_AUTO || algo == PB_GEMM_DMMA)
      return gemm_dmma_f64(d, map, batch, M, N, K, (const double*)A, (const double*)B, (double*)C);
    PB_FAIL(PB_ERR_UNSUPPORTED, "float64 GEMM runs on the DMMA or the DFMA (SIMT) kernel");
  }
  if (algo == PB_GEMM_DMMA) PB_FAIL(PB_ERR_UNSUPPORTED, "DMMA is the float64 kernel");
  return gemm_f32_algo(d, map, batch, M, N, K, (const float*)A, (const float*)B, (float*)C, algo);
}

}  // namespace pb

extern "C" {

int pb_gemm(pb_ctx* ctx, int dev, int dtype, int batch_ndim, const int64_t* batch_shape,
            const int64_t* a_bstride, const int64_t* b_bstride, int64_t M, int64_t N, int64_t K,
            const void* A, const void* B, void* C) {
  return pb::gemm_dispatch(ctx, dev, dtype, batch_ndim, batch_shape, a_bstride, b_bstride, M, N,
                           K, A, B, C, 0);
}

int pb_gemm_ex(pb_ctx* ctx, int dev, int dtype, int batch_ndim, const int64_t* batch_shape,
               const int64_t* a_bstride, const int64_t* b_bstride, int64_t M, int64_t N,
               int64_t K, const void* A, const void* B, void* C, int algo) {
  return pb::gemm_dispatch(ctx, dev, dtype, batch_ndim, batch_shape, a_bstride, b_bstride, M, N,
                           K, A, B, C, algo);
}

}  // extern "C"
