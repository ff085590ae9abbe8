// pb_gemm_host: a product whose operands and result are in host memory,
// with the copies overlapped with each other and with the GEMM.
//
// The reference's CUDA backend uploads the operands, multiplies and
// downloads the result one step after another (CUDABackend.upload / matmul /
// download, src/openpacho/_cuda.py:241-281, 493-517); its benchmarks time
// exactly that sequence (src/openpacho/cli.py:54-72).  Here the product is cut
// into chunks along the leading batch dimension (or the rows of A): chunk i's
// A goes up on one copy stream while chunk i-1 multiplies on the device
// stream and chunk i-2's C comes down on a third, so the host link carries
// both directions at once and the GEMM hides behind them.
#include "pb_internal.cuh"

namespace pb {
namespace {

int host_streams(Device* d, size_t events) {
  if (!d->up) PB_CUDA(cudaStreamCreateWithFlags(&d->up, cudaStreamNonBlocking));
  if (!d->down) PB_CUDA(cudaStreamCreateWithFlags(&d->down, cudaStreamNonBlocking));
  while (d->host_events.size() < events) {
    cudaEvent_t e;
    PB_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    d->host_events.push_back(e);
  }
  return PB_OK;
}

// True when an operand's matrices are laid out densely in C order over its
// own (unbroadcast) batch dimensions and it is batched along `lead`: then its
// matrices for index l of dimension `lead` (all earlier extents being 1) are
// [l * st[lead], (l + 1) * st[lead]).
bool dense_along(int nd, const int64_t* shape, const int64_t* st, int lead) {
  int64_t expect = 1;
  for (int j = nd - 1; j >= 0; --j) {
    if (st[j] == 0 || shape[j] == 1) continue;
    if (st[j] != expect) return false;
    expect *= shape[j];
  }
  return st[lead] != 0;
}

}  // namespace
}  // namespace pb

extern "C" {

int pb_gemm_host(pb_ctx* ctx, int dev, int dtype, int batch_ndim, const int64_t* batch_shape,
                 const int64_t* a_bstride, const int64_t* b_bstride, int64_t M, int64_t N,
                 int64_t K, const void* A, const void* B, void* C, int chunks) {
  using namespace pb;
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (dtype != PB_F32 && dtype != PB_F64) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  if (M < 0 || N < 0 || K < 0) PB_FAIL(PB_ERR_INVALID, "negative GEMM extent");
  if (batch_ndim < 0 || batch_ndim > 8) PB_FAIL(PB_ERR_UNSUPPORTED, "at most 8 batch dimensions");
  if (batch_ndim && (!batch_shape || !a_bstride || !b_bstride))
    PB_FAIL(PB_ERR_INVALID, "null batch description");
  const size_t isz = dtype == PB_F64 ? 8 : 4;
  int64_t batch = 1, nA = 1, nB = 1;
  for (int j = 0; j < batch_ndim; ++j) {
    if (batch_shape[j] < 0 || a_bstride[j] < 0 || b_bstride[j] < 0)
      PB_FAIL(PB_ERR_INVALID, "negative batch extent");
    batch *= batch_shape[j];
    if (a_bstride[j]) nA += (batch_shape[j] - 1) * a_bstride[j];
    if (b_bstride[j]) nB += (batch_shape[j] - 1) * b_bstride[j];
  }
  const size_t a_bytes = (size_t)(nA * M * K) * isz, b_bytes = (size_t)(nB * K * N) * isz;
  const size_t c_bytes = (size_t)(batch * M * N) * isz;
  if (!c_bytes) return PB_OK;
  if (!C || (K && (!A || !B))) PB_FAIL(PB_ERR_INVALID, "null operand");

  // The cut: along the first batch dimension longer than 1 when A is dense
  // along it (B broadcast along it or dense too), else along the rows of A
  // when there is no batch, else one piece.
  int lead = 0;
  while (lead < batch_ndim - 1 && batch_shape[lead] == 1) ++lead;
  const bool by_batch = batch_ndim > 0 && batch_shape[lead] > 1 &&
                        dense_along(batch_ndim, batch_shape, a_bstride, lead) &&
                        (b_bstride[lead] == 0 || dense_along(batch_ndim, batch_shape, b_bstride, lead));
  const int64_t outer = by_batch ? batch_shape[lead] : batch_ndim == 0 ? M : 1;
  int64_t pieces = chunks > 0 ? chunks : 8;
  if (!K) pieces = 1;
  // At least 4 MiB of traffic per piece: smaller copies do not reach the
  // link's rate.
  const int64_t by_size = (int64_t)((a_bytes + c_bytes) / (4u << 20));
  if (pieces > by_size) pieces = by_size > 1 ? by_size : 1;
  if (pieces > outer) pieces = outer;
  if (pieces < 1) pieces = 1;

  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "pb_gemm_host cannot run during stream capture");
  PB_CHECK(host_streams(d, (size_t)(2 * pieces + 2)));
  cudaEvent_t* ev = d->host_events.data();  // [0] buffers, [1] B up, [2+2i] A_i up, [3+2i] C_i done

  void *dA = nullptr, *dB = nullptr, *dC = nullptr;
  int status = PB_OK;
  auto fail_cuda = [&](cudaError_t e, const char* what) {
    if (e == cudaSuccess || status != PB_OK) return;
    set_error("%s: %s", what, cudaGetErrorString(e));
    status = e == cudaErrorMemoryAllocation ? PB_ERR_OOM : PB_ERR_CUDA;
  };
  fail_cuda(cudaMallocAsync(&dC, c_bytes, d->pool, d->stream), "cudaMallocAsync");
  if (K) {
    fail_cuda(cudaMallocAsync(&dA, a_bytes ? a_bytes : 16, d->pool, d->stream), "cudaMallocAsync");
    fail_cuda(cudaMallocAsync(&dB, b_bytes ? b_bytes : 16, d->pool, d->stream), "cudaMallocAsync");
  }
  // The copy streams start after the buffers exist (and after the device's
  // earlier work).
  fail_cuda(cudaEventRecord(ev[0], d->stream), "cudaEventRecord");
  fail_cuda(cudaStreamWaitEvent(d->up, ev[0], 0), "cudaStreamWaitEvent");
  fail_cuda(cudaStreamWaitEvent(d->down, ev[0], 0), "cudaStreamWaitEvent");

  const int64_t inner = by_batch ? batch / batch_shape[lead] : 1;
  const int64_t a_per = by_batch ? a_bstride[lead] * M * K : batch_ndim == 0 ? K : 0;
  const int64_t b_per = by_batch ? b_bstride[lead] * K * N : 0;
  const int64_t c_per = by_batch ? inner * M * N : batch_ndim == 0 ? N : 0;
  const bool b_whole = !(by_batch && b_bstride[lead]);
  if (K && b_whole && status == PB_OK) {
    fail_cuda(cudaMemcpyAsync(dB, B, b_bytes, cudaMemcpyHostToDevice, d->up), "cudaMemcpyAsync");
    fail_cuda(cudaEventRecord(ev[1], d->up), "cudaEventRecord");
    fail_cuda(cudaStreamWaitEvent(d->stream, ev[1], 0), "cudaStreamWaitEvent");
  }
  int64_t shape2[8], as2[8], bs2[8];
  for (int j = 0; j < batch_ndim; ++j) {
    shape2[j] = batch_shape[j];
    as2[j] = a_bstride[j];
    bs2[j] = b_bstride[j];
  }
  for (int64_t i = 0; i < pieces && status == PB_OK; ++i) {
    const int64_t lo = outer * i / pieces, hi = outer * (i + 1) / pieces;
    if (pieces == 1 && !by_batch && batch_ndim) {
      // One piece of a batched product: everything at once.
      if (K) {
        fail_cuda(cudaMemcpyAsync(dA, A, a_bytes, cudaMemcpyHostToDevice, d->up), "cudaMemcpyAsync");
        if (!b_whole)
          fail_cuda(cudaMemcpyAsync(dB, B, b_bytes, cudaMemcpyHostToDevice, d->up), "cudaMemcpyAsync");
      }
    } else if (K) {
      const size_t off = (size_t)(lo * a_per) * isz, len = (size_t)((hi - lo) * a_per) * isz;
      fail_cuda(cudaMemcpyAsync((char*)dA + off, (const char*)A + off, len, cudaMemcpyHostToDevice,
                                d->up),
                "cudaMemcpyAsync");
      if (!b_whole) {
        const size_t bo = (size_t)(lo * b_per) * isz, bl = (size_t)((hi - lo) * b_per) * isz;
        fail_cuda(cudaMemcpyAsync((char*)dB + bo, (const char*)B + bo, bl, cudaMemcpyHostToDevice,
                                  d->up),
                  "cudaMemcpyAsync");
      }
    }
    fail_cuda(cudaEventRecord(ev[2 + 2 * i], d->up), "cudaEventRecord");
    fail_cuda(cudaStreamWaitEvent(d->stream, ev[2 + 2 * i], 0), "cudaStreamWaitEvent");
    if (status != PB_OK) break;
    // The piece's product on the device stream.
    const size_t coff = (size_t)(lo * c_per) * isz;
    if (by_batch) {
      shape2[lead] = hi - lo;
      status = gemm_dispatch(ctx, dev, dtype, batch_ndim, shape2, as2, bs2, M, N, K,
                             K ? (const char*)dA + (size_t)(lo * a_per) * isz : nullptr,
                             K ? (const char*)dB + (b_whole ? 0 : (size_t)(lo * b_per) * isz) : nullptr,
                             (char*)dC + coff, 0);
    } else if (batch_ndim == 0) {
      status = gemm_dispatch(ctx, dev, dtype, 0, nullptr, nullptr, nullptr, hi - lo, N, K,
                             K ? (const char*)dA + (size_t)(lo * a_per) * isz : nullptr, dB,
                             (char*)dC + coff, 0);
    } else {
      status = gemm_dispatch(ctx, dev, dtype, batch_ndim, batch_shape, a_bstride, b_bstride, M, N,
                             K, dA, dB, dC, 0);
    }
    if (status != PB_OK) break;
    fail_cuda(cudaEventRecord(ev[3 + 2 * i], d->stream), "cudaEventRecord");
    fail_cuda(cudaStreamWaitEvent(d->down, ev[3 + 2 * i], 0), "cudaStreamWaitEvent");
    const size_t clen = by_batch || batch_ndim == 0 ? (size_t)((hi - lo) * c_per) * isz : c_bytes;
    fail_cuda(cudaMemcpyAsync((char*)C + coff, (char*)dC + coff, clen, cudaMemcpyDeviceToHost, d->down),
              "cudaMemcpyAsync");
  }
  // The device stream ends after the last download; the buffers go back to
  // the pool in its order, and the call returns with C on the host.
  cudaEventRecord(ev[1], d->down);
  cudaStreamWaitEvent(d->stream, ev[1], 0);
  cudaEventRecord(ev[0], d->up);
  cudaStreamWaitEvent(d->stream, ev[0], 0);
  if (dA) cudaFreeAsync(dA, d->stream);
  if (dB) cudaFreeAsync(dB, d->stream);
  if (dC) cudaFreeAsync(dC, d->stream);
  const cudaError_t e = cudaStreamSynchronize(d->stream);
  fail_cuda(e, "cudaStreamSynchronize");
  if (status != PB_OK) return status;
  return check_kernel_error(d);
}

}  // extern "C"
