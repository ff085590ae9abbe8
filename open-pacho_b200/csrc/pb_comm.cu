// Multi-GPU layer: one process per GPU, NCCL over NVLink/NVSwitch.
//
// The reference is single-device (src/openpacho/_cuda.py:138-199) and has no
// collective call sites; this file adds the exchanges the sharded paths need:
//  * broadcast of the shared B operand for row-block sharded GEMM;
//  * the merge of per-rank (scale exponent, ssq, class) norm partials;
//  * a sum all-reduce for sharded DOT.
// NCCL is loaded with dlopen on first use (PB_NCCL_LIB overrides the name) so
// single-GPU use has no NCCL dependency.  Communicators are non-blocking; every
// wait on them is bounded (PB_COMM_TIMEOUT_S, default 300 s) and ends in
// ncclCommAbort plus an error status rather than a hang.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "pb_internal.cuh"

namespace pb {

int norm_pairs_finalize(Device* d, int dtype, const void* pairs, int n, void* out);
int norm_pair_zero(Device* d, int dtype, void* pair);
int norm_sharded_p2p(Device* d, int dtype, int64_t n, const void* x, void* out);

namespace {

struct NcclApi {
  bool loaded = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

int load_nccl() {
  std::lock_guard<std::mutex> g(g_nccl_mu);
  if (g_nccl.loaded) return PB_OK;
  const char* name = getenv("PB_NCCL_LIB");
  void* h = dlopen(name && *name ? name : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) PB_FAIL(PB_ERR_NCCL, "cannot load NCCL: %s", dlerror());
#define PB_SYM(field, sym)                                               \
  g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, sym)); \
  if (!g_nccl.field) PB_FAIL(PB_ERR_NCCL, "NCCL symbol %s missing", sym);
  PB_SYM(GetUniqueId, "ncclGetUniqueId");
  PB_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
  PB_SYM(CommDestroy, "ncclCommDestroy");
  PB_SYM(CommAbort, "ncclCommAbort");
  PB_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
  PB_SYM(AllReduce, "ncclAllReduce");
  PB_SYM(Broadcast, "ncclBroadcast");
  PB_SYM(AllGather, "ncclAllGather");
  PB_SYM(GetErrorString, "ncclGetErrorString");
#undef PB_SYM
  g_nccl.loaded = true;
  return PB_OK;
}

double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

double comm_timeout_s() {
  const char* s = getenv("PB_COMM_TIMEOUT_S");
  double v = s ? atof(s) : 0.0;
  return v > 0 ? v : 300.0;
}

void abort_comm(Device* d) {
  if (d->comm) g_nccl.CommAbort((ncclComm_t)d->comm);
  d->comm = nullptr;
  d->nranks = 1;
  d->rank = 0;
}

// Wait until the non-blocking communicator has no operation in progress:
// spin for the first millisecond (enqueues normally finish in microseconds),
// then poll with short sleeps until the deadline.
int settle(Device* d, ncclResult_t r) {
  const double start = now_s();
  const double deadline = start + comm_timeout_s();
  while (r == ncclInProgress) {
    const double t = now_s();
    if (t > deadline) {
      abort_comm(d);
      PB_FAIL(PB_ERR_NCCL, "NCCL operation timed out; communicator aborted");
    }
    if (t - start > 1e-3) usleep(20);
    g_nccl.CommGetAsyncError((ncclComm_t)d->comm, &r);
  }
  if (r != ncclSuccess) {
    const char* msg = g_nccl.GetErrorString(r);
    abort_comm(d);
    PB_FAIL(PB_ERR_NCCL, "NCCL error: %s; communicator aborted", msg);
  }
  return PB_OK;
}

int need_comm(Device* d) {
  if (!d->comm) PB_FAIL(PB_ERR_INVALID, "device has no communicator; call pb_comm_init");
  return PB_OK;
}

}  // namespace

// Bounded stream wait that also watches the communicator (used by pb_sync
// callers through pb_comm_sync).
int comm_stream_wait(Device* d) {
  const double deadline = now_s() + comm_timeout_s();
  for (;;) {
    cudaError_t q = cudaStreamQuery(d->stream);
    if (q == cudaSuccess) return PB_OK;
    if (q != cudaErrorNotReady) PB_FAIL(PB_ERR_CUDA, "stream failed: %s", cudaGetErrorString(q));
    if (d->comm) {
      ncclResult_t r;
      g_nccl.CommGetAsyncError((ncclComm_t)d->comm, &r);
      if (r != ncclSuccess && r != ncclInProgress) return settle(d, r);
    }
    if (now_s() > deadline) {
      abort_comm(d);
      PB_FAIL(PB_ERR_NCCL, "collective did not finish in time; communicator aborted");
    }
    usleep(20);
  }
}

}  // namespace pb

using namespace pb;

extern "C" {

int pb_comm_unique_id(unsigned char id[128]) {
  if (!id) PB_FAIL(PB_ERR_INVALID, "null id buffer");
  PB_CHECK(load_nccl());
  ncclUniqueId u;
  ncclResult_t r = g_nccl.GetUniqueId(&u);
  if (r != ncclSuccess) PB_FAIL(PB_ERR_NCCL, "ncclGetUniqueId: %s", g_nccl.GetErrorString(r));
  static_assert(sizeof(u) == 128, "ncclUniqueId is 128 bytes");
  memcpy(id, &u, 128);
  return PB_OK;
}

int pb_comm_init(pb_ctx* ctx, int dev, int nranks, int rank, const unsigned char id[128]) {
  if (!ctx || !id) PB_FAIL(PB_ERR_INVALID, "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) PB_FAIL(PB_ERR_INVALID, "bad rank %d/%d", rank, nranks);
  PB_CHECK(load_nccl());
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->comm) PB_FAIL(PB_ERR_INVALID, "device already has a communicator");
  ncclUniqueId u;
  memcpy(&u, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = g_nccl.CommInitRankConfig(&comm, nranks, u, rank, &cfg);
  d->comm = comm;
  d->nranks = nranks;
  d->rank = rank;
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm) g_nccl.CommAbort(comm);
    d->comm = nullptr;
    PB_FAIL(PB_ERR_NCCL, "ncclCommInitRankConfig: %s", g_nccl.GetErrorString(r));
  }
  if (r == ncclInProgress) g_nccl.CommGetAsyncError(comm, &r);
  return settle(d, r);
}

int pb_comm_destroy(pb_ctx* ctx, int dev) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!d->comm) return PB_OK;
  int st = comm_stream_wait(d);
  if (d->comm) {
    ncclResult_t r = g_nccl.CommDestroy((ncclComm_t)d->comm);
    if (r != ncclSuccess && r != ncclInProgress) g_nccl.CommAbort((ncclComm_t)d->comm);
  }
  d->comm = nullptr;
  d->nranks = 1;
  d->rank = 0;
  return st;
}

int pb_comm_abort(pb_ctx* ctx, int dev) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  abort_comm(d);
  return PB_OK;
}

int pb_broadcast(pb_ctx* ctx, int dev, void* buf, size_t bytes, int root) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  PB_CHECK(need_comm(d));
  if (root < 0 || root >= d->nranks) PB_FAIL(PB_ERR_INVALID, "bad root %d", root);
  if (!bytes) return PB_OK;
  ncclResult_t r =
      g_nccl.Broadcast(buf, buf, bytes, ncclUint8, root, (ncclComm_t)d->comm, d->stream);
  return settle(d, r);
}

int pb_allreduce_sum(pb_ctx* ctx, int dev, int dtype, void* buf, size_t count) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (dtype != PB_F32 && dtype != PB_F64) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  PB_CHECK(need_comm(d));
  if (!count) return PB_OK;
  ncclResult_t r = g_nccl.AllReduce(buf, buf, count, dtype == PB_F32 ? ncclFloat32 : ncclFloat64,
                                    ncclSum, (ncclComm_t)d->comm, d->stream);
  return settle(d, r);
}

int pb_norm_sharded(pb_ctx* ctx, int dev, int dtype, int64_t n, const void* x, void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (dtype != PB_F32 && dtype != PB_F64) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  if (n < 0) PB_FAIL(PB_ERR_INVALID, "negative length");
  if (!out) PB_FAIL(PB_ERR_INVALID, "null output");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (n > 0 && !x) PB_FAIL(PB_ERR_INVALID, "null input");
  if (d->capturing)
    PB_FAIL(PB_ERR_UNSUPPORTED, "the sharded norm cannot be captured: its exchange advances "
                                "sequence numbers and allocates with every call");
  // With peer mailboxes mapped: push over NVLink from the norm kernel itself.
  if (d->box_ranks > 1) return norm_sharded_p2p(d, dtype, n, x, out);
  PB_CHECK(need_comm(d));
  // pairs[r] = rank r's (scale exponent, ssq, class); one all-gather, then
  // every rank merges them in rank order (identical result everywhere).
  void* buf;
  const size_t bytes = (size_t)d->nranks * sizeof(NormPair);
  PB_CUDA(cudaMallocAsync(&buf, bytes, d->pool, d->stream));
  NormPair* pairs = (NormPair*)buf;
  int st = PB_OK;
  if (n > 0) {
    if (!x) st = (set_error("null input"), PB_ERR_INVALID);
    else st = norm_pair_global(d, dtype, n, x, pairs + d->rank);
  } else {
    st = norm_pair_zero(d, dtype, pairs + d->rank);
  }
  if (st == PB_OK)
    st = settle(d, g_nccl.AllGather(pairs + d->rank, pairs, sizeof(NormPair), ncclUint8,
                                    (ncclComm_t)d->comm, d->stream));
  if (st == PB_OK) st = norm_pairs_finalize(d, dtype, pairs, d->nranks, out);
  cudaFreeAsync(buf, d->stream);
  return st;
}

}  // extern "C"
