// Peer mailboxes: the sharded norm and DOT exchange their one per-rank
// partial over NVLink with plain stores into each peer's memory, in the same
// kernel that computes it (the norm) or the launch right after (the DOT),
// instead of an NCCL collective.  The reference is single-device; the
// exchange replaces the all-gather / all-reduce of the NCCL path
// (pb_comm.cu), which stays as the fallback when CUDA IPC is unavailable.
//
// Setup (once per group): each rank allocates its mailbox with cudaMalloc,
// exports it (pb_peer_export), the 64-byte IPC handles travel through the
// host store, and each rank maps every peer's mailbox (pb_peer_import).
// Every later exchange is: push (payload, system fence, release store of the
// call's sequence number into slot [rank][seq % 2] of every mailbox), then one
// thread per rank waits for all sequence numbers (acquire loads, bounded at
// the context's wait limit, 10 s unless pb_peer_set_wait changed it; error flag on timeout) and merges in rank order, so every
// rank computes identical bits.
#include <string.h>

#include "pb_internal.cuh"

namespace pb {

int mailbox_norm(Device* d, int dtype, int parity, unsigned long long seq, void* out);
int norm_push_empty(Device* d, int dtype, const PushArgs& a);
int dot_device(Device* d, int dtype, int64_t n, const void* x, const void* y, void* out);

namespace {

constexpr size_t kBoxBytes = (size_t)kMaxRanks * 2 * sizeof(MailSlot);

PushArgs push_args(Device* d, unsigned long long seq) {
  PushArgs a{};
  for (int r = 0; r < d->box_ranks; ++r) a.box[r] = d->box[r];
  a.nranks = d->box_ranks;
  a.rank = d->box_rank;
  a.parity = (int)(seq & 1);
  a.seq = seq;
  return a;
}

template <typename T>
__global__ void push_value_kernel(const T* v, const PushArgs a) {
  if (threadIdx.x == 0) push_slot(a, (double)*v, 0, 0);
}

// Sum of every rank's partial, in rank order.
template <typename T>
__global__ void mailbox_sum_kernel(const MailSlot* box, int nranks, int parity,
                                   unsigned long long seq, T* out, int* err,
                                   unsigned long long wait_ns) {
  if (threadIdx.x != 0) return;
  double s = 0.0;
  for (int r = 0; r < nranks; ++r) {
    const MailSlot* slot = box + r * 2 + parity;
    if (!mailbox_wait(slot, seq, err, wait_ns)) return;
    s += *(volatile const double*)&slot->a;
  }
  *out = (T)s;
}

int close_boxes(Device* d) {
  int st = PB_OK;
  for (int r = 0; r < kMaxRanks; ++r) {
    if (!d->box[r]) continue;
    cudaError_t e = r == d->box_rank ? cudaFree(d->box[r]) : cudaIpcCloseMemHandle(d->box[r]);
    if (e != cudaSuccess && st == PB_OK) {
      set_error("closing mailbox of rank %d: %s", r, cudaGetErrorString(e));
      st = PB_ERR_CUDA;
    }
    d->box[r] = nullptr;
  }
  d->box_ranks = 0;
  return st;
}

}  // namespace

// Unmap the peers' mailboxes and free this one (context teardown).
int peer_close(Device* d) { return close_boxes(d); }

}  // namespace pb

using namespace pb;

extern "C" {

int pb_peer_export(pb_ctx* ctx, int dev, int nranks, int rank, unsigned char handle[64]) {
  if (!ctx || !handle) PB_FAIL(PB_ERR_INVALID, "null argument");
  if (nranks < 2 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
    PB_FAIL(PB_ERR_INVALID, "peer mailboxes take 2..%d ranks (got rank %d of %d)", kMaxRanks, rank,
            nranks);
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  PB_CHECK(close_boxes(d));
  void* p = nullptr;
  PB_CUDA(cudaMalloc(&p, kBoxBytes));  // IPC needs a cudaMalloc allocation
  cudaError_t e = cudaMemset(p, 0, kBoxBytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    PB_FAIL(PB_ERR_UNAVAILABLE, "mailbox export: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  memcpy(handle, &h, 64);
  d->box[rank] = static_cast<MailSlot*>(p);
  d->box_rank = rank;
  d->box_seq = 0;
  return PB_OK;
}

int pb_peer_import(pb_ctx* ctx, int dev, int nranks, const unsigned char* handles) {
  if (!ctx || !handles) PB_FAIL(PB_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!d->box[d->box_rank]) PB_FAIL(PB_ERR_INVALID, "pb_peer_export first");
  if (nranks < 2 || nranks > kMaxRanks || d->box_rank >= nranks)
    PB_FAIL(PB_ERR_INVALID, "bad rank count %d", nranks);
  for (int r = 0; r < nranks; ++r) {
    if (r == d->box_rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, handles + 64 * r, 64);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      cudaGetLastError();
      close_boxes(d);
      PB_FAIL(PB_ERR_UNAVAILABLE, "mapping the mailbox of rank %d: %s", r, cudaGetErrorString(e));
    }
    d->box[r] = static_cast<MailSlot*>(p);
  }
  d->box_ranks = nranks;
  return PB_OK;
}

int pb_peer_close(pb_ctx* ctx, int dev) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  PB_CUDA(cudaStreamSynchronize(d->stream));
  return close_boxes(d);
}

int pb_peer_set_wait(pb_ctx* ctx, int dev, uint64_t limit_ns) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  d->box_wait_ns = limit_ns ? (unsigned long long)limit_ns : kMailboxWaitNs;
  return PB_OK;
}

int pb_dot_sharded(pb_ctx* ctx, int dev, int dtype, int64_t n, const void* x, const void* y,
                   void* out) {
  if (!ctx || !out) PB_FAIL(PB_ERR_INVALID, "null argument");
  if (dtype != PB_F32 && dtype != PB_F64) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  if (n < 0) PB_FAIL(PB_ERR_INVALID, "negative length");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->box_ranks < 2) PB_FAIL(PB_ERR_INVALID, "no peer mailboxes; call pb_peer_export/import");
  if (d->capturing)
    PB_FAIL(PB_ERR_UNSUPPORTED, "the mailbox exchange cannot be captured: its sequence numbers "
                                "advance with every call");
  PB_CHECK(dot_device(d, dtype, n, x, y, out));  // local partial into out
  const unsigned long long seq = ++d->box_seq;
  const PushArgs a = push_args(d, seq);
  if (dtype == PB_F32) {
    push_value_kernel<float><<<1, 32, 0, d->stream>>>((const float*)out, a);
    PB_LAUNCHED(d);
    mailbox_sum_kernel<float><<<1, 32, 0, d->stream>>>(d->box[d->box_rank], d->box_ranks, a.parity,
                                                       seq, (float*)out, d->err_dev, d->box_wait_ns);
  } else {
    push_value_kernel<double><<<1, 32, 0, d->stream>>>((const double*)out, a);
    PB_LAUNCHED(d);
    mailbox_sum_kernel<double><<<1, 32, 0, d->stream>>>(d->box[d->box_rank], d->box_ranks,
                                                        a.parity, seq, (double*)out, d->err_dev,
                                                        d->box_wait_ns);
  }
  PB_LAUNCHED(d);
  return PB_OK;
}

}  // extern "C"

namespace pb {

// The sharded norm over the mailboxes: the local norm kernel pushes its pair
// to every rank, then the merge.  Called by pb_norm_sharded when mapped.
int norm_sharded_p2p(Device* d, int dtype, int64_t n, const void* x, void* out) {
  const unsigned long long seq = ++d->box_seq;
  const PushArgs a = push_args(d, seq);
  if (n > 0)
    PB_CHECK(norm_pair_global(d, dtype, n, x, nullptr, &a));
  else
    PB_CHECK(norm_push_empty(d, dtype, a));  // an empty slice: the neutral pair
  return mailbox_norm(d, dtype, a.parity, seq, out);
}

}  // namespace pb
