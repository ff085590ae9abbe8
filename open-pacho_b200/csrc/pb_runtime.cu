// Context, memory, copies, errors and timers of libpacho_b200.
//
// Behavioural model: CUDABackend in src/openpacho/_cuda.py -- one
// non-blocking stream per device (:157-160), synchronous snapshot uploads
// (:293-303), downloads that synchronise first (:305-311), a reusable memory
// pool (:232-274) and explicit close (:644-673).  The pool here is CUDA's
// stream-ordered allocator instead of a Python LRU of cuMemAlloc blocks.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <string.h>

#include <vector>

#include "pb_internal.cuh"

namespace pb {

static thread_local char g_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int enter(pb_ctx* ctx, int dev, Device** out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (dev < 0 || dev >= ctx->ndev) PB_FAIL(PB_ERR_INVALID, "device index %d out of range", dev);
  Device* d = &ctx->devs[dev];
  PB_CUDA(cudaSetDevice(d->ordinal));
  *out = d;
  return PB_OK;
}

// During a stream capture nothing may allocate: a call that would grow a
// buffer fails and asks for one uncaptured call of the same shape first.
#define PB_NO_GROWTH_IN_CAPTURE(d)                                                          \
  do {                                                                                      \
    if ((d)->capturing)                                                                     \
      PB_FAIL(PB_ERR_UNSUPPORTED,                                                           \
              "a buffer would grow during stream capture: make one uncaptured call of the " \
              "same shape first");                                                          \
  } while (0)

// Frees a library buffer, or keeps it until the last graph is destroyed.
static int release_buffer(Device* d, void* p) {
  if (!p) return PB_OK;
  if (d->graphs_live > 0) {
    d->retired.push_back(p);
    return PB_OK;
  }
  PB_CUDA(cudaFreeAsync(p, d->stream));
  return PB_OK;
}

int scratch(Device* d, size_t bytes, void** out) {
  if (bytes > d->scratch_bytes) {
    PB_NO_GROWTH_IN_CAPTURE(d);
    PB_CHECK(release_buffer(d, d->scratch));
    d->scratch = nullptr;
    d->scratch_bytes = 0;
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    PB_CUDA(cudaMallocAsync(&d->scratch, want, d->pool, d->stream));
    d->scratch_bytes = want;
  }
  *out = d->scratch;
  return PB_OK;
}

int counters(Device* d, size_t n, unsigned int** out) {
  if (n > d->counters_n) {
    PB_NO_GROWTH_IN_CAPTURE(d);
    PB_CHECK(release_buffer(d, d->counters));
    d->counters = nullptr;
    d->counters_n = 0;
    size_t want = n < 4096 ? 4096 : n;
    PB_CUDA(cudaMallocAsync((void**)&d->counters, want * sizeof(unsigned int), d->pool,
                            d->stream));
    PB_CUDA(cudaMemsetAsync(d->counters, 0, want * sizeof(unsigned int), d->stream));
    d->counters_n = want;
  }
  *out = d->counters;
  return PB_OK;
}

int operand_tags(Device* d, size_t n, unsigned int** out, unsigned int* gen) {
  if (n > d->tags_n || d->tag_gen == UINT32_MAX) {
    PB_NO_GROWTH_IN_CAPTURE(d);
    const size_t want = n > d->tags_n ? (n < 65536 ? 65536 : n) : d->tags_n;
    if (want > d->tags_n) {
      PB_CHECK(release_buffer(d, d->tags));
      d->tags = nullptr;
      d->tags_n = 0;
      PB_CUDA(cudaMallocAsync((void**)&d->tags, want * sizeof(unsigned int), d->pool, d->stream));
      d->tags_n = want;
    }
    PB_CUDA(cudaMemsetAsync(d->tags, 0, d->tags_n * sizeof(unsigned int), d->stream));
    d->tag_gen = 0;
  }
  *out = d->tags;
  *gen = ++d->tag_gen;
  return PB_OK;
}

constexpr size_t kMaxTimedLaunches = 4096;

int kt_begin(Device* d) {
  if (!d->kt_on) return PB_OK;
  if (d->kt_used >= kMaxTimedLaunches)
    PB_FAIL(PB_ERR_UNSUPPORTED, "kernel timer holds at most %zu launches between reads",
            kMaxTimedLaunches);
  if (d->kt_used == d->kt_events.size()) {
    cudaEvent_t a, b;
    PB_CUDA(cudaEventCreate(&a));
    if (cudaEventCreate(&b) != cudaSuccess) {
      cudaEventDestroy(a);
      PB_FAIL(PB_ERR_CUDA, "cudaEventCreate failed");
    }
    d->kt_events.emplace_back(a, b);
  }
  // Inside a capture the pair must become event nodes of the graph.
  PB_CUDA(cudaEventRecordWithFlags(d->kt_events[d->kt_used].first, d->stream,
                                   d->capturing ? cudaEventRecordExternal : cudaEventRecordDefault));
  return PB_OK;
}

int kt_end(Device* d) {
  if (!d->kt_on) return PB_OK;
  PB_CUDA(cudaEventRecordWithFlags(d->kt_events[d->kt_used].second, d->stream,
                                   d->capturing ? cudaEventRecordExternal : cudaEventRecordDefault));
  ++d->kt_used;
  return PB_OK;
}

int tensor_map_encoder(void** fn) {
  static std::once_flag once;
  static void* encoder = nullptr;
  static cudaError_t status = cudaSuccess;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &encoder, cudaEnableDefault, &q);
    if (status == cudaSuccess && q != cudaDriverEntryPointSuccess) status = cudaErrorNotSupported;
  });
  if (status != cudaSuccess || !encoder)
    PB_FAIL(PB_ERR_UNAVAILABLE, "cuTensorMapEncodeTiled unavailable: %s",
            cudaGetErrorString(status));
  *fn = encoder;
  return PB_OK;
}

static void release_device(Device* d) {
  if (d->ordinal < 0) return;
  cudaSetDevice(d->ordinal);
  if (d->stream) cudaStreamSynchronize(d->stream);
  peer_close(d);
  if (d->scratch) cudaFreeAsync(d->scratch, d->stream);
  if (d->counters) cudaFreeAsync(d->counters, d->stream);
  if (d->tags) cudaFreeAsync(d->tags, d->stream);
  for (void* p : d->retired) cudaFreeAsync(p, d->stream);
  d->retired.clear();
  if (d->stream) cudaStreamSynchronize(d->stream);
  if (d->t0) cudaEventDestroy(d->t0);
  if (d->t1) cudaEventDestroy(d->t1);
  if (d->order_ev) cudaEventDestroy(d->order_ev);
  for (auto& ev : d->kt_events) {
    cudaEventDestroy(ev.first);
    cudaEventDestroy(ev.second);
  }
  d->kt_events.clear();
  d->kt_used = 0;
  d->dot_static = nullptr;
  if (d->err_host) cudaFreeHost(d->err_host);
  for (cudaEvent_t e : d->host_events) cudaEventDestroy(e);
  d->host_events.clear();
  if (d->up) cudaStreamSynchronize(d->up), cudaStreamDestroy(d->up);
  if (d->down) cudaStreamSynchronize(d->down), cudaStreamDestroy(d->down);
  d->up = d->down = nullptr;
  if (d->stream) cudaStreamDestroy(d->stream);
  if (d->pool) cudaMemPoolTrimTo(d->pool, 0);
  d->scratch = nullptr;
  d->counters = nullptr;
  d->tags = nullptr;
  d->tags_n = 0;
  d->err_host = d->err_dev = nullptr;
  d->stream = nullptr;
}

// Kernel error word check (after a synchronisation).
int check_kernel_error(Device* d) {
  if (d->err_host && *(volatile int*)d->err_host != KERR_NONE) {
    int code = *(volatile int*)d->err_host;
    *(volatile int*)d->err_host = KERR_NONE;
    // An aborted kernel may have left arrival counters or marks behind; the
    // stream is idle here, so zero them before the next launch reads them.
    if (d->counters) cudaMemsetAsync(d->counters, 0, d->counters_n * sizeof(unsigned int), d->stream);
    PB_FAIL(PB_ERR_DEVICE, "kernel reported error %d (%s)", code,
            code == KERR_WAIT_TIMEOUT ? "bounded wait timed out" : "bad argument");
  }
  return PB_OK;
}

}  // namespace pb

using namespace pb;

extern "C" {

const char* pb_last_error(void) { return g_error; }

int pb_abi_version(void) { return PB_ABI_VERSION; }

int pb_device_count(int* count) {
  if (!count) PB_FAIL(PB_ERR_INVALID, "null count");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *count = 0;
    PB_FAIL(PB_ERR_UNAVAILABLE, "no CUDA device: %s", cudaGetErrorString(e));
  }
  *count = n;
  return PB_OK;
}

int pb_driver_version(int* version) {
  if (!version) PB_FAIL(PB_ERR_INVALID, "null version");
  *version = 0;
  cudaError_t e = cudaDriverGetVersion(version);
  if (e != cudaSuccess) PB_FAIL(PB_ERR_UNAVAILABLE, "no CUDA driver: %s", cudaGetErrorString(e));
  return PB_OK;
}

int pb_device_info(int ordinal, char* name, size_t name_len, size_t* total_bytes, int* sm_count,
                   int* cc_major, int* cc_minor) {
  cudaDeviceProp p;
  cudaError_t e = cudaGetDeviceProperties(&p, ordinal);
  if (e != cudaSuccess) PB_FAIL(PB_ERR_UNAVAILABLE, "device %d: %s", ordinal, cudaGetErrorString(e));
  if (name && name_len) {
    strncpy(name, p.name, name_len - 1);
    name[name_len - 1] = 0;
  }
  if (total_bytes) *total_bytes = p.totalGlobalMem;
  if (sm_count) *sm_count = p.multiProcessorCount;
  if (cc_major) *cc_major = p.major;
  if (cc_minor) *cc_minor = p.minor;
  return PB_OK;
}

int pb_init(int ndev, const int* ordinals, pb_ctx** out) {
  if (!out || ndev <= 0 || !ordinals) PB_FAIL(PB_ERR_INVALID, "pb_init needs >=1 device");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    PB_FAIL(PB_ERR_UNAVAILABLE, "no CUDA device: %s", cudaGetErrorString(e));
  pb_ctx* ctx = new pb_ctx();
  ctx->ndev = ndev;
  ctx->devs = new Device[ndev];
  int status = PB_OK;
  for (int i = 0; i < ndev && status == PB_OK; ++i) {
    Device* d = &ctx->devs[i];
    int ord = ordinals[i];
    if (ord < 0 || ord >= count) {
      set_error("CUDA device %d not found (%d visible)", ord, count);
      status = PB_ERR_UNAVAILABLE;
      break;
    }
    cudaDeviceProp p;
    if ((e = cudaGetDeviceProperties(&p, ord)) != cudaSuccess) {
      set_error("cudaGetDeviceProperties: %s", cudaGetErrorString(e));
      status = PB_ERR_UNAVAILABLE;
      break;
    }
    if (p.major != 10) {
      set_error("device %d (%s, sm_%d%d) is not a B200-class sm_100 GPU", ord, p.name, p.major,
                p.minor);
      status = PB_ERR_UNAVAILABLE;
      break;
    }
    d->ordinal = ord;
    d->sm_count = p.multiProcessorCount;
    auto fail = [&](const char* what, cudaError_t err) {
      set_error("%s: %s", what, cudaGetErrorString(err));
      status = err == cudaErrorMemoryAllocation ? PB_ERR_OOM : PB_ERR_CUDA;
    };
    if ((e = cudaSetDevice(ord)) != cudaSuccess) { fail("cudaSetDevice", e); break; }
    if ((e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking)) != cudaSuccess) {
      fail("cudaStreamCreate", e);
      break;
    }
    if ((e = cudaDeviceGetDefaultMemPool(&d->pool, ord)) != cudaSuccess) {
      fail("cudaDeviceGetDefaultMemPool", e);
      break;
    }
    // Keep freed blocks cached in the pool (no release at each sync point).
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(d->pool, cudaMemPoolAttrReleaseThreshold, &keep);
    if ((e = cudaHostAlloc((void**)&d->err_host, sizeof(int), cudaHostAllocMapped)) !=
        cudaSuccess) {
      fail("cudaHostAlloc(error word)", e);
      break;
    }
    *d->err_host = KERR_NONE;
    if ((e = cudaHostGetDevicePointer((void**)&d->err_dev, d->err_host, 0)) != cudaSuccess) {
      fail("cudaHostGetDevicePointer", e);
      break;
    }
    if ((e = cudaEventCreate(&d->t0)) != cudaSuccess || (e = cudaEventCreate(&d->t1)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&d->order_ev, cudaEventDisableTiming)) != cudaSuccess) {
      fail("cudaEventCreate", e);
      break;
    }
    if ((status = dot_static_prepare(d)) != PB_OK) break;
  }
  if (status != PB_OK) {
    for (int i = 0; i < ndev; ++i) release_device(&ctx->devs[i]);
    delete[] ctx->devs;
    delete ctx;
    return status;
  }
  *out = ctx;
  return PB_OK;
}

int pb_comm_destroy(pb_ctx* ctx, int dev);

int pb_destroy(pb_ctx* ctx) {
  if (!ctx) return PB_OK;
  {
    std::lock_guard<std::recursive_mutex> g(ctx->mu);
    for (int i = 0; i < ctx->ndev; ++i) {
      if (ctx->devs[i].comm) pb_comm_destroy(ctx, i);
      release_device(&ctx->devs[i]);
    }
  }
  delete[] ctx->devs;
  delete ctx;
  return PB_OK;
}

int pb_alloc(pb_ctx* ctx, int dev, size_t bytes, void** ptr) {
  if (!ptr || !ctx) PB_FAIL(PB_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  if (bytes == 0) bytes = 16;
  PB_CUDA(cudaMallocAsync(ptr, bytes, d->pool, d->stream));
  return PB_OK;
}

int pb_free(pb_ctx* ctx, int dev, void* ptr) {
  if (!ptr) return PB_OK;
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  PB_CUDA(cudaFreeAsync(ptr, d->stream));
  return PB_OK;
}

int pb_h2d(pb_ctx* ctx, int dev, void* dst, const void* src, size_t bytes, int blocking) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (!bytes) return PB_OK;
  if (!dst || !src) PB_FAIL(PB_ERR_INVALID, "null pointer in pb_h2d");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (blocking && d->capturing)
    PB_FAIL(PB_ERR_UNSUPPORTED, "a blocking copy cannot run during stream capture");
  PB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, d->stream));
  if (blocking) PB_CUDA(cudaStreamSynchronize(d->stream));
  return PB_OK;
}

int pb_d2h(pb_ctx* ctx, int dev, void* dst, const void* src, size_t bytes) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  if (bytes) {
    if (!dst || !src) PB_FAIL(PB_ERR_INVALID, "null pointer in pb_d2h");
    PB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, d->stream));
  }
  PB_CUDA(cudaStreamSynchronize(d->stream));
  return check_kernel_error(d);
}

int pb_d2h_async(pb_ctx* ctx, int dev, void* dst, const void* src, size_t bytes) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (!bytes) return PB_OK;
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  PB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, d->stream));
  return PB_OK;
}

int pb_d2d(pb_ctx* ctx, int dev, void* dst, const void* src, size_t bytes) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (!bytes) return PB_OK;
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  PB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, d->stream));
  return PB_OK;
}

int pb_sync(pb_ctx* ctx, int dev) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  if (d->comm) PB_CHECK(comm_stream_wait(d));
  else PB_CUDA(cudaStreamSynchronize(d->stream));
  return check_kernel_error(d);
}

int pb_host_register(void* ptr, size_t bytes) {
  if (!ptr || !bytes) PB_FAIL(PB_ERR_INVALID, "empty host range");
  PB_CUDA(cudaHostRegister(ptr, bytes, cudaHostRegisterDefault));
  return PB_OK;
}

int pb_host_unregister(void* ptr) {
  if (!ptr) return PB_OK;
  PB_CUDA(cudaHostUnregister(ptr));
  return PB_OK;
}

int pb_trim(pb_ctx* ctx, int dev) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->graphs_live > 0)
    PB_FAIL(PB_ERR_UNSUPPORTED, "pb_trim would free buffers that live graphs use");
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  if (d->scratch) PB_CUDA(cudaFreeAsync(d->scratch, d->stream));
  d->scratch = nullptr;
  d->scratch_bytes = 0;
  if (d->tags) PB_CUDA(cudaFreeAsync(d->tags, d->stream));
  d->tags = nullptr;
  d->tags_n = 0;
  PB_CUDA(cudaStreamSynchronize(d->stream));
  PB_CUDA(cudaMemPoolTrimTo(d->pool, 0));
  return PB_OK;
}

int pb_timer_start(pb_ctx* ctx, int dev) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  PB_CUDA(cudaEventRecord(d->t0, d->stream));
  return PB_OK;
}

int pb_timer_stop(pb_ctx* ctx, int dev, float* ms) {
  if (!ctx || !ms) PB_FAIL(PB_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  PB_CUDA(cudaEventRecord(d->t1, d->stream));
  PB_CUDA(cudaEventSynchronize(d->t1));
  PB_CUDA(cudaEventElapsedTime(ms, d->t0, d->t1));
  return check_kernel_error(d);
}

int pb_ktimer_enable(pb_ctx* ctx, int dev, int enable) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "the kernel timer cannot change during capture");
  d->kt_on = enable < 0 || enable > 2 ? 1 : enable;
  d->kt_used = 0;
  return PB_OK;
}

// ---- several devices in one context ---------------------------------------

int pb_peer_enable(pb_ctx* ctx, int* all_pairs) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  int all = 1;
  for (int i = 0; i < ctx->ndev; ++i) {
    for (int j = 0; j < ctx->ndev; ++j) {
      const int a = ctx->devs[i].ordinal, b = ctx->devs[j].ordinal;
      if (a == b) continue;
      int can = 0;
      PB_CUDA(cudaDeviceCanAccessPeer(&can, a, b));
      if (!can) {
        all = 0;
        continue;
      }
      PB_CUDA(cudaSetDevice(a));
      const cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
      } else if (e != cudaSuccess) {
        PB_FAIL(PB_ERR_CUDA, "cudaDeviceEnablePeerAccess(%d -> %d): %s", a, b,
                cudaGetErrorString(e));
      }
    }
  }
  if (all_pairs) *all_pairs = all;
  return PB_OK;
}

// Peer copies go device to device over NVLink only where the remote side of
// the copy is mapped into the issuing device: memory from cudaMalloc, which
// peer access maps, unlike the stream-ordered pools.
int pb_alloc_mapped(pb_ctx* ctx, int dev, size_t bytes, void** ptr) {
  if (!ctx || !ptr) PB_FAIL(PB_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  PB_CUDA(cudaMalloc(ptr, bytes ? bytes : 16));
  return PB_OK;
}

int pb_free_mapped(pb_ctx* ctx, int dev, void* ptr) {
  if (!ptr) return PB_OK;
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  PB_CUDA(cudaStreamSynchronize(d->stream));  // the device's work on it is done
  PB_CUDA(cudaFree(ptr));
  return PB_OK;
}

// Stream `which` of a device: 0 its stream (every kernel of the library runs
// there), 1 its copy stream (created on first use).
static int device_stream(Device* d, int which, cudaStream_t* out) {
  if (which == 0) {
    *out = d->stream;
    return PB_OK;
  }
  if (which != 1) PB_FAIL(PB_ERR_INVALID, "stream %d: 0 (the device's) or 1 (its copy stream)", which);
  if (!d->up) {
    PB_CUDA(cudaSetDevice(d->ordinal));
    PB_CUDA(cudaStreamCreateWithFlags(&d->up, cudaStreamNonBlocking));
  }
  *out = d->up;
  return PB_OK;
}

int pb_stream_wait(pb_ctx* ctx, int waiter, int waiter_stream, int signal, int signal_stream) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device *w, *s;
  PB_CHECK(enter(ctx, signal, &s));
  PB_CHECK(enter(ctx, waiter, &w));
  if (w->capturing || s->capturing)
    PB_FAIL(PB_ERR_UNSUPPORTED, "pb_stream_wait cannot run during stream capture");
  cudaStream_t ws, ss;
  PB_CHECK(device_stream(w, waiter_stream, &ws));
  PB_CHECK(device_stream(s, signal_stream, &ss));
  if (ws == ss) return PB_OK;
  PB_CUDA(cudaSetDevice(s->ordinal));
  PB_CUDA(cudaEventRecord(s->order_ev, ss));
  PB_CUDA(cudaSetDevice(w->ordinal));
  PB_CUDA(cudaStreamWaitEvent(ws, s->order_ev, 0));
  return PB_OK;
}

int pb_copy_peer(pb_ctx* ctx, int dst_dev, void* dst, int src_dev, const void* src, size_t bytes,
                 int stream_dev, int stream) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (!bytes) return PB_OK;
  if (!dst || !src) PB_FAIL(PB_ERR_INVALID, "null pointer in pb_copy_peer");
  if (stream_dev != dst_dev && stream_dev != src_dev)
    PB_FAIL(PB_ERR_INVALID, "pb_copy_peer runs on a stream of the source or the destination");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device *t, *s, *on;
  PB_CHECK(enter(ctx, src_dev, &s));
  PB_CHECK(enter(ctx, dst_dev, &t));
  PB_CHECK(enter(ctx, stream_dev, &on));
  if (on->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "pb_copy_peer cannot run during stream capture");
  cudaStream_t st;
  PB_CHECK(device_stream(on, stream, &st));
  PB_CUDA(cudaSetDevice(on->ordinal));
  if (t == s)
    PB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st));
  else
    PB_CUDA(cudaMemcpyPeerAsync(dst, t->ordinal, src, s->ordinal, bytes, st));
  return PB_OK;
}

int pb_capture_begin(pb_ctx* ctx, int dev) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_INVALID, "a capture is already in progress");
  PB_CUDA(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeRelaxed));
  d->capturing = 1;
  return PB_OK;
}

int pb_capture_end(pb_ctx* ctx, int dev, void** graph) {
  if (!ctx || !graph) PB_FAIL(PB_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!d->capturing) PB_FAIL(PB_ERR_INVALID, "no capture in progress");
  d->capturing = 0;
  cudaGraph_t cg = nullptr;
  PB_CUDA(cudaStreamEndCapture(d->stream, &cg));
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, cg, 0);
  cudaGraphDestroy(cg);
  if (e != cudaSuccess)
    PB_FAIL(PB_ERR_CUDA, "cudaGraphInstantiate failed: %s", cudaGetErrorString(e));
  *graph = exec;
  ++d->graphs_live;
  return PB_OK;
}

int pb_graph_launch(pb_ctx* ctx, int dev, void* graph) {
  if (!ctx || !graph) PB_FAIL(PB_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  PB_CUDA(cudaGraphLaunch((cudaGraphExec_t)graph, d->stream));
  return PB_OK;
}

int pb_graph_destroy(pb_ctx* ctx, int dev, void* graph) {
  if (!graph) return PB_OK;
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  // The graph may still run on the stream: destroying the executable is safe
  // then, freeing what it uses is ordered after it on the same stream.
  PB_CUDA(cudaGraphExecDestroy((cudaGraphExec_t)graph));
  if (d->graphs_live > 0 && --d->graphs_live == 0) {
    for (void* p : d->retired) PB_CUDA(cudaFreeAsync(p, d->stream));
    d->retired.clear();
  }
  return PB_OK;
}

int pb_ktimer_read(pb_ctx* ctx, int dev, double* total_ms, uint64_t* launches) {
  if (!ctx || !total_ms || !launches) PB_FAIL(PB_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (d->capturing) PB_FAIL(PB_ERR_UNSUPPORTED, "%s cannot run during stream capture", __func__);
  PB_CUDA(cudaStreamSynchronize(d->stream));
  double total = 0.0;
  for (size_t i = 0; i < d->kt_used; ++i) {
    float ms = 0.0f;
    PB_CUDA(cudaEventElapsedTime(&ms, d->kt_events[i].first, d->kt_events[i].second));
    total += ms;
  }
  *total_ms = total;
  *launches = d->kt_used;
  if (d->kt_on != 2) d->kt_used = 0;
  return check_kernel_error(d);
}

int pb_memory_stats(pb_ctx* ctx, int dev, size_t* pool_reserved, size_t* pool_used,
                    size_t* scratch_bytes, size_t* device_free) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  uint64_t reserved = 0, used = 0;
  PB_CUDA(cudaMemPoolGetAttribute(d->pool, cudaMemPoolAttrReservedMemCurrent, &reserved));
  PB_CUDA(cudaMemPoolGetAttribute(d->pool, cudaMemPoolAttrUsedMemCurrent, &used));
  size_t free_b = 0, total_b = 0;
  PB_CUDA(cudaMemGetInfo(&free_b, &total_b));
  if (pool_reserved) *pool_reserved = (size_t)reserved;
  if (pool_used) *pool_used = (size_t)used;
  if (scratch_bytes) *scratch_bytes = d->scratch_bytes;
  if (device_free) *device_free = free_b;
  return PB_OK;
}

int pb_launch_count(pb_ctx* ctx, int dev, uint64_t* count) {
  if (!ctx || !count) PB_FAIL(PB_ERR_INVALID, "null argument");
  if (dev < 0 || dev >= ctx->ndev) PB_FAIL(PB_ERR_INVALID, "device index %d out of range", dev);
  *count = ctx->devs[dev].launches.load();
  return PB_OK;
}

}  // extern "C"
