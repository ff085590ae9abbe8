/*
 * pacho_b200.h -- C ABI of libpacho_b200.so, the B200 (sm_100a) backend for
 * OpenPacho's linear-algebra hot path: batched GEMM with broadcast leading
 * dimensions, GEMV, DOT and the overflow-safe scaled Euclidean/Frobenius norm.
 *
 * Conventions
 *  - Every entry point returns an int status (PB_OK == 0).  On failure the
 *    message is available from pb_last_error(), which is thread-local.
 *  - Device pointers are plain `void*` obtained from pb_alloc(); sizes are
 *    element or byte counts as documented; no C++ or framework types appear.
 *  - All work of one device is ordered on one non-blocking CUDA stream owned
 *    by the context.  Calls return after *submission*; pb_sync() and
 *    pb_d2h() synchronise.  A host mutex per context serialises submission,
 *    mirroring the reference CUDA backend's RLock (src/openpacho/_cuda.py:148,
 *    201-220).
 *  - Matrices are C-contiguous (row-major).  Batched operands are a sequence
 *    of contiguous matrices; broadcast is expressed by per-dimension batch
 *    strides counted in whole matrices, 0 for a broadcast dimension.
 *  - There is no CPU fallback anywhere: an unsupported request is an error.
 */
#ifndef PACHO_B200_H
#define PACHO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Only the entry points below are exported from the shared library. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define PB_ABI_VERSION 1

/* Status codes. */
enum {
  PB_OK = 0,
  PB_ERR_INVALID = 1,     /* bad argument (shape, pointer, dtype value)          */
  PB_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed                    */
  PB_ERR_UNSUPPORTED = 3, /* valid request this library does not implement       */
  PB_ERR_OOM = 4,         /* device allocation failed                            */
  PB_ERR_NCCL = 5,        /* NCCL missing or a collective failed                  */
  PB_ERR_DEVICE = 6,      /* a kernel reported an error (e.g. a bounded wait ran out) */
  PB_ERR_UNAVAILABLE = 7  /* no usable device / driver                           */
};

/* Element types (the reference supports float32 and float64 on this path,
 * plus bool storage for comparisons and masks: src/openpacho/_cuda.py:226-230).
 * PB_BOOL is one byte per element, 0 or 1 (nonzero reads as true). */
enum { PB_F32 = 0, PB_F64 = 1, PB_BOOL = 2 };

typedef struct pb_ctx pb_ctx;

/* ---- errors / discovery ------------------------------------------------ */

/* Thread-local message of the last failing call on this thread. */
const char* pb_last_error(void);
/* PB_ABI_VERSION of the loaded library. */
int pb_abi_version(void);
/* Replaces cuda_devices() (src/openpacho/_cuda.py, used by backends.devices
 * at src/openpacho/backends.py:55-60). */
int pb_device_count(int* count);
/* Name, memory, SM count and compute capability of one CUDA ordinal: the
 * fields of the reference's DeviceInfo records (src/openpacho/_cuda.py:68-94). */
int pb_device_info(int ordinal, char* name, size_t name_len, size_t* total_bytes,
                   int* sm_count, int* cc_major, int* cc_minor);
/* CUDA driver version (e.g. 13000), the `driver` field of the reference's
 * DeviceInfo records (src/openpacho/_cuda.py:68-94). */
int pb_driver_version(int* version);

/* ---- context / memory (CUDABackend.__init__/empty/upload/download/close,
 *      src/openpacho/_cuda.py:138-199, 232-311, 644-673) ------------------ */

/* Create a context over `ndev` CUDA ordinals; one stream and one stream-ordered
 * memory pool per device. */
int pb_init(int ndev, const int* ordinals, pb_ctx** out);
/* Synchronise and release every resource of the context (CUDABackend.close,
 * src/openpacho/_cuda.py:644-673). */
int pb_destroy(pb_ctx* ctx);
/* Stream-ordered device allocation (never returns NULL for bytes > 0);
 * replaces CUDABackend.empty's cuMemAlloc or pool reuse (src/openpacho/_cuda.py:241-256). */
int pb_alloc(pb_ctx* ctx, int dev, size_t bytes, void** ptr);
/* Stream-ordered release back to the device pool; replaces the release of an
 * _Allocation into the backend's pool (src/openpacho/_cuda.py:113-125, 258-289). */
int pb_free(pb_ctx* ctx, int dev, void* ptr);
/* Host -> device copy on the context stream.  blocking != 0 waits for the copy
 * (snapshot semantics of CUDABackend.upload, _cuda.py:293-303). */
int pb_h2d(pb_ctx* ctx, int dev, void* dst, const void* src, size_t bytes, int blocking);
/* Device -> host copy; synchronises the stream first (download, _cuda.py:305-311). */
int pb_d2h(pb_ctx* ctx, int dev, void* dst, const void* src, size_t bytes);
/* Asynchronous device -> host copy into pinned memory (no synchronisation).
 * No counterpart in the reference, whose download always synchronises. */
int pb_d2h_async(pb_ctx* ctx, int dev, void* dst, const void* src, size_t bytes);
/* Device -> device copy on the context stream.  No counterpart in the
 * reference's backend protocol (its copies go through host memory). */
int pb_d2d(pb_ctx* ctx, int dev, void* dst, const void* src, size_t bytes);
/* Fill `count` elements with `value` (CUDABackend.full, _cuda.py:404-414);
 * PB_BOOL stores value != 0. */
int pb_fill(pb_ctx* ctx, int dev, int dtype, void* dst, size_t count, double value);
/* Wait for all submitted work; reports kernel-side error flags
 * (CUDABackend.synchronize, src/openpacho/_cuda.py:237-239). */
int pb_sync(pb_ctx* ctx, int dev);
/* Page-lock host memory for asynchronous copies, and undo it.  No
 * counterpart in the reference. */
int pb_host_register(void* ptr, size_t bytes);
int pb_host_unregister(void* ptr);
/* Return pooled device memory and scratch to the driver
 * (release_cached_memory, _cuda.py:262-274). */
int pb_trim(pb_ctx* ctx, int dev);
/* CUDA-event timer on the device stream (for benchmarks): start, then stop and
 * read the elapsed milliseconds.  No counterpart in the reference. */
int pb_timer_start(pb_ctx* ctx, int dev);
int pb_timer_stop(pb_ctx* ctx, int dev, float* ms);
/* Number of kernels this library launched on `dev` since pb_init.  No
 * counterpart in the reference. */
int pb_launch_count(pb_ctx* ctx, int dev, uint64_t* count);
/* Per-kernel timer for rooflines: while enabled, every entry point brackets
 * its main kernel (the GEMM tile kernel, the GEMV/DOT/norm/elementwise/
 * reduction kernel -- not the operand-split or partial-merge helpers) with
 * CUDA events on the device stream.  pb_ktimer_read waits for the stream,
 * returns the summed milliseconds and the number of bracketed launches since
 * the last enable/read, and starts a new count.  At most 4096 launches are
 * kept between reads (PB_ERR_UNSUPPORTED beyond).  An event between two
 * chained launches serialises them, so time the whole step with the timer off.
 * enable = 2 is for a captured step: the event pairs become nodes of the graph,
 * each replay re-records them, and a read returns the last replay's times
 * without starting a new count.  No counterpart in the reference. */
int pb_ktimer_enable(pb_ctx* ctx, int dev, int enable);
int pb_ktimer_read(pb_ctx* ctx, int dev, double* total_ms, uint64_t* launches);
/* Several GPUs in one context (pb_init with ndev > 1; `dev` is the index
 * into its ordinals).  pb_peer_enable turns on peer access between every pair
 * of the context's devices that supports it and reports in *all_pairs (may be
 * NULL) whether every pair does.  Peer access maps memory from
 * pb_alloc_mapped (cudaMalloc) into the other devices, not the stream-ordered
 * pool memory of pb_alloc: a peer copy runs device to device over NVLink when
 * the side of it that is remote to the issuing device comes from
 * pb_alloc_mapped (else the driver stages it).  pb_free_mapped waits for the
 * device's stream before it frees.  Each device has two streams: 0, where
 * every kernel of the library runs, and 1, a copy stream.  pb_copy_peer queues
 * a copy of `bytes` from `src` on device index `src_dev` to `dst` on `dst_dev`
 * on stream `stream` of `stream_dev` (one of the two devices) and orders
 * nothing else; pb_stream_wait makes stream `waiter_stream` of `waiter` wait
 * for the work queued so far on stream `signal_stream` of `signal`.  The
 * caller orders each copy after the producer of its source and the
 * allocation of its destination, and the consumer (or a free) after the
 * copy.  No counterpart in the reference, which drives one device
 * (src/openpacho/_cuda.py:138-199). */
int pb_peer_enable(pb_ctx* ctx, int* all_pairs);
int pb_alloc_mapped(pb_ctx* ctx, int dev, size_t bytes, void** ptr);
int pb_free_mapped(pb_ctx* ctx, int dev, void* ptr);
int pb_copy_peer(pb_ctx* ctx, int dst_dev, void* dst, int src_dev, const void* src, size_t bytes,
                 int stream_dev, int stream);
int pb_stream_wait(pb_ctx* ctx, int waiter, int waiter_stream, int signal, int signal_stream);

/* CUDA graphs of hot-path calls.  pb_capture_begin starts a (relaxed) capture
 * of the device stream; the entry points called until pb_capture_end are
 * recorded, not run, and pb_capture_end returns an instantiated graph that
 * pb_graph_launch replays on the device stream (same pointers, shapes and
 * scalars as captured; the data in the buffers is read afresh every replay).
 * During a capture, calls that synchronise, allocate, free or grow the
 * context's internal buffers, and the sharded mailbox / NCCL exchanges, fail
 * with PB_ERR_UNSUPPORTED: make one uncaptured call of the same shapes first so
 * the buffers have their size.  A failed call leaves the capture open; end it
 * with pb_capture_end (which may then fail) before anything else.  While any
 * graph lives, buffers that grow are kept until the last graph is destroyed,
 * and pb_trim is refused.  Destroy graphs before pb_shutdown.  A 3xTF32 GEMM
 * replays the operand generation it was captured with, so an operand row or
 * column group that held a tiny value (nonzero, below 2^-57) in an earlier
 * replay stays on the float32-FMA recompute in later ones (within the same
 * error bound, slower) until the graph is captured again.  No counterpart in
 * the reference,
 * whose CUDA backend launches eagerly (src/openpacho/_cuda.py). */
int pb_capture_begin(pb_ctx* ctx, int dev);
int pb_capture_end(pb_ctx* ctx, int dev, void** graph);
int pb_graph_launch(pb_ctx* ctx, int dev, void* graph);
int pb_graph_destroy(pb_ctx* ctx, int dev, void* graph);
/* Device memory in use by this context on `dev`: bytes the stream-ordered
 * pool holds reserved from the driver and in use, the size of the context's
 * grow-only scratch buffer, and the device's free memory (cudaMemGetInfo).
 * Memory statistics of the kind the reference's pool keeps in Python
 * (src/openpacho/_cuda.py:232-274). */
int pb_memory_stats(pb_ctx* ctx, int dev, size_t* pool_reserved, size_t* pool_used,
                    size_t* scratch_bytes, size_t* device_free);

/* ---- hot path ---------------------------------------------------------- */

/* C[b] = A[a_off(b)] @ B[b_off(b)] for every index b of the broadcast batch
 * shape `batch_shape[0..batch_ndim)`; a_off/b_off = sum(idx_i * stride_i)
 * with strides in whole matrices (0 = broadcast).  A matrices are M x K,
 * B matrices K x N, C (batch x M x N) is written densely.  K == 0 writes
 * zeros.  float32 uses error-compensated 3xTF32 on tcgen05 tensor cores
 * (never plain TF32), float64 the FP64 tensor cores (DMMA).
 * Replaces NumpyBackend.matmul (src/openpacho/backends.py:139-142) and
 * CUDABackend.matmul (src/openpacho/_cuda.py:493-637) with the register GEMM
 * (src/openpacho/_gemm.py:102-137) and broadcast offsets (_gemm.py:13-21). */
int pb_gemm(pb_ctx* ctx, int dev, int dtype, int batch_ndim, const int64_t* batch_shape,
            const int64_t* a_bstride, const int64_t* b_bstride, int64_t M, int64_t N,
            int64_t K, const void* A, const void* B, void* C);

/* pb_gemm with an explicit kernel choice: PB_GEMM_AUTO (what pb_gemm does),
 * PB_GEMM_SIMT (register-tiled CUDA-core FFMA/DFMA kernel), PB_GEMM_TF32X3
 * (float32; picks one of the two 3xTF32 kernels by size),
 * PB_GEMM_TF32X3_PRESPLIT (operands split into hi/lo copies in HBM first),
 * PB_GEMM_TF32X3_FUSED (A split inside the kernel, into tensor memory;
 * needs K % 4 == 0), PB_GEMM_DMMA (float64 only, FP64 tensor cores) or
 * PB_GEMM_SKINNY (M <= 8: one pass over B with 16-byte loads along N; what
 * pb_gemm uses for M <= 8, vector @ matrix included).  The
 * reference exposes the same kind of provider choice as
 * CUDABackend(blas="custom"|"cublas")
 * (src/openpacho/_cuda.py:138-141). */
enum {
  PB_GEMM_AUTO = 0,
  PB_GEMM_SIMT = 1,
  PB_GEMM_TF32X3 = 2,
  PB_GEMM_DMMA = 3,
  PB_GEMM_TF32X3_PRESPLIT = 4,
  PB_GEMM_TF32X3_FUSED = 5,
  PB_GEMM_SKINNY = 6
};
int pb_gemm_ex(pb_ctx* ctx, int dev, int dtype, int batch_ndim, const int64_t* batch_shape,
               const int64_t* a_bstride, const int64_t* b_bstride, int64_t M, int64_t N,
               int64_t K, const void* A, const void* B, void* C, int algo);

/* pb_gemm with A, B and C in HOST memory: returns when C holds the product.
 * The reference's CUDA backend uploads, multiplies and downloads one step
 * after another (CUDABackend.upload / matmul / download,
 * src/openpacho/_cuda.py:241-281, 493-517).  Here the product is cut into
 * `chunks` pieces (0 = up to 8; at least 4 MiB of traffic each) along the
 * leading batch dimension when A is dense along it (B broadcast along it or
 * dense too), else along the rows of A when there is no batch, else one
 * piece; each piece's A goes up on a host-to-device stream while the previous
 * piece multiplies and the one before comes down on a device-to-host stream,
 * so both directions of the host link and the GEMM overlap.  Host buffers
 * registered with pb_host_register (pinned) let the copies run
 * asynchronously; pageable ones work, with the driver's staged copies. */
int pb_gemm_host(pb_ctx* ctx, int dev, int dtype, int batch_ndim, const int64_t* batch_shape,
                 const int64_t* a_bstride, const int64_t* b_bstride, int64_t M, int64_t N,
                 int64_t K, const void* A, const void* B, void* C, int chunks);

/* y[r] = sum_k A[r,k] * x[k] for r < rows (leading dims flattened into rows).
 * Replaces matvec_data (src/openpacho/_cuda_gemv.py:47-95) and the cuBLAS
 * ?gemv loop (src/openpacho/_cuda_blas.py:32-61). */
int pb_gemv(pb_ctx* ctx, int dev, int dtype, int64_t rows, int64_t K, const void* A,
            const void* x, void* y);

/* out[r] = b[r] - (A @ x)[r] for r < rows: the GEMV with the compiled plan's
 * residual subtraction in its epilogue, so the product never goes to HBM.
 * The product is rounded to the dtype before the subtraction, as in the
 * eager b - A @ x; results are bit-identical to pb_gemv followed by an
 * elementwise subtract.  K == 0 copies b.  `out` may alias `b`.  Replaces
 * residual_matvec_data (src/openpacho/_gemv.py:10-60), which the compiled
 * plans reach through the lowering hook (src/openpacho/_compiler.py:157-176,
 * 306-307). */
int pb_gemv_residual(pb_ctx* ctx, int dev, int dtype, int64_t rows, int64_t K, const void* A,
                     const void* x, const void* b, void* out);

/* *out = sum_i x[i] * y[i] written to device memory.  Replaces the long-DOT
 * chunked path (src/openpacho/_cuda_gemv.py:67-84) and cuBLAS ?dot in
 * device-pointer mode (src/openpacho/_cuda_blas.py:18-30). */
int pb_dot(pb_ctx* ctx, int dev, int dtype, int64_t n, const void* x, const void* y,
           void* out);

/* pb_dot for callers that cannot call cudaMalloc -- for example an engine
 * that hands all device memory to its own allocator up front and forbids
 * other allocations, or a latency-critical loop that must never enter the
 * driver's allocator (which can block, or fail when memory is fully
 * reserved).  Same kernel and result as pb_dot; it allocates nothing.  The
 * caller passes x, y and out as usual.  The DOT's partial sums go to a fixed
 * 33 KiB device array inside the library (room for 4096 partials; a DOT uses
 * at most 16 per SM, 2368 on a B200), which every GPU that loads the library
 * keeps until the process exits; a plan needing more is rejected with
 * PB_ERR_UNSUPPORTED.  pb_init looks the array's device address up for each
 * device of the context, with that device current, and loads the DOT
 * kernels there, so no pb_dot_noalloc call loads code or data onto the
 * device (with lazy module loading, that load could allocate).  The call
 * zeroes the array's arrival counter (a stream-ordered memset of existing
 * memory) before the kernel.  All calls share the one array: calls ordered on one
 * context's stream are safe, calls that overlap on the GPU (other streams or
 * contexts on the same device) race.  No counterpart in the reference. */
int pb_dot_noalloc(pb_ctx* ctx, int dev, int dtype, int64_t n, const void* x, const void* y,
                   void* out);

/* out[o*inner + i] = || x[o, :, i] ||_2 over the middle axis of the
 * contiguous view (outer, reduced, inner).  Overflow/underflow-safe; NaN
 * dominates Inf; -0.0 yields +0.0; reduced == 0 yields 0.
 * Replaces norm_data (src/openpacho/_norm.py:39-118) for any contiguous run
 * of reduced axes. */
int pb_norm(pb_ctx* ctx, int dev, int dtype, int64_t outer, int64_t reduced, int64_t inner,
            const void* x, void* out);

/* General axis sets: output element o (row-major over out_shape) reduces the
 * elements at sum(out_idx*out_strides) + sum(red_idx*red_strides) (element
 * strides) for every index of red_shape.  ndims <= 8 each.  Same semantics
 * as pb_norm; replaces the _index() addressing of src/openpacho/_norm.py:12-25. */
int pb_norm_strided(pb_ctx* ctx, int dev, int dtype, int out_ndim, const int64_t* out_shape,
                    const int64_t* out_strides, int red_ndim, const int64_t* red_shape,
                    const int64_t* red_strides, const void* x, void* out);

/* ---- around the path: elementwise, gather, reductions ----------------- */

/* Elementwise operations, in the names of the reference's expression table
 * (src/openpacho/_cuda.py:21-46) and ufunc list (src/openpacho/_ops.py:5-29). */
enum {
  PB_EW_ADD = 0,
  PB_EW_SUBTRACT,
  PB_EW_MULTIPLY,
  PB_EW_DIVIDE, /* true_divide and divide */
  PB_EW_POWER,
  PB_EW_NEGATIVE,
  PB_EW_POSITIVE,
  PB_EW_ABSOLUTE,
  PB_EW_SQRT,
  PB_EW_EXP,
  PB_EW_LOG,
  PB_EW_SIN,
  PB_EW_COS,
  PB_EW_TANH,
  PB_EW_EQUAL,
  PB_EW_NOT_EQUAL,
  PB_EW_LESS,
  PB_EW_LESS_EQUAL,
  PB_EW_GREATER,
  PB_EW_GREATER_EQUAL,
  PB_EW_ISFINITE,
  PB_EW_CAST,
  PB_EW_WHERE /* a != 0 ? b : c */
};

/* out[i] = op(args...) over the output shape `shape[0..ndim)` (C order).
 * Operand j has dtype arg_dtypes[j] and element strides
 * arg_strides[j*ndim + d] per output dimension (0 = broadcast).  Values are
 * computed in float64 and rounded once to out_dtype (bool: != 0).  Binary ops
 * take 2 operands, where 3, the rest 1.  Replaces CUDABackend.elementwise
 * (src/openpacho/_cuda.py:416-434); oracle NumpyBackend.elementwise
 * (src/openpacho/backends.py:109-116). */
int pb_elementwise(pb_ctx* ctx, int dev, int op, int nargs, const void* const* args,
                   const int* arg_dtypes, const int64_t* arg_strides, int ndim,
                   const int64_t* shape, int out_dtype, void* out);

/* out[i] = src[offset + sum_d idx_d(i) * strides[d]] (element units, strides
 * may be negative): the strided copy behind transpose, diag and slicing.
 * Replaces CUDABackend.gather (src/openpacho/_cuda.py:436-447); oracle
 * NumpyBackend.gather (src/openpacho/backends.py:118-128). */
int pb_gather(pb_ctx* ctx, int dev, int dtype, const void* src, int ndim, const int64_t* shape,
              int64_t offset, const int64_t* strides, void* out);

/* Reductions over the axes set in axes_mask (bit d = axis d) of a C-order
 * array of shape[0..ndim); output in the order of the kept axes.  Sums
 * accumulate in float64 (bool input counts trues; a bool output sum is
 * unsupported, as in the reference); min/max propagate NaN and prefer -0 /
 * +0 on zero ties (src/openpacho/_reductions.py:45-72).  An empty sum
 * writes zeros; an empty extremum is an error.  Replaces CUDABackend.reduce
 * (src/openpacho/_cuda.py:449-492); oracle NumpyBackend.reduce
 * (src/openpacho/backends.py:130-136). */
enum { PB_REDUCE_SUM = 0, PB_REDUCE_MIN = 1, PB_REDUCE_MAX = 2 };
int pb_reduce(pb_ctx* ctx, int dev, int op, int in_dtype, const void* src, int ndim,
              const int64_t* shape, uint32_t axes_mask, int out_dtype, void* out);

/* ---- multi-GPU (one process per GPU; NCCL loaded on first use) --------- *
 * None of these has a counterpart in the reference, which is single-device
 * (src/openpacho/_cuda.py:138-199). */

/* Opaque NCCL unique id (128 bytes) made by rank 0 and shared out of band. */
int pb_comm_unique_id(unsigned char id[128]);
/* Join the communicator of `nranks` processes as `rank` for device `dev`;
 * leave it (waiting for peers) with pb_comm_destroy. */
int pb_comm_init(pb_ctx* ctx, int dev, int nranks, int rank, const unsigned char id[128]);
int pb_comm_destroy(pb_ctx* ctx, int dev);
/* Abandon the communicator without waiting for peers (after a peer failed);
 * outstanding collectives are aborted by NCCL. */
int pb_comm_abort(pb_ctx* ctx, int dev);
/* In-place broadcast of `bytes` from `root` (used to give every GPU the
 * shared B operand of a row-block sharded GEMM). */
int pb_broadcast(pb_ctx* ctx, int dev, void* buf, size_t bytes, int root);
/* Full-array norm of a tensor sliced contiguously across ranks: each rank
 * passes its own slice (n local elements, possibly 0); every rank receives
 * the global norm in `out` (device, 1 element).  Each rank's local
 * (scale exponent, ssq, NaN/Inf class) triple is exchanged -- pushed over
 * NVLink into every peer's mailbox by the reduction kernel itself when peer
 * mailboxes are mapped (pb_peer_import), else one NCCL all-gather of 16 bytes
 * per rank -- and merged on the device in rank order, so every rank computes
 * the identical result.  No counterpart in the reference, which is
 * single-device (src/openpacho/_cuda.py:138-199). */
int pb_norm_sharded(pb_ctx* ctx, int dev, int dtype, int64_t n, const void* x, void* out);
/* Peer mailboxes for the sharded norm and DOT: after them, pb_norm_sharded and
 * pb_dot_sharded exchange each rank's partial with NVLink stores into every
 * peer's memory (the norm from inside its reduction kernel), merged in rank
 * order with waits bounded at 10 s (PB_ERR_DEVICE on timeout) -- no NCCL call.
 * pb_peer_export allocates this rank's mailbox and returns its 64-byte CUDA
 * IPC handle; once every rank's handle is known, pb_peer_import maps them
 * (handles: nranks x 64 bytes in rank order).  PB_ERR_UNAVAILABLE when CUDA
 * IPC is not available: keep using the NCCL path.  2 <= nranks <= 8.
 * pb_peer_close unmaps the peers' mailboxes and frees this rank's. */
int pb_peer_export(pb_ctx* ctx, int dev, int nranks, int rank, unsigned char handle[64]);
int pb_peer_import(pb_ctx* ctx, int dev, int nranks, const unsigned char* handles);
int pb_peer_close(pb_ctx* ctx, int dev);
/* Limit, in nanoseconds, of each wait of the mailbox merge kernels for a
 * peer's partial (default 10 s; 0 restores it).  A wait that runs out sets the
 * kernel error word and the kernel returns, so the next pb_sync reports
 * PB_ERR_DEVICE and the context stays usable; the group's sequence numbers
 * are then out of step and the mailboxes must be closed and set up again.
 * No counterpart in the reference (single-device). */
int pb_peer_set_wait(pb_ctx* ctx, int dev, uint64_t limit_ns);
/* *out = sum over ranks of the DOT of each rank's (x, y) slice (peer
 * mailboxes required), the same value on every rank. */
int pb_dot_sharded(pb_ctx* ctx, int dev, int dtype, int64_t n, const void* x, const void* y,
                   void* out);

/* NCCL sum all-reduce of `count` elements in place (the sharded DOT's
 * fallback when peer mailboxes are not mapped). */
int pb_allreduce_sum(pb_ctx* ctx, int dev, int dtype, void* buf, size_t count);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* PACHO_B200_H */
