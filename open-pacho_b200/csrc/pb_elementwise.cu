// Elementwise operations, strided gather and reductions: the operations the
// callers of the path need around it (astype and the arithmetic of compiled
// solver steps, sum/mean/min/max, transpose/diag views).
//
// Reference: CUDABackend.elementwise / gather / reduce
// (src/openpacho/_cuda.py:416-492) with its expression table _EXPRESSIONS
// (src/openpacho/_cuda.py:21-46) and the extrema algebra of
// src/openpacho/_reductions.py:15-72 (NaN propagates; min prefers -0 and max
// +0 on zero ties; bool min/max are and/or); oracle NumpyBackend
// (src/openpacho/backends.py:109-136).
//
// Values are computed in float64 and rounded once to the output type.  For
// float32 +, -, *, / and sqrt that is the correctly rounded float32 result
// (53 >= 2*24 + 2 bits), bit for bit what float32 arithmetic gives; the
// transcendental functions come out within an ulp of the float32 ones.
// Broadcast operands carry per-dimension element strides (0 = broadcast);
// contiguous and one-element operands skip the index arithmetic.
#include <array>
#include <utility>

#include "pb_internal.cuh"

namespace pb {
namespace {

constexpr int kMaxDims = 8;
constexpr int kThreads = 256;

struct EwParams {
  int op, nargs, ndim, out_dtype;
  int dtype[3];
  int kind[3];  // 0 strided, 1 contiguous like the output, 2 one element
  const void* arg[3];
  int64_t shape[kMaxDims];
  int64_t stride[3][kMaxDims];
  void* out;
  int64_t count;
};

__device__ __forceinline__ double load(const void* p, int dtype, int64_t i) {
  if (dtype == PB_F32) return (double)__ldg(static_cast<const float*>(p) + i);
  if (dtype == PB_F64) return __ldg(static_cast<const double*>(p) + i);
  return static_cast<const unsigned char*>(p)[i] ? 1.0 : 0.0;
}

__device__ __forceinline__ void store(void* p, int dtype, int64_t i, double v) {
  if (dtype == PB_F32)
    static_cast<float*>(p)[i] = (float)v;
  else if (dtype == PB_F64)
    static_cast<double*>(p)[i] = v;
  else
    static_cast<unsigned char*>(p)[i] = v != 0.0;
}

__device__ __forceinline__ double apply(int op, double a, double b, double c) {
  switch (op) {
    case PB_EW_ADD: return a + b;
    case PB_EW_SUBTRACT: return a - b;
    case PB_EW_MULTIPLY: return a * b;
    case PB_EW_DIVIDE: return a / b;
    case PB_EW_POWER: return pow(a, b);
    case PB_EW_NEGATIVE: return -a;
    case PB_EW_POSITIVE: return a;
    case PB_EW_ABSOLUTE: return fabs(a);
    case PB_EW_SQRT: return sqrt(a);
    case PB_EW_EXP: return exp(a);
    case PB_EW_LOG: return log(a);
    case PB_EW_SIN: return sin(a);
    case PB_EW_COS: return cos(a);
    case PB_EW_TANH: return tanh(a);
    case PB_EW_EQUAL: return a == b;
    case PB_EW_NOT_EQUAL: return a != b;
    case PB_EW_LESS: return a < b;
    case PB_EW_LESS_EQUAL: return a <= b;
    case PB_EW_GREATER: return a > b;
    case PB_EW_GREATER_EQUAL: return a >= b;
    case PB_EW_ISFINITE: return isfinite(a);
    case PB_EW_CAST: return a;
    default: return a != 0.0 ? b : c;  // PB_EW_WHERE
  }
}

__global__ void __launch_bounds__(kThreads) elementwise_kernel(const EwParams p) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  bool strided = false;
  for (int j = 0; j < p.nargs; ++j) strided |= p.kind[j] == 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.count; i += stride) {
    int64_t off[3] = {i, i, i};
    if (strided) {
      int64_t rest = i, o0 = 0, o1 = 0, o2 = 0;
      for (int d = p.ndim - 1; d >= 0; --d) {
        const int64_t c = rest % p.shape[d];
        rest /= p.shape[d];
        o0 += c * p.stride[0][d];
        o1 += c * p.stride[1][d];
        o2 += c * p.stride[2][d];
      }
      off[0] = o0, off[1] = o1, off[2] = o2;
    }
    double v[3] = {0.0, 0.0, 0.0};
    for (int j = 0; j < p.nargs; ++j)
      v[j] = load(p.arg[j], p.dtype[j], p.kind[j] == 2 ? 0 : p.kind[j] == 1 ? i : off[j]);
    store(p.out, p.out_dtype, i, apply(p.op, v[0], v[1], v[2]));
  }
}

// Every operand contiguous like the output or a single element: groups of
// four elements, 16-byte loads and stores where the type allows (float32
// operands, float32 output), two groups in flight per thread.
__device__ __forceinline__ void load4(const void* p, int dtype, int kind, int64_t i, double (&v)[4]) {
  if (kind == 2) {
    v[0] = v[1] = v[2] = v[3] = load(p, dtype, 0);
  } else if (dtype == PB_F32) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
    v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
  } else if (dtype == PB_F64) {
    const double2 a = __ldg(reinterpret_cast<const double2*>(static_cast<const double*>(p) + i));
    const double2 b = __ldg(reinterpret_cast<const double2*>(static_cast<const double*>(p) + i + 2));
    v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
  } else {
    const uchar4 q = *reinterpret_cast<const uchar4*>(static_cast<const unsigned char*>(p) + i);
    v[0] = q.x ? 1.0 : 0.0, v[1] = q.y ? 1.0 : 0.0, v[2] = q.z ? 1.0 : 0.0, v[3] = q.w ? 1.0 : 0.0;
  }
}

__device__ __forceinline__ void store4(void* p, int dtype, int64_t i, const double (&v)[4]) {
  if (dtype == PB_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(p) + i) =
        make_float4((float)v[0], (float)v[1], (float)v[2], (float)v[3]);
  } else if (dtype == PB_F64) {
    double2* d = reinterpret_cast<double2*>(static_cast<double*>(p) + i);
    d[0] = make_double2(v[0], v[1]);
    d[1] = make_double2(v[2], v[3]);
  } else {
    *reinterpret_cast<uchar4*>(static_cast<unsigned char*>(p) + i) =
        make_uchar4(v[0] != 0.0, v[1] != 0.0, v[2] != 0.0, v[3] != 0.0);
  }
}

constexpr int operands(int op) {
  return op == PB_EW_WHERE ? 3
         : (op <= PB_EW_POWER || (op >= PB_EW_EQUAL && op <= PB_EW_GREATER_EQUAL)) ? 2 : 1;
}

// One instantiation per operation: the operand count is a compile-time
// constant (operands stay in registers) and only OP's arithmetic is compiled.
template <int OP>
__global__ void __launch_bounds__(kThreads) elementwise_dense_kernel(const EwParams p) {
  constexpr int NA = operands(OP);
  const int64_t groups = p.count / 4;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  auto group = [&](int64_t g) {
    double v[3][4] = {};
#pragma unroll
    for (int j = 0; j < NA; ++j) load4(p.arg[j], p.dtype[j], p.kind[j], 4 * g, v[j]);
    double r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) r[e] = apply(OP, v[0][e], v[1][e], v[2][e]);
    store4(p.out, p.out_dtype, 4 * g, r);
  };
  int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; g + step < groups; g += 2 * step) {
    group(g);
    group(g + step);
  }
  if (g < groups) group(g);
  // The last count % 4 elements.
  const int64_t tail = groups * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (tail < p.count) {
    double v[3] = {0.0, 0.0, 0.0};
#pragma unroll
    for (int j = 0; j < NA; ++j) v[j] = load(p.arg[j], p.dtype[j], p.kind[j] == 2 ? 0 : tail);
    store(p.out, p.out_dtype, tail, apply(OP, v[0], v[1], v[2]));
  }
}

// Correctly rounded operations on float32 operands into float32 (or bool)
// give the same bits in float32 as in float64 rounded once, so they run in
// float32: no conversions, fewer registers, more resident blocks.
constexpr bool exact_in_f32(int op) {
  return op != PB_EW_POWER && !(op >= PB_EW_EXP && op <= PB_EW_TANH);
}

__device__ __forceinline__ float apply_f32(int op, float a, float b, float c) {
  switch (op) {
    case PB_EW_ADD: return a + b;
    case PB_EW_SUBTRACT: return a - b;
    case PB_EW_MULTIPLY: return a * b;
    case PB_EW_DIVIDE: return a / b;
    case PB_EW_NEGATIVE: return -a;
    case PB_EW_POSITIVE: return a;
    case PB_EW_ABSOLUTE: return fabsf(a);
    case PB_EW_SQRT: return sqrtf(a);
    case PB_EW_EQUAL: return a == b;
    case PB_EW_NOT_EQUAL: return a != b;
    case PB_EW_LESS: return a < b;
    case PB_EW_LESS_EQUAL: return a <= b;
    case PB_EW_GREATER: return a > b;
    case PB_EW_GREATER_EQUAL: return a >= b;
    case PB_EW_ISFINITE: return isfinite(a);
    case PB_EW_CAST: return a;
    default: return a != 0.0f ? b : c;  // PB_EW_WHERE
  }
}

// Every operand and the output float32 (bool output for comparisons),
// operation exact in float32: float4 in, float4 (or uchar4) out.
template <int OP>
__global__ void __launch_bounds__(kThreads) elementwise_f32_kernel(const EwParams p) {
  constexpr int NA = operands(OP);
  const int64_t groups = p.count / 4;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  auto load4f = [&](int j, int64_t i) {
    if (p.kind[j] == 2) {
      const float v = __ldg(static_cast<const float*>(p.arg[j]));
      return make_float4(v, v, v, v);
    }
    return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.arg[j]) + i));
  };
  auto group = [&](int64_t g) {
    float4 v[3] = {};
#pragma unroll
    for (int j = 0; j < NA; ++j) v[j] = load4f(j, 4 * g);
    const float4 r = make_float4(apply_f32(OP, v[0].x, v[1].x, v[2].x), apply_f32(OP, v[0].y, v[1].y, v[2].y),
                                 apply_f32(OP, v[0].z, v[1].z, v[2].z), apply_f32(OP, v[0].w, v[1].w, v[2].w));
    if (p.out_dtype == PB_F32)
      *reinterpret_cast<float4*>(static_cast<float*>(p.out) + 4 * g) = r;
    else
      *reinterpret_cast<uchar4*>(static_cast<unsigned char*>(p.out) + 4 * g) =
          make_uchar4(r.x != 0.0f, r.y != 0.0f, r.z != 0.0f, r.w != 0.0f);
  };
  int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; g + step < groups; g += 2 * step) {
    group(g);
    group(g + step);
  }
  if (g < groups) group(g);
  const int64_t tail = groups * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (tail < p.count) {
    float v[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < NA; ++j) v[j] = __ldg(static_cast<const float*>(p.arg[j]) + (p.kind[j] == 2 ? 0 : tail));
    const float r = apply_f32(OP, v[0], v[1], v[2]);
    if (p.out_dtype == PB_F32)
      static_cast<float*>(p.out)[tail] = r;
    else
      static_cast<unsigned char*>(p.out)[tail] = r != 0.0f;
  }
}

using DenseKernel = void (*)(const EwParams);
template <int... OPS>
constexpr auto dense_table(std::integer_sequence<int, OPS...>) {
  return std::array<DenseKernel, sizeof...(OPS)>{&elementwise_dense_kernel<OPS>...};
}
template <int... OPS>
constexpr auto f32_table(std::integer_sequence<int, OPS...>) {
  return std::array<DenseKernel, sizeof...(OPS)>{
      (exact_in_f32(OPS) ? &elementwise_f32_kernel<exact_in_f32(OPS) ? OPS : 0> : nullptr)...};
}
constexpr auto kDense = dense_table(std::make_integer_sequence<int, PB_EW_WHERE + 1>{});
constexpr auto kDenseF32 = f32_table(std::make_integer_sequence<int, PB_EW_WHERE + 1>{});

struct GatherParams {
  const unsigned char* src;
  unsigned char* out;
  int itemsize, ndim;
  int64_t offset;
  int64_t shape[kMaxDims];
  int64_t stride[kMaxDims];
  int64_t count;
};

template <typename W>
__global__ void __launch_bounds__(kThreads) gather_kernel(const GatherParams p) {
  const W* src = reinterpret_cast<const W*>(p.src);
  W* out = reinterpret_cast<W*>(p.out);
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.count; i += step) {
    int64_t rest = i, off = p.offset;
    for (int d = p.ndim - 1; d >= 0; --d) {
      off += (rest % p.shape[d]) * p.stride[d];
      rest /= p.shape[d];
    }
    out[i] = src[off];
  }
}

// ------------------------------------------------------------- reduction --

struct ReduceParams {
  const void* src;
  int in_dtype, out_dtype, op;
  int ondim, rndim;
  int64_t oshape[kMaxDims], ostride[kMaxDims];  // kept dims: extents, input strides
  int64_t rshape[kMaxDims], rstride[kMaxDims];  // reduced dims
  int64_t count, reduced;
  int trailing;      // the reduced axes are the last ones: offset = base + r
  int chunks;        // reduced range split into chunks (block per output x chunk)
  int64_t chunk;     // reduced indices per chunk
  double* partial;   // count x chunks when chunks > 1
  void* out;
};

__device__ __forceinline__ double identity(int op) {
  return op == PB_REDUCE_SUM ? 0.0 : op == PB_REDUCE_MIN ? __longlong_as_double(0x7ff0000000000000ll)
                                                          : -__longlong_as_double(0x7ff0000000000000ll);
}

// src/openpacho/_reductions.py:45-72: NaN propagates; on a zero tie min takes
// the negative zero and max the positive one.
__device__ __forceinline__ double combine(int op, double l, double r) {
  if (op == PB_REDUCE_SUM) return l + r;
  if (isnan(l)) return l;
  if (isnan(r)) return r;
  if (l == 0.0 && r == 0.0) {
    const bool neg = signbit(l);
    return op == PB_REDUCE_MIN ? (neg ? l : r) : (neg ? r : l);
  }
  return op == PB_REDUCE_MIN ? (l < r ? l : r) : (l > r ? l : r);
}

__device__ __forceinline__ int64_t offset_of(const int64_t* shape, const int64_t* stride, int n,
                                             int64_t index) {
  int64_t off = 0;
  for (int d = n - 1; d >= 0; --d) {
    off += (index % shape[d]) * stride[d];
    index /= shape[d];
  }
  return off;
}

// Block per (output, chunk): 256 threads stride over the chunk's reduced
// indices, then a fixed shuffle + shared-memory tree.
// Aligned float32 body [r, body) of one block's chunk: four accumulator lanes
// (one per float4 component), eight 16-byte loads in flight per thread.
template <int OP>
__device__ __forceinline__ double trailing_f32(const float* __restrict__ x, int64_t r,
                                               int64_t body) {
  double lane[4] = {identity(OP), identity(OP), identity(OP), identity(OP)};
  int64_t q = r + 4 * (int64_t)threadIdx.x;
  for (; q + 28 * kThreads < body; q += 32 * kThreads) {
    float4 u[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) u[i] = __ldg(reinterpret_cast<const float4*>(x + q + 4 * kThreads * i));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      lane[0] = combine(OP, lane[0], (double)u[i].x);
      lane[1] = combine(OP, lane[1], (double)u[i].y);
      lane[2] = combine(OP, lane[2], (double)u[i].z);
      lane[3] = combine(OP, lane[3], (double)u[i].w);
    }
  }
  for (; q < body; q += 4 * kThreads) {
    const float4 u = __ldg(reinterpret_cast<const float4*>(x + q));
    lane[0] = combine(OP, lane[0], (double)u.x);
    lane[1] = combine(OP, lane[1], (double)u.y);
    lane[2] = combine(OP, lane[2], (double)u.z);
    lane[3] = combine(OP, lane[3], (double)u.w);
  }
  return combine(OP, combine(OP, lane[0], lane[1]), combine(OP, lane[2], lane[3]));
}

__global__ void __launch_bounds__(kThreads) reduce_blocks_kernel(const ReduceParams p) {
  __shared__ double warp_part[kThreads / 32];
  const int64_t o = blockIdx.x / p.chunks;
  const int c = (int)(blockIdx.x % p.chunks);
  const int64_t base = offset_of(p.oshape, p.ostride, p.ondim, o);
  const int64_t r0 = (int64_t)c * p.chunk, r1 = min(p.reduced, r0 + p.chunk);
  double acc = identity(p.op);
  if (p.trailing && p.in_dtype == PB_F32) {
    // The reduced axes are the trailing ones: [base + r0, base + r1) is
    // contiguous.  Scalar head up to 16-byte alignment, float4 body, tail.
    const float* x = static_cast<const float*>(p.src) + base;
    int64_t r = r0;
    const int64_t head = min(r1, r0 + (int64_t)((4 - ((uintptr_t)(x + r0) >> 2 & 3)) & 3));
    if (r + threadIdx.x < head) acc = combine(p.op, acc, (double)__ldg(x + r + threadIdx.x));
    r = head;
    const int64_t body = r + (r1 - r) / 4 * 4;
    const double lanes = p.op == PB_REDUCE_SUM ? trailing_f32<PB_REDUCE_SUM>(x, r, body)
                         : p.op == PB_REDUCE_MIN ? trailing_f32<PB_REDUCE_MIN>(x, r, body)
                                                 : trailing_f32<PB_REDUCE_MAX>(x, r, body);
    acc = combine(p.op, acc, lanes);
    if (body + threadIdx.x < r1) acc = combine(p.op, acc, (double)__ldg(x + body + threadIdx.x));
  } else if (p.trailing) {
    for (int64_t r = r0 + threadIdx.x; r < r1; r += kThreads)
      acc = combine(p.op, acc, load(p.src, p.in_dtype, base + r));
  } else {
    for (int64_t r = r0 + threadIdx.x; r < r1; r += kThreads)
      acc = combine(p.op, acc, load(p.src, p.in_dtype, base + offset_of(p.rshape, p.rstride, p.rndim, r)));
  }
  for (int s = 16; s > 0; s >>= 1) acc = combine(p.op, acc, __shfl_down_sync(0xffffffffu, acc, s));
  if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = warp_part[0];
    for (int w = 1; w < kThreads / 32; ++w) t = combine(p.op, t, warp_part[w]);
    if (p.chunks == 1)
      store(p.out, p.out_dtype, o, t);
    else
      p.partial[o * p.chunks + c] = t;
  }
}

// Thread per output (short reductions, many outputs), or the final pass over
// the chunk partials in chunk order.
__global__ void __launch_bounds__(kThreads) reduce_threads_kernel(const ReduceParams p, int merge) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < p.count; o += step) {
    double acc;
    if (merge) {
      acc = p.partial[o * p.chunks];
      for (int c = 1; c < p.chunks; ++c) acc = combine(p.op, acc, p.partial[o * p.chunks + c]);
    } else {
      const int64_t base = offset_of(p.oshape, p.ostride, p.ondim, o);
      acc = identity(p.op);
      for (int64_t r = 0; r < p.reduced; ++r)
        acc = combine(p.op, acc, load(p.src, p.in_dtype, base + offset_of(p.rshape, p.rstride, p.rndim, r)));
    }
    store(p.out, p.out_dtype, o, acc);
  }
}

int64_t grid_for(Device* d, int64_t count) {
  int64_t blocks = ceil_div(count, (int64_t)kThreads);
  const int64_t cap = (int64_t)d->sm_count * 16;
  return blocks < 1 ? 1 : blocks > cap ? cap : blocks;
}

// Blocks of kThreads that fit on the device at once (one wave), for a
// grid-stride kernel: more would leave a second, partial wave.
template <typename K>
int64_t wave(Device* d, K kernel) {
  return resident_blocks(d, (const void*)kernel, kThreads);
}

bool valid_dtype(int t) { return t == PB_F32 || t == PB_F64 || t == PB_BOOL; }
size_t itemsize(int t) { return t == PB_F32 ? 4 : t == PB_F64 ? 8 : 1; }

}  // namespace
}  // namespace pb

using namespace pb;

extern "C" {

int pb_elementwise(pb_ctx* ctx, int dev, int op, int nargs, const void* const* args,
                   const int* arg_dtypes, const int64_t* arg_strides, int ndim,
                   const int64_t* shape, int out_dtype, void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (op < 0 || op > PB_EW_WHERE) PB_FAIL(PB_ERR_INVALID, "unknown elementwise operation %d", op);
  const int want = op == PB_EW_WHERE ? 3 : op <= PB_EW_POWER || (op >= PB_EW_EQUAL && op <= PB_EW_GREATER_EQUAL) ? 2 : 1;
  if (nargs != want) PB_FAIL(PB_ERR_INVALID, "operation %d takes %d operands, got %d", op, want, nargs);
  if (ndim < 0 || ndim > kMaxDims) PB_FAIL(PB_ERR_UNSUPPORTED, "at most %d dimensions", kMaxDims);
  if (!valid_dtype(out_dtype)) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", out_dtype);
  EwParams p = {};
  p.op = op;
  p.nargs = nargs;
  p.ndim = ndim;
  p.out_dtype = out_dtype;
  p.out = out;
  p.count = 1;
  for (int d = 0; d < ndim; ++d) {
    if (shape[d] < 0) PB_FAIL(PB_ERR_INVALID, "negative extent");
    p.shape[d] = shape[d];
    p.count *= shape[d];
  }
  if (!p.count) return PB_OK;
  if (!out || !args) PB_FAIL(PB_ERR_INVALID, "null operand");
  for (int j = 0; j < nargs; ++j) {
    if (!args[j]) PB_FAIL(PB_ERR_INVALID, "null operand %d", j);
    if (!valid_dtype(arg_dtypes[j])) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", arg_dtypes[j]);
    p.arg[j] = args[j];
    p.dtype[j] = arg_dtypes[j];
    bool zero = true, contiguous = true;
    int64_t dense = 1;
    for (int d = ndim - 1; d >= 0; --d) {
      const int64_t s = arg_strides[j * ndim + d];
      p.stride[j][d] = s;
      zero &= s == 0 || shape[d] == 1;
      contiguous &= s == dense || shape[d] == 1;
      dense *= shape[d];
    }
    p.kind[j] = zero ? 2 : contiguous ? 1 : 0;
  }
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  bool dense = ((uintptr_t)out & 15) == 0;
  for (int j = 0; j < nargs; ++j) dense &= p.kind[j] != 0 && ((uintptr_t)p.arg[j] & 15) == 0;
  PB_CHECK(kt_begin(d));
  if (dense) {
    bool f32 = kDenseF32[op] != nullptr && (out_dtype == PB_F32 || out_dtype == PB_BOOL);
    for (int j = 0; j < nargs; ++j) f32 &= p.dtype[j] == PB_F32;
    if (op == PB_EW_WHERE) f32 = false;  // a bool condition operand
    const DenseKernel kernel = f32 ? kDenseF32[op] : kDense[op];
    int64_t blocks = ceil_div(p.count / 4 + 1, (int64_t)kThreads);
    const int64_t cap = wave(d, kernel);
    kernel<<<(unsigned)(blocks < cap ? blocks : cap), kThreads, 0, d->stream>>>(p);
  } else {
    elementwise_kernel<<<(unsigned)grid_for(d, p.count), kThreads, 0, d->stream>>>(p);
  }
  PB_LAUNCHED(d);
  return kt_end(d);
}

int pb_gather(pb_ctx* ctx, int dev, int dtype, const void* src, int ndim, const int64_t* shape,
              int64_t offset, const int64_t* strides, void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (!valid_dtype(dtype)) PB_FAIL(PB_ERR_INVALID, "unknown dtype %d", dtype);
  if (ndim < 0 || ndim > kMaxDims) PB_FAIL(PB_ERR_UNSUPPORTED, "at most %d dimensions", kMaxDims);
  GatherParams p = {};
  p.src = static_cast<const unsigned char*>(src);
  p.out = static_cast<unsigned char*>(out);
  p.itemsize = (int)itemsize(dtype);
  p.ndim = ndim;
  p.offset = offset;
  p.count = 1;
  for (int k = 0; k < ndim; ++k) {
    if (shape[k] < 0) PB_FAIL(PB_ERR_INVALID, "negative extent");
    p.shape[k] = shape[k];
    p.stride[k] = strides[k];
    p.count *= shape[k];
  }
  if (!p.count) return PB_OK;
  if (!src || !out) PB_FAIL(PB_ERR_INVALID, "null operand");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  const unsigned grid = (unsigned)grid_for(d, p.count);
  if (p.itemsize == 8)
    gather_kernel<unsigned long long><<<grid, kThreads, 0, d->stream>>>(p);
  else if (p.itemsize == 4)
    gather_kernel<unsigned int><<<grid, kThreads, 0, d->stream>>>(p);
  else
    gather_kernel<unsigned char><<<grid, kThreads, 0, d->stream>>>(p);
  PB_LAUNCHED(d);
  return PB_OK;
}

int pb_reduce(pb_ctx* ctx, int dev, int op, int in_dtype, const void* src, int ndim,
              const int64_t* shape, uint32_t axes_mask, int out_dtype, void* out) {
  if (!ctx) PB_FAIL(PB_ERR_INVALID, "null context");
  if (op != PB_REDUCE_SUM && op != PB_REDUCE_MIN && op != PB_REDUCE_MAX)
    PB_FAIL(PB_ERR_INVALID, "unknown reduction %d", op);
  if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype)) PB_FAIL(PB_ERR_INVALID, "unknown dtype");
  if (op == PB_REDUCE_SUM && out_dtype == PB_BOOL)
    PB_FAIL(PB_ERR_UNSUPPORTED, "boolean sums are not implemented");
  if (ndim < 0 || ndim > kMaxDims) PB_FAIL(PB_ERR_UNSUPPORTED, "at most %d dimensions", kMaxDims);
  ReduceParams p = {};
  p.src = src;
  p.in_dtype = in_dtype;
  p.out_dtype = out_dtype;
  p.op = op;
  p.out = out;
  p.count = 1;
  p.reduced = 1;
  int64_t stride = 1;
  int64_t strides[kMaxDims];
  for (int k = ndim - 1; k >= 0; --k) {
    if (shape[k] < 0) PB_FAIL(PB_ERR_INVALID, "negative extent");
    strides[k] = stride;
    stride *= shape[k];
  }
  int first_reduced = ndim;
  for (int k = 0; k < ndim; ++k)
    if ((axes_mask >> k & 1u) && first_reduced == ndim) first_reduced = k;
  p.trailing = 1;
  for (int k = first_reduced; k < ndim; ++k) p.trailing &= (int)(axes_mask >> k & 1u);
  for (int k = 0; k < ndim; ++k) {
    if (axes_mask >> k & 1u) {
      p.rshape[p.rndim] = shape[k];
      p.rstride[p.rndim++] = strides[k];
      p.reduced *= shape[k];
    } else {
      p.oshape[p.ondim] = shape[k];
      p.ostride[p.ondim++] = strides[k];
      p.count *= shape[k];
    }
  }
  if (!p.count) return PB_OK;
  if (!out) PB_FAIL(PB_ERR_INVALID, "null output");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  Device* d;
  PB_CHECK(enter(ctx, dev, &d));
  if (!p.reduced) {
    if (op != PB_REDUCE_SUM) PB_FAIL(PB_ERR_INVALID, "empty extremum reduction");
    return fill_device(d, out_dtype, out, (size_t)p.count, 0.0);
  }
  if (!src) PB_FAIL(PB_ERR_INVALID, "null input");
  if (p.reduced < 256 && p.count >= (int64_t)d->sm_count * kThreads) {
    p.chunks = 1;
    PB_CHECK(kt_begin(d));
    reduce_threads_kernel<<<(unsigned)grid_for(d, p.count), kThreads, 0, d->stream>>>(p, 0);
    PB_LAUNCHED(d);
    return kt_end(d);
  }
  // One wave of blocks, at least 4096 reduced indices each.
  int64_t chunks = wave(d, reduce_blocks_kernel) / p.count;
  const int64_t most = ceil_div(p.reduced, (int64_t)4096);
  if (chunks > most) chunks = most;
  if (chunks < 1) chunks = 1;
  p.chunk = ceil_div(p.reduced, chunks);
  p.chunks = (int)ceil_div(p.reduced, p.chunk);
  if (p.count * p.chunks > INT32_MAX) PB_FAIL(PB_ERR_UNSUPPORTED, "reduction grid too large");
  if (p.chunks > 1) {
    void* ws;
    PB_CHECK(scratch(d, (size_t)p.count * p.chunks * sizeof(double), &ws));
    p.partial = static_cast<double*>(ws);
  }
  PB_CHECK(kt_begin(d));
  reduce_blocks_kernel<<<(unsigned)(p.count * p.chunks), kThreads, 0, d->stream>>>(p);
  PB_LAUNCHED(d);
  PB_CHECK(kt_end(d));
  if (p.chunks > 1) {
    reduce_threads_kernel<<<(unsigned)grid_for(d, p.count), kThreads, 0, d->stream>>>(p, 1);
    PB_LAUNCHED(d);
  }
  return PB_OK;
}

}  // extern "C"
