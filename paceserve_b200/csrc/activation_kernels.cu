// Gated activations (silu/gelu/gelu-tanh and mul) and the element-wise tanh
// GELUs (gelu_new, gelu_fast) for sm_100a.
//
// Semantics:
//  * silu_and_mul: out = (T)((T)silu(x) * y), silu in fp32
//    (reference csrc/activation_kernels.cu:8-25: silu returns T, the multiply
//    is a T*T operation, i.e. fp32 multiply then rounding to T).
//  * gelu_and_mul / gelu_tanh_and_mul: same rounding points, with the erf GELU
//    and the tanh-approximated GELU (no reference kernel; they match the
//    PyTorch composition F.gelu(x[:, :d], approximate=...) * x[:, d:]).
//  * gelu_new / gelu_fast: the reference's formulas with every intermediate
//    rounded where the reference's T-typed arithmetic rounds
//    (csrc/activation_kernels.cu:86-98).
//
// Design: pure streaming.  2-D grid of (column chunk, row) -- chunk-major, so
// CTAs dispatched together stream neighbouring pieces of one row; each thread
// loads its 16-byte vector of both input halves before any math and stores one
// vector.
// Unaligned shapes use a scalar kernel with the same arithmetic.
#include "common.cuh"

namespace pace {
namespace {

template <typename T>
__device__ __forceinline__ float R(float v) {
  return Traits<T>::round(v);
}

// Gated activations for 16-bit outputs use the hardware's approximate exp2
// and reciprocal (__expf, __fdividef: a few fp32 ulps) -- hidden by the
// rounding to bf16/fp16 in all but ~1e-4 of elements, at a third of the
// instructions, which keeps these streaming kernels memory-bound.  fp32
// outputs use the correctly rounded library functions.
template <typename T>
constexpr bool kFast = sizeof(T) == 2;

struct SiluOp {
  template <typename T>
  __device__ __forceinline__ static float act(float x) {
    if constexpr (kFast<T>) return R<T>(__fdividef(x, 1.0f + __expf(-x)));
    return R<T>(x / (1.0f + expf(-x)));
  }
};

// erf by Abramowitz & Stegun, Handbook of Mathematical Functions, 7.1.26:
// erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2),
// t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7.
__device__ __forceinline__ float erf_as(float x) {
  const float z = fabsf(x);
  const float t = __fdividef(1.0f, fmaf(0.3275911f, z, 1.0f));
  float poly = fmaf(1.061405429f, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  poly *= t;
  const float e = 1.0f - poly * __expf(-z * z);
  return copysignf(e, x);
}

struct GeluErfOp {
  template <typename T>
  __device__ __forceinline__ static float act(float x) {
    const float u = x * 0.70710678118654752440f;  // x / sqrt(2)
    if constexpr (kFast<T>) return R<T>(0.5f * x * (1.0f + erf_as(u)));
    return R<T>(0.5f * x * (1.0f + erff(u)));
  }
};

struct GeluTanhOp {
  template <typename T>
  __device__ __forceinline__ static float act(float x) {
    // sqrt(2/pi) and the cubic coefficient of the tanh approximation.
    const float kBeta = 0.79788456080286535588f;
    const float kKappa = 0.044715f;
    const float x3 = x * x * x;
    const float inner = kBeta * (x + kKappa * x3);
    if constexpr (kFast<T>) {
      // tanh(u) = 1 - 2 / (exp(2u) + 1)
      const float th = 1.0f - __fdividef(2.0f, __expf(2.0f * inner) + 1.0f);
      return R<T>(0.5f * x * (1.0f + th));
    }
    return R<T>(0.5f * x * (1.0f + tanhf(inner)));
  }
};

// gelu_new with the reference's T-typed intermediate roundings
// (csrc/activation_kernels.cu:86-91).
struct GeluNewOp {
  template <typename T>
  __device__ __forceinline__ static float act(float x) {
    const float x3 = R<T>(R<T>(x * x) * x);
    const float a = R<T>(0.044715f * x3);
    const float b = R<T>(x + a);
    const float c = R<T>(0.79788456f * b);
    const float t = R<T>(tanhf(c));
    return R<T>(R<T>(0.5f * x) * R<T>(1.0f + t));
  }
};

// gelu_fast (csrc/activation_kernels.cu:93-98).
struct GeluFastOp {
  template <typename T>
  __device__ __forceinline__ static float act(float x) {
    const float a = R<T>(x * 0.79788456f);
    const float b = R<T>(0.044715f * x);
    const float d = R<T>(1.0f + R<T>(b * x));
    const float t = R<T>(tanhf(R<T>(a * d)));
    return R<T>(R<T>(0.5f * x) * R<T>(1.0f + t));
  }
};

// GATED: in row = [x (d) | y (d)], out = act(x) * y.  Otherwise out = act(x).
template <typename T, typename Op, int U, bool GATED>
__global__ void __launch_bounds__(256)
    act_vec_kernel(T* __restrict__ out, const T* __restrict__ in, int64_t d, int64_t in_stride,
                   int64_t out_stride, int chunk_major) {
  using Tr = Traits<T>;
  constexpr int V = Tr::kVec;
  // chunk_major: grid (chunks, rows), so CTAs dispatched together stream
  // neighbouring pieces of one row; otherwise grid (rows, chunks).
  const int64_t row = chunk_major ? blockIdx.y : blockIdx.x;
  const int64_t nvec = d / V;
  const int64_t first = (int64_t)(chunk_major ? blockIdx.x : blockIdx.y) * (blockDim.x * U);
  const int64_t base = first + threadIdx.x;
  const T* xr = in + row * in_stride;
  T* orow = out + row * out_stride;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    const int64_t span = (int64_t)blockDim.x * U;
    const int64_t nv = nvec - first < span ? nvec - first : span;
    prefetch_l2(xr + first * V, nv * 16);
    if (GATED) prefetch_l2(xr + d + first * V, nv * 16);
  }
  pdl_wait();
  uint4 xv[U], yv[U];
#pragma unroll
  for (int j = 0; j < U; ++j) {
    const int64_t c = base + (int64_t)j * blockDim.x;
    if (c < nvec) {
      xv[j] = ld_nc_v4(xr + c * V);
      if (GATED) yv[j] = ld_nc_v4(xr + d + c * V);
    }
  }
#pragma unroll
  for (int j = 0; j < U; ++j) {
    const int64_t c = base + (int64_t)j * blockDim.x;
    if (c < nvec) {
      float x[V], o[V];
      Tr::unpack(xv[j], x);
      if (GATED) {
        float y[V];
        Tr::unpack(yv[j], y);
#pragma unroll
        for (int e = 0; e < V; ++e) o[e] = Op::template act<T>(x[e]) * y[e];
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) o[e] = Op::template act<T>(x[e]);
      }
      st_v4(orow + c * V, Tr::pack(o));
    }
  }
}

template <typename T, typename Op, bool GATED>
__global__ void __launch_bounds__(256)
    act_scalar_kernel(T* __restrict__ out, const T* __restrict__ in, int64_t d, int64_t in_stride,
                      int64_t out_stride) {
  using Tr = Traits<T>;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const T* xr = in + row * in_stride;
  T* orow = out + row * out_stride;
  for (int64_t i = (int64_t)blockIdx.y * blockDim.x + threadIdx.x; i < d;
       i += (int64_t)gridDim.y * blockDim.x) {
    const float x = Tr::to_f(xr[i]);
    float o = Op::template act<T>(x);
    if (GATED) o = o * Tr::to_f(xr[d + i]);
    orow[i] = Tr::from_f(o);
  }
}

template <typename T, typename Op, bool GATED>
int launch_act(void* out, const void* in, int64_t num_tokens, int64_t d, int64_t in_stride,
               int64_t out_stride, cudaStream_t stream, const char* name) {
  constexpr int V = Traits<T>::kVec;
  T* o = static_cast<T*>(out);
  const T* x = static_cast<const T*>(in);
  const bool vec = (d % V == 0) && (in_stride % V == 0) && (out_stride % V == 0) &&
                   aligned16(out) && aligned16(in);
  cudaError_t err;
  if (vec) {
    const int64_t nvec = d / V;
    // One vector pair per thread, 256-thread CTAs: many small CTAs (8 per SM)
    // balance the last wave best -- on B200 this shape moved silu_and_mul at
    // [512, 2 x 14336] 13 % faster than 4 vectors per thread (128- and
    // 512-thread CTAs were 3-15 % slower).  Chunk-major order (consecutive CTAs
    // on consecutive pieces of the same row) is 3-4 % faster than row-major
    // at every T >= 512; rows beyond the grid's y limit use row-major.
    // Decode batches (T <= 64) use 128-thread CTAs: twice the CTAs spread the
    // few rows over more SMs (T = 1: 12 % faster; at T = 128 the 70B width was
    // 8 % slower).
    const int threads = num_tokens <= 64 ? 128 : 256;
    const int64_t chunks = ceil_div(nvec, threads);
    const bool cm = num_tokens <= 65535;
    const dim3 grid = cm ? dim3((unsigned)chunks, (unsigned)num_tokens)
                         : dim3((unsigned)num_tokens, (unsigned)chunks);
    err = launch(act_vec_kernel<T, Op, 1, GATED>, grid, dim3(threads), 0, stream, o, x, d,
                 in_stride, out_stride, cm ? 1 : 0);
  } else {
    const int64_t bx = ceil_div(d, 256) < 64 ? ceil_div(d, 256) : 64;
    const dim3 grid((unsigned)num_tokens, (unsigned)bx);
    err = launch(act_scalar_kernel<T, Op, GATED>, grid, dim3(256), 0, stream, o, x, d, in_stride,
                 out_stride);
  }
  if (err != cudaSuccess) return cuda_fail(err, name);
  return PACE_OK;
}

template <typename Op, bool GATED>
int act_entry(void* out, const void* input, int64_t num_tokens, int64_t d, int64_t in_stride,
              int64_t out_stride, int dtype, cudaStream_t stream, const char* name) {
  if (num_tokens < 0 || d < 0 || num_tokens > INT32_MAX)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad shape [%lld, %lld]", name,
                (long long)num_tokens, (long long)d);
  // Past 65535 rows the grid is row-major, with the row's chunks (256 x 4
  // fp32 elements at least) in grid.y.
  if (num_tokens > 65535 && d / 4 > 65535LL * 256)
    return fail(PACE_ERR_TOO_LARGE, "%s: row width %lld too large", name, (long long)d);
  const int64_t in_w = GATED ? 2 * d : d;
  if (in_stride < in_w || out_stride < d)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: row stride smaller than the row", name);
  if (num_tokens == 0 || d == 0) return PACE_OK;
  if (!out || !input) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  StreamDeviceGuard guard(stream);
  return PACE_DISPATCH_FLOAT(dtype, name, [&] {
    return launch_act<scalar_t, Op, GATED>(out, input, num_tokens, d, in_stride, out_stride,
                                           stream, name);
  });
}

}  // namespace
}  // namespace pace

extern "C" int pace_silu_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                                 int64_t input_row_stride, int64_t out_row_stride, int dtype,
                                 cudaStream_t stream) {
  return pace::act_entry<pace::SiluOp, true>(out, input, num_tokens, d, input_row_stride,
                                             out_row_stride, dtype, stream, "silu_and_mul");
}

extern "C" int pace_gelu_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                                 int64_t input_row_stride, int64_t out_row_stride, int dtype,
                                 cudaStream_t stream) {
  return pace::act_entry<pace::GeluErfOp, true>(out, input, num_tokens, d, input_row_stride,
                                                out_row_stride, dtype, stream, "gelu_and_mul");
}

extern "C" int pace_gelu_tanh_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                                      int64_t input_row_stride, int64_t out_row_stride, int dtype,
                                      cudaStream_t stream) {
  return pace::act_entry<pace::GeluTanhOp, true>(out, input, num_tokens, d, input_row_stride,
                                                 out_row_stride, dtype, stream,
                                                 "gelu_tanh_and_mul");
}

extern "C" int pace_gelu_new(void* out, const void* input, int64_t num_tokens, int64_t d,
                             int64_t input_row_stride, int64_t out_row_stride, int dtype,
                             cudaStream_t stream) {
  return pace::act_entry<pace::GeluNewOp, false>(out, input, num_tokens, d, input_row_stride,
                                                 out_row_stride, dtype, stream, "gelu_new");
}

extern "C" int pace_gelu_fast(void* out, const void* input, int64_t num_tokens, int64_t d,
                              int64_t input_row_stride, int64_t out_row_stride, int dtype,
                              cudaStream_t stream) {
  return pace::act_entry<pace::GeluFastOp, false>(out, input, num_tokens, d, input_row_stride,
                                                  out_row_stride, dtype, stream, "gelu_fast");
}
