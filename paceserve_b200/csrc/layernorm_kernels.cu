// RMSNorm and fused residual-add + RMSNorm for sm_100a.
//
// Semantics follow the reference kernel (csrc/layernorm_kernels.cu:10-35):
// fp32 sum of squares, inv = rsqrtf(sum / H + eps), and the normalised value
// is rounded to the storage type BEFORE the weight multiply
// (out = (T)((T)(x * inv) * w), layernorm_kernels.cu:33).  The fused variant
// restates the PyTorch composition at paceserve/model_executor/models/llama.py:
// 248-252: residual <- (T)(x + residual), then rms_norm of that rounded sum.
//
// Design: one CTA per token row (two rows for the plain norm at large T); the
// row is read once with 16-byte vectors and held in registers across the
// reduction (the reference reads it twice with 2-byte loads); warp-shuffle
// then shared-memory reduction, fixed order so all threads derive the
// identical inv.  The Llama-3 widths (4096, 8192) in 16-bit types run a kernel
// whose CTA shape and row width are compile-time constants (no per-vector
// guards, a constant divisor), 8-45 % faster at T <= 1024; other widths run
// the general vector kernel.  Rows that do not meet the vector alignment go
// through a scalar two-pass kernel.
#include "common.cuh"

namespace pace {
namespace {

constexpr int kMaxThreads = 512;  // vector path: rows up to 4 x 512 vectors

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Sum of `v` over the CTA; every thread gets the same value.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = (blockDim.x + 31) >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (nwarps > 8) {
    // Every warp reduces the partials with the same butterfly, so every thread
    // gets the same total; with 16 warps this is 3 % faster than a serial sum.
    const float t = lane < nwarps ? red[lane] : 0.f;
    return warp_sum(t);
  }
  float total = 0.f;
  for (int i = 0; i < nwarps; ++i) total += red[i];
  return total;
}

// Vector path.  NV = 16-byte vectors per thread (at most 4 with up to 512
// threads, so a row of up to 2048 vectors -- H = 16384 in bf16 -- stays in
// registers).  Shape, measured on B200: the fused norm (two input rows per
// thread) runs up to 512 threads x 1 vector per row (10 % faster than 256 x 2
// at H = 4096); the plain norm keeps 256 x 2, since one load per thread halves
// the bytes in flight per SM and cost it 25 % at large T.  FUSED: x_in == x_out is the
// hidden-state row (read, then overwritten with the normalised row) and
// `res` is the residual row (overwritten with x + res).
template <typename T, int NV, bool FUSED>
__global__ void __launch_bounds__(kMaxThreads)
    rms_norm_vec_kernel(const T* x_in, T* x_out, T* res, const T* __restrict__ weight, float eps,
                        int hidden, int64_t in_stride, int64_t out_stride, int64_t res_stride) {
  using Tr = Traits<T>;
  constexpr int V = Tr::kVec;
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = hidden / V;
  const T* xr = x_in + row * in_stride;
  T* orow = x_out + row * out_stride;
  T* rr = FUSED ? res + row * res_stride : nullptr;

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    prefetch_l2(xr, (int64_t)hidden * sizeof(T));
    if (FUSED) prefetch_l2(rr, (int64_t)hidden * sizeof(T));
    if (row < 4) prefetch_l2(weight, (int64_t)hidden * sizeof(T));
  }
  pdl_wait();

  float v[NV][V];
  uint4 raw[NV];
  uint4 rraw[NV];
  uint4 wraw[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < nvec) {
      if (FUSED) {
        raw[j] = ld_v4(xr + (int64_t)c * V);
        rraw[j] = ld_v4(rr + (int64_t)c * V);
      } else {
        raw[j] = ld_nc_v4(xr + (int64_t)c * V);
      }
      wraw[j] = __ldg(reinterpret_cast<const uint4*>(weight) + c);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < nvec) {
      Tr::unpack(raw[j], v[j]);
      if (FUSED) {
        float r[V];
        Tr::unpack(rraw[j], r);
#pragma unroll
        for (int e = 0; e < V; ++e) v[j][e] = Tr::round(v[j][e] + r[e]);
        st_v4(rr + (int64_t)c * V, Tr::pack(v[j]));
      }
#pragma unroll
      for (int e = 0; e < V; ++e) ss += v[j][e] * v[j][e];
    }
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total / (float)hidden + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < nvec) {
      float w[V];
      Tr::unpack(wraw[j], w);
      float o[V];
#pragma unroll
      for (int e = 0; e < V; ++e) o[e] = Tr::round(v[j][e] * inv) * w[e];
      st_v4(orow + (int64_t)c * V, Tr::pack(o));
    }
  }
}

// Plain rms_norm, R rows per CTA: each thread holds NV vectors of each of the
// R rows, so a CTA has R times the bytes in flight of the one-row kernel and
// one barrier serves R rows.  Rows past `rows` (the last CTA) are skipped.
template <typename T, int NV, int R>
__global__ void __launch_bounds__(kMaxThreads)
    rms_norm_rows_kernel(const T* __restrict__ x_in, T* __restrict__ x_out,
                         const T* __restrict__ weight, float eps, int hidden, int64_t rows,
                         int64_t in_stride, int64_t out_stride) {
  using Tr = Traits<T>;
  constexpr int V = Tr::kVec;
  __shared__ float red[R][32];
  const int64_t row0 = (int64_t)blockIdx.x * R;
  const int nvec = hidden / V;
  pdl_launch_dependents();
  if (threadIdx.x < R && row0 + threadIdx.x < rows)
    prefetch_l2(x_in + (row0 + threadIdx.x) * in_stride, (int64_t)hidden * sizeof(T));
  if (threadIdx.x == R && blockIdx.x < 4) prefetch_l2(weight, (int64_t)hidden * sizeof(T));
  pdl_wait();

  uint4 raw[R][NV];
  uint4 wraw[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < nvec) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (row0 + r < rows) raw[r][j] = ld_nc_v4(x_in + (row0 + r) * in_stride + (int64_t)c * V);
      wraw[j] = __ldg(reinterpret_cast<const uint4*>(weight) + c);
    }
  }
  float ss[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    ss[r] = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c < nvec && row0 + r < rows) {
        float v[V];
        Tr::unpack(raw[r][j], v);
#pragma unroll
        for (int e = 0; e < V; ++e) ss[r] += v[e] * v[e];
      }
    }
    ss[r] = warp_sum(ss[r]);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = (blockDim.x + 31) >> 5;
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) red[r][warp] = ss[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (row0 + r >= rows) break;
    float total = 0.f;
    for (int i = 0; i < nwarps; ++i) total += red[r][i];
    const float inv = rsqrtf(total / (float)hidden + eps);
    T* orow = x_out + (row0 + r) * out_stride;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c < nvec) {
        float v[V], w[V], o[V];
        Tr::unpack(raw[r][j], v);
        Tr::unpack(wraw[j], w);
#pragma unroll
        for (int e = 0; e < V; ++e) o[e] = Tr::round(v[e] * inv) * w[e];
        st_v4(orow + (int64_t)c * V, Tr::pack(o));
      }
    }
  }
}

// Exact-fit vector path for 16-bit rows: hidden == NT * NV * 8 at compile
// time, so every thread owns exactly NV vectors (no per-vector guards), the
// CTA size and warp count are constants, and the mean's divisor is a
// constant (a power of two becomes an exact multiply).  WASM: the weight is
// loaded with the same ordered vector load as the row, so it is in flight
// together with the row instead of wherever the compiler schedules it.
// Arithmetic, rounding points and reduction order per thread/warp are those
// of rms_norm_vec_kernel.
template <typename T, int NT, int NV, bool FUSED, bool WASM>
__global__ void __launch_bounds__(NT)
    rms_norm_exact_kernel(const T* x_in, T* x_out, T* res, const T* __restrict__ weight, float eps,
                          int64_t in_stride, int64_t out_stride, int64_t res_stride) {
  using Tr = Traits<T>;
  constexpr int V = Tr::kVec;
  constexpr int HID = NT * NV * V;
  constexpr int NW = NT / 32;
  static_assert(NT % 32 == 0 && NW <= 32, "");
  __shared__ float red[NW];
  const int64_t row = blockIdx.x;
  const T* xr = x_in + row * in_stride;
  T* orow = x_out + row * out_stride;
  T* rr = FUSED ? res + row * res_stride : nullptr;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    prefetch_l2(xr, HID * (int)sizeof(T));
    if (FUSED) prefetch_l2(rr, HID * (int)sizeof(T));
    if (row < 4) prefetch_l2(weight, HID * (int)sizeof(T));
  }
  pdl_wait();
  uint4 a[NV], b[NV], wv[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = threadIdx.x + j * NT;
    if (FUSED) {
      a[j] = ld_v4(xr + c * V);
      b[j] = ld_v4(rr + c * V);
    } else {
      a[j] = ld_nc_v4(xr + c * V);
    }
    wv[j] = WASM ? ld_nc_v4(weight + c * V) : __ldg(reinterpret_cast<const uint4*>(weight) + c);
  }
  float v[NV][V];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = threadIdx.x + j * NT;
    Tr::unpack(a[j], v[j]);
    if (FUSED) {
      float q[V];
      Tr::unpack(b[j], q);
#pragma unroll
      for (int e = 0; e < V; ++e) v[j][e] = Tr::round(v[j][e] + q[e]);
      st_v4(rr + c * V, Tr::pack(v[j]));
    }
#pragma unroll
    for (int e = 0; e < V; ++e) ss += v[j][e] * v[j][e];
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float total = ss;
  if (NW > 1) {
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (NW > 8) {
      total = warp_sum(lane < NW ? red[lane] : 0.f);
    } else {
      total = 0.f;
#pragma unroll
      for (int i = 0; i < NW; ++i) total += red[i];
    }
  }
  const float inv = rsqrtf(total / (float)HID + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = threadIdx.x + j * NT;
    float w[V], o[V];
    Tr::unpack(wv[j], w);
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = Tr::round(v[j][e] * inv) * w[e];
    st_v4(orow + c * V, Tr::pack(o));
  }
}

// Rows per CTA of the plain norm's vector path (1 = rms_norm_vec_kernel).
// Measured on B200: two rows per CTA are 8-9 % faster (8B) and 3-4 % faster
// (70B) at T >= 8192, 5 % slower at T = 2048 and 45 % slower at T = 512, where
// halving the CTA count leaves SMs idle.
inline int norm_rows_per_cta(int64_t num_tokens) { return num_tokens >= 8192 ? 2 : 1; }

// Scalar fallback for any hidden size, stride or alignment.
template <typename T, bool FUSED>
__global__ void __launch_bounds__(256)
    rms_norm_scalar_kernel(const T* x_in, T* x_out, T* res, const T* __restrict__ weight,
                           float eps, int hidden, int64_t in_stride, int64_t out_stride,
                           int64_t res_stride) {
  using Tr = Traits<T>;
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const T* xr = x_in + row * in_stride;
  T* orow = x_out + row * out_stride;
  T* rr = FUSED ? res + row * res_stride : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    float x = Tr::to_f(xr[i]);
    if (FUSED) {
      x = Tr::round(x + Tr::to_f(rr[i]));
      rr[i] = Tr::from_f(x);
    }
    ss += x * x;
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total / (float)hidden + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    // Each thread re-reads only elements it read (and, fused, wrote) itself.
    const float x = FUSED ? Tr::to_f(rr[i]) : Tr::to_f(xr[i]);
    orow[i] = Tr::from_f(Tr::round(x * inv) * Tr::to_f(weight[i]));
  }
}

// Exact-fit shape (threads x vectors per thread) for a 16-bit row of `hidden`
// elements at `num_tokens` rows, or {0, 0} when the general kernels serve it.
// Measured on B200 (32 back-to-back launches over distinct buffers, us):
//   fused, H = 4096: T=1 1.54 (256x2), T=128 2.12 (256x2; 512x1 2.44),
//     T=512 3.20 (512x1; 256x2 4.29, general kernel 3.46), T=2048 11.45,
//     T=16384 79.3 (256x2; 512x1 81.8);  H = 8192: 512x2 at every T (equal to
//     the general kernel, 256x4 1-8 % slower).
//   plain, H = 4096: 256x2 up to T=1024 (T=1 1.03 against 1.48, T=512 2.19
//     against 3.07), 128x4 up to 8192 (T=2048 6.60 against 7.24), then the
//     two-row kernel;  H = 8192: 512x2 up to T=128 (2.13 against 3.07), 256x4 up
//     to 2048 (T=512 3.61 against 3.92), then the two-row kernel.
struct ExactShape {
  int threads, nv;
};
inline ExactShape exact_shape(bool fused, int64_t hidden, int64_t num_tokens) {
  if (hidden == 4096) {
    if (fused) return num_tokens > 128 && num_tokens <= 1024 ? ExactShape{512, 1} : ExactShape{256, 2};
    if (num_tokens <= 1024) return {256, 2};
    if (num_tokens < 8192) return {128, 4};
    return {0, 0};
  }
  if (hidden == 8192) {
    if (fused) return {512, 2};
    if (num_tokens <= 128) return {512, 2};
    if (num_tokens <= 2048) return {256, 4};
    return {0, 0};
  }
  return {0, 0};
}

template <typename T, bool FUSED>
int launch_norm(const void* x_in, void* x_out, void* res, const void* weight, float eps,
                int64_t num_tokens, int64_t hidden, int64_t in_stride, int64_t out_stride,
                int64_t res_stride, cudaStream_t stream, const char* name) {
  constexpr int V = Traits<T>::kVec;
  const T* xi = static_cast<const T*>(x_in);
  T* xo = static_cast<T*>(x_out);
  T* r = static_cast<T*>(res);
  const T* w = static_cast<const T*>(weight);
  const int64_t nvec = hidden / V;
  bool vec = (hidden % V == 0) && (in_stride % V == 0) && (out_stride % V == 0) &&
             aligned16(x_in) && aligned16(x_out) && aligned16(weight) &&
             nvec <= 4 * kMaxThreads;
  if (FUSED) vec = vec && (res_stride % V == 0) && aligned16(res);
  cudaError_t err;
  const dim3 grid((unsigned)num_tokens);
  if constexpr (V == 8) {
    const ExactShape sh = vec ? exact_shape(FUSED, hidden, num_tokens) : ExactShape{0, 0};
    if (sh.threads > 0) {
      switch (sh.threads * 10 + sh.nv) {
#define PACE_EXACT_CASE(NT, NV)                                                                 \
  case NT * 10 + NV:                                                                            \
    err = launch(rms_norm_exact_kernel<T, NT, NV, FUSED, false>, grid, dim3(NT), 0, stream, xi, \
                 xo, r, w, eps, in_stride, out_stride, res_stride);                             \
    break;
        PACE_EXACT_CASE(512, 1)
        PACE_EXACT_CASE(256, 2)
        PACE_EXACT_CASE(128, 4)
        PACE_EXACT_CASE(512, 2)
        PACE_EXACT_CASE(256, 4)
#undef PACE_EXACT_CASE
        default: return fail(PACE_ERR_INVALID_ARGUMENT, "%s: internal exact shape", name);
      }
      if (err != cudaSuccess) return cuda_fail(err, name);
      return PACE_OK;
    }
  }
  if (vec) {
    // Threads per row, measured on B200: the fused norm up to 512, but 256 for
    // T <= 128 with rows of <= 512 vectors (H = 4096 bf16: 20 % faster at
    // T = 128, 1-3 % below; wider rows were 3 % slower); the plain norm up to
    // 256, and 128 for 1024 <= T < 8192 (4 vectors per thread at H = 4096: 8-15 %
    // faster there, 0-13 % slower below).
    const int max_threads =
        FUSED ? (num_tokens <= 128 && nvec <= 512 ? 256 : kMaxThreads)
              : (num_tokens >= 1024 && num_tokens < 8192 ? 128 : kMaxThreads / 2);
    int nv = 1;
    while (nv < 4 && ceil_div(nvec, nv) > max_threads) nv *= 2;
    int threads = (int)ceil_div(ceil_div(nvec, nv), 32) * 32;
    if (threads > kMaxThreads) threads = kMaxThreads;
    const int h = (int)hidden;
    const int rows_per_cta = FUSED ? 1 : norm_rows_per_cta(num_tokens);
    if (!FUSED && rows_per_cta > 1) {
      const dim3 g((unsigned)ceil_div(num_tokens, (int64_t)rows_per_cta));
      switch (nv * 10 + rows_per_cta) {
#define PACE_ROWS_CASE(N, R)                                                                  \
  case N * 10 + R:                                                                            \
    err = launch(rms_norm_rows_kernel<T, N, R>, g, dim3(threads), 0, stream, xi, xo, w, eps, h, \
                 num_tokens, in_stride, out_stride);                                          \
    break;
        PACE_ROWS_CASE(1, 2)
        PACE_ROWS_CASE(2, 2)
        PACE_ROWS_CASE(4, 2)
#undef PACE_ROWS_CASE
        default: return fail(PACE_ERR_INVALID_ARGUMENT, "%s: internal row split", name);
      }
      if (err != cudaSuccess) return cuda_fail(err, name);
      return PACE_OK;
    }
    switch (nv) {
#define PACE_NORM_CASE(N)                                                                     \
  case N:                                                                                     \
    err = launch(rms_norm_vec_kernel<T, N, FUSED>, grid, dim3(threads), 0, stream, xi, xo, r, \
                 w, eps, h, in_stride, out_stride, res_stride);                               \
    break;
      PACE_NORM_CASE(1)
      PACE_NORM_CASE(2)
      PACE_NORM_CASE(4)
#undef PACE_NORM_CASE
      default: return fail(PACE_ERR_INVALID_ARGUMENT, "%s: internal vector split", name);
    }
  } else {
    err = launch(rms_norm_scalar_kernel<T, FUSED>, grid, dim3(256), 0, stream, xi, xo, r, w, eps,
                 (int)hidden, in_stride, out_stride, res_stride);
  }
  if (err != cudaSuccess) return cuda_fail(err, name);
  return PACE_OK;
}

}  // namespace
}  // namespace pace

extern "C" int pace_rms_norm(void* out, const void* input, const void* weight, float epsilon,
                             int64_t num_tokens, int64_t hidden_size, int64_t input_row_stride,
                             int64_t out_row_stride, int dtype, cudaStream_t stream) {
  using namespace pace;
  if (num_tokens < 0 || hidden_size <= 0 || hidden_size > INT32_MAX || num_tokens > INT32_MAX)
    return fail(PACE_ERR_INVALID_ARGUMENT, "rms_norm: bad shape [%lld, %lld]",
                (long long)num_tokens, (long long)hidden_size);
  if (input_row_stride < hidden_size || out_row_stride < hidden_size)
    return fail(PACE_ERR_INVALID_ARGUMENT, "rms_norm: row stride smaller than hidden size");
  if (num_tokens == 0) return PACE_OK;
  if (!out || !input || !weight) return fail(PACE_ERR_INVALID_ARGUMENT, "rms_norm: null pointer");
  StreamDeviceGuard guard(stream);
  return PACE_DISPATCH_FLOAT(dtype, "rms_norm", [&] {
    return launch_norm<scalar_t, false>(input, out, nullptr, weight, epsilon, num_tokens,
                                        hidden_size, input_row_stride, out_row_stride, 0, stream,
                                        "rms_norm");
  });
}

extern "C" int pace_fused_add_rms_norm(void* input, void* residual, const void* weight,
                                       float epsilon, int64_t num_tokens, int64_t hidden_size,
                                       int64_t input_row_stride, int64_t residual_row_stride,
                                       int dtype, cudaStream_t stream) {
  using namespace pace;
  if (num_tokens < 0 || hidden_size <= 0 || hidden_size > INT32_MAX || num_tokens > INT32_MAX)
    return fail(PACE_ERR_INVALID_ARGUMENT, "fused_add_rms_norm: bad shape [%lld, %lld]",
                (long long)num_tokens, (long long)hidden_size);
  if (input_row_stride < hidden_size || residual_row_stride < hidden_size)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "fused_add_rms_norm: row stride smaller than hidden size");
  if (num_tokens == 0) return PACE_OK;
  if (!input || !residual || !weight)
    return fail(PACE_ERR_INVALID_ARGUMENT, "fused_add_rms_norm: null pointer");
  StreamDeviceGuard guard(stream);
  return PACE_DISPATCH_FLOAT(dtype, "fused_add_rms_norm", [&] {
    return launch_norm<scalar_t, true>(input, input, residual, weight, epsilon, num_tokens,
                                       hidden_size, input_row_stride, input_row_stride,
                                       residual_row_stride, stream, "fused_add_rms_norm");
  });
}

// Row sum-of-squares partials for the RMSNorm that the GEMM epilogues apply:
// out[t, g] = sum of x[t, c]^2 over the 32 columns c of group g, in fp32.
// One CTA per row, one thread per group (four 16-byte loads).
namespace pace {
namespace {
template <typename T>
__global__ void __launch_bounds__(256)
    row_sumsq_kernel(float* __restrict__ out, const T* __restrict__ x, int groups,
                     int64_t in_stride) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const T* xr = x + row * in_stride;
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float v[8];
      Traits<T>::unpack(ld_nc_v4(xr + g * 32 + q * 8), v);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
    }
    out[row * groups + g] = ss;
  }
}
}  // namespace
}  // namespace pace

extern "C" int pace_row_sumsq(float* row_sumsq, const void* input, int64_t num_tokens,
                              int64_t hidden_size, int64_t input_row_stride, int dtype,
                              cudaStream_t stream) {
  using namespace pace;
  if (num_tokens < 0 || num_tokens > INT32_MAX || hidden_size <= 0 || hidden_size % 32 != 0 ||
      hidden_size / 32 > INT32_MAX)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "row_sumsq: hidden size %lld must be a positive multiple of 32",
                (long long)hidden_size);
  if (input_row_stride < hidden_size || input_row_stride % 8 != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "row_sumsq: row stride must be >= the row and a multiple of 8");
  if (num_tokens == 0) return PACE_OK;
  if (!row_sumsq || !input) return fail(PACE_ERR_INVALID_ARGUMENT, "row_sumsq: null pointer");
  if (!aligned16(input)) return fail(PACE_ERR_INVALID_ARGUMENT, "row_sumsq: input not 16-byte aligned");
  StreamDeviceGuard guard(stream);
  const int groups = (int)(hidden_size / 32);
  const dim3 block((unsigned)(groups < 256 ? (groups + 31) / 32 * 32 : 256));
  cudaError_t err;
  if (dtype == PACE_BF16)
    err = launch(row_sumsq_kernel<__nv_bfloat16>, dim3((unsigned)num_tokens), block, 0, stream,
                 row_sumsq, static_cast<const __nv_bfloat16*>(input), groups, input_row_stride);
  else if (dtype == PACE_F16)
    err = launch(row_sumsq_kernel<__half>, dim3((unsigned)num_tokens), block, 0, stream,
                 row_sumsq, static_cast<const __half*>(input), groups, input_row_stride);
  else
    return fail(PACE_ERR_UNSUPPORTED_DTYPE, "row_sumsq: dtype %d must be bfloat16 or float16", dtype);
  if (err != cudaSuccess) return cuda_fail(err, "row_sumsq");
  return PACE_OK;
}
