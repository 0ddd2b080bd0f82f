// Shared helpers for the sm_100a kernels: dtype traits, 16-byte vector
// packing, programmatic-dependent-launch (PDL) hooks, status reporting and a
// stream-device guard for the C-ABI entry points.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "pace_b200.h"

namespace pace {

// ---------------------------------------------------------------- status --
// Records a message for pace_last_error() on this thread and returns `code`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Maps a CUDA error to PACE_ERR_CUDA with the call site in the message.
int cuda_fail(cudaError_t err, const char* what);
bool pdl_enabled();
// Number of SMs of `device`, cached.
int sm_count(int device);
// cudaFuncSetAttribute(func, MaxDynamicSharedMemorySize, bytes) on `device`,
// done once per (function, device) and size: repeated launches skip the call.
cudaError_t ensure_dynamic_smem(const void* func, int device, int bytes);

// The device the entry point launches on: the calling thread's current
// device, which must own the stream (as for any CUDA launch).  No query is
// made on the stream itself: querying a stream that is being captured into a
// CUDA graph invalidates the capture.
class StreamDeviceGuard {
 public:
  explicit StreamDeviceGuard(cudaStream_t) {
    if (cudaGetDevice(&dev_) != cudaSuccess) dev_ = 0;
  }
  int device() const { return dev_; }

 private:
  int dev_ = 0;
};

// Launch with the PDL attribute (when enabled) so the kernel's CTAs may be
// scheduled while the previous kernel in the stream drains; every kernel
// launched this way calls pdl_wait() before touching global memory that an
// earlier kernel may write or read.
template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  cfg.numAttrs = 0;
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cfg.attrs = attr;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same for kernels run as clusters of two CTAs (one per SM of a TPC).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pairs(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.numAttrs = 1;
  if (pdl_enabled()) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cfg.attrs = attr;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ------------------------------------------------------------ device side --
__device__ __forceinline__ void pdl_wait() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
__device__ __forceinline__ void pdl_launch_dependents() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

// Asks the bulk-copy engine to pull [p, p + bytes) into L2 (p 16-byte aligned,
// bytes a multiple of 16).  Kernels issue it for their input rows BEFORE
// pdl_wait(): L2 is the point of coherence, so a line fetched early and then
// written by the still-running predecessor holds the predecessor's data when
// this kernel reads it after the wait.  The DRAM latency of the first touch
// then overlaps the predecessor's tail instead of following it.
__device__ __forceinline__ void prefetch_l2(const void* p, int64_t bytes) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  const char* c = static_cast<const char*>(p);
  while (bytes > 0) {
    const uint32_t n = bytes > 32768 ? 32768u : static_cast<uint32_t>(bytes);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
    c += n;
    bytes -= n;
  }
#endif
}

// 16-byte global accesses.  *_nc: read-only path for inputs that the kernel
// does not write; L1::no_allocate keeps single-use streams out of L1.
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
// 8-byte load cached at L2 only: a second read of a location sees what L2
// holds now, never a stale L1 line from a read earlier in the same kernel.
__device__ __forceinline__ int64_t ld_cg_s64(const int64_t* p) {
  int64_t v;
  asm volatile("ld.global.cg.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_v4(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
// 32 bytes in one store (sm_100 256-bit access): a whole L2 sector per thread.
// p must be 32-byte aligned.
__device__ __forceinline__ void st_v8(void* p, const uint4& lo, const uint4& hi) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(lo.x),
               "r"(lo.y), "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
               : "memory");
}

// ------------------------------------------------------------ dtype traits --
template <typename T>
struct Traits;

template <>
struct Traits<float> {
  static constexpr int kVec = 4;  // elements per 16-byte vector
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static float from_f(float x) { return x; }
  // float(T(x)): the value after rounding to T
  __device__ __forceinline__ static float round(float x) { return x; }
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};

template <>
struct Traits<__half> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
  __device__ __forceinline__ static float round(float x) { return __half2float(__float2half_rn(x)); }
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

template <>
struct Traits<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    // bf16 -> fp32 is a 16-bit shift: the low half of each word is element 2i.
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

inline int dtype_size(int dtype) {
  switch (dtype) {
    case PACE_F32: return 4;
    case PACE_F16: return 2;
    case PACE_BF16: return 2;
    case PACE_U8: return 1;
    case PACE_I8: return 1;
    case PACE_I16: return 2;
    case PACE_I32: return 4;
    case PACE_I64: return 8;
    default: return 0;
  }
}

}  // namespace pace

// Expands BODY with `scalar_t` bound to the C++ type of a float dtype code;
// returns PACE_ERR_UNSUPPORTED_DTYPE for anything else.
#define PACE_DISPATCH_FLOAT(DTYPE, NAME, ...)                                         \
  [&]() -> int {                                                                      \
    switch (DTYPE) {                                                                  \
      case PACE_F32: { using scalar_t = float; return __VA_ARGS__(); }                \
      case PACE_F16: { using scalar_t = __half; return __VA_ARGS__(); }               \
      case PACE_BF16: { using scalar_t = __nv_bfloat16; return __VA_ARGS__(); }       \
      default:                                                                        \
        return pace::fail(PACE_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype code %d", \
                          NAME, (int)(DTYPE));                                        \
    }                                                                                 \
  }()
