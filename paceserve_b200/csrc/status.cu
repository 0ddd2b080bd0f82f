// Status reporting, version, process-wide launch settings and the small
// device-attribute cache shared by all entry points.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "common.cuh"

namespace pace {

namespace {
thread_local std::string g_last_error;
std::atomic<int> g_pdl{-1};  // -1: not yet read from the environment
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
}  // namespace

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(PACE_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

bool pdl_enabled() {
  int v = g_pdl.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* env = getenv("PACE_PDL");
    v = (env && env[0] == '0') ? 0 : 1;
    g_pdl.store(v, std::memory_order_relaxed);
  }
  return v != 0;
}

cudaError_t ensure_dynamic_smem(const void* func, int device, int bytes) {
  static std::mutex mu;
  static std::vector<std::tuple<const void*, int, int>> done;  // (func, device, bytes set)
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : done)
    if (std::get<0>(e) == func && std::get<1>(e) == device && std::get<2>(e) >= bytes)
      return cudaSuccess;
  const cudaError_t err =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess) done.emplace_back(func, device, bytes);
  return err;
}

int sm_count(int device) {
  if (device < 0 || device >= kMaxDevices) return 148;
  int v = g_sm_count[device].load(std::memory_order_relaxed);
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
      v = 148;
    g_sm_count[device].store(v, std::memory_order_relaxed);
  }
  return v;
}

}  // namespace pace

extern "C" {

const char* pace_last_error(void) { return pace::g_last_error.c_str(); }

const char* pace_status_string(int status) {
  switch (status) {
    case PACE_OK: return "PACE_OK";
    case PACE_ERR_INVALID_ARGUMENT: return "PACE_ERR_INVALID_ARGUMENT";
    case PACE_ERR_UNSUPPORTED_DTYPE: return "PACE_ERR_UNSUPPORTED_DTYPE";
    case PACE_ERR_CUDA: return "PACE_ERR_CUDA";
    case PACE_ERR_PEER_ACCESS: return "PACE_ERR_PEER_ACCESS";
    case PACE_ERR_TOO_LARGE: return "PACE_ERR_TOO_LARGE";
    default: return "PACE_ERR_UNKNOWN";
  }
}

int pace_version(void) { return (0 << 16) | (1 << 8) | 0; }

void pace_set_pdl(int enable) { pace::g_pdl.store(enable ? 1 : 0, std::memory_order_relaxed); }

int pace_get_pdl(void) { return pace::pdl_enabled() ? 1 : 0; }

}  // extern "C"
