// Paged-KV block transfer for sm_100a: block copy between two paged caches
// (the LP -> HP promotion, over NVLink when the caches live on different
// GPUs), gather of blocks into a contiguous buffer and scatter back (the
// KVhelper get/insert path), plus peer-access and CUDA IPC helpers.
//
// Reference behaviour replaced: KVhelper.get_kv_cache / insert_kv_cache
// (paceserve/kv_transfer/kv_utils.py:33-56) move a sequence's blocks with one
// fancy-index gather per layer into a CPU tensor, through the Ray object
// store, and one index-put per layer on the other GPU.  Cache layout
// (paceserve/model_executor/attention/flashinfer_attention_wrapper.py:53-73):
// one tensor per layer, [num_blocks, 2, block_size, kv_heads, head_dim], so a
// (layer, block) pair is one contiguous slab.
//
// Design: one kernel moves every (layer, pair) slab of the request set.  The
// work unit is a fixed-size chunk of one slab; CTAs stride over units.
//  * SIMT path: each thread issues U 16-byte loads before its U stores, so a
//    CTA keeps 256 * U * 16 bytes in flight -- enough to cover NVLink latency
//    from every SM.
//  * Bulk path: one elected thread per CTA drives a ring of shared-memory
//    stages with the bulk-async copy engine (cp.async.bulk global->shared with
//    an mbarrier, then shared->global bulk store).  No cluster multicast is
//    used anywhere: sources may be a peer GPU's memory.  Every mbarrier wait
//    is bounded by %globaltimer; on expiry the kernel flags the error, drains
//    what it issued (again bounded) and returns.
// Pair ids are validated on the device: an id outside the cache is skipped and
// counted, never dereferenced.
#include <cuda.h>

#include <algorithm>
#include <vector>

#include "common.cuh"

namespace pace {
namespace {

constexpr int kMaxLayers = 256;
constexpr int kThreads = 256;
constexpr int kUnroll = 8;                              // 16-byte vectors per thread
constexpr int64_t kChunk = kThreads * kUnroll * 16;     // 32 KiB per SIMT unit
constexpr int kBulkStages = 6;
constexpr int64_t kBulkChunk = 16 * 1024;               // bytes per bulk stage
constexpr unsigned long long kDefaultWaitLimitNs = 2000000000ull;  // 2 s
constexpr int32_t kTimeoutFlag = PACE_KV_TIMEOUT_FLAG;
constexpr int32_t kDrainTimeoutFlag = PACE_KV_DRAIN_TIMEOUT_FLAG;

struct LayerTable {
  char* p[kMaxLayers];
};

enum Mode { kPagedToPaged = 0, kPagedToContig = 1, kContigToPaged = 2 };

struct Job {
  int num_layers;
  int64_t num_pairs;
  int64_t block_bytes;
  int64_t src_blocks;  // bound for src ids (paged source)
  int64_t dst_blocks;  // bound for dst ids (paged destination)
  unsigned long long wait_limit_ns;  // bulk path: bound of every mbarrier wait
  uint32_t overarm_bytes;            // bulk path, tests only (pace_kv_copy_opts)
};

// Source/destination address of (layer l, pair j), or nullptr if the pair's
// id is out of range.
template <int MODE>
__device__ __forceinline__ bool locate(const Job& job, const LayerTable& src, const LayerTable& dst,
                                       const char* src_flat, char* dst_flat,
                                       const int32_t* src_ids, const int32_t* dst_ids, int l,
                                       int64_t j, const char** s, char** d) {
  const int64_t B = job.block_bytes;
  if (MODE == kContigToPaged) {
    *s = src_flat + ((int64_t)l * job.num_pairs + j) * B;
  } else {
    const int64_t sb = src_ids[j];
    if (sb < 0 || sb >= job.src_blocks) return false;
    *s = src.p[l] + sb * B;
  }
  if (MODE == kPagedToContig) {
    *d = dst_flat + ((int64_t)l * job.num_pairs + j) * B;
  } else {
    const int64_t db = dst_ids[j];
    if (db < 0 || db >= job.dst_blocks) return false;
    *d = dst.p[l] + db * B;
  }
  return true;
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads)
    kv_copy_simt_kernel(const __grid_constant__ LayerTable src, const __grid_constant__ LayerTable dst,
                        const char* src_flat, char* dst_flat, const int32_t* __restrict__ src_ids,
                        const int32_t* __restrict__ dst_ids, Job job, int32_t* bad) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t per_slab = ceil_div(job.block_bytes, kChunk);
  const int64_t units = (int64_t)job.num_layers * job.num_pairs * per_slab;
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int64_t slab = u / per_slab;
    const int64_t c = u - slab * per_slab;
    const int l = (int)(slab / job.num_pairs);
    const int64_t j = slab - (int64_t)l * job.num_pairs;
    const char* s;
    char* d;
    if (!locate<MODE>(job, src, dst, src_flat, dst_flat, src_ids, dst_ids, l, j, &s, &d)) {
      if (bad && l == 0 && c == 0 && threadIdx.x == 0) atomicAdd(bad, 1);
      continue;
    }
    const int64_t off0 = c * kChunk;
    const int64_t lim = job.block_bytes - off0;  // bytes of this slab left
    uint4 v[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const int64_t o = ((int64_t)k * kThreads + threadIdx.x) * 16;
      if (o < lim) v[k] = ld_stream(s + off0 + o);
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const int64_t o = ((int64_t)k * kThreads + threadIdx.x) * 16;
      if (o < lim) st_v4(d + off0 + o, v[k]);
    }
  }
}

// ------------------------------------------------------------ bulk path ----
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false when `limit_ns` expired.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) return false;
  }
  return true;
}
// expect_bytes is `bytes` except in the over-arm test, where the barrier is
// told to expect more than the copy delivers, so its phase never completes.
__device__ __forceinline__ void bulk_load(uint32_t dst_smem, const void* src, uint32_t bytes,
                                          uint32_t bar, uint32_t expect_bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(expect_bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_smem),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(src_smem), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int MODE>
__global__ void __launch_bounds__(32)
    kv_copy_bulk_kernel(const __grid_constant__ LayerTable src, const __grid_constant__ LayerTable dst,
                        const char* src_flat, char* dst_flat, const int32_t* __restrict__ src_ids,
                        const int32_t* __restrict__ dst_ids, Job job, int32_t* bad) {
  extern __shared__ __align__(128) unsigned char stage_mem[];
  __shared__ __align__(8) uint64_t bars[kBulkStages];
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x != 0) return;  // one thread drives the copy engine
  for (int s = 0; s < kBulkStages; ++s)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bars[s])) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  const int64_t per_slab = ceil_div(job.block_bytes, kBulkChunk);
  const int64_t units = (int64_t)job.num_layers * job.num_pairs * per_slab;
  // This CTA's units are u = blockIdx.x + i * gridDim.x, i = 0, 1, ...
  const int64_t my_units =
      units > blockIdx.x ? ceil_div(units - blockIdx.x, gridDim.x) : 0;

  // Per stage: destination and size of the unit it holds, whether its load
  // is still in flight, and how many loads it has completed (the parity).
  char* st_dst[kBulkStages];
  uint32_t st_bytes[kBulkStages];
  uint32_t uses[kBulkStages];
  bool pending[kBulkStages];
  for (int s = 0; s < kBulkStages; ++s) {
    st_dst[s] = nullptr;
    st_bytes[s] = 0;
    uses[s] = 0;
    pending[s] = false;
  }
  bool timed_out = false;

  // Issue the load of this CTA's i-th unit into stage s (skips invalid pairs).
  auto issue = [&](int64_t i, int s) {
    const int64_t u = blockIdx.x + i * (int64_t)gridDim.x;
    const int64_t slab = u / per_slab;
    const int64_t c = u - slab * per_slab;
    const int l = (int)(slab / job.num_pairs);
    const int64_t j = slab - (int64_t)l * job.num_pairs;
    const char* sp;
    char* dp;
    st_dst[s] = nullptr;
    if (!locate<MODE>(job, src, dst, src_flat, dst_flat, src_ids, dst_ids, l, j, &sp, &dp)) {
      if (bad && l == 0 && c == 0) atomicAdd(bad, 1);
      return;
    }
    const int64_t off = c * kBulkChunk;
    const int64_t left = job.block_bytes - off;
    const uint32_t bytes = (uint32_t)(left < kBulkChunk ? left : kBulkChunk);
    st_dst[s] = dp + off;
    st_bytes[s] = bytes;
    pending[s] = true;
    const uint32_t expect = (i == 0 && blockIdx.x == 0) ? bytes + job.overarm_bytes : bytes;
    bulk_load(smem_addr(stage_mem + s * kBulkChunk), sp + off, bytes, smem_addr(&bars[s]), expect);
  };

  const int64_t pro = my_units < kBulkStages ? my_units : kBulkStages;
  for (int64_t i = 0; i < pro; ++i) issue(i, (int)i);
  for (int64_t i = 0; i < my_units; ++i) {
    const int s = (int)(i % kBulkStages);
    if (pending[s]) {
      if (!mbar_wait(smem_addr(&bars[s]), uses[s] & 1u, job.wait_limit_ns)) {
        timed_out = true;
        break;
      }
      pending[s] = false;
      uses[s]++;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bulk_store(st_dst[s], smem_addr(stage_mem + s * kBulkChunk), st_bytes[s]);
    }
    const int64_t next = i + kBulkStages;
    if (next < my_units) {
      // The store just issued from stage s must have read its data out of
      // shared memory before the stage is refilled.
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      issue(next, s);
    }
  }
  if (timed_out) {
    // No new load is issued after a timeout.  Every load still in flight is
    // waited for once more (same bound) so that none lands in this CTA's shared
    // memory after it exits.  A load that outlasts that second bound too (a
    // source that stopped answering) cannot be cancelled: the drain flag tells
    // the caller the device may hold a late write and must not be trusted.
    int32_t flags = kTimeoutFlag;
    for (int s = 0; s < kBulkStages; ++s)
      if (pending[s] && !mbar_wait(smem_addr(&bars[s]), uses[s] & 1u, job.wait_limit_ns))
        flags |= kDrainTimeoutFlag;
    atomicOr(bad, flags);
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Device-side address of a flat gather/scatter buffer: device memory as is,
// page-locked host memory through its mapping.  Pageable host memory is
// rejected (the kernel cannot reach it).
int device_view(const void* p, const void** out, const char* what) {
  cudaPointerAttributes a;
  cudaError_t err = cudaPointerGetAttributes(&a, p);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: buffer is not CUDA-visible memory", what);
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
    *out = p;
    return PACE_OK;
  }
  if (a.type == cudaMemoryTypeHost && a.devicePointer != nullptr) {
    *out = a.devicePointer;
    return PACE_OK;
  }
  return fail(PACE_ERR_INVALID_ARGUMENT,
              "%s: buffer must be device memory or page-locked host memory", what);
}

int check_layers(void* const* layers, int num_layers, const char* what) {
  if (!layers) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null layer table", what);
  for (int l = 0; l < num_layers; ++l) {
    if (!layers[l]) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: layer %d pointer is null", what, l);
    if (!aligned16(layers[l]))
      return fail(PACE_ERR_INVALID_ARGUMENT, "%s: layer %d pointer not 16-byte aligned", what, l);
  }
  return PACE_OK;
}

struct CopyOpts {
  int method = 0;          // 0 auto, 1 SIMT, 2 bulk
  int max_ctas = 0;        // 0: no cap
  unsigned long long wait_limit_ns = kDefaultWaitLimitNs;
  uint32_t overarm_bytes = 0;
};

template <int MODE>
int run_copy(void* const* src_layers, void* const* dst_layers, const void* src_flat, void* dst_flat,
             int num_layers, const int32_t* src_ids, const int32_t* dst_ids, int64_t n,
             int64_t block_bytes, int64_t src_blocks, int64_t dst_blocks, int32_t* bad,
             const CopyOpts& opt, cudaStream_t stream, const char* what) {
  const int method = opt.method;
  if (num_layers <= 0 || num_layers > kMaxLayers)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: num_layers %d outside [1, %d]", what, num_layers,
                kMaxLayers);
  if (n < 0 || block_bytes <= 0 || block_bytes % 16 != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: need num_pairs >= 0 and block_bytes a positive multiple of 16 (got %lld)",
                what, (long long)block_bytes);
  if (n == 0) return PACE_OK;
  LayerTable st = {}, dt = {};
  if (MODE != kContigToPaged) {
    int rc = check_layers(src_layers, num_layers, what);
    if (rc) return rc;
    if (!src_ids) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null source ids", what);
    for (int l = 0; l < num_layers; ++l) st.p[l] = static_cast<char*>(src_layers[l]);
  } else if (!src_flat || !aligned16(src_flat)) {
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: source buffer null or unaligned", what);
  }
  if (MODE != kPagedToContig) {
    int rc = check_layers(dst_layers, num_layers, what);
    if (rc) return rc;
    if (!dst_ids) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null destination ids", what);
    for (int l = 0; l < num_layers; ++l) dt.p[l] = static_cast<char*>(dst_layers[l]);
  } else if (!dst_flat || !aligned16(dst_flat)) {
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: destination buffer null or unaligned", what);
  }
  if (method == 2 && !bad)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: the bulk method reports wait timeouts only through bad_pairs, which must "
                "not be NULL", what);
  if (opt.max_ctas < 0 || opt.overarm_bytes % 16 != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad copy options", what);
  Job job{num_layers, n,  block_bytes, src_blocks, dst_blocks, opt.wait_limit_ns,
          opt.overarm_bytes};
  StreamDeviceGuard guard(stream);
  if (MODE == kContigToPaged) {
    int rc = device_view(src_flat, &src_flat, what);
    if (rc) return rc;
  }
  if (MODE == kPagedToContig) {
    const void* d = nullptr;
    int rc = device_view(dst_flat, &d, what);
    if (rc) return rc;
    dst_flat = const_cast<void*>(d);
  }
  const int sms = sm_count(guard.device());
  cudaError_t err;
  if (method == 2) {
    const int64_t units = (int64_t)num_layers * n * ceil_div(block_bytes, kBulkChunk);
    int64_t grid = units < 2 * sms ? units : 2 * sms;
    if (opt.max_ctas > 0 && grid > opt.max_ctas) grid = opt.max_ctas;
    const size_t smem = (size_t)kBulkStages * kBulkChunk;
    auto kern = kv_copy_bulk_kernel<MODE>;
    err = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), guard.device(), (int)smem);
    if (err != cudaSuccess) return cuda_fail(err, what);
    err = launch(kern, dim3((unsigned)grid), dim3(32), smem, stream, st, dt,
                 static_cast<const char*>(src_flat), static_cast<char*>(dst_flat), src_ids,
                 dst_ids, job, bad);
  } else {
    // One short CTA per 32 KiB unit (grid-stride only past the grid limit):
    // on B200 this moves 1.1 GB HBM -> HBM at 3258 GB/s (99.5 % of the measured
    // copy peak in HBM traffic) against 2963 GB/s with one resident wave of
    // 8 CTAs per SM looping over the units.
    const int64_t units = (int64_t)num_layers * n * ceil_div(block_bytes, kChunk);
    int64_t grid = units < INT32_MAX ? units : INT32_MAX;
    if (opt.max_ctas > 0 && grid > opt.max_ctas) grid = opt.max_ctas;
    err = launch(kv_copy_simt_kernel<MODE>, dim3((unsigned)grid), dim3(kThreads), 0, stream, st,
                 dt, static_cast<const char*>(src_flat), static_cast<char*>(dst_flat), src_ids,
                 dst_ids, job, bad);
  }
  if (err != cudaSuccess) return cuda_fail(err, what);
  return PACE_OK;
}

}  // namespace
}  // namespace pace

extern "C" int pace_kv_copy_blocks(void* const* src_layers, void* const* dst_layers,
                                   int num_layers, const int32_t* src_block_ids,
                                   const int32_t* dst_block_ids, int64_t num_pairs,
                                   int64_t block_bytes, int64_t src_num_blocks,
                                   int64_t dst_num_blocks, int32_t* bad_pairs, int method,
                                   cudaStream_t stream) {
  pace_kv_copy_opts opts = {};
  opts.method = method;
  return pace_kv_copy_blocks_ex(src_layers, dst_layers, num_layers, src_block_ids, dst_block_ids,
                                num_pairs, block_bytes, src_num_blocks, dst_num_blocks, bad_pairs,
                                &opts, stream);
}

extern "C" int pace_kv_copy_blocks_ex(void* const* src_layers, void* const* dst_layers,
                                      int num_layers, const int32_t* src_block_ids,
                                      const int32_t* dst_block_ids, int64_t num_pairs,
                                      int64_t block_bytes, int64_t src_num_blocks,
                                      int64_t dst_num_blocks, int32_t* bad_pairs,
                                      const pace_kv_copy_opts* opts, cudaStream_t stream) {
  using namespace pace;
  if (!opts) return fail(PACE_ERR_INVALID_ARGUMENT, "kv_copy_blocks: null options");
  if (opts->method < 0 || opts->method > 2)
    return fail(PACE_ERR_INVALID_ARGUMENT, "kv_copy_blocks: method %d not in {0,1,2}",
                opts->method);
  CopyOpts o;
  o.method = opts->method;
  o.max_ctas = opts->max_ctas;
  o.wait_limit_ns = opts->wait_limit_ns ? opts->wait_limit_ns : kDefaultWaitLimitNs;
  if (opts->test_overarm_bytes < 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "kv_copy_blocks: negative test_overarm_bytes");
  o.overarm_bytes = (uint32_t)opts->test_overarm_bytes;
  if (o.overarm_bytes && o.method != 2)
    return fail(PACE_ERR_INVALID_ARGUMENT, "kv_copy_blocks: test_overarm_bytes needs method 2");
  return run_copy<kPagedToPaged>(src_layers, dst_layers, nullptr, nullptr, num_layers,
                                 src_block_ids, dst_block_ids, num_pairs, block_bytes,
                                 src_num_blocks, dst_num_blocks, bad_pairs, o, stream,
                                 "kv_copy_blocks");
}

extern "C" int pace_kv_gather_blocks(void* const* layers, int num_layers, const int32_t* block_ids,
                                     int64_t n, int64_t block_bytes, int64_t num_blocks, void* out,
                                     int32_t* bad_ids, cudaStream_t stream) {
  using namespace pace;
  CopyOpts o;
  o.method = 1;
  return run_copy<kPagedToContig>(layers, nullptr, nullptr, out, num_layers, block_ids, nullptr, n,
                                  block_bytes, num_blocks, 0, bad_ids, o, stream,
                                  "kv_gather_blocks");
}

extern "C" int pace_kv_scatter_blocks(const void* in, void* const* layers, int num_layers,
                                      const int32_t* block_ids, int64_t n, int64_t block_bytes,
                                      int64_t num_blocks, int32_t* bad_ids, cudaStream_t stream) {
  using namespace pace;
  CopyOpts o;
  o.method = 1;
  return run_copy<kContigToPaged>(nullptr, layers, in, nullptr, num_layers, nullptr, block_ids, n,
                                  block_bytes, 0, num_blocks, bad_ids, o, stream,
                                  "kv_scatter_blocks");
}

// ------------------------------------------------- copy-engine path ------
// Block copy with the GPU's copy engines instead of its SMs: one
// cudaMemcpyAsync per run of pairs whose source and destination ids are both
// consecutive, per layer -- or one cudaMemcpy2DAsync per run covering every
// layer when both layer tables are evenly spaced (one allocation viewed per
// layer).  No kernel runs, so a promotion this way leaves every SM to the
// serving instance.  The ids are host arrays (the block manager's tables);
// pairs are ordered by source id before the runs are formed.
namespace pace {
namespace {

struct Pair {
  int64_t s, d;
};

// Byte distance between consecutive layer pointers when it is the same for all
// layers and positive, else 0.
int64_t uniform_stride(void* const* layers, int num_layers) {
  if (num_layers < 2) return 0;
  const int64_t st = reinterpret_cast<const char*>(layers[1]) - reinterpret_cast<const char*>(layers[0]);
  if (st <= 0) return 0;
  for (int l = 2; l < num_layers; ++l)
    if (reinterpret_cast<const char*>(layers[l]) - reinterpret_cast<const char*>(layers[l - 1]) != st)
      return 0;
  return st;
}

}  // namespace
}  // namespace pace

extern "C" int pace_kv_copy_blocks_ce(void* const* src_layers, void* const* dst_layers,
                                      int num_layers, const int32_t* src_block_ids,
                                      const int32_t* dst_block_ids, int64_t num_pairs,
                                      int64_t block_bytes, int64_t src_num_blocks,
                                      int64_t dst_num_blocks, int64_t* bad_pairs,
                                      int64_t* copies_issued, cudaStream_t stream) {
  using namespace pace;
  const char* what = "kv_copy_blocks_ce";
  if (num_layers <= 0 || num_layers > kMaxLayers)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: num_layers %d outside [1, %d]", what, num_layers,
                kMaxLayers);
  if (num_pairs < 0 || block_bytes <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: need num_pairs >= 0 and block_bytes > 0", what);
  if (bad_pairs) *bad_pairs = 0;
  if (copies_issued) *copies_issued = 0;
  if (num_pairs == 0) return PACE_OK;
  if (!src_block_ids || !dst_block_ids)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null block id array", what);
  int rc = check_layers(src_layers, num_layers, what);
  if (rc) return rc;
  rc = check_layers(dst_layers, num_layers, what);
  if (rc) return rc;
  std::vector<Pair> pairs;
  pairs.reserve((size_t)num_pairs);
  int64_t bad = 0;
  for (int64_t j = 0; j < num_pairs; ++j) {
    const int64_t sb = src_block_ids[j], db = dst_block_ids[j];
    if (sb < 0 || sb >= src_num_blocks || db < 0 || db >= dst_num_blocks) {
      ++bad;
      continue;
    }
    pairs.push_back({sb, db});
  }
  if (bad_pairs) *bad_pairs = bad;
  std::stable_sort(pairs.begin(), pairs.end(), [](const Pair& a, const Pair& b) { return a.s < b.s; });
  const int64_t ss = uniform_stride(src_layers, num_layers);
  const int64_t ds = uniform_stride(dst_layers, num_layers);
  const bool two_d = ss >= block_bytes && ds >= block_bytes;
  int64_t issued = 0;
  size_t i = 0;
  while (i < pairs.size()) {
    size_t j = i + 1;
    while (j < pairs.size() && pairs[j].s == pairs[j - 1].s + 1 && pairs[j].d == pairs[j - 1].d + 1)
      ++j;
    const size_t run = (size_t)(j - i) * (size_t)block_bytes;
    const int64_t so = pairs[i].s * block_bytes, doff = pairs[i].d * block_bytes;
    if (two_d && (size_t)ss >= run && (size_t)ds >= run) {
      const cudaError_t err = cudaMemcpy2DAsync(
          static_cast<char*>(dst_layers[0]) + doff, (size_t)ds,
          static_cast<const char*>(src_layers[0]) + so, (size_t)ss, run, (size_t)num_layers,
          cudaMemcpyDefault, stream);
      if (err != cudaSuccess) return cuda_fail(err, what);
      ++issued;
    } else {
      for (int l = 0; l < num_layers; ++l) {
        const cudaError_t err =
            cudaMemcpyAsync(static_cast<char*>(dst_layers[l]) + doff,
                            static_cast<const char*>(src_layers[l]) + so, run, cudaMemcpyDefault,
                            stream);
        if (err != cudaSuccess) return cuda_fail(err, what);
        ++issued;
      }
    }
    i = j;
  }
  if (copies_issued) *copies_issued = issued;
  return PACE_OK;
}

// ------------------------------------------------------ peer access / IPC --

extern "C" int pace_can_access_peer(int device, int peer, int* can) {
  using namespace pace;
  if (!can) return fail(PACE_ERR_INVALID_ARGUMENT, "can_access_peer: null output");
  *can = 0;
  if (device == peer) {
    *can = 1;
    return PACE_OK;
  }
  int v = 0;
  cudaError_t err = cudaDeviceCanAccessPeer(&v, device, peer);
  if (err != cudaSuccess) return cuda_fail(err, "can_access_peer");
  *can = v;
  return PACE_OK;
}

extern "C" int pace_enable_peer_access(int device, int peer) {
  using namespace pace;
  if (device == peer) return PACE_OK;
  int can = 0;
  int rc = pace_can_access_peer(device, peer, &can);
  if (rc) return rc;
  if (!can)
    return fail(PACE_ERR_PEER_ACCESS, "enable_peer_access: device %d cannot address device %d",
                device, peer);
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t err = cudaSetDevice(device);
  if (err == cudaSuccess) err = cudaDeviceEnablePeerAccess(peer, 0);
  if (err == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();  // clear the sticky-free "already enabled" status
    err = cudaSuccess;
  }
  cudaSetDevice(prev);
  if (err != cudaSuccess) return fail(PACE_ERR_PEER_ACCESS, "enable_peer_access: %s", cudaGetErrorString(err));
  return PACE_OK;
}

namespace {
typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (GetAddressRangeFn) nullptr;
    return reinterpret_cast<GetAddressRangeFn>(p);
  }();
  return fn;
}
}  // namespace

extern "C" int pace_ipc_get_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  using namespace pace;
  static_assert(sizeof(cudaIpcMemHandle_t) == PACE_IPC_HANDLE_BYTES, "IPC handle size");
  if (!dev_ptr || !handle_out || !offset_out)
    return fail(PACE_ERR_INVALID_ARGUMENT, "ipc_get_handle: null argument");
  GetAddressRangeFn range = address_range_fn();
  if (!range) return fail(PACE_ERR_CUDA, "ipc_get_handle: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(PACE_ERR_INVALID_ARGUMENT, "ipc_get_handle: pointer is not device memory");
  cudaIpcMemHandle_t h;
  cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) return cuda_fail(err, "ipc_get_handle");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return PACE_OK;
}

extern "C" int pace_ipc_open_handle(const void* handle, int device, void** base_out) {
  using namespace pace;
  if (!handle || !base_out) return fail(PACE_ERR_INVALID_ARGUMENT, "ipc_open_handle: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t err = cudaSetDevice(device);
  void* p = nullptr;
  if (err == cudaSuccess) err = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  cudaSetDevice(prev);
  if (err != cudaSuccess) return fail(PACE_ERR_PEER_ACCESS, "ipc_open_handle: %s", cudaGetErrorString(err));
  *base_out = p;
  return PACE_OK;
}

extern "C" int pace_ipc_close_handle(void* base) {
  using namespace pace;
  if (!base) return fail(PACE_ERR_INVALID_ARGUMENT, "ipc_close_handle: null base");
  cudaError_t err = cudaIpcCloseMemHandle(base);
  if (err != cudaSuccess) return cuda_fail(err, "ipc_close_handle");
  return PACE_OK;
}
