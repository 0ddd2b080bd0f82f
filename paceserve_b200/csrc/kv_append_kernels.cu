// Append of new K/V tokens into the paged KV cache, for sm_100a.
//
// Replaces flashinfer.page.append_paged_kv_cache (FlashInfer, pinned at
// 0.2.0 in PaceServe's requirements.txt:40; not vendored), which PaceServe
// calls once per layer per step at
// paceserve/model_executor/attention/flashinfer_attention_wrapper.py:239-255,
// after deriving every token's request and position with FlashInfer's
// get_seq_lens + get_batch_indices_positions.  Published semantics restated:
// the cache is [num_pages, 2, page_size, kv_heads, head_dim] (NHD, K then V);
// token i of request b at sequence position p is written to page
// kv_indices[kv_indptr[b] + p / page_size], slot p % page_size.  With the
// append-indptr form, the tokens of request b are the last
// append_indptr[b+1] - append_indptr[b] tokens of a sequence of length
// (kv_indptr[b+1] - kv_indptr[b] - 1) * page_size + kv_last_page_len[b].
//
// Design: one CTA per token, one 16-byte vector of K or V per thread.  The
// K/V row loads are issued first (they do not depend on the indices), then the
// short index chain (request -> page table -> page), then the stores.  K/V
// rows may be strided views of a fused qkv tensor.  A token whose request,
// position or page is out of range is skipped and counted.
#include "common.cuh"

namespace pace {
namespace {

constexpr int kAppendThreads = 256;
// Requests whose per-request metadata (append_indptr, kv_indptr,
// kv_last_page_len) each CTA stages in shared memory: 3 x 2049 x 4 B.
constexpr int64_t kMaxStagedBatch = 2048;

struct AppendJob {
  int64_t nnz;
  int heads;
  int head_dim;
  int64_t key_stride;
  int64_t value_stride;
  int64_t num_pages;
  int page_size;
  int64_t batch;
  int64_t num_indices;  // entries of kv_indices
};

// Page and slot of a token of request b at sequence position pos, or false
// if any index is out of range.  ip / last: kv_indptr and kv_last_page_len
// (global or staged copies).  A last-page length outside [1, page_size] makes
// the request's length inconsistent with its page count, so its tokens are
// rejected rather than placed on a page past the request's range.
__device__ __forceinline__ bool locate_token(const AppendJob& j, int b, int64_t pos,
                                             const int32_t* kv_indices, const int32_t* ip,
                                             const int32_t* last, int64_t* page, int* slot) {
  if (b < 0 || b >= j.batch || pos < 0) return false;
  const int64_t p0 = ip[b];
  const int64_t np = (int64_t)ip[b + 1] - p0;
  if (np <= 0 || p0 < 0 || p0 + np > j.num_indices) return false;
  const int64_t lp = last[b];
  if (lp < 1 || lp > j.page_size) return false;
  const int64_t seq_len = (np - 1) * j.page_size + lp;
  if (pos >= seq_len) return false;  // so pos / page_size < np
  const int64_t pg = kv_indices[p0 + pos / j.page_size];
  if (pg < 0 || pg >= j.num_pages) return false;
  *page = pg;
  *slot = (int)(pos % j.page_size);
  return true;
}

// Request of token i from append_indptr (ascending, batch + 1 entries).
__device__ __forceinline__ int find_request(const int32_t* indptr, int64_t batch, int64_t i) {
  int lo = 0, hi = (int)batch - 1;  // largest b with indptr[b] <= i
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (indptr[mid] <= i)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// BY_INDPTR: derive (request, position) from append_indptr; otherwise read
// batch_indices / positions.  VEC: 16-byte vectors; otherwise elements.
// STAGED: the per-request arrays are copied to shared memory first, so the
// token's index chain after the K/V loads is shared-memory lookups plus one
// global load (its kv_indices entry) instead of three dependent global loads.
template <typename T, bool BY_INDPTR, bool VEC, bool STAGED>
__global__ void __launch_bounds__(kAppendThreads)
    kv_append_kernel(const T* key, const T* value, const int32_t* __restrict__ batch_indices,
                     const int32_t* __restrict__ positions, const int32_t* __restrict__ append_indptr,
                     T* cache, const int32_t* __restrict__ kv_indices,
                     const int32_t* __restrict__ kv_indptr,
                     const int32_t* __restrict__ kv_last_page_len, AppendJob job, int32_t* bad) {
  extern __shared__ int32_t sh[];  // STAGED: kv_indptr | kv_last_page_len | append_indptr
  constexpr int V = VEC ? Traits<T>::kVec : 1;
  const int64_t i = blockIdx.x;
  const int64_t row = (int64_t)job.heads * job.head_dim;  // elements per K (or V) row
  const int64_t units = row / V;                          // per K or V
  pdl_launch_dependents();
  if (VEC && threadIdx.x == 0) {
    prefetch_l2(key + i * job.key_stride, row * (int64_t)sizeof(T));
    prefetch_l2(value + i * job.value_stride, row * (int64_t)sizeof(T));
  }
  pdl_wait();
  // Token -> request and position inputs that need no staged data.
  int b = 0;
  int64_t pos = 0;
  if (!BY_INDPTR) {
    b = batch_indices[i];
    pos = positions[i];
  }
  int32_t* s_ip = sh;
  int32_t* s_last = sh + job.batch + 1;
  int32_t* s_ai = sh + 2 * job.batch + 1;
  if (STAGED) {
    for (int64_t k = threadIdx.x; k <= job.batch; k += blockDim.x) {
      s_ip[k] = kv_indptr[k];
      if (k < job.batch) s_last[k] = kv_last_page_len[k];
      if (BY_INDPTR) s_ai[k] = append_indptr[k];
    }
    __syncthreads();
  }
  const int32_t* ip = STAGED ? s_ip : kv_indptr;
  const int32_t* last = STAGED ? s_last : kv_last_page_len;
  for (int64_t u0 = 0; u0 < 2 * units; u0 += blockDim.x) {
    const int64_t u = u0 + threadIdx.x;
    const bool is_v = u >= units;
    const int64_t c = is_v ? u - units : u;
    const bool live = u < 2 * units;
    const T* src = (is_v ? value + i * job.value_stride : key + i * job.key_stride) + c * V;
    uint4 vec = make_uint4(0, 0, 0, 0);
    T elem{};
    if (live) {
      if (VEC)
        vec = ld_nc_v4(src);
      else
        elem = *src;
    }
    if (BY_INDPTR) {
      const int32_t* ai = STAGED ? s_ai : append_indptr;
      b = find_request(ai, job.batch, i);
      if (i < (int64_t)ai[b] || i >= (int64_t)ai[b + 1]) {
        // append_indptr does not cover token i (it does not start at 0, or is
        // not ascending): no request owns the token.
        b = -1;
      } else {
        const int64_t np = (int64_t)ip[b + 1] - ip[b];
        const int64_t seq_len = (np - 1) * job.page_size + last[b];
        pos = seq_len - ((int64_t)ai[b + 1] - ai[b]) + (i - ai[b]);
      }
    }
    int64_t page;
    int slot;
    const bool ok = locate_token(job, b, pos, kv_indices, ip, last, &page, &slot);
    if (!ok) {
      if (bad && u0 == 0 && threadIdx.x == 0) atomicAdd(bad, 1);
      return;
    }
    if (live) {
      T* dst = cache + ((page * 2 + (is_v ? 1 : 0)) * job.page_size + slot) * row + c * V;
      if (VEC)
        st_v4(dst, vec);
      else
        *dst = elem;
    }
  }
}

template <bool BY_INDPTR>
int run_append(const void* key, const void* value, int64_t nnz, int heads, int head_dim,
               int64_t key_stride, int64_t value_stride, const int32_t* batch_indices,
               const int32_t* positions, const int32_t* append_indptr, void* cache,
               int64_t num_pages, int page_size, const int32_t* kv_indices,
               const int32_t* kv_indptr, const int32_t* kv_last_page_len, int64_t batch,
               int64_t num_indices, int32_t* bad, int dtype, cudaStream_t stream,
               const char* what) {
  if (nnz < 0 || nnz > INT32_MAX || heads <= 0 || head_dim <= 0 || page_size <= 0 ||
      num_pages < 0 || batch < 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad shape", what);
  const int64_t row = (int64_t)heads * head_dim;
  if (key_stride < row || value_stride < row)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: row stride smaller than kv_heads * head_dim", what);
  if (nnz == 0) return PACE_OK;
  if (batch == 0) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: tokens but no requests", what);
  if (!key || !value || !cache || !kv_indices || !kv_indptr || !kv_last_page_len ||
      (BY_INDPTR ? !append_indptr : (!batch_indices || !positions)))
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  StreamDeviceGuard guard(stream);
  AppendJob job{nnz, heads, head_dim, key_stride, value_stride, num_pages, page_size, batch,
                num_indices};
  const bool staged = batch <= kMaxStagedBatch;
  const size_t smem = staged ? (size_t)(3 * batch + 2) * 4 : 0;
  return PACE_DISPATCH_FLOAT(dtype, what, [&] {
    using T = scalar_t;
    constexpr int V = Traits<T>::kVec;
    const bool vec = row % V == 0 && key_stride % V == 0 && value_stride % V == 0 &&
                     aligned16(key) && aligned16(value) && aligned16(cache);
    const int64_t units = 2 * (vec ? row / V : row);
    const int threads = units >= kAppendThreads ? kAppendThreads : (int)ceil_div(units, 32) * 32;
    const T* k = static_cast<const T*>(key);
    const T* v = static_cast<const T*>(value);
    T* c = static_cast<T*>(cache);
    auto go = [&](auto kernel) {
      return launch(kernel, dim3((unsigned)nnz), dim3(threads), smem, stream, k, v, batch_indices,
                    positions, append_indptr, c, kv_indices, kv_indptr, kv_last_page_len, job,
                    bad);
    };
    cudaError_t err;
    if (vec)
      err = staged ? go(kv_append_kernel<T, BY_INDPTR, true, true>)
                   : go(kv_append_kernel<T, BY_INDPTR, true, false>);
    else
      err = staged ? go(kv_append_kernel<T, BY_INDPTR, false, true>)
                   : go(kv_append_kernel<T, BY_INDPTR, false, false>);
    if (err != cudaSuccess) return cuda_fail(err, what);
    return PACE_OK;
  });
}

}  // namespace
}  // namespace pace

extern "C" int pace_append_paged_kv_cache(const void* key, const void* value, int64_t nnz,
                                          int num_kv_heads, int head_dim, int64_t key_row_stride,
                                          int64_t value_row_stride, const int32_t* batch_indices,
                                          const int32_t* positions, void* paged_cache,
                                          int64_t num_pages, int page_size,
                                          const int32_t* kv_indices, int64_t num_kv_indices,
                                          const int32_t* kv_indptr,
                                          const int32_t* kv_last_page_len, int64_t batch_size,
                                          int32_t* bad_tokens, int dtype, cudaStream_t stream) {
  return pace::run_append<false>(key, value, nnz, num_kv_heads, head_dim, key_row_stride,
                                 value_row_stride, batch_indices, positions, nullptr, paged_cache,
                                 num_pages, page_size, kv_indices, kv_indptr, kv_last_page_len,
                                 batch_size, num_kv_indices, bad_tokens, dtype, stream,
                                 "append_paged_kv_cache");
}

extern "C" int pace_append_paged_kv_cache_by_indptr(
    const void* key, const void* value, int64_t nnz, int num_kv_heads, int head_dim,
    int64_t key_row_stride, int64_t value_row_stride, const int32_t* append_indptr,
    void* paged_cache, int64_t num_pages, int page_size, const int32_t* kv_indices,
    int64_t num_kv_indices, const int32_t* kv_indptr, const int32_t* kv_last_page_len,
    int64_t batch_size, int32_t* bad_tokens, int dtype, cudaStream_t stream) {
  return pace::run_append<true>(key, value, nnz, num_kv_heads, head_dim, key_row_stride,
                                value_row_stride, nullptr, nullptr, append_indptr, paged_cache,
                                num_pages, page_size, kv_indices, kv_indptr, kv_last_page_len,
                                batch_size, num_kv_indices, bad_tokens, dtype, stream,
                                "append_paged_kv_cache_by_indptr");
}
