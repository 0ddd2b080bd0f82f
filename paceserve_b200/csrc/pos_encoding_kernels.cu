// In-place rotary position embedding on query and key for sm_100a.
//
// Semantics follow the reference (csrc/pos_encoding_kernels.cu:8-76): the
// cache row for position p is [cos(rot_dim/2) | sin(rot_dim/2)]; GPT-NeoX style
// rotates the pair (i, i + rot_dim/2) of every head, GPT-J style the pair
// (2i, 2i+1), both with x' = x cos - y sin, y' = y cos + x sin; elements past
// rot_dim in a head are untouched; q/k row strides are honoured (the q and k
// views of a fused qkv projection).  Differences, by design: the math runs in
// fp32 (the reference rounds every product to the storage type), the cache
// may be fp32 while q/k are bf16/fp16, and a token whose position is outside
// [0, max_position) is left unchanged instead of reading outside the cache.
//
// Design: a thread owns one "unit" of one head: for NeoX a 16-byte vector of
// the first half plus the matching vector of the second half, for GPT-J one
// 16-byte vector of interleaved pairs, so every q/k access is a coalesced
// 16-byte load/store and cos/sin are fetched as vectors too.  A token's units
// are covered by one CTA, or (NeoX) split over several CTAs whose size depends
// on the batch (see launch_rope).
#include "common.cuh"

namespace pace {
namespace {

// N consecutive cache entries as floats, with one or two vector loads.
template <typename C, int N>
__device__ __forceinline__ void load_cs(const C* p, float* out) {
  if constexpr (sizeof(C) == 4) {
    static_assert(N == 8 || N == 4 || N == 2, "");
    if constexpr (N == 8) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p));
      const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
      out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
      out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
    } else if constexpr (N == 4) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p));
      out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    } else {
      const float2 a = __ldg(reinterpret_cast<const float2*>(p));
      out[0] = a.x; out[1] = a.y;
    }
  } else {
    static_assert(N == 8 || N == 4, "");
    if constexpr (N == 8) {
      Traits<C>::unpack(__ldg(reinterpret_cast<const uint4*>(p)), out);
    } else {
      const uint2 a = __ldg(reinterpret_cast<const uint2*>(p));
      float tmp[8];
      Traits<C>::unpack(make_uint4(a.x, a.y, 0u, 0u), tmp);
      out[0] = tmp[0]; out[1] = tmp[1]; out[2] = tmp[2]; out[3] = tmp[3];
    }
  }
}

// SPLIT_MAJOR: the token's units are split over several CTAs ("parts") and
// the grid is (parts, tokens); otherwise it is (tokens, parts).  A compile-time
// choice: selecting the indices at run time cost 12 registers and occupancy.
// TIGHT: at most 32 registers (4 CTAs of 512 threads per SM), for the
// multi-part launches above T = 128, where the extra residency pays: 70B at
// T=512 16 % faster, long prefills 1-4 %.  One-part launches keep the
// compiler's 40 registers (32 cost the 8B shape at T=512 26 %).
template <typename T, typename C, bool NEOX, bool SPLIT_MAJOR, bool TIGHT>
__global__ void __launch_bounds__(512, TIGHT ? 4 : 0)
    rope_vec_kernel(const int64_t* __restrict__ positions, T* query, T* key, int num_heads,
                    int num_kv_heads, int head_size, int64_t q_stride, int64_t k_stride,
                    const C* __restrict__ cache, int rot_dim, int64_t max_position) {
  using Tr = Traits<T>;
  constexpr int V = Tr::kVec;
  const int64_t tok = SPLIT_MAJOR ? blockIdx.y : blockIdx.x;
  const int part_idx = SPLIT_MAJOR ? blockIdx.x : blockIdx.y;
  const int nparts = SPLIT_MAJOR ? gridDim.x : gridDim.y;
  pdl_launch_dependents();
  const int embed = rot_dim / 2;
  // units per head: NeoX pairs a vector of each half; GPT-J one vector of pairs
  const int uph = NEOX ? embed / V : rot_dim / V;
  const int total = (num_heads + num_kv_heads) * uph;
  if (threadIdx.x == 0) {
    // Prefetch the heads this CTA rotates (all of them with one part).
    const int u0 = part_idx * blockDim.x;
    const int u1 = nparts == 1 ? total : min(total, u0 + (int)blockDim.x);
    if (u1 > u0) {
      const int ha = u0 / uph, hb = (u1 - 1) / uph;  // heads [ha, hb]
      const int qb = min(hb, num_heads - 1);
      if (qb >= ha)
        prefetch_l2(query + tok * q_stride + (int64_t)ha * head_size,
                    (int64_t)(qb - ha + 1) * head_size * sizeof(T));
      const int ka = max(ha, num_heads) - num_heads, kb = hb - num_heads;
      if (kb >= ka)
        prefetch_l2(key + tok * k_stride + (int64_t)ka * head_size,
                    (int64_t)(kb - ka + 1) * head_size * sizeof(T));
    }
  }
  if (NEOX && total <= (int)(blockDim.x * nparts)) {
    // One unit per thread (the token's units split over `nparts` CTAs).
    const int u = part_idx * blockDim.x + threadIdx.x;
    const bool live = u < total;
    const int head = live ? u / uph : 0;
    const int part = live ? u - head * uph : 0;
    T* hp = head < num_heads ? query + tok * q_stride + (int64_t)head * head_size
                             : key + tok * k_stride + (int64_t)(head - num_heads) * head_size;
    const int i0 = part * V;
    pdl_wait();
    // issue the q/k loads before the position load so the two latencies overlap
    uint4 xv = make_uint4(0, 0, 0, 0), yv = xv;
    if (live) {
      xv = ld_v4(hp + i0);
      yv = ld_v4(hp + embed + i0);
    }
    const int64_t pos = positions[tok];
    if (!live || pos < 0 || pos >= max_position) return;
    const C* cos_row = cache + pos * rot_dim;
    float c[V], s[V], x[V], y[V];
    load_cs<C, V>(cos_row + i0, c);
    load_cs<C, V>(cos_row + embed + i0, s);
    Tr::unpack(xv, x);
    Tr::unpack(yv, y);
    float xo[V], yo[V];
#pragma unroll
    for (int e = 0; e < V; ++e) {
      xo[e] = x[e] * c[e] - y[e] * s[e];
      yo[e] = y[e] * c[e] + x[e] * s[e];
    }
    st_v4(hp + i0, Tr::pack(xo));
    st_v4(hp + embed + i0, Tr::pack(yo));
    return;
  }
  pdl_wait();
  const int64_t pos = positions[tok];
  if (pos < 0 || pos >= max_position) return;
  const C* cos_row = cache + pos * rot_dim;
  const C* sin_row = cos_row + embed;
  for (int u = threadIdx.x; u < total; u += blockDim.x) {
    const int head = u / uph;
    const int part = u - head * uph;
    T* hp = head < num_heads ? query + tok * q_stride + (int64_t)head * head_size
                             : key + tok * k_stride + (int64_t)(head - num_heads) * head_size;
    if (NEOX) {
      const int i0 = part * V;
      float c[V], s[V], x[V], y[V];
      const uint4 xv = ld_v4(hp + i0);
      const uint4 yv = ld_v4(hp + embed + i0);
      load_cs<C, V>(cos_row + i0, c);
      load_cs<C, V>(sin_row + i0, s);
      Tr::unpack(xv, x);
      Tr::unpack(yv, y);
      float xo[V], yo[V];
#pragma unroll
      for (int e = 0; e < V; ++e) {
        xo[e] = x[e] * c[e] - y[e] * s[e];
        yo[e] = y[e] * c[e] + x[e] * s[e];
      }
      st_v4(hp + i0, Tr::pack(xo));
      st_v4(hp + embed + i0, Tr::pack(yo));
    } else {
      const int e0 = part * V;  // element offset; pairs e0/2 .. e0/2 + V/2
      float c[V / 2], s[V / 2], a[V];
      const uint4 av = ld_v4(hp + e0);
      load_cs<C, V / 2>(cos_row + e0 / 2, c);
      load_cs<C, V / 2>(sin_row + e0 / 2, s);
      Tr::unpack(av, a);
      float o[V];
#pragma unroll
      for (int p = 0; p < V / 2; ++p) {
        const float x = a[2 * p], y = a[2 * p + 1];
        o[2 * p] = x * c[p] - y * s[p];
        o[2 * p + 1] = y * c[p] + x * s[p];
      }
      st_v4(hp + e0, Tr::pack(o));
    }
  }
}

// Lean NeoX kernel for 16-bit q/k: one unit (a 16-byte vector of each half of
// one head) per thread, UPH units per head at compile time (rot_dim = 16 * UPH),
// grid (tokens, parts) with each token's units split over `parts` CTAs.  Head
// and unit indices are shifts, so the kernel stays at 32 registers (the general
// kernel above needs 46-52, which costs occupancy).
//
// SPEC (speculation): the token's position and its cos/sin slice are read
// BEFORE waiting for the previous kernel in the stream, so they arrive while
// it drains; after the wait only the q/k loads stand between the kernel and
// its stores (one L2 round trip instead of position -> cos/sin -> math).  The
// position is read again after the wait (at L2, past the incoherent L1) and the
// slice reloaded if it changed, so a position written by the previous kernel
// is honoured.  The cos/sin table is a constant of the model: it must not be
// written by a kernel that is still running when this one starts.  Chosen only
// when the whole grid is resident in one wave: a CTA of a later wave starts
// after its predecessor has finished, and the early position load would only
// delay its q/k loads.  Measured on B200 (Llama-3-8B, 32 back-to-back
// launches, T = 512): 2.39 us against 3.23 us without it.
template <typename T, typename C, int UPH, bool SPEC>
__global__ void __launch_bounds__(512)
    rope_neox_kernel(const int64_t* __restrict__ positions, T* query, T* key, int num_heads,
                     int num_kv_heads, int head_size, int64_t q_stride, int64_t k_stride,
                     const C* __restrict__ cache, int64_t max_position) {
  using Tr = Traits<T>;
  constexpr int V = Tr::kVec;
  static_assert(V == 8, "16-bit q/k");
  constexpr int EMBED = UPH * V;
  constexpr int ROT = 2 * EMBED;
  const int64_t tok = blockIdx.x;
  const int u = blockIdx.y * blockDim.x + threadIdx.x;
  const int heads = num_heads + num_kv_heads;
  const bool live = u < heads * UPH;
  const int head = u / UPH;
  const int i0 = (u % UPH) * V;
  T* hp = head < num_heads ? query + tok * q_stride + (int64_t)head * head_size
                           : key + tok * k_stride + (int64_t)(head - num_heads) * head_size;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    const int ha = blockIdx.y * blockDim.x / UPH;
    const int hb = min(heads - 1, (int)((blockIdx.y + 1) * blockDim.x - 1) / UPH);
    const int qb = min(hb, num_heads - 1);
    if (qb >= ha)
      prefetch_l2(query + tok * q_stride + (int64_t)ha * head_size,
                  (int64_t)(qb - ha + 1) * head_size * sizeof(T));
    const int ka = max(ha, num_heads) - num_heads, kb = hb - num_heads;
    if (kb >= ka)
      prefetch_l2(key + tok * k_stride + (int64_t)ka * head_size,
                  (int64_t)(kb - ka + 1) * head_size * sizeof(T));
  }
  float c[V], s[V];
  int64_t spec = -1;
  if (SPEC && live) {
    spec = ld_cg_s64(positions + tok);
    if (spec >= 0 && spec < max_position) {
      load_cs<C, V>(cache + spec * ROT + i0, c);
      load_cs<C, V>(cache + spec * ROT + EMBED + i0, s);
    }
  }
  pdl_wait();
  if (!live) return;
  const uint4 xv = ld_v4(hp + i0);
  const uint4 yv = ld_v4(hp + EMBED + i0);
  const int64_t pos = SPEC ? ld_cg_s64(positions + tok) : positions[tok];
  if (pos < 0 || pos >= max_position) return;
  if (!SPEC || pos != spec) {
    load_cs<C, V>(cache + pos * ROT + i0, c);
    load_cs<C, V>(cache + pos * ROT + EMBED + i0, s);
  }
  float x[V], y[V], xo[V], yo[V];
  Tr::unpack(xv, x);
  Tr::unpack(yv, y);
#pragma unroll
  for (int e = 0; e < V; ++e) {
    xo[e] = x[e] * c[e] - y[e] * s[e];
    yo[e] = y[e] * c[e] + x[e] * s[e];
  }
  st_v4(hp + i0, Tr::pack(xo));
  st_v4(hp + EMBED + i0, Tr::pack(yo));
}

// Scalar fallback: one thread per rotated pair.
template <typename T, typename C, bool NEOX>
__global__ void __launch_bounds__(256)
    rope_scalar_kernel(const int64_t* __restrict__ positions, T* query, T* key, int num_heads,
                       int num_kv_heads, int head_size, int64_t q_stride, int64_t k_stride,
                       const C* __restrict__ cache, int rot_dim, int64_t max_position) {
  using Tr = Traits<T>;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t tok = blockIdx.x;
  const int64_t pos = positions[tok];
  if (pos < 0 || pos >= max_position) return;
  const int embed = rot_dim / 2;
  const int total = (num_heads + num_kv_heads) * embed;
  const C* cos_row = cache + pos * rot_dim;
  const C* sin_row = cos_row + embed;
  for (int u = threadIdx.x; u < total; u += blockDim.x) {
    const int head = u / embed;
    const int i = u - head * embed;
    T* hp = head < num_heads ? query + tok * q_stride + (int64_t)head * head_size
                             : key + tok * k_stride + (int64_t)(head - num_heads) * head_size;
    const int xi = NEOX ? i : 2 * i;
    const int yi = NEOX ? embed + i : 2 * i + 1;
    const float c = Traits<C>::to_f(cos_row[i]);
    const float s = Traits<C>::to_f(sin_row[i]);
    const float x = Tr::to_f(hp[xi]);
    const float y = Tr::to_f(hp[yi]);
    hp[xi] = Tr::from_f(x * c - y * s);
    hp[yi] = Tr::from_f(y * c + x * s);
  }
}

template <typename T, typename C>
int launch_rope(const int64_t* positions, void* query, void* key, int64_t num_tokens,
                int num_heads, int num_kv_heads, int head_size, int64_t q_stride,
                int64_t k_stride, const void* cache, int rot_dim, int64_t max_position,
                bool neox, cudaStream_t stream) {
  constexpr int V = Traits<T>::kVec;
  T* q = static_cast<T*>(query);
  T* k = static_cast<T*>(key);
  const C* cs = static_cast<const C*>(cache);
  const int embed = rot_dim / 2;
  bool vec = (head_size % V == 0) && (q_stride % V == 0) && aligned16(query) &&
             aligned16(cache) && ((int64_t)rot_dim * (int64_t)sizeof(C)) % 16 == 0;
  if (num_kv_heads > 0) vec = vec && (k_stride % V == 0) && aligned16(key);
  if (neox)
    vec = vec && (embed % V == 0);
  else
    vec = vec && (rot_dim % V == 0);
  dim3 grid((unsigned)num_tokens);
  cudaError_t err;
  if constexpr (V == 8) {
    // Lean NeoX kernel for rot_dim 64 / 128 / 256.  Parts per token, measured on
    // B200: CTAs of about 96 threads up to T = 128 (8B, T=128: 1.48 us against
    // 1.58), two parts per token above (8B, T=512: 2.39 us with speculation;
    // 70B, T=512: 3.34 against 3.50 for the general kernel).  Speculation only
    // when every thread of the grid is resident at once (see rope_neox_kernel).
    const int uph = embed / V;
    if (vec && neox && (uph == 4 || uph == 8 || uph == 16) && num_tokens <= INT32_MAX) {
      const int64_t units = (int64_t)(num_heads + num_kv_heads) * uph;
      int64_t parts = num_tokens <= 128 ? ceil_div(units, 96) : (units > 256 ? 2 : 1);
      int threads = (int)ceil_div(ceil_div(units, parts), 32) * 32;
      if (threads > 512) {
        parts = ceil_div(units, 512);
        threads = (int)ceil_div(ceil_div(units, parts), 32) * 32;
      }
      if (parts <= 65535) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
        const bool spec =
            num_tokens * parts * threads <= (int64_t)sm_count(dev) * 2048;
        const dim3 g((unsigned)num_tokens, (unsigned)parts);
        auto go = [&](auto kernel) {
          return launch(kernel, g, dim3(threads), 0, stream, positions, q, k, num_heads,
                        num_kv_heads, head_size, q_stride, k_stride, cs, max_position);
        };
        switch (uph * 2 + (spec ? 1 : 0)) {
          case 8: err = go(rope_neox_kernel<T, C, 4, false>); break;
          case 9: err = go(rope_neox_kernel<T, C, 4, true>); break;
          case 16: err = go(rope_neox_kernel<T, C, 8, false>); break;
          case 17: err = go(rope_neox_kernel<T, C, 8, true>); break;
          case 32: err = go(rope_neox_kernel<T, C, 16, false>); break;
          default: err = go(rope_neox_kernel<T, C, 16, true>); break;
        }
        if (err != cudaSuccess) return cuda_fail(err, "rotary_embedding");
        return PACE_OK;
      }
    }
  }
  if (vec) {
    const int uph = neox ? embed / V : rot_dim / V;
    const int64_t units = (int64_t)(num_heads + num_kv_heads) * uph;
    // NeoX: a token's units (one per thread) may be split over several CTAs.
    // Measured on B200 (Llama-3-8B, 320 units): 2-warp CTAs are fastest for
    // decode-sized batches (T <= 128: 13-18 % over one CTA per token), one CTA
    // per token up to T = 512, 5-warp CTAs above (T = 768-1024: 12-14 %; long
    // prefills: 9 %).
    int64_t per_cta = 512;
    if (neox) per_cta = num_tokens <= 128 ? 64 : (num_tokens > 512 ? 160 : 512);
    int64_t split = neox ? ceil_div(units, per_cta) : 1;
    if (split > 65535) split = 1;  // grid.y limit: one CTA per token loops over the units
    int threads = (int)ceil_div(ceil_div(units, split), 32) * 32;
    if (threads > 512) threads = 512;
    if (threads < 32) threads = 32;
    // Order of the split CTAs, measured on B200: a token's parts adjacent
    // (split-major) is 2-7 % faster for T <= 128; for long prefills one part
    // of every token, then the next part (token-major), is 15-20 % faster.
    const int sm = (split > 1 && num_tokens <= 128) ? 1 : 0;
    if (sm)
      grid = dim3((unsigned)split, (unsigned)num_tokens);
    else
      grid.y = (unsigned)split;
    auto go = [&](auto kernel) {
      return launch(kernel, grid, dim3(threads), 0, stream, positions, q, k, num_heads,
                    num_kv_heads, head_size, q_stride, k_stride, cs, rot_dim, max_position);
    };
    const bool tight = split > 1 && num_tokens > 128;
    err = !neox ? go(rope_vec_kernel<T, C, false, false, false>)
          : sm  ? go(rope_vec_kernel<T, C, true, true, false>)
          : tight ? go(rope_vec_kernel<T, C, true, false, true>)
                  : go(rope_vec_kernel<T, C, true, false, false>);
  } else {
    err = neox ? launch(rope_scalar_kernel<T, C, true>, grid, dim3(256), 0, stream, positions, q,
                        k, num_heads, num_kv_heads, head_size, q_stride, k_stride, cs, rot_dim,
                        max_position)
               : launch(rope_scalar_kernel<T, C, false>, grid, dim3(256), 0, stream, positions,
                        q, k, num_heads, num_kv_heads, head_size, q_stride, k_stride, cs, rot_dim,
                        max_position);
  }
  if (err != cudaSuccess) return cuda_fail(err, "rotary_embedding");
  return PACE_OK;
}

}  // namespace
}  // namespace pace

extern "C" int pace_rotary_embedding(const int64_t* positions, void* query, void* key,
                                     int64_t num_tokens, int num_heads, int num_kv_heads,
                                     int head_size, int64_t query_row_stride,
                                     int64_t key_row_stride, const void* cos_sin_cache,
                                     int cache_dtype, int rot_dim, int64_t max_position,
                                     int is_neox, int dtype, cudaStream_t stream) {
  using namespace pace;
  if (num_tokens < 0 || num_tokens > INT32_MAX || num_heads < 0 || num_kv_heads < 0 ||
      head_size <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "rotary_embedding: bad shape");
  if (rot_dim <= 0 || rot_dim % 2 != 0 || rot_dim > head_size)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "rotary_embedding: rot_dim %d must be even and in (0, head_size=%d]", rot_dim,
                head_size);
  if (max_position <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "rotary_embedding: empty cos_sin_cache");
  if (query_row_stride < (int64_t)num_heads * head_size ||
      (num_kv_heads > 0 && key_row_stride < (int64_t)num_kv_heads * head_size))
    return fail(PACE_ERR_INVALID_ARGUMENT, "rotary_embedding: row stride smaller than the row");
  if (num_tokens == 0 || num_heads + num_kv_heads == 0) return PACE_OK;
  if (!positions || !cos_sin_cache || (num_heads > 0 && !query) || (num_kv_heads > 0 && !key))
    return fail(PACE_ERR_INVALID_ARGUMENT, "rotary_embedding: null pointer");
  StreamDeviceGuard guard(stream);
  const bool neox = is_neox != 0;
  return PACE_DISPATCH_FLOAT(dtype, "rotary_embedding", [&] {
    if (cache_dtype == PACE_F32)
      return launch_rope<scalar_t, float>(positions, query, key, num_tokens, num_heads,
                                          num_kv_heads, head_size, query_row_stride,
                                          key_row_stride, cos_sin_cache, rot_dim, max_position,
                                          neox, stream);
    if (cache_dtype == dtype)
      return launch_rope<scalar_t, scalar_t>(positions, query, key, num_tokens, num_heads,
                                             num_kv_heads, head_size, query_row_stride,
                                             key_row_stride, cos_sin_cache, rot_dim,
                                             max_position, neox, stream);
    return fail(PACE_ERR_UNSUPPORTED_DTYPE,
                "rotary_embedding: cos_sin_cache dtype %d must be float32 or the q/k dtype %d",
                cache_dtype, dtype);
  });
}
