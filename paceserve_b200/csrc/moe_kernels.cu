// MoE routing for sm_100a: fused softmax + top-k over expert logits, and the
// block-aligned counting sort of (token, expert) assignments.
//
// topk_softmax (reference csrc/moe_topk_softmax_kernels.cu:182-380, host
// :476-503).  Output semantics: softmax in fp32 (max-subtract, expf, one
// reciprocal of the row sum, multiply), then k rounds of argmax with ties to
// the lowest expert index; token_expert_indices[t, j] = j*T + t.
// For power-of-two E <= 256 each row is split over TPR lanes that own the same
// expert columns as the reference's fused kernel, so the fp32 row sum is
// accumulated in the same association (per-lane sequential sum, then an XOR
// butterfly over the lanes of the row).  That makes the probabilities -- and
// therefore the selected indices, including exact ties -- bit-identical to the
// reference.  Other E (the reference falls back to two kernels and a
// workspace) use one warp per row and no workspace; probabilities then agree
// to fp32 rounding.
//
// moe_align_block_size (reference csrc/moe_align_block_size_kernels.cu:23-109).
// Output semantics: per-expert counts padded to a multiple of block_size,
// expert_ids per block, and sorted_token_ids holding, for each expert, its flat
// indices in ASCENDING order.  Design: one CTA of up to 32 warps; the expert ids
// are staged once into shared memory as int16 (vector loads, all in flight
// together) when they fit; each warp owns a contiguous slice of the flat index
// range.  For E <= 32 a warp counts and ranks each 32-entry group with one
// ballot per expert (lane x keeps expert x's count and next slot in a
// register); larger E use shared-memory atomics and match-any.  A
// shared-memory scan gives every (warp, expert) its start, and the second pass
// scatters by rank within the group -- a stable counting sort with no global
// scratch and no global atomics.
#include "common.cuh"

namespace pace {
namespace {

// --------------------------------------------------------------- top-k ----

// Column ownership of a power-of-two row of E fp32 logits: vectors of LDG
// floats, VECS of them per lane, TPR lanes per row.  Lane g of a row owns the
// columns (v * TPR + g) * LDG + j for v < VECS, j < LDG.
template <int E>
struct RowSplit {
  static constexpr int LDG = E < 4 ? E : 4;
  static constexpr int VECS = (E / (LDG * 32)) > 0 ? E / (LDG * 32) : 1;
  static constexpr int VPT = VECS * LDG;
  static constexpr int TPR = E / VPT;
  static constexpr int ROWS_PER_WARP = 32 / TPR;
  __device__ __forceinline__ static int col(int g, int v, int j) { return (v * TPR + g) * LDG + j; }
};

template <int E, bool ALIGNED>
__global__ void __launch_bounds__(64)
    topk_softmax_pow2_kernel(const float* __restrict__ gating, float* __restrict__ weights,
                             int32_t* __restrict__ indices, int32_t* __restrict__ source_rows,
                             int64_t num_rows, int k, int renormalize) {
  using S = RowSplit<E>;
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t row = warp_global * S::ROWS_PER_WARP + lane / S::TPR;
  const int g = lane % S::TPR;
  const bool live = row < num_rows;
  // Lanes past the last row compute on row 0 and store nothing, so every lane
  // stays in the shuffles below.
  const float* rp = gating + (live ? row : 0) * (int64_t)E;

  float x[S::VPT];
#pragma unroll
  for (int v = 0; v < S::VECS; ++v) {
    const float* p = rp + S::col(g, v, 0);
    if constexpr (ALIGNED && S::LDG == 4) {
      const float4 q = *reinterpret_cast<const float4*>(p);
      x[v * 4 + 0] = q.x; x[v * 4 + 1] = q.y; x[v * 4 + 2] = q.z; x[v * 4 + 3] = q.w;
    } else if constexpr (ALIGNED && S::LDG == 2) {
      const float2 q = *reinterpret_cast<const float2*>(p);
      x[v * 2 + 0] = q.x; x[v * 2 + 1] = q.y;
    } else {
#pragma unroll
      for (int j = 0; j < S::LDG; ++j) x[v * S::LDG + j] = p[j];
    }
  }

  float mx = x[0];
#pragma unroll
  for (int i = 1; i < S::VPT; ++i) mx = fmaxf(mx, x[i]);
#pragma unroll
  for (int m = S::TPR / 2; m > 0; m >>= 1)
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m, S::TPR));

  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < S::VPT; ++i) {
    x[i] = expf(x[i] - mx);
    sum += x[i];
  }
#pragma unroll
  for (int m = S::TPR / 2; m > 0; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m, S::TPR);
  const float rcp = 1.f / sum;
#pragma unroll
  for (int i = 0; i < S::VPT; ++i) x[i] *= rcp;

  float* wrow = weights + (live ? row : 0) * (int64_t)k;
  int32_t* irow = indices + (live ? row : 0) * (int64_t)k;
  float picked_sum = 0.f;
  for (int kk = 0; kk < k; ++kk) {
    // Lane-local argmax in ascending column order; strict > keeps the lowest.
    float bv = x[0];
    int be = S::col(g, 0, 0);
#pragma unroll
    for (int v = 0; v < S::VECS; ++v)
#pragma unroll
      for (int j = 0; j < S::LDG; ++j)
        if (x[v * S::LDG + j] > bv) {
          bv = x[v * S::LDG + j];
          be = S::col(g, v, j);
        }
#pragma unroll
    for (int m = S::TPR / 2; m > 0; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m, S::TPR);
      const int oe = __shfl_xor_sync(0xffffffffu, be, m, S::TPR);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if (live && g == 0) {
      wrow[kk] = bv;
      irow[kk] = be;
      source_rows[row * k + kk] = (int32_t)(kk * num_rows + row);
      picked_sum += bv;
    }
    // The owning lane retires the winner (probabilities are >= 0).
#pragma unroll
    for (int v = 0; v < S::VECS; ++v)
#pragma unroll
      for (int j = 0; j < S::LDG; ++j)
        if (S::col(g, v, j) == be) x[v * S::LDG + j] = -10000.f;
  }
  if (renormalize && live && g == 0) {
    for (int kk = 0; kk < k; ++kk) wrow[kk] = wrow[kk] / picked_sum;
  }
}

// One warp per row, any E <= 32 * EPT; lane l owns columns l, l+32, ...
template <int EPT>
__global__ void __launch_bounds__(128)
    topk_softmax_warp_kernel(const float* __restrict__ gating, float* __restrict__ weights,
                             int32_t* __restrict__ indices, int32_t* __restrict__ source_rows,
                             int64_t num_rows, int num_experts, int k, int renormalize) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= num_rows) return;  // whole warp leaves together
  const float* rp = gating + row * (int64_t)num_experts;
  float x[EPT];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int c = lane + 32 * i;
    x[i] = c < num_experts ? rp[c] : -INFINITY;
    mx = fmaxf(mx, x[i]);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int c = lane + 32 * i;
    x[i] = c < num_experts ? expf(x[i] - mx) : -1.f;
    if (c < num_experts) sum += x[i];
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
  const float rcp = 1.f / sum;
#pragma unroll
  for (int i = 0; i < EPT; ++i)
    if (lane + 32 * i < num_experts) x[i] *= rcp;
  float picked_sum = 0.f;
  for (int kk = 0; kk < k; ++kk) {
    float bv = -2.f;
    int be = num_experts;
#pragma unroll
    for (int i = 0; i < EPT; ++i)
      if (lane + 32 * i < num_experts && x[i] > bv) {
        bv = x[i];
        be = lane + 32 * i;
      }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oe = __shfl_xor_sync(0xffffffffu, be, m);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if (lane == 0) {
      weights[row * k + kk] = bv;
      indices[row * k + kk] = be;
      source_rows[row * k + kk] = (int32_t)(kk * num_rows + row);
      picked_sum += bv;
    }
#pragma unroll
    for (int i = 0; i < EPT; ++i)
      if (lane + 32 * i == be) x[i] = -1.f;
  }
  if (renormalize && lane == 0)
    for (int kk = 0; kk < k; ++kk) weights[row * k + kk] = weights[row * k + kk] / picked_sum;
}

template <int E>
cudaError_t launch_topk_pow2(const float* g, float* w, int32_t* idx, int32_t* src, int64_t T,
                             int k, int renorm, cudaStream_t stream) {
  using S = RowSplit<E>;
  constexpr int kThreads = 64;
  const int64_t rows_per_cta = (kThreads / 32) * S::ROWS_PER_WARP;
  const dim3 grid((unsigned)ceil_div(T, rows_per_cta));
  const bool aligned = (reinterpret_cast<uintptr_t>(g) % (sizeof(float) * S::LDG)) == 0;
  if (aligned)
    return launch(topk_softmax_pow2_kernel<E, true>, grid, dim3(kThreads), 0, stream, g, w, idx,
                  src, T, k, renorm);
  return launch(topk_softmax_pow2_kernel<E, false>, grid, dim3(kThreads), 0, stream, g, w, idx,
                src, T, k, renorm);
}

template <int EPT>
cudaError_t launch_topk_warp(const float* g, float* w, int32_t* idx, int32_t* src, int64_t T,
                             int E, int k, int renorm, cudaStream_t stream) {
  const dim3 grid((unsigned)ceil_div(T, 4));
  return launch(topk_softmax_warp_kernel<EPT>, grid, dim3(128), 0, stream, g, w, idx, src, T, E,
                k, renorm);
}

// ----------------------------------------------------- moe_align_block_size --

template <typename I>
__device__ __forceinline__ int load_expert(const I* ids, int64_t i, int num_experts) {
  const int64_t e = (int64_t)ids[i];
  return (e >= 0 && e < num_experts) ? (int)e : -1;
}

// Number of 4-byte words before the staged expert ids in shared memory:
// cnt[NW][E] | cum[E+1] | tot[E] | scan[32], rounded up to 8 bytes.
__host__ __device__ inline int64_t moe_align_words(int nw, int num_experts) {
  const int64_t w = (int64_t)nw * num_experts + 2LL * num_experts + 1 + 32;
  return (w + 1) & ~1LL;
}

// Expert of every flat entry as int16 in shared memory (-1 for ids outside
// [0, E)), read with all loads of a thread issued before its stores: 16-byte
// vectors for 4-byte ids on a 16-byte boundary, 8 scalar loads in flight
// otherwise.
template <typename I>
__device__ __forceinline__ void stage_experts(const I* __restrict__ ids, int64_t numel, int E,
                                              int16_t* ex) {
  const int tid = threadIdx.x, nt = blockDim.x;
  if constexpr (sizeof(I) == 4) {
    if ((reinterpret_cast<uintptr_t>(ids) & 15u) == 0) {
      const int64_t nv = numel / 4;
      const int4* v4 = reinterpret_cast<const int4*>(ids);
      for (int64_t base = tid; base < nv; base += (int64_t)nt * 4) {
        int4 r[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t v = base + (int64_t)k * nt;
          if (v < nv) r[k] = __ldg(v4 + v);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t v = base + (int64_t)k * nt;
          if (v < nv) {
            const int q[4] = {r[k].x, r[k].y, r[k].z, r[k].w};
            short4 o;
            o.x = (short)((q[0] >= 0 && q[0] < E) ? q[0] : -1);
            o.y = (short)((q[1] >= 0 && q[1] < E) ? q[1] : -1);
            o.z = (short)((q[2] >= 0 && q[2] < E) ? q[2] : -1);
            o.w = (short)((q[3] >= 0 && q[3] < E) ? q[3] : -1);
            *reinterpret_cast<short4*>(ex + 4 * v) = o;
          }
        }
      }
      for (int64_t i = nv * 4 + tid; i < numel; i += nt) ex[i] = (int16_t)load_expert(ids, i, E);
      return;
    }
  }
  for (int64_t base = tid; base < numel; base += (int64_t)nt * 8) {
    int v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t i = base + (int64_t)k * nt;
      v[k] = i < numel ? load_expert(ids, i, E) : -1;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t i = base + (int64_t)k * nt;
      if (i < numel) ex[i] = (int16_t)v[k];
    }
  }
}

// STAGED: the expert ids are first copied into shared memory (when they fit),
// so the two counting passes never wait on global memory inside their loops.
template <typename I, bool STAGED>
__global__ void __launch_bounds__(1024)
    moe_align_kernel(const I* __restrict__ ids, int64_t numel, int num_experts, int block_size,
                     int32_t* __restrict__ sorted_ids, int64_t sorted_capacity,
                     int32_t* __restrict__ expert_ids, int32_t* __restrict__ total_post_pad,
                     int fill_padding) {
  extern __shared__ int smem[];
  const int E = num_experts;
  const int NW = blockDim.x >> 5;
  int* cnt = smem;
  int* cum = cnt + NW * E;
  int* tot = cum + E + 1;
  int* scan = tot + E;
  int16_t* ex = reinterpret_cast<int16_t*>(smem + moe_align_words(NW, E));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();
  pdl_wait();

  if (STAGED) stage_experts(ids, numel, E, ex);
  for (int i = tid; i < NW * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();

  const int64_t chunk = ceil_div(ceil_div(numel, NW), 32) * 32;
  const int64_t begin = (int64_t)warp * chunk;
  const int64_t end = begin + chunk < numel ? begin + chunk : numel;
  int* wcnt = cnt + warp * E;
  const unsigned lt_mask = (1u << lane) - 1u;

  // Pass 1: per-warp counts.  E <= 32: one ballot per expert per 32 entries,
  // lane x accumulating expert x; otherwise shared-memory atomics.
  if (E <= 32) {
    int c = 0;
    for (int64_t base = begin; base < end; base += 32) {
      const int64_t i = base + lane;
      const int e = i < end ? (STAGED ? (int)ex[i] : load_expert(ids, i, E)) : -1;
      for (int x = 0; x < E; ++x) {
        const unsigned b = __ballot_sync(0xffffffffu, e == x);
        if (lane == x) c += __popc(b);
      }
    }
    if (lane < E) wcnt[lane] = c;
  } else {
    for (int64_t i = begin + lane; i < end; i += 32) {
      const int e = STAGED ? (int)ex[i] : load_expert(ids, i, E);
      if (e >= 0) atomicAdd(&wcnt[e], 1);
    }
  }
  __syncthreads();

  // Per expert: exclusive prefix over warps, and the total.
  for (int e = tid; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < NW; ++w) {
      const int c = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += c;
    }
    tot[e] = run;
  }
  __syncthreads();

  // Exclusive scan of the padded counts over experts: each thread sums a
  // contiguous run of experts, then a block scan over the thread sums.
  const int per = (E + blockDim.x - 1) / blockDim.x;
  const int e0 = tid * per;
  int local = 0;
  for (int e = e0; e < e0 + per && e < E; ++e) local += (tot[e] + block_size - 1) / block_size * block_size;
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = lane < NW ? scan[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v += u;
    }
    if (lane < NW) scan[lane] = v;  // inclusive warp totals
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? scan[warp - 1] : 0);
  for (int e = e0; e < e0 + per && e < E; ++e) {
    cum[e] = run;
    run += (tot[e] + block_size - 1) / block_size * block_size;
  }
  if (tid == blockDim.x - 1) cum[E] = run;  // the last thread holds the grand total
  __syncthreads();

  const int total = cum[E];
  if (tid == 0) *total_post_pad = total;
  // Each expert's blocks and padding slots, one warp per expert.
  for (int e = warp; e < E; e += NW) {
    for (int b = cum[e] / block_size + lane; b < cum[e + 1] / block_size; b += 32) expert_ids[b] = e;
    if (fill_padding)
      for (int p = cum[e] + tot[e] + lane; p < cum[e + 1]; p += 32) sorted_ids[p] = (int32_t)numel;
  }
  if (fill_padding)
    for (int64_t p = total + tid; p < sorted_capacity; p += blockDim.x) sorted_ids[p] = (int32_t)numel;

  // Pass 2: stable scatter; an entry's slot is its expert's next free slot in
  // this warp's range plus its rank among the group's lanes with that expert.
  if (E <= 32) {
    int next = lane < E ? cum[lane] + wcnt[lane] : 0;  // lane x: next slot of expert x
    for (int64_t base = begin; base < end; base += 32) {
      const int64_t i = base + lane;
      const int e = i < end ? (STAGED ? (int)ex[i] : load_expert(ids, i, E)) : -1;
      unsigned peers = 0;
      int grown = 0;
      for (int x = 0; x < E; ++x) {
        const unsigned b = __ballot_sync(0xffffffffu, e == x);
        if (e == x) peers = b;
        if (lane == x) grown = __popc(b);
      }
      const int slot = __shfl_sync(0xffffffffu, next, e >= 0 ? e : 0);
      if (e >= 0) sorted_ids[slot + __popc(peers & lt_mask)] = (int32_t)i;
      next += grown;
    }
  } else {
    for (int64_t base = begin; base < end; base += 32) {
      const int64_t i = base + lane;
      const int e = i < end ? (STAGED ? (int)ex[i] : load_expert(ids, i, E)) : -1;
      const unsigned active = __ballot_sync(0xffffffffu, e >= 0);
      unsigned peers = 0;
      if (e >= 0) {
        peers = __match_any_sync(active, e);
        sorted_ids[cum[e] + wcnt[e] + __popc(peers & lt_mask)] = (int32_t)i;
      }
      __syncwarp();
      if (e >= 0 && (peers & lt_mask) == 0) wcnt[e] += __popc(peers);
      __syncwarp();
    }
  }
}

// ---------------------------------------------- cluster version, E <= 32 --
// For large inputs the counting sort is spread over a thread-block cluster of
// G <= 8 CTAs (one per SM): CTA r stages and counts the r-th slice, the
// per-CTA expert totals are exchanged through distributed shared memory
// across a cluster barrier, and every CTA then scatters its own slice.  No
// global scratch is used.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// Address of `p` (this CTA's shared memory) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(out)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
  return out;
}
__device__ __forceinline__ int ld_cluster(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

constexpr int kClusterMax = 8;  // portable cluster size
constexpr int kClusterWarps = 16;

// Shared layout (ints): cnt[NW][32] | ctot[32] | base[32] | tot[32] | cum[33] (+pad) | ex[int16]
template <typename I>
__global__ void __launch_bounds__(kClusterWarps * 32)
    moe_align_cluster_kernel(const I* __restrict__ ids, int64_t numel, int num_experts,
                             int block_size, int32_t* __restrict__ sorted_ids,
                             int64_t sorted_capacity, int32_t* __restrict__ expert_ids,
                             int32_t* __restrict__ total_post_pad, int fill_padding,
                             int64_t slice) {
  extern __shared__ int smem[];
  const int E = num_experts;
  const int NW = blockDim.x >> 5;
  int* cnt = smem;               // [NW][32]: per-warp counts, then exclusive prefixes
  int* ctot = cnt + NW * 32;     // this CTA's totals (read by the other CTAs)
  int* base = ctot + 32;         // entries of each expert in earlier CTAs
  int* tot = base + 32;          // cluster-wide totals
  int* cum = tot + 32;           // padded exclusive cumsum [E+1]
  int16_t* ex = reinterpret_cast<int16_t*>(cum + 34);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_rank();
  const int G = gridDim.x;
  const unsigned lt_mask = (1u << lane) - 1u;
  pdl_launch_dependents();
  pdl_wait();

  const int64_t s0 = (int64_t)rank * slice;
  const int64_t s1 = s0 + slice < numel ? s0 + slice : numel;
  const int64_t n = s1 > s0 ? s1 - s0 : 0;
  stage_experts(ids + s0, n, E, ex);
  __syncthreads();

  const int64_t chunk = ceil_div(ceil_div(n, NW), 32) * 32;
  const int64_t begin = (int64_t)warp * chunk;
  const int64_t end = begin + chunk < n ? begin + chunk : n;
  int c = 0;
  for (int64_t b = begin; b < end; b += 32) {
    const int64_t i = b + lane;
    const int e = i < end ? (int)ex[i] : -1;
    for (int x = 0; x < E; ++x) {
      const unsigned m = __ballot_sync(0xffffffffu, e == x);
      if (lane == x) c += __popc(m);
    }
  }
  cnt[warp * 32 + lane] = c;
  __syncthreads();
  if (tid < 32) {
    int run = 0;
    for (int w = 0; w < NW; ++w) {
      const int v = cnt[w * 32 + tid];
      cnt[w * 32 + tid] = run;
      run += v;
    }
    ctot[tid] = run;
  }
  cluster_sync_all();  // every CTA's ctot is complete and visible
  if (tid < 32) {
    int t = 0, bs = 0;
    for (int r = 0; r < G; ++r) {
      const int v = ld_cluster(cluster_addr(&ctot[tid], (uint32_t)r));
      t += v;
      if (r < (int)rank) bs += v;
    }
    tot[tid] = t;
    base[tid] = bs;
  }
  cluster_sync_all();  // no CTA leaves while another may still read its ctot
  if (warp == 0) {
    const int padded = lane < E ? (tot[lane] + block_size - 1) / block_size * block_size : 0;
    int incl = padded;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    cum[lane] = incl - padded;
    if (lane == 31) cum[32] = incl;
  }
  __syncthreads();
  const int total = cum[32];
  if (rank == 0 && tid == 0) *total_post_pad = total;
  const int gw = (int)rank * NW + warp;
  for (int e = gw; e < E; e += G * NW) {
    for (int b = cum[e] / block_size + lane; b < cum[e + 1] / block_size; b += 32) expert_ids[b] = e;
    if (fill_padding)
      for (int p = cum[e] + tot[e] + lane; p < cum[e + 1]; p += 32) sorted_ids[p] = (int32_t)numel;
  }
  if (fill_padding)
    for (int64_t p = total + (int64_t)rank * blockDim.x + tid; p < sorted_capacity;
         p += (int64_t)G * blockDim.x)
      sorted_ids[p] = (int32_t)numel;

  int next = lane < E ? cum[lane] + base[lane] + cnt[warp * 32 + lane] : 0;
  for (int64_t b = begin; b < end; b += 32) {
    const int64_t i = b + lane;
    const int e = i < end ? (int)ex[i] : -1;
    unsigned peers = 0;
    int grown = 0;
    for (int x = 0; x < E; ++x) {
      const unsigned m = __ballot_sync(0xffffffffu, e == x);
      if (e == x) peers = m;
      if (lane == x) grown = __popc(m);
    }
    const int slot = __shfl_sync(0xffffffffu, next, e >= 0 ? e : 0);
    if (e >= 0) sorted_ids[slot + __popc(peers & lt_mask)] = (int32_t)(s0 + i);
    next += grown;
  }
}

}  // namespace
}  // namespace pace

extern "C" int pace_topk_softmax(float* topk_weights, int32_t* topk_indices,
                                 int32_t* token_expert_indices, const float* gating_output,
                                 int64_t num_tokens, int num_experts, int topk, int renormalize,
                                 cudaStream_t stream) {
  using namespace pace;
  if (num_tokens < 0 || num_experts <= 0 || topk <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "topk_softmax: bad shape T=%lld E=%d k=%d",
                (long long)num_tokens, num_experts, topk);
  if (topk > num_experts)
    return fail(PACE_ERR_INVALID_ARGUMENT, "topk_softmax: k=%d exceeds num_experts=%d", topk,
                num_experts);
  if (num_experts > 1024)
    return fail(PACE_ERR_TOO_LARGE, "topk_softmax: num_experts=%d exceeds 1024", num_experts);
  if ((int64_t)topk * num_tokens > INT32_MAX)
    return fail(PACE_ERR_TOO_LARGE, "topk_softmax: k*T exceeds int32");
  if (num_tokens == 0) return PACE_OK;
  if (!topk_weights || !topk_indices || !token_expert_indices || !gating_output)
    return fail(PACE_ERR_INVALID_ARGUMENT, "topk_softmax: null pointer");
  StreamDeviceGuard guard(stream);
  const float* g = gating_output;
  float* w = topk_weights;
  int32_t* idx = topk_indices;
  int32_t* src = token_expert_indices;
  const int64_t T = num_tokens;
  const int k = topk, rn = renormalize ? 1 : 0;
  cudaError_t err;
  switch (num_experts) {
    case 1: err = launch_topk_pow2<1>(g, w, idx, src, T, k, rn, stream); break;
    case 2: err = launch_topk_pow2<2>(g, w, idx, src, T, k, rn, stream); break;
    case 4: err = launch_topk_pow2<4>(g, w, idx, src, T, k, rn, stream); break;
    case 8: err = launch_topk_pow2<8>(g, w, idx, src, T, k, rn, stream); break;
    case 16: err = launch_topk_pow2<16>(g, w, idx, src, T, k, rn, stream); break;
    case 32: err = launch_topk_pow2<32>(g, w, idx, src, T, k, rn, stream); break;
    case 64: err = launch_topk_pow2<64>(g, w, idx, src, T, k, rn, stream); break;
    case 128: err = launch_topk_pow2<128>(g, w, idx, src, T, k, rn, stream); break;
    case 256: err = launch_topk_pow2<256>(g, w, idx, src, T, k, rn, stream); break;
    default: {
      const int E = num_experts;
      if (E <= 32)
        err = launch_topk_warp<1>(g, w, idx, src, T, E, k, rn, stream);
      else if (E <= 64)
        err = launch_topk_warp<2>(g, w, idx, src, T, E, k, rn, stream);
      else if (E <= 128)
        err = launch_topk_warp<4>(g, w, idx, src, T, E, k, rn, stream);
      else if (E <= 256)
        err = launch_topk_warp<8>(g, w, idx, src, T, E, k, rn, stream);
      else if (E <= 512)
        err = launch_topk_warp<16>(g, w, idx, src, T, E, k, rn, stream);
      else
        err = launch_topk_warp<32>(g, w, idx, src, T, E, k, rn, stream);
    }
  }
  if (err != cudaSuccess) return cuda_fail(err, "topk_softmax");
  return PACE_OK;
}

extern "C" int pace_moe_align_block_size(const void* topk_ids, int ids_dtype, int64_t numel,
                                         int num_experts, int block_size,
                                         int32_t* sorted_token_ids, int64_t sorted_capacity,
                                         int32_t* expert_ids, int64_t expert_ids_capacity,
                                         int32_t* num_tokens_post_pad, int fill_padding,
                                         cudaStream_t stream) {
  using namespace pace;
  if (numel < 0 || num_experts <= 0 || block_size <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "moe_align_block_size: bad arguments numel=%lld E=%d block_size=%d",
                (long long)numel, num_experts, block_size);
  const int64_t need = numel + (int64_t)num_experts * (block_size - 1);
  if (need > INT32_MAX)
    return fail(PACE_ERR_TOO_LARGE, "moe_align_block_size: padded size exceeds int32");
  if (sorted_capacity < need)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "moe_align_block_size: sorted_token_ids holds %lld < numel + E*(block_size-1) "
                "= %lld",
                (long long)sorted_capacity, (long long)need);
  if (expert_ids_capacity < ceil_div(need, block_size))
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "moe_align_block_size: expert_ids holds %lld < %lld blocks",
                (long long)expert_ids_capacity, (long long)ceil_div(need, block_size));
  if (!sorted_token_ids || !expert_ids || !num_tokens_post_pad || (numel > 0 && !topk_ids))
    return fail(PACE_ERR_INVALID_ARGUMENT, "moe_align_block_size: null pointer");
  StreamDeviceGuard guard(stream);
  // Inputs above 2048 entries with E <= 32: a cluster of up to 8 CTAs, >= 1024
  // entries each.
  if (numel > 2048 && num_experts <= 32) {
    int g = (int)ceil_div(numel, 1024);
    if (g > kClusterMax) g = kClusterMax;
    const int64_t slice = ceil_div(ceil_div(numel, g), 32) * 32;
    const int64_t csmem = (kClusterWarps * 32 + 32 * 3 + 34) * 4 + ((slice * 2 + 7) & ~7LL);
    if (csmem <= 200 * 1024) {
      auto run_cluster = [&](auto type_tag) -> int {
        using I = decltype(type_tag);
        auto kern = moe_align_cluster_kernel<I>;
        cudaError_t e = cudaSuccess;
        if (csmem > 48 * 1024)
          e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), guard.device(),
                                  (int)csmem);
        if (e != cudaSuccess) return cuda_fail(e, "moe_align_block_size: cluster attributes");
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(g);
        cfg.blockDim = dim3(kClusterWarps * 32);
        cfg.dynamicSmemBytes = (size_t)csmem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = g;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.numAttrs = 1;
        if (pdl_enabled()) {
          attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
          attr[1].val.programmaticStreamSerializationAllowed = 1;
          cfg.numAttrs = 2;
        }
        cfg.attrs = attr;
        e = cudaLaunchKernelEx(&cfg, kern, static_cast<const I*>(topk_ids), numel, num_experts,
                               block_size, sorted_token_ids, sorted_capacity, expert_ids,
                               num_tokens_post_pad, fill_padding, slice);
        if (e != cudaSuccess) return cuda_fail(e, "moe_align_block_size (cluster)");
        return PACE_OK;
      };
      switch (ids_dtype) {
        case PACE_U8: return run_cluster(uint8_t{});
        case PACE_I8: return run_cluster(int8_t{});
        case PACE_I16: return run_cluster(int16_t{});
        case PACE_I32: return run_cluster(int32_t{});
        case PACE_I64: return run_cluster(int64_t{});
        default:
          return fail(PACE_ERR_UNSUPPORTED_DTYPE,
                      "moe_align_block_size: unsupported ids dtype %d", ids_dtype);
      }
    }
  }
  // One CTA: 4 to 32 warps, each owning >= 64 entries when there are enough
  // (>= 256 above 2048 entries), and per-warp counters that fit in shared memory.
  int nw = (int)ceil_div(numel, numel > 2048 ? 256 : 64);
  if (nw < 4) nw = 4;
  if (nw > 32) nw = 32;
  const int64_t max_smem = 200 * 1024;
  while (nw > 1 && moe_align_words(nw, num_experts) * 4 > max_smem) nw >>= 1;
  const int64_t counters = moe_align_words(nw, num_experts) * 4;
  // Stage the ids in shared memory as int16 when they fit next to the counters.
  const int64_t staged_bytes = counters + ((numel * 2 + 7) & ~7LL);
  const bool staged = num_experts <= 32767 && staged_bytes <= max_smem;
  const int64_t smem = staged ? staged_bytes : counters;
  if (counters > max_smem)
    return fail(PACE_ERR_TOO_LARGE, "moe_align_block_size: num_experts=%d too large",
                num_experts);
  auto run = [&](auto type_tag) -> int {
    using I = decltype(type_tag);
    auto kern = staged ? moe_align_kernel<I, true> : moe_align_kernel<I, false>;
    if (smem > 48 * 1024) {
      cudaError_t e =
          ensure_dynamic_smem(reinterpret_cast<const void*>(kern), guard.device(), (int)smem);
      if (e != cudaSuccess) return cuda_fail(e, "moe_align_block_size: smem attribute");
    }
    cudaError_t err = launch(kern, dim3(1), dim3(nw * 32), (size_t)smem, stream,
                             static_cast<const I*>(topk_ids), numel, num_experts, block_size,
                             sorted_token_ids, sorted_capacity, expert_ids, num_tokens_post_pad,
                             fill_padding);
    if (err != cudaSuccess) return cuda_fail(err, "moe_align_block_size");
    return PACE_OK;
  };
  switch (ids_dtype) {
    case PACE_U8: return run(uint8_t{});
    case PACE_I8: return run(int8_t{});
    case PACE_I16: return run(int16_t{});
    case PACE_I32: return run(int32_t{});
    case PACE_I64: return run(int64_t{});
    default:
      return fail(PACE_ERR_UNSUPPORTED_DTYPE, "moe_align_block_size: unsupported ids dtype %d",
                  ids_dtype);
  }
}
