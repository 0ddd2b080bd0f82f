// GEMMs with the layer's elementwise work in their epilogues, for sm_100a
// (tcgen05 tensor cores): out = epilogue(A @ W^T), A [T, K] rows, W [N, K].
//
// Epilogues (each replaces a reference op that would run after the GEMM):
//  * rope: the qkv projection followed by the in-place rotary embedding of
//    the q and k heads (paceserve/model_executor/models/llama.py:176-178,
//    csrc/pos_encoding_kernels.cu:38-76; cache row = [cos(rot/2) | sin(rot/2)]),
//    applied to the fp32 accumulator, so q/k are rounded once and the rope
//    launch and its 4 (nq + nkv) hd bytes per token disappear;
//  * rope with the input RMSNorm as a per-row factor (norm weight folded into
//    W, the row statistics written by the GEMM before);
//  * residual: o_proj / down_proj plus the residual add, writing the new
//    rows' sum of squares per 32 columns for the next norm;
//  * gate/up: silu(gate) * up from a tile holding 128 gate and the matching
//    128 up columns (W = [gate rows; up rows], llama.py:70-104), optionally
//    with the post-attention RMSNorm factor.
//
// Tiles are 128 rows x 256 accumulator columns (for rope two whole heads, so
// both halves of every NeoX pair (i, i + 64) and every GPT-J pair (2i, 2i + 1)
// sit in one tile), or 256 rows on a CTA pair (PAIR, T > 128: a two-CTA
// cluster sharing cta_group::2 MMAs, each CTA holding its 128 rows and half
// of B), in 64-element K blocks.  The workers (CTAs or pairs, one per SM or
// SM pair, persistent) take whole tiles round-robin, then either one more
// data-parallel round on fewer workers or a stream-K split of the leftover
// tiles' (tile, K block) units over all of them (schedule_workers).  A
// segment that covers a whole tile is finished from TMEM.  Any other stores
// its fp32 partial in the caller's workspace, and the tile is finished later
// from the partials, added in worker order so the result does not depend on
// timing: at decode sizes (<= 32 rows) by its last contributor (a per-tile
// counter; no CTA waits), otherwise after one grid-wide barrier by all
// epilogue warps of the grid, a (column pair, 32 rows) piece each.  The grid
// is co-resident (at most one CTA per SM) and every wait is bounded.
//
// Inside a CTA: a shared-memory ring of A (128 x 64) and B (256 or, PAIR,
// 128 x 64) blocks filled by TMA (128-byte swizzle, no multicast; warp 8),
// tcgen05.mma (M=128 or 256, N=256, K=16, fp32) issued by one thread of warp 9
// (of the pair leader) into one of two 256-column TMEM accumulators, and 8
// epilogue warps (warp w owns TMEM lanes 32(w % 4)..+31, i.e. tile rows, and
// head w / 4 of the tile) that drain one accumulator while the MMAs fill the
// other.  Every mbarrier wait is bounded by %globaltimer; on expiry the CTA
// records bit 30 in the caller's fault word, stops issuing, waits (bounded
// again) for its own copies and MMAs, frees TMEM and returns.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "tcgen05.cuh"

namespace pace {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, HEAD = 128;
constexpr int A_BYTES = BM * BK * 2;
// Shared-memory stage ring by CTA mode.  One CTA per 128 x 256 tile: A
// 128 x 64 and B 256 x 64 per stage, 4 stages of 48 KB.  A CTA pair per
// 256 x 256 tile (tcgen05 cta_group::2: each CTA holds its 128 rows of A and
// half of B, 128 x 64): 6 stages of 32 KB.  192 KB either way.
template <bool PAIR>
struct Ring {
  static constexpr int kB = (PAIR ? BN / 2 : BN) * BK * 2;  // B bytes per CTA and stage
  static constexpr int kStage = A_BYTES + kB;
  static constexpr int kStages = PAIR ? 6 : 4;
};
constexpr int RING_BYTES = 4 * Ring<false>::kStage;
static_assert(Ring<true>::kStages * Ring<true>::kStage == RING_BYTES, "");
constexpr int MAX_STAGES = 6;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter: one per head of the tile
constexpr int THREADS = (EPI_WARPS + 2) * 32;
constexpr int TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = RING_BYTES + 1024 + 256;
constexpr int SLOT_FLOATS = BM * BN;  // one partial tile
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait
constexpr int32_t kFaultTimeout = 1 << 30;
constexpr int kEpiBarrier = 1;  // named barrier of the 256 epilogue threads

struct Ctl {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem;
  int abort;
  int ready;  // epilogue: thread 0's grid-barrier wait succeeded
  int nfin;   // decode sizes: shared tiles this CTA completed last ...
  int fin[4];  // ... (at most 2: a range's first and last segment)
};
static_assert(sizeof(Ctl) <= 256, "");

// Static split of the (tile, K block) units over the persistent CTAs.
struct Split {
  int64_t units;  // tiles * k_blocks
  int ctas;
  int k_blocks;
  __device__ __forceinline__ int64_t start(int c) const { return (int64_t)c * units / ctas; }
  // the CTA whose range contains unit u
  __device__ __forceinline__ int owner(int64_t u) const {
    return (int)(((u + 1) * ctas - 1) / units);
  }
};

// A CTA's segments, in order: first whole tiles cta, cta + ctas, ... of the
// rounds that every CTA can fill (data-parallel), then its stream-K range of
// the units of the tiles left over.  Tiles are numbered n fastest, so the
// CTAs running together read a few rows of A and the whole weight, which
// stays in L2, instead of every tile of both.
struct Walk {
  int64_t t_next, t_stop, step;  // data-parallel tiles t_next, +step, ... < t_stop
  int64_t u, u_end;              // stream-K units, relative to tile t_stop
  int k_blocks;
  __device__ __forceinline__ bool next(int64_t& t, int& kb0, int& kb1) {
    if (t_next < t_stop) {
      t = t_next;
      t_next += step;
      kb0 = 0;
      kb1 = k_blocks;
      return true;
    }
    if (u >= u_end) return false;
    const int64_t rt = u / k_blocks;
    t = t_stop + rt;
    kb0 = (int)(u - rt * k_blocks);
    kb1 = (int)min((int64_t)k_blocks, kb0 + (u_end - u));
    u += kb1 - kb0;
    return true;
  }
};

__device__ __forceinline__ void raise_fault(Ctl* ctl, int32_t* fault) {
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
  if (fault) atomicOr(fault, kFaultTimeout);
}

__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kEpiBarrier), "n"(EPI_WARPS * 32) : "memory");
}
// Barrier of the epilogue threads that also ANDs `pred` over them, so every
// epilogue warp takes the same branch.
__device__ __forceinline__ bool epi_all(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "n"(kEpiBarrier), "n"(EPI_WARPS * 32)
      : "memory");
  return r != 0;
}

// n cache entries (n = 8 or 16) starting at p (16-byte aligned) as floats.
template <typename C, int N>
__device__ __forceinline__ void load_cs(const C* p, float* out) {
  if constexpr (sizeof(C) == 4) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p) + i);
      out[4 * i] = v.x;
      out[4 * i + 1] = v.y;
      out[4 * i + 2] = v.z;
      out[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N / 8; ++i)
      Traits<C>::unpack(__ldg(reinterpret_cast<const uint4*>(p) + i), out + 8 * i);
  }
}

// 16 values of a tile row: one 32-byte store when the address allows (a full
// sector; the rows of a warp are far apart, so two 16-byte stores would each
// write half sectors), else two 16-byte stores.
template <typename T>
__device__ __forceinline__ void store16(T* p, const float* v) {
  const uint4 lo = Traits<T>::pack(v), hi = Traits<T>::pack(v + 8);
  if ((reinterpret_cast<uintptr_t>(p) & 31u) == 0) {
    st_v8(p, lo, hi);
  } else {
    st_v4(p, lo);
    st_v4(p + 8, hi);
  }
}

// Partials go through L2 only (.cg): the CTA that reads them back runs on
// another SM, whose L1 may hold stale lines of the same slot from an earlier
// call.
__device__ __forceinline__ void st_cg_f4(float* p, float a, float b, float c, float d) {
  __stcg(reinterpret_cast<float4*>(p), make_float4(a, b, c, d));
}
__device__ __forceinline__ float4 ld_cg_f4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

// Partial-tile layout in the workspace: [16-column chunk][quarter q][row][4
// floats], so one warp instruction (32 rows, the same chunk and quarter) reads
// or writes 512 contiguous bytes.
__device__ __forceinline__ float* slot_q(float* slot, int chunk, int q, int row) {
  return slot + ((int64_t)(chunk * 4 + q) * BM + row) * 4;
}

// ---- epilogue ------------------------------------------------------------
// Epilogue kinds: the rotary embedding of the q/k heads (NeoX or GPT-J
// pairs), the residual add of o_proj / down_proj, or SiLU-and-mul of the
// gate/up projection (a tile holds 128 gate columns and the matching 128 up
// columns; the output is 128 columns).  NORM (rope and gate/up kinds):
// each row of the accumulator is first scaled by its RMSNorm factor
// inv = rsqrt(sum of the row's squares / K + eps), from the sum-of-squares
// partials the producer of the input rows wrote (the residual epilogue, or
// pace_row_sumsq); the norm weight is folded into the GEMM weight by the
// caller, so x_norm @ W^T = inv * (h @ (W diag(w))^T).
constexpr int EPI_ROPE_NEOX = 0, EPI_ROPE_GPTJ = 1, EPI_RESIDUAL = 2, EPI_GATEUP_SILU = 3;
constexpr int SUMSQ_GROUP = 32;  // columns per sum-of-squares partial

struct EpiParams {
  // rope
  const int64_t* positions;
  const void* cache;
  int64_t max_position;
  int rot_heads, total_heads;
  // NORM: the input rows' sum-of-squares partials [rows, sumsq_in_groups]
  const float* sumsq_in;
  int sumsq_in_groups;
  float inv_k, eps;
  // residual: partials of the new residual rows [rows, n_cols / 32], or null
  float* sumsq_out;
  int n_cols;  // output columns (rope: total_heads * 128)
};

// A thread finishes 16-column pieces of one tile row of one 128-column group
// ("head"): step i (0..3) holds a at head column col_a(i) and b at col_b(i).
//   NeoX : a = x = [16i, 16i+16), b = y = [64+16i, +16), cache entries 16i + e;
//   GPT-J: a = [32i, 32i+16), b = [32i+16, 32i+32), pairs (2p, 2p+1) with cache
//          entries 16i + p;
//   residual: the same columns as GPT-J; step i is sum-of-squares group 4h + i.
template <int EPI>
__device__ __forceinline__ int col_a(int i) { return EPI == EPI_ROPE_NEOX ? 16 * i : 32 * i; }
template <int EPI>
__device__ __forceinline__ int col_b(int i) {
  return EPI == EPI_ROPE_NEOX ? 64 + 16 * i : 32 * i + 16;
}

template <typename C>
__device__ __forceinline__ void load_step_cs(const C* cs, int i, float* cv, float* sv) {
  load_cs<C, 16>(cs + 16 * i, cv);
  load_cs<C, 16>(cs + HEAD / 2 + 16 * i, sv);
}

template <int EPI>
__device__ __forceinline__ void rotate(float* a, float* b, const float* cv, const float* sv) {
  if (EPI == EPI_ROPE_NEOX) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float x = a[e], y = b[e];
      a[e] = x * cv[e] - y * sv[e];
      b[e] = y * cv[e] + x * sv[e];
    }
  } else {
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const float x0 = a[2 * p], y0 = a[2 * p + 1];
      a[2 * p] = x0 * cv[p] - y0 * sv[p];
      a[2 * p + 1] = y0 * cv[p] + x0 * sv[p];
      const float x1 = b[2 * p], y1 = b[2 * p + 1];
      b[2 * p] = x1 * cv[8 + p] - y1 * sv[8 + p];
      b[2 * p + 1] = y1 * cv[8 + p] + x1 * sv[8 + p];
    }
  }
}

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* v) {
  Traits<T>::unpack(ld_v4(p), v);
  Traits<T>::unpack(ld_v4(p + 8), v + 8);
}

__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// What one thread needs to finish its head of one tile row.
template <typename C>
struct RowState {
  const C* cs;  // rope: the token's cache row, or null (not rotated)
  float inv;    // NORM factor (1 without NORM)
  bool store;   // the row exists and the head is inside the output
};

// Row state of row m, 128-column group `head` (global index).  NORM: the
// partials are added in group order, so every thread of a row derives the
// same factor.
template <typename C, int EPI, bool NORM>
__device__ __forceinline__ RowState<C> row_state(const EpiParams& ep, int m, bool valid,
                                                 int head) {
  RowState<C> s;
  s.cs = nullptr;
  s.inv = 1.f;
  s.store = valid && (EPI == EPI_GATEUP_SILU ? true
                       : EPI == EPI_RESIDUAL  ? head * HEAD < ep.n_cols
                                              : head < ep.total_heads);
  if ((EPI == EPI_ROPE_NEOX || EPI == EPI_ROPE_GPTJ) && valid && head < ep.rot_heads) {
    const int64_t pos = ep.positions[m];
    if (pos >= 0 && pos < ep.max_position) {
      s.cs = static_cast<const C*>(ep.cache) + pos * HEAD;
      // the epilogue's four steps read the whole cache row (read-only data,
      // cached in L1): fetch it while the MMAs run
#pragma unroll
      for (int l = 0; l < HEAD * (int)sizeof(C); l += 128)
        prefetch_l1(reinterpret_cast<const char*>(s.cs) + l);
    }
  }
  if (NORM && valid) {
    const float* p = ep.sumsq_in + (int64_t)m * ep.sumsq_in_groups;
    float ss = 0.f;
    int g = 0;
    for (; g + 4 <= ep.sumsq_in_groups; g += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p + g));
      ss += v.x;
      ss += v.y;
      ss += v.z;
      ss += v.w;
    }
    for (; g < ep.sumsq_in_groups; ++g) ss += __ldg(p + g);
    s.inv = rsqrtf(ss * ep.inv_k + ep.eps);
  }
  return s;
}

// Step i of a row: a (at col_a) and b (at col_b) hold the fp32 accumulator;
// o is the row's output at the head's first column.  Returns the step's sum
// of squares (residual), else 0.
// The memory inputs of step i besides the accumulator: rope, the cache's 16
// cos and 16 sin values (x, y) when the head is rotated; residual, the 16 + 16
// residual values at col_a / col_b.  Issued early by callers that can overlap
// them with other loads.
template <typename T, typename C, int EPI>
__device__ __forceinline__ void load_step_inputs(const RowState<C>& s, int i, const T* o,
                                                 float* x, float* y) {
  if (EPI == EPI_RESIDUAL) {
    if (s.store) {
      load16(o + col_a<EPI>(i), x);
      load16(o + col_b<EPI>(i), y);
    }
  } else if (s.cs) {
    load_step_cs(s.cs, i, x, y);
  }
}

template <typename T, typename C, int EPI, bool NORM>
__device__ __forceinline__ float apply_step_with(const RowState<C>& s, int i, float* a, float* b,
                                                 T* o, const float* x, const float* y) {
  if (NORM) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      a[e] *= s.inv;
      b[e] *= s.inv;
    }
  }
  float ss = 0.f;
  if (EPI == EPI_RESIDUAL) {
    if (s.store) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        a[e] = Traits<T>::round(a[e] + x[e]);
        b[e] = Traits<T>::round(b[e] + y[e]);
        ss += a[e] * a[e] + b[e] * b[e];
      }
    }
  } else if (s.cs) {
    rotate<EPI>(a, b, x, y);
  }
  if (s.store) {
    store16(o + col_a<EPI>(i), a);
    store16(o + col_b<EPI>(i), b);
  }
  return ss;
}

template <typename T, typename C, int EPI, bool NORM>
__device__ __forceinline__ float apply_step(const RowState<C>& s, int i, float* a, float* b,
                                            T* o) {
  float x[16], y[16];
  load_step_inputs<T, C, EPI>(s, i, o, x, y);
  return apply_step_with<T, C, EPI, NORM>(s, i, a, b, o, x, y);
}

// A whole tile from TMEM: this thread's row, one head (128 columns at TMEM
// address `taddr`).  All lanes of the warp call it (TMEM loads are
// warp-wide).  ss_out: the row's sum-of-squares partials (residual), or null.
template <typename T, typename C, int EPI, bool NORM>
__device__ __forceinline__ void finish_head_tmem(uint32_t taddr, T* o, const RowState<C>& s,
                                                 float* ss_out, int head) {
  if (EPI == EPI_RESIDUAL && s.store) {
    // the head's residual values: 128 columns, fetched while TMEM is read
#pragma unroll
    for (int l = 0; l < HEAD * (int)sizeof(T); l += 128)
      prefetch_l1(reinterpret_cast<const char*>(o) + l);
  }
  // step i + 1's TMEM loads are issued before step i is processed
  uint32_t ra[16], rb[16];
  tc::tmem_ld16(taddr + col_a<EPI>(0), ra);
  tc::tmem_ld16(taddr + col_b<EPI>(0), rb);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    tc::tmem_wait_ld(ra);
    tc::tmem_wait_ld(rb);
    float a[16], b[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      a[e] = __uint_as_float(ra[e]);
      b[e] = __uint_as_float(rb[e]);
    }
    if (i < 3) {
      tc::tmem_ld16(taddr + col_a<EPI>(i + 1), ra);
      tc::tmem_ld16(taddr + col_b<EPI>(i + 1), rb);
    }
    const float ss = apply_step<T, C, EPI, NORM>(s, i, a, b, o);
    if (EPI == EPI_RESIDUAL && ss_out && s.store) ss_out[head * 4 + i] = ss;
  }
}

// This thread's row and head of a shared tile, as a partial sum: TMEM ->
// workspace slot (chunk = head * 8 + j for the head's 16-column chunk j).
__device__ __forceinline__ void store_partial(uint32_t taddr, float* slot, int head_in_tile,
                                              int row, bool valid) {
#pragma unroll 1
  for (int j = 0; j < HEAD / 16; j += 2) {
    uint32_t ra[16], rb[16];
    tc::tmem_ld16(taddr + 16 * j, ra);
    tc::tmem_ld16(taddr + 16 * j + 16, rb);
    tc::tmem_wait_ld(ra);
    tc::tmem_wait_ld(rb);
    if (valid) {
      const int ca = head_in_tile * 8 + j, cb = ca + 1;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        st_cg_f4(slot_q(slot, ca, q, row), __uint_as_float(ra[4 * q]),
                 __uint_as_float(ra[4 * q + 1]), __uint_as_float(ra[4 * q + 2]),
                 __uint_as_float(ra[4 * q + 3]));
        st_cg_f4(slot_q(slot, cb, q, row), __uint_as_float(rb[4 * q]),
                 __uint_as_float(rb[4 * q + 1]), __uint_as_float(rb[4 * q + 2]),
                 __uint_as_float(rb[4 * q + 3]));
      }
    }
  }
}

// SiLU-and-mul of gate value g and up value u (NORM: both scaled by the row's
// factor first).
template <bool NORM>
__device__ __forceinline__ float silu_mul(float g, float u, float inv) {
  if (NORM) {
    g *= inv;
    u *= inv;
  }
  return g / (1.f + __expf(-g)) * u;
}
// The same for 16 gate values a and 16 up values b, into a.
template <bool NORM>
__device__ __forceinline__ void silu_mul16(float* a, const float* b, float inv) {
#pragma unroll
  for (int e = 0; e < 16; ++e) a[e] = silu_mul<NORM>(a[e], b[e], inv);
}

// A whole gate/up tile from TMEM: this thread's row, output columns
// [64 half, 64 half + 64) = gate accumulator columns of the same offsets and
// up columns 128 + those.  `taddr` addresses the row's accumulator start;
// o is the row's output at the tile's first column.
template <typename T, typename C, bool NORM>
__device__ __forceinline__ void finish_gateup_tmem(uint32_t taddr, int half, T* o,
                                                   const RowState<C>& s) {
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const int c = half * 64 + 16 * i;
    uint32_t rg[16], ru[16];
    tc::tmem_ld16(taddr + c, rg);
    tc::tmem_ld16(taddr + HEAD + c, ru);
    tc::tmem_wait_ld(rg);
    tc::tmem_wait_ld(ru);
    float a[16], b[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      a[e] = __uint_as_float(rg[e]);
      b[e] = __uint_as_float(ru[e]);
    }
    silu_mul16<NORM>(a, b, s.inv);
    if (s.store) store16(o + c, a);
  }
}

// Grid-wide barrier, called by thread 0 of every CTA once its epilogue
// threads' partial stores are issued (and ordered before the call by the
// epilogue barrier).  bar[0] counts arrivals and is reset to zero by the last
// one, which then advances the generation bar[kGenOffset] (its own 128-byte
// line, so the waiters' polls do not contend with the arrivals) that the
// others wait on (bounded).  The whole grid is co-resident (at most one CTA
// per SM, grid <= SMs or resident CTA pairs), so every CTA arrives.
// Arrival on a counter: a gpu-scope acquire-release add, so the caller's
// earlier writes (and those of the threads ordered before it by a CTA
// barrier) are released with the arrival, and an arriver that sees the
// final count has acquired every earlier arriver's writes.
__device__ __forceinline__ int arrive_acq_rel(int* counter) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;"
               : "=r"(old)
               : "l"(counter)
               : "memory");
  return old;
}

constexpr int kGenOffset = 32;
// Per-tile arrival counters (decode sizes) start after the barrier's 256 bytes.
constexpr int kTileCounterOffset = 64;
__device__ __forceinline__ bool grid_barrier(int* bar, int ctas, const Ctl* ctl) {
  int* gen = bar + kGenOffset;
  int gen0;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(gen0) : "l"(gen) : "memory");
  if (arrive_acq_rel(bar) == ctas - 1) {
    *reinterpret_cast<volatile int*>(bar) = 0;  // re-armed for the next call
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(gen), "r"(gen0 + 1) : "memory");
    return true;
  }
  const uint64_t t0 = tc::globaltimer_ns();
  for (;;) {
    int g;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(g) : "l"(gen) : "memory");
    if (g != gen0) break;
    if (*reinterpret_cast<const volatile int*>(&ctl->abort)) return false;
    if (tc::globaltimer_ns() - t0 > kWaitLimitNs) return false;
    __nanosleep(20);
  }
  return true;
}

// Partial slot of contributor c to shared tile t: a segment that starts at
// the tile's first K block is its CTA's last (slot 2c + 1); any other is its
// CTA's first (slot 2c).
__device__ __forceinline__ const float* slot_of(const float* slots, int c, bool tile_start) {
  return slots + (int64_t)(2 * c + (tile_start ? 1 : 0)) * SLOT_FLOATS;
}

// v_a, v_b += the partials of workers w0..w1 at chunks ca, cb of tile row r,
// in worker order; worker w's CTA is w * mul + add (PAIR: the CTA of the pair
// holding these rows).  The loads of two workers are issued together.
__device__ __forceinline__ void sum_partials(float* va, float* vb, const float* slots, int w0,
                                             int w1, int mul, int add, int ca, int cb, int r) {
  constexpr int NB = 2;
#pragma unroll 1
  for (int w = w0; w <= w1; w += NB) {
    float4 x[NB][8];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      if (w + k > w1) break;
      float* sl = const_cast<float*>(slot_of(slots, (w + k) * mul + add, w + k == w0));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        x[k][q] = ld_cg_f4(slot_q(sl, ca, q, r));
        x[k][4 + q] = ld_cg_f4(slot_q(sl, cb, q, r));
      }
    }
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      if (w + k > w1) break;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        va[4 * q] += x[k][q].x;
        va[4 * q + 1] += x[k][q].y;
        va[4 * q + 2] += x[k][q].z;
        va[4 * q + 3] += x[k][q].w;
        vb[4 * q] += x[k][4 + q].x;
        vb[4 * q + 1] += x[k][4 + q].y;
        vb[4 * q + 2] += x[k][4 + q].z;
        vb[4 * q + 3] += x[k][4 + q].w;
      }
    }
  }
}

// One piece of a shared stream-K tile: column pair p, 32-row group g of the
// tile's 128-row half h, summed over the contributing workers w0..w1 and
// finished.  A lane takes one row, so each load of a warp reads 512
// contiguous bytes of a slot.  Column pair p: rope and residual, step p % 4
// of head p / 4 (the two 16-column pieces a step combines); gate/up, output
// columns [16p, 16p + 16) from gate chunk p and up chunk 8 + p.
template <typename T, typename C, int EPI, bool NORM, bool PAIR>
__device__ __forceinline__ void finish_piece(const float* slots, int w0, int w1, int m0, int nt,
                                             int p, int g, int h, T* out, int64_t out_stride,
                                             const EpiParams& ep, int num_tokens, int lane,
                                             bool decode) {
  constexpr int HALVES = PAIR ? 2 : 1;
  // Decode sizes (g == 0, at most 32 rows): the warp's lanes split into
  // groups of R >= rows lanes; group k sums workers w0 + k, w0 + k + groups,
  // ... for its rows, and the groups are added in a fixed tree, so a few
  // rows with many contributors cost one round of loads, not one per
  // contributor.  Otherwise a lane takes one row and every worker.
  int rows_here = 32, R = 32;
  if (decode) {
    rows_here = min(32, num_tokens - m0);
    R = 1;
    while (R < rows_here) R <<= 1;
  }
  const int grp = lane / R, groups = 32 / R;
  const int r = 32 * g + lane % R, m = m0 + r;
  const bool row_ok = m < num_tokens && lane % R < rows_here;
  if (!decode && !row_ok) return;
  int ca, cb, head, i;
  if (EPI == EPI_GATEUP_SILU) {
    ca = p, cb = 8 + p, head = 0, i = 0;
  } else {
    const int hh = p >> 2;
    i = p & 3;
    ca = hh * 8 + col_a<EPI>(i) / 16;
    cb = hh * 8 + col_b<EPI>(i) / 16;
    head = nt * (BN / HEAD) + hh;
  }
  // The row's own inputs (position, norm partials, then the cache row or
  // residual values) are requested before and between the partial loads,
  // so their latencies overlap; a head past the output (odd head counts)
  // only skips the store.
  const RowState<C> s = row_state<C, EPI, NORM>(ep, row_ok ? m : m0, row_ok, head);
  T* o = out + (int64_t)m * out_stride + (int64_t)head * HEAD;
  float x[16], y[16];
  if constexpr (EPI != EPI_GATEUP_SILU) {
    if (grp == 0) load_step_inputs<T, C, EPI>(s, i, o, x, y);
  }
  float a[16], b[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) a[e] = b[e] = 0.f;
  if (!decode) {
    sum_partials(a, b, slots, w0, w1, HALVES, h, ca, cb, r);
  } else {
    if (row_ok) {
#pragma unroll 1
      for (int w = w0 + grp; w <= w1; w += groups) {
        float* sl = const_cast<float*>(slot_of(slots, w * HALVES + h, w == w0));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 fa = ld_cg_f4(slot_q(sl, ca, q, r));
          const float4 fb = ld_cg_f4(slot_q(sl, cb, q, r));
          a[4 * q] += fa.x;
          a[4 * q + 1] += fa.y;
          a[4 * q + 2] += fa.z;
          a[4 * q + 3] += fa.w;
          b[4 * q] += fb.x;
          b[4 * q + 1] += fb.y;
          b[4 * q + 2] += fb.z;
          b[4 * q + 3] += fb.w;
        }
      }
    }
    for (int off = 16; off >= R; off >>= 1) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        a[e] += __shfl_down_sync(0xffffffffu, a[e], off);
        b[e] += __shfl_down_sync(0xffffffffu, b[e], off);
      }
    }
    if (grp != 0 || !row_ok) return;
  }
  if (!s.store) return;
  if constexpr (EPI == EPI_GATEUP_SILU) {
    silu_mul16<NORM>(a, b, s.inv);
    store16(out + (int64_t)m * out_stride + (int64_t)nt * HEAD + 16 * p, a);
  } else {
    const float ss = apply_step_with<T, C, EPI, NORM>(s, i, a, b, o, x, y);
    if (EPI == EPI_RESIDUAL && ep.sumsq_out)
      ep.sumsq_out[(int64_t)m * (ep.n_cols / SUMSQ_GROUP) + head * 4 + i] = ss;
  }
}

// One persistent CTA per SM (grid = min(SMs, units)); see the file comment.
// PAIR: clusters of two CTAs (launched with cluster dimension 2) share each
// 256 x 256 tile through cta_group::2 MMAs; the pair is the unit of the
// data-parallel and stream-K schedule ("worker"), each CTA keeps its 128 rows.
// m_tiles counts tiles of 128 (one CTA) or 256 rows (PAIR).
// slots: 2 partial tiles of BM x BN floats per CTA; counters: the grid
// barrier (arrival count, zero before the call and left zero by it;
// generation).
template <typename T, typename C, int EPI, bool NORM, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_epi_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    T* __restrict__ out, int64_t out_stride, int num_tokens, int m_tiles,
                    int k_blocks, const EpiParams ep, int* __restrict__ counters,
                    float* __restrict__ slots, int32_t* fault) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Ctl* ctl = reinterpret_cast<Ctl*>(tiles + RING_BYTES);
  constexpr int NST = Ring<PAIR>::kStages, SB = Ring<PAIR>::kStage;
  constexpr int PM = PAIR ? 2 * BM : BM;  // rows per tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const uint32_t rank = PAIR ? tc::cluster_rank() : 0u;  // rows rank * 128 of the tile
  const int worker = PAIR ? cta >> 1 : cta;
  const int workers = PAIR ? (int)gridDim.x >> 1 : (int)gridDim.x;
  // output columns per tile: 128 for gate/up (each tile holds gate and up), else 256
  const int n_tiles = EPI == EPI_GATEUP_SILU ? ep.n_cols / HEAD : (ep.n_cols + BN - 1) / BN;
  const int64_t n_all = (int64_t)m_tiles * n_tiles;
  const int64_t t_stop = n_all / workers * workers;  // first stream-K tile
  Split sp;  // stream-K split of the units of tiles [t_stop, n_all)
  sp.units = (n_all - t_stop) * k_blocks;
  // at most one worker per unit, so every stream-K range is non-empty and a
  // tile's contributors are consecutive workers
  sp.ctas = (int)min((int64_t)workers, sp.units);
  sp.k_blocks = k_blocks;
  const bool streams = worker < sp.ctas;
  const int64_t u_begin = streams ? sp.start(worker) : 0;
  const int64_t u_end = streams ? sp.start(worker + 1) : 0;
  const Walk walk0{worker, t_stop, (int64_t)workers, u_begin, u_end, k_blocks};
  // at most 32 rows (single CTAs): shared tiles are finished by their last
  // contributor instead of after a grid barrier
  const bool decode = !PAIR && num_tokens <= 32;
  int* tile_counters = counters + kTileCounterOffset;

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(&ctl->full[s], 1);
      tc::mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&ctl->tmem_full[b], 1);
      // PAIR: the epilogue warps of both CTAs free the leader's accumulator
      tc::mbar_init(&ctl->tmem_empty[b], PAIR ? 2 * EPI_WARPS : EPI_WARPS);
    }
    tc::mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    ctl->nfin = 0;
    tc::fence_barrier_init();
  }
  if (warp == EPI_WARPS && lane == 0) {
    tc::tma_prefetch_desc(&tm_a);
    tc::tma_prefetch_desc(&tm_b);
  }
  if (warp == 0) {
    if constexpr (PAIR)
      tc::tmem_alloc_pair(&ctl->tmem, TMEM_COLS);
    else
      tc::tmem_alloc(&ctl->tmem, TMEM_COLS);
  }
  tc::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) tc::cluster_sync();  // both CTAs' barriers initialised
  tc::tc_fence_after();
  const uint32_t tmem = ctl->tmem;
  // hidden states, positions and the workspace may be in use by the previous
  // kernel of the stream
  pdl_wait();

  if (warp == EPI_WARPS) {
    // ---- TMA producer: every K block of every segment, in order ---------
    if (lane == 0) {
      int64_t i = 0;
      bool ok = true;
      Walk walk = walk0;
      int64_t t;
      int kb0, kb1;
      // PAIR: both CTAs' copies complete on the leader's barrier, which
      // expects the bytes of both
      const uint32_t full0 = PAIR ? tc::map_to_rank(&ctl->full[0], 0) : 0u;
      while (ok && walk.next(t, kb0, kb1)) {
        const int m0 = (int)(t / n_tiles) * PM + (int)rank * BM;
        const int nt = (int)(t % n_tiles);
        // B rows of this CTA: gate/up, gate rows [128 nt, +128) and up rows
        // [n_cols + 128 nt, +128) (PAIR: rank 0 the gate, rank 1 the up rows);
        // otherwise rows [256 nt, +256) (PAIR: rank r the 128 rows 128 r on)
        const int n0 = EPI == EPI_GATEUP_SILU ? (int)rank * ep.n_cols + nt * HEAD
                                              : nt * BN + (int)rank * (BN / 2);
        for (int kb = kb0; kb < kb1; ++kb, ++i) {
          const int s = (int)(i % NST);
          const uint32_t use = (uint32_t)(i / NST);
          if (use > 0 &&
              !tc::mbar_wait(&ctl->empty[s], (use - 1) & 1u, kWaitLimitNs, &ctl->abort)) {
            ok = false;
            break;
          }
          uint8_t* a = tiles + s * SB;
          if constexpr (PAIR) {
            const uint32_t bar = full0 + (uint32_t)(s * sizeof(uint64_t));
            if (rank == 0) tc::mbar_arrive_expect_tx(&ctl->full[s], 2 * SB);
            tc::tma_load_2d_pair(a, &tm_a, kb * BK, m0, bar);
            tc::tma_load_2d_pair(a + A_BYTES, &tm_b, kb * BK, n0, bar);
          } else {
            tc::mbar_arrive_expect_tx(&ctl->full[s], SB);
            tc::tma_load_2d(a, &tm_a, kb * BK, m0, &ctl->full[s]);
            tc::tma_load_2d(a + A_BYTES, &tm_b, kb * BK, n0, &ctl->full[s]);
            if (EPI == EPI_GATEUP_SILU)
              tc::tma_load_2d(a + A_BYTES + HEAD * BK * 2, &tm_b, kb * BK, ep.n_cols + n0,
                              &ctl->full[s]);
          }
        }
      }
      if (!ok) raise_fault(ctl, fault);
      // every copy issued has landed before the CTA's shared memory is released
      // (immediate when the MMAs consumed them all).  PAIR: the leader's
      // barriers count both CTAs' copies; the partner leaves only after the
      // leader, at the closing cluster barrier.
      if (!PAIR || rank == 0)
        for (int64_t q = i > NST ? i - NST : 0; q < i; ++q)
          tc::mbar_wait(&ctl->full[q % NST], (uint32_t)(q / NST) & 1u, kWaitLimitNs, nullptr);
    }
  } else if (warp == EPI_WARPS + 1) {
    // ---- MMA issuer ----------------------------------------------------
    if (lane == 0 && rank == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idesc = tc::umma_idesc_f16(kBf16, PM, BN);
      int64_t i = 0;
      int j = 0;
      bool ok = true;
      Walk walk = walk0;
      int64_t t;
      int kb0, kb1;
      for (; ok && walk.next(t, kb0, kb1); ++j) {
        const int b = j & 1;
        const uint32_t use_b = (uint32_t)(j >> 1);
        if (use_b > 0 &&
            !tc::mbar_wait(&ctl->tmem_empty[b], (use_b - 1) & 1u, kWaitLimitNs, &ctl->abort)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        for (int kb = kb0; kb < kb1; ++kb, ++i) {
          const int s = (int)(i % NST);
          if (!tc::mbar_wait(&ctl->full[s], (uint32_t)(i / NST) & 1u, kWaitLimitNs,
                             &ctl->abort)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_addr = tc::smem_u32(tiles + s * SB);
          const uint64_t ad = tc::umma_desc_sw128(a_addr);
          const uint64_t bd = tc::umma_desc_sw128(a_addr + A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            if constexpr (PAIR)
              tc::umma_f16_pair(d, ad + 2 * k, bd + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            else
              tc::umma_f16(d, ad + 2 * k, bd + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          // the stage is free in both CTAs (PAIR) once these MMAs complete
          if constexpr (PAIR)
            tc::umma_commit_pair_both(&ctl->empty[s]);
          else
            tc::umma_commit(&ctl->empty[s]);
        }
        if (ok) {
          if constexpr (PAIR)
            tc::umma_commit_pair_both(&ctl->tmem_full[b]);
          else
            tc::umma_commit(&ctl->tmem_full[b]);
        }
      }
      if (!ok) raise_fault(ctl, fault);
      // every MMA issued has completed before TMEM is freed
      if constexpr (PAIR)
        tc::umma_commit_pair(&ctl->drain);
      else
        tc::umma_commit(&ctl->drain);
      tc::mbar_wait(&ctl->drain, 0, kWaitLimitNs, nullptr);
    }
  } else {
    // ---- epilogue: warp w drains TMEM lanes 32 (w % 4) .. +31, head w / 4 ----
    const int quarter = warp % 4, hh = warp / 4;
    const int row = quarter * 32 + lane;
    // the accumulator buffers are freed on the pair leader's barriers
    const uint32_t tmem_empty0 = PAIR ? tc::map_to_rank(&ctl->tmem_empty[0], 0) : 0u;
    int j = 0;
    Walk walk = walk0;
    int64_t t;
    int kb0, kb1;
    for (; walk.next(t, kb0, kb1); ++j) {
      const int b = j & 1;
      const int mt = (int)(t / n_tiles), nt = (int)(t % n_tiles);
      const int m0 = mt * PM + (int)rank * BM, m = m0 + row;
      const bool valid = m < num_tokens;
      const int head = nt * (BN / HEAD) + hh;
      const bool whole = kb0 == 0 && kb1 == k_blocks;
      // the row's position / cache row / norm factor are read while the MMAs run
      RowState<C> rs;
      if (whole) rs = row_state<C, EPI, NORM>(ep, m, valid, head);
      bool ready = tc::mbar_wait(&ctl->tmem_full[b], (uint32_t)(j >> 1) & 1u, kWaitLimitNs,
                                 &ctl->abort);
      ready = epi_all(ready);
      if (!ready) {
        raise_fault(ctl, fault);
        break;
      }
      tc::tc_fence_after();
      const uint32_t taddr = tmem + (uint32_t)(b * BN + hh * HEAD) +
                             (static_cast<uint32_t>(quarter * 32) << 16);
      if (!whole) {
        // a shared stream-K tile: publish this CTA's partial (finished in the
        // second phase, or by the tile's last contributor for decode sizes)
        store_partial(taddr, const_cast<float*>(slot_of(slots, cta, kb0 == 0)), hh, row, valid);
      } else if constexpr (EPI == EPI_GATEUP_SILU) {
        T* o = out + (int64_t)(valid ? m : 0) * out_stride + (int64_t)nt * HEAD;
        finish_gateup_tmem<T, C, NORM>(taddr - (uint32_t)(hh * HEAD), hh, o, rs);
      } else {
        T* o = out + (int64_t)(valid ? m : 0) * out_stride + (int64_t)head * HEAD;
        finish_head_tmem<T, C, EPI, NORM>(
            taddr, o, rs,
            EPI == EPI_RESIDUAL && ep.sumsq_out
                ? ep.sumsq_out + (int64_t)(valid ? m : 0) * (ep.n_cols / SUMSQ_GROUP)
                : nullptr,
            head);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          tc::mbar_arrive_cluster(tmem_empty0 + (uint32_t)(b * sizeof(uint64_t)));
        else
          tc::mbar_arrive(&ctl->tmem_empty[b]);
      }
      if (!PAIR && !whole && decode) {
        // Decode sizes: the tile's last contributor finishes it, after its
        // walk (below), so no CTA waits.  All epilogue threads' partial
        // stores are ordered before thread 0's arrival by the barrier.
        const int64_t tile_u0 = (t - t_stop) * k_blocks;
        const int c0 = sp.owner(tile_u0), c1 = sp.owner(tile_u0 + k_blocks - 1);
        epi_sync();
        if (threadIdx.x == 0 && arrive_acq_rel(&tile_counters[t]) == c1 - c0) {
          tile_counters[t] = 0;  // re-armed for the next call
          if (ctl->nfin < 4) ctl->fin[ctl->nfin++] = (int)t;
        }
      }
    }
    if (sp.units > 0) {
      // Second phase (same for every CTA: it depends on the shape only).
      // Decode sizes: the shared tiles this CTA contributed to last, its 8
      // warps one column pair each (rows 0-31).  Otherwise every CTA meets
      // at the grid barrier (arriving even after a fault, so the others do
      // not wait it out) and takes a share of all shared tiles' pieces.
      epi_sync();
      bool go = true;
      if (PAIR || !decode) {
        if (threadIdx.x == 0) ctl->ready = grid_barrier(counters, gridDim.x, ctl);
        epi_sync();
        go = *reinterpret_cast<volatile int*>(&ctl->ready) != 0;
        if (!go) raise_fault(ctl, fault);
      }
      constexpr int HALVES = PAIR ? 2 : 1;  // 128-row halves of a tile
      const bool spread = PAIR || !decode;
      const int64_t items = spread ? (n_all - t_stop) * 32 * HALVES
                                   : *reinterpret_cast<volatile int*>(&ctl->nfin);
      const int64_t first = spread ? (int64_t)blockIdx.x * EPI_WARPS + warp : 0;
      const int64_t step = spread ? (int64_t)gridDim.x * EPI_WARPS : 1;
#pragma unroll 1
      for (int64_t it = first; go && it < items; it += step) {
        const int64_t tp = spread ? t_stop + it / (32 * HALVES)
                                  : *reinterpret_cast<volatile int*>(&ctl->fin[it]);
        const int h = PAIR ? (int)(it / 32) & 1 : 0;
        const int p = spread ? (int)(it % 32) >> 2 : warp, g = spread ? (int)(it & 3) : 0;
        const int64_t tile_u0 = (tp - t_stop) * k_blocks;
        const int c0 = sp.owner(tile_u0), c1 = sp.owner(tile_u0 + k_blocks - 1);
        const int m0p = (int)(tp / n_tiles) * PM + h * BM;
        if (c0 == c1 || m0p + 32 * g >= num_tokens) continue;  // whole, or no rows here
        finish_piece<T, C, EPI, NORM, PAIR>(slots, c0, c1, m0p, (int)(tp % n_tiles), p, g, h,
                                            out, out_stride, ep, num_tokens, lane, !spread);
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) {
    // neither CTA leaves (nor frees TMEM) while its partner may still signal
    // its barriers or read its shared memory
    tc::cluster_sync();
    if (warp == 0) tc::tmem_dealloc_pair(tmem, TMEM_COLS);
  } else {
    if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------ decode batches on CUDA cores --
// With at most kGemvTokens rows a projection is a stream of its weight (50 MB
// for Llama-3-8B's qkv, 235 MB for gate/up) past a few hidden rows:
// HBM-bound, with a 128-row MMA tile almost all padding and the split-K
// reduction that the tile schedule needs at this size costing more than the
// stream itself.  The work unit is a pair of weight rows: a rotation pair of
// output columns (NeoX: head columns i and i + 64; GPT-J: 2i and 2i + 1), or
// the gate and up rows of one output column (SiLU-and-mul), or two adjacent
// output columns (residual add, for o_proj and down_proj).  A CTA owns up to
// kGemvPairs units over the whole K, so no sum crosses CTAs; the units are
// spread evenly over three CTAs per SM (more CTAs, in waves, when there are
// more than 8 units per CTA).  One producer
// thread streams the pairs' weight rows through a ring of kGemvStages
// shared-memory stages with bulk copies (kGemvChunk elements of every row per
// stage, 64 KB in flight per CTA: register loads could not keep enough bytes
// in flight to cover the DRAM latency).  Consumer warp j copies pair j's two
// row chunks to registers, releases the stage, and dots them with the hidden
// rows (read through L1, which the CTA's warps share); after the last chunk it
// reduces across the warp, and lane t finishes token t as the tensor-core
// epilogue does: norm factor, then the rotation, SiLU-and-mul or residual
// add in fp32, one rounding.  Every wait is bounded; on expiry the CTA sets bit 30 of the
// fault word, stops, and the producer waits (bounded) for its copies before
// leaving.
constexpr int kGemvTokens = 2, kGemvPairs = 8, kGemvChunk = 512, kGemvStages = 4;
constexpr int kGemvStageElems = 2 * kGemvPairs * kGemvChunk;  // 16-bit weights
constexpr int kGemvThreads = (kGemvPairs + 1) * 32;
constexpr int kGemvVec = kGemvChunk / 256;  // 16-byte vectors per lane, row and chunk
struct GemvCtl {
  uint64_t full[kGemvStages], empty[kGemvStages];
  int abort;
};
constexpr int kGemvSmem = kGemvStages * kGemvStageElems * 2 + (int)sizeof(GemvCtl);

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Plain (non-multicast) bulk copy global -> this CTA's shared memory,
// completing `bytes` of transaction count on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          tc::smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
      : "memory");
}

// The two weight rows of work unit `unit`: a rotation pair of output columns
// (rope; head and i locate the pair's cache entry), gate row `unit` and up
// row n_cols + unit of output column `unit` (SiLU-and-mul), or output columns
// 2 unit and 2 unit + 1 (residual).
template <int EPI>
__device__ __forceinline__ void pair_columns(int unit, int n_cols, int& head, int& i, int& c1,
                                             int& c2) {
  if (EPI == EPI_GATEUP_SILU || EPI == EPI_RESIDUAL) {
    head = i = 0;
    c1 = EPI == EPI_RESIDUAL ? 2 * unit : unit;
    c2 = EPI == EPI_RESIDUAL ? c1 + 1 : n_cols + unit;
    return;
  }
  head = unit / (HEAD / 2);
  i = unit % (HEAD / 2);
  c1 = head * HEAD + (EPI == EPI_ROPE_NEOX ? i : 2 * i);
  c2 = c1 + (EPI == EPI_ROPE_NEOX ? HEAD / 2 : 1);
}
template <int EPI>
__host__ __device__ __forceinline__ int gemv_units(int n_cols) {
  return EPI == EPI_GATEUP_SILU ? n_cols : n_cols / 2;
}

// NT: tokens the loops are unrolled for (num_tokens <= NT).  Measured on
// B200 (Llama-3-8B qkv, 50 MB of weight): 9.8 us at one token, 12.9 at two,
// against 11.9 for cuBLAS's GEMM alone; from three tokens on the tensor-core
// kernel is faster, so kGemvTokens is 2.
template <typename T, typename C, int EPI, bool NORM, int NT>
__global__ void __launch_bounds__(kGemvThreads, 3)
    gemv_epi_kernel(const T* __restrict__ hidden, int64_t hidden_stride,
                     const T* __restrict__ weight, int64_t k, T* __restrict__ out,
                     int64_t out_stride, int num_tokens, const EpiParams ep, int32_t* fault) {
  extern __shared__ __align__(16) uint8_t gemv_smem[];
  T* ring = reinterpret_cast<T*>(gemv_smem);
  GemvCtl* ctl = reinterpret_cast<GemvCtl*>(gemv_smem + kGemvStages * kGemvStageElems * 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = gemv_units<EPI>(ep.n_cols);
  const int unit0 = (int)((int64_t)blockIdx.x * units / gridDim.x);
  const int pairs = (int)((int64_t)(blockIdx.x + 1) * units / gridDim.x) - unit0;
  const int chunks = (int)ceil_div(k, kGemvChunk);
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemvStages; ++s) {
      tc::mbar_init(&ctl->full[s], 1);
      tc::mbar_init(&ctl->empty[s], kGemvPairs);
    }
    ctl->abort = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();

  if (warp == kGemvPairs) {
    // ---- producer: every chunk of both rows of the CTA's units -----------
    if (lane != 0) return;
    pdl_wait();
    int c = 0;
    bool ok = true;
    for (; c < chunks; ++c) {
      const int s = c % kGemvStages;
      if (c >= kGemvStages && !tc::mbar_wait(&ctl->empty[s], (uint32_t)(c / kGemvStages - 1) & 1u,
                                             kWaitLimitNs, &ctl->abort)) {
        ok = false;
        break;
      }
      const int64_t k0 = (int64_t)c * kGemvChunk;
      const uint32_t bytes = (uint32_t)(min((int64_t)kGemvChunk, k - k0) * (int64_t)sizeof(T));
      tc::mbar_arrive_expect_tx(&ctl->full[s], bytes * 2u * (uint32_t)pairs);
      T* st = ring + (size_t)s * kGemvStageElems;
      for (int j = 0; j < pairs; ++j) {
        int head, i, c1, c2;
        pair_columns<EPI>(unit0 + j, ep.n_cols, head, i, c1, c2);
        bulk_g2s(st + (2 * j) * kGemvChunk, weight + (int64_t)c1 * k + k0, bytes, &ctl->full[s]);
        bulk_g2s(st + (2 * j + 1) * kGemvChunk, weight + (int64_t)c2 * k + k0, bytes,
                 &ctl->full[s]);
      }
    }
    if (!ok) {
      *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
      if (fault) atomicOr(fault, kFaultTimeout);
    }
    // every copy issued has landed before the CTA's shared memory is released
    for (int q = c > kGemvStages ? c - kGemvStages : 0; q < c; ++q)
      tc::mbar_wait(&ctl->full[q % kGemvStages], (uint32_t)(q / kGemvStages) & 1u, kWaitLimitNs,
                    nullptr);
    return;
  }

  // ---- consumer warp `warp`: unit unit0 + warp ----------------------------
  const bool has = warp < pairs;
  int head = 0, i = 0, c1 = 0, c2 = 0;
  if (has) pair_columns<EPI>(unit0 + warp, ep.n_cols, head, i, c1, c2);
  float acc1[NT], acc2[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc1[t] = acc2[t] = 0.f;
  // the hidden rows (NORM: and their partials) may be written by the previous kernel
  pdl_wait();
  bool ok = true;
  for (int c = 0; c < chunks; ++c) {
    const int s = c % kGemvStages;
    const int64_t k0 = (int64_t)c * kGemvChunk;
    const int nvc = (int)(min((int64_t)kGemvChunk, k - k0) / 8);  // 16-byte vectors per row
    // this chunk's hidden vectors, issued before the wait on the ring
    uint4 xv[kGemvVec][NT];
#pragma unroll
    for (int q = 0; q < kGemvVec; ++q) {
      const int v = lane + 32 * q;
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (has && t < num_tokens && v < nvc)
          xv[q][t] = __ldg(reinterpret_cast<const uint4*>(hidden + t * hidden_stride + k0) + v);
    }
    if (!tc::mbar_wait(&ctl->full[s], (uint32_t)(c / kGemvStages) & 1u, kWaitLimitNs,
                       &ctl->abort)) {
      ok = false;
      break;
    }
    // the pair's row chunks to registers; the stage is free for the next copy
    uint4 wa[kGemvVec], wb[kGemvVec];
    const T* st = ring + (size_t)s * kGemvStageElems;
#pragma unroll
    for (int q = 0; q < kGemvVec; ++q) {
      const int v = lane + 32 * q;
      if (has && v < nvc) {
        wa[q] = *reinterpret_cast<const uint4*>(st + (2 * warp) * kGemvChunk + 8 * v);
        wb[q] = *reinterpret_cast<const uint4*>(st + (2 * warp + 1) * kGemvChunk + 8 * v);
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&ctl->empty[s]);
#pragma unroll
    for (int q = 0; q < kGemvVec; ++q) {
      const int v = lane + 32 * q;
      if (has && v < nvc) {
        float w1[8], w2[8];
        Traits<T>::unpack(wa[q], w1);
        Traits<T>::unpack(wb[q], w2);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < num_tokens) {
            float x[8];
            Traits<T>::unpack(xv[q][t], x);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              acc1[t] = fmaf(w1[e], x[e], acc1[t]);
              acc2[t] = fmaf(w2[e], x[e], acc2[t]);
            }
          }
        }
      }
    }
  }
  if (!ok) {
    *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
    if (fault && lane == 0) atomicOr(fault, kFaultTimeout);
    return;
  }
  if (!has) return;
  float f[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    acc1[t] = warp_sum(acc1[t]);
    acc2[t] = warp_sum(acc2[t]);
    f[t] = 1.f;
    if (NORM && t < num_tokens) {
      const float* p = ep.sumsq_in + (int64_t)t * ep.sumsq_in_groups;
      float ss = 0.f;
      for (int g = lane; g < ep.sumsq_in_groups; g += 32) ss += __ldg(p + g);
      f[t] = rsqrtf(warp_sum(ss) * ep.inv_k + ep.eps);
    }
  }
  if (lane >= num_tokens) return;
  float x1 = 0.f, x2 = 0.f, inv = 1.f;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    if (t == lane) {
      x1 = acc1[t];
      x2 = acc2[t];
      inv = f[t];
    }
  }
  T* o = out + (int64_t)lane * out_stride;
  if (EPI == EPI_GATEUP_SILU) {
    o[c1] = Traits<T>::from_f(silu_mul<NORM>(x1, x2, inv));
    return;
  }
  if (EPI == EPI_RESIDUAL) {  // the row's residual, updated in place
    o[c1] = Traits<T>::from_f(x1 + Traits<T>::to_f(o[c1]));
    o[c2] = Traits<T>::from_f(x2 + Traits<T>::to_f(o[c2]));
    return;
  }
  if (NORM) {
    x1 *= inv;
    x2 *= inv;
  }
  const int64_t pos = ep.positions[lane];
  if (head < ep.rot_heads && pos >= 0 && pos < ep.max_position) {
    const C* cs = static_cast<const C*>(ep.cache) + pos * HEAD;
    const float cv = Traits<C>::to_f(cs[i]), sv = Traits<C>::to_f(cs[HEAD / 2 + i]);
    const float y1 = x1 * cv - x2 * sv, y2 = x2 * cv + x1 * sv;
    x1 = y1;
    x2 = y2;
  }
  o[c1] = Traits<T>::from_f(x1);
  o[c2] = Traits<T>::from_f(x2);
}

// ---------------------------------------------------------------- host ----
// Workspace layout: 2 partial slots per SM (a fixed size for the device),
// then 256 bytes for the grid barrier, then one int32 counter per 128-row
// tile (decode sizes).  Both sit at offsets that do not depend on the shape
// and are left zero (the barrier's generation aside), so a workspace that a
// call of one shape left valid serves a call of any other shape that fits.
struct QkvShape {
  int m_tiles, n_tiles, k_blocks, ctas;
  bool pair;  // 256-row tiles on CTA pairs (m_tiles counts those)
  size_t slot_bytes, workspace_bytes;
};

// CTA pairs once the rows fill more than one 128-row tile: they halve the B
// bytes each SM stages per MMA.  One 128-row tile runs on single CTAs (a
// pair would spend half its MMAs on rows that do not exist).
QkvShape qkv_shape(int64_t num_tokens, int64_t hidden_size, int total_heads, int sms) {
  QkvShape s;
  s.pair = num_tokens > BM;
  s.m_tiles = (int)ceil_div(num_tokens, s.pair ? 2 * BM : BM);
  s.n_tiles = (int)ceil_div((int64_t)total_heads * HEAD, BN);
  s.k_blocks = (int)ceil_div(hidden_size, BK);
  const int64_t units = (int64_t)s.m_tiles * s.n_tiles * s.k_blocks;
  const int64_t workers = s.pair ? sms / 2 : sms;
  s.ctas = (int)((units < workers ? units : workers) * (s.pair ? 2 : 1));
  s.slot_bytes = (size_t)2 * sms * SLOT_FLOATS * sizeof(float);
  s.workspace_bytes =
      s.slot_bytes + kTileCounterOffset * sizeof(int) +
      ((size_t)ceil_div(num_tokens, BM) * s.n_tiles * sizeof(int) + 255) / 256 * 256;
  return s;
}

// Clusters of two of this kernel that the device holds at once, per device
// (the same for every instantiation: one CTA per SM by shared memory).
template <typename K>
int pairs_resident(K kernel, int dev) {
  static std::mutex mu;
  static int cached[64] = {};
  if (dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) return 0;
    cached[dev] = n;
  }
  return cached[dev];
}

// Workers (CTAs, or CTA pairs) to run n_all tiles of k_blocks K blocks on,
// given `workers` available.  Stream-K spreads the tiles left after the last
// full round over every worker, at the price of writing and re-reading fp32
// partials and a grid barrier (measured at about 10 us on B200).  When the
// leftover round is nearly full, one more data-parallel round on fewer
// workers is cheaper: its idle share of a round costs (1 - leftover/workers)
// tile times (a 64-block K loop takes about 0.38 us per block on one SM or
// pair).  T=512 on the Llama-3-8B qkv projection: 48 tiles on 48 pairs.
int schedule_workers(int64_t n_all, int k_blocks, int workers) {
  constexpr double kBlockUs = 0.38, kStreamKUs = 10.0;
  if (n_all <= 0 || workers <= 0) return workers;
  const int64_t rounds = n_all / workers, left = n_all % workers;
  if (left == 0) return workers;
  if ((1.0 - (double)left / workers) * k_blocks * kBlockUs < kStreamKUs)
    return (int)ceil_div(n_all, rounds + 1);
  return workers;
}

template <typename T, typename C, int EPI, bool NORM, bool PAIR>
int launch_gemm_epi_mode(const CUtensorMap& ma, const CUtensorMap& mb, void* out,
                         int64_t out_stride, int64_t num_tokens, const QkvShape& sh,
                         const EpiParams& ep, void* workspace, int32_t* fault, int dev,
                         cudaStream_t stream, const char* name) {
  auto kernel = gemm_epi_kernel<T, C, EPI, NORM, PAIR>;
  cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), dev, SMEM_BYTES);
  if (err != cudaSuccess) return cuda_fail(err, name);
  float* slots = static_cast<float*>(workspace);
  int* counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + sh.slot_bytes);
  int ctas = sh.ctas;
  if constexpr (PAIR) {
    // every CTA must be resident at once (grid barrier)
    const int pairs = pairs_resident(kernel, dev);
    if (pairs < 1)
      return fail(PACE_ERR_CUDA, "%s: the device holds no cluster of two CTAs", name);
    ctas = ctas < 2 * pairs ? ctas : 2 * pairs;
    ctas = 2 * schedule_workers((int64_t)sh.m_tiles * sh.n_tiles, sh.k_blocks, ctas / 2);
    err = launch_pairs(kernel, dim3((unsigned)ctas), dim3(THREADS), SMEM_BYTES, stream, ma, mb,
                       static_cast<T*>(out), out_stride, (int)num_tokens, sh.m_tiles,
                       sh.k_blocks, ep, counters, slots, fault);
  } else {
    ctas = schedule_workers((int64_t)sh.m_tiles * sh.n_tiles, sh.k_blocks, ctas);
    err = launch(kernel, dim3((unsigned)ctas), dim3(THREADS), SMEM_BYTES, stream, ma, mb,
                 static_cast<T*>(out), out_stride, (int)num_tokens, sh.m_tiles, sh.k_blocks, ep,
                 counters, slots, fault);
  }
  if (err != cudaSuccess) return cuda_fail(err, name);
  return PACE_OK;
}

template <typename T, typename C, int EPI, bool NORM>
int launch_gemm_epi(const CUtensorMap& ma, const CUtensorMap& mb, void* out, int64_t out_stride,
                    int64_t num_tokens, const QkvShape& sh, const EpiParams& ep, void* workspace,
                    int32_t* fault, int dev, cudaStream_t stream, const char* name) {
  if (sh.pair)
    return launch_gemm_epi_mode<T, C, EPI, NORM, true>(ma, mb, out, out_stride, num_tokens, sh,
                                                       ep, workspace, fault, dev, stream, name);
  return launch_gemm_epi_mode<T, C, EPI, NORM, false>(ma, mb, out, out_stride, num_tokens, sh,
                                                      ep, workspace, fault, dev, stream, name);
}

EpiParams rope_params(const int64_t* positions, const void* cache, int64_t max_position,
                      int rot_heads, int total_heads) {
  EpiParams ep = {};
  ep.positions = positions;
  ep.cache = cache;
  ep.max_position = max_position;
  ep.rot_heads = rot_heads;
  ep.total_heads = total_heads;
  ep.n_cols = total_heads * HEAD;
  return ep;
}

// Whether a call of num_tokens rows and reduction length k takes the
// CUDA-core kernel: always for one token; for two, up to k = 8192 (measured on
// B200: at two tokens and k = 14336, Llama-3-8B's down_proj, the tensor-core
// kernel is faster).
inline bool gemv_path(int64_t num_tokens, int64_t k) {
  return num_tokens <= 1 || (num_tokens <= kGemvTokens && k <= 8192);
}

template <typename T, typename C, int EPI, bool NORM, int NT>
cudaError_t launch_gemv_nt(const void* hidden, int64_t hidden_stride, const void* weight,
                           int64_t k, void* out, int64_t out_stride, int64_t num_tokens,
                           const EpiParams& ep, int32_t* fault, int dev, cudaStream_t stream) {
  auto kernel = gemv_epi_kernel<T, C, EPI, NORM, NT>;
  cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), dev, kGemvSmem);
  if (err != cudaSuccess) return err;
  // three CTAs per SM, so the whole grid is resident at once (set once per
  // kernel and device)
  static std::atomic<bool> carveout_set[64];
  if (dev >= 0 && dev < 64 && !carveout_set[dev].load(std::memory_order_acquire)) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (err != cudaSuccess) return err;
    carveout_set[dev].store(true, std::memory_order_release);
  }
  // the units spread over three CTAs per SM, at most kGemvPairs per CTA
  const int64_t units = gemv_units<EPI>(ep.n_cols);
  const int64_t grid =
      std::max<int64_t>(ceil_div(units, kGemvPairs), std::min<int64_t>(units, 3 * sm_count(dev)));
  return launch(kernel, dim3((unsigned)grid), dim3(kGemvThreads), kGemvSmem, stream,
                static_cast<const T*>(hidden), hidden_stride, static_cast<const T*>(weight), k,
                static_cast<T*>(out), out_stride, (int)num_tokens, ep, fault);
}

template <typename T, typename C, int EPI, bool NORM>
cudaError_t launch_gemv_t(const void* hidden, int64_t hidden_stride, const void* weight,
                          int64_t k, void* out, int64_t out_stride, int64_t num_tokens,
                          const EpiParams& ep, int32_t* fault, int dev, cudaStream_t stream) {
  if (num_tokens == 1)
    return launch_gemv_nt<T, C, EPI, NORM, 1>(hidden, hidden_stride, weight, k, out, out_stride,
                                              num_tokens, ep, fault, dev, stream);
  return launch_gemv_nt<T, C, EPI, NORM, kGemvTokens>(hidden, hidden_stride, weight, k, out,
                                                      out_stride, num_tokens, ep, fault, dev,
                                                      stream);
}

// The decode-batch qkv projection for the dtype pair.
template <bool NORM>
int launch_gemv_rope(const void* hidden, int64_t hidden_stride, const void* weight, int64_t k,
                     void* out, int64_t out_stride, int64_t num_tokens, const EpiParams& ep,
                     int dtype, int cache_dtype, bool neox, int32_t* fault, int dev,
                     cudaStream_t stream, const char* name) {
#define PACE_GEMV(T, C, NX)                                                                      \
  launch_gemv_t<T, C, NX ? EPI_ROPE_NEOX : EPI_ROPE_GPTJ, NORM>(                                 \
      hidden, hidden_stride, weight, k, out, out_stride, num_tokens, ep, fault, dev, stream)
  cudaError_t err;
  const bool f32c = cache_dtype == PACE_F32;
  if (dtype == PACE_BF16) {
    if (f32c)
      err = neox ? PACE_GEMV(__nv_bfloat16, float, true) : PACE_GEMV(__nv_bfloat16, float, false);
    else
      err = neox ? PACE_GEMV(__nv_bfloat16, __nv_bfloat16, true)
                 : PACE_GEMV(__nv_bfloat16, __nv_bfloat16, false);
  } else {
    if (f32c)
      err = neox ? PACE_GEMV(__half, float, true) : PACE_GEMV(__half, float, false);
    else
      err = neox ? PACE_GEMV(__half, __half, true) : PACE_GEMV(__half, __half, false);
  }
#undef PACE_GEMV
  if (err != cudaSuccess) return cuda_fail(err, name);
  return PACE_OK;
}

template <typename T, typename C, bool NEOX>
int launch_qkv_rope(const CUtensorMap& ma, const CUtensorMap& mb, void* out, int64_t out_stride,
                    const int64_t* positions, const void* cache, int64_t max_position,
                    int64_t num_tokens, const QkvShape& sh, int rot_heads, int total_heads,
                    void* workspace, int32_t* fault, int dev, cudaStream_t stream) {
  const EpiParams ep = rope_params(positions, cache, max_position, rot_heads, total_heads);
  return launch_gemm_epi<T, C, NEOX ? EPI_ROPE_NEOX : EPI_ROPE_GPTJ, false>(
      ma, mb, out, out_stride, num_tokens, sh, ep, workspace, fault, dev, stream,
      "qkv_proj_rope");
}

}  // namespace
}  // namespace pace

extern "C" size_t pace_qkv_proj_rope_workspace_size(int64_t num_tokens, int64_t hidden_size,
                                                    int num_heads, int num_kv_heads,
                                                    int device) {
  using namespace pace;
  if (num_tokens <= 0 || hidden_size <= 0 || num_heads < 0 || num_kv_heads < 0 ||
      num_heads + num_kv_heads <= 0)
    return 0;
  if (gemv_path(num_tokens, hidden_size)) return 0;  // the CUDA-core kernel needs none
  return qkv_shape(num_tokens, hidden_size, num_heads + 2 * num_kv_heads, sm_count(device))
      .workspace_bytes;
}

extern "C" int pace_qkv_proj_rope(void* qkv_out, const void* hidden, const void* weight,
                                  const int64_t* positions, int64_t num_tokens,
                                  int64_t hidden_size, int num_heads, int num_kv_heads,
                                  int head_size, int64_t hidden_row_stride,
                                  int64_t out_row_stride, const void* cos_sin_cache,
                                  int cache_dtype, int rot_dim, int64_t max_position, int is_neox,
                                  int dtype, void* workspace, size_t workspace_bytes,
                                  int32_t* fault_flags, cudaStream_t stream) {
  using namespace pace;
  const char* name = "qkv_proj_rope";
  if (num_tokens < 0 || num_tokens > INT32_MAX || hidden_size <= 0 || num_heads < 0 ||
      num_kv_heads < 0 || num_heads + num_kv_heads <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad shape", name);
  if (head_size != HEAD || rot_dim != head_size)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: head_size and rot_dim must both be %d (got %d, %d)", name, HEAD, head_size,
                rot_dim);
  if (dtype != PACE_BF16 && dtype != PACE_F16)
    return fail(PACE_ERR_UNSUPPORTED_DTYPE, "%s: dtype %d must be bfloat16 or float16", name,
                dtype);
  if (cache_dtype != PACE_F32 && cache_dtype != dtype)
    return fail(PACE_ERR_UNSUPPORTED_DTYPE,
                "%s: cos_sin_cache dtype %d must be float32 or the q/k dtype %d", name,
                cache_dtype, dtype);
  const int heads = num_heads + 2 * num_kv_heads;
  const int64_t n = (int64_t)heads * head_size;
  if (hidden_row_stride < hidden_size || out_row_stride < n)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: row stride smaller than the row", name);
  if (hidden_size % 8 != 0 || hidden_row_stride % 8 != 0 || out_row_stride % 8 != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: hidden size and row strides must be multiples of 8 elements", name);
  if (hidden_size > (int64_t)INT32_MAX * BK || num_tokens > (int64_t)1 << 24)
    return fail(PACE_ERR_TOO_LARGE, "%s: shape too large", name);
  if (max_position <= 0) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: empty cos_sin_cache", name);
  if (num_tokens == 0) return PACE_OK;
  // at most kGemvTokens tokens: the CUDA-core kernel, no workspace
  const bool gemv = gemv_path(num_tokens, hidden_size);
  if (!qkv_out || !hidden || !weight || !positions || !cos_sin_cache || (!workspace && !gemv))
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(qkv_out) || !aligned16(hidden) || !aligned16(weight) ||
      !aligned16(cos_sin_cache) || (!gemv && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0))
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: pointers must be 16-byte aligned (the workspace 256-byte aligned)", name);
  StreamDeviceGuard guard(stream);
  const int dev = guard.device();
  const QkvShape sh = qkv_shape(num_tokens, hidden_size, heads, sm_count(dev));
  if (!gemv && workspace_bytes < sh.workspace_bytes)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes, %zu needed", name,
                workspace_bytes, sh.workspace_bytes);
  const int rot_heads = num_heads + num_kv_heads;
  if (gemv)
    return launch_gemv_rope<false>(
        hidden, hidden_row_stride, weight, hidden_size, qkv_out, out_row_stride, num_tokens,
        rope_params(positions, cos_sin_cache, max_position, rot_heads, heads), dtype,
        cache_dtype, is_neox != 0, fault_flags, dev, stream, name);
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  int st = tc::make_kmajor_map(&ma, hidden, bf16, num_tokens, hidden_size, hidden_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, weight, bf16, n, hidden_size, hidden_size,
                           sh.pair ? BN / 2 : BN, name);
  if (st != PACE_OK) return st;
#define PACE_QKV_ROPE(T, C, NX)                                                                 \
  launch_qkv_rope<T, C, NX>(ma, mb, qkv_out, out_row_stride, positions, cos_sin_cache,         \
                            max_position, num_tokens, sh, rot_heads, heads, workspace,         \
                            fault_flags, dev, stream)
  const bool neox = is_neox != 0;
  const bool f32c = cache_dtype == PACE_F32;
  if (bf16) {
    if (f32c)
      return neox ? PACE_QKV_ROPE(__nv_bfloat16, float, true)
                  : PACE_QKV_ROPE(__nv_bfloat16, float, false);
    return neox ? PACE_QKV_ROPE(__nv_bfloat16, __nv_bfloat16, true)
                : PACE_QKV_ROPE(__nv_bfloat16, __nv_bfloat16, false);
  }
  if (f32c) return neox ? PACE_QKV_ROPE(__half, float, true) : PACE_QKV_ROPE(__half, float, false);
  return neox ? PACE_QKV_ROPE(__half, __half, true) : PACE_QKV_ROPE(__half, __half, false);
#undef PACE_QKV_ROPE
}

// ------------------------------------------------ RMSNorm around the GEMMs --
namespace pace {
namespace {
// Shape and pointer checks shared by the two entry points below.
int check_gemm_args(const char* name, int64_t num_tokens, int64_t n, int64_t k, int64_t a_stride,
                    int64_t out_stride, int dtype, const void* out, const void* a, const void* w,
                    const void* workspace, bool need_workspace = true) {
  if (num_tokens < 0 || num_tokens > ((int64_t)1 << 24) || n <= 0 || k <= 0 ||
      n > (int64_t)INT32_MAX || k > (int64_t)INT32_MAX * BK)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad shape", name);
  if (dtype != PACE_BF16 && dtype != PACE_F16)
    return fail(PACE_ERR_UNSUPPORTED_DTYPE, "%s: dtype %d must be bfloat16 or float16", name,
                dtype);
  if (a_stride < k || out_stride < n)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: row stride smaller than the row", name);
  if (k % 8 != 0 || a_stride % 8 != 0 || out_stride % 8 != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: K and row strides must be multiples of 8 elements", name);
  if (num_tokens == 0) return PACE_OK;
  if (!out || !a || !w || (need_workspace && !workspace))
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(out) || !aligned16(a) || !aligned16(w) ||
      (need_workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0))
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: pointers must be 16-byte aligned (the workspace 256-byte aligned)", name);
  return PACE_OK;
}
}  // namespace
}  // namespace pace

extern "C" size_t pace_linear_residual_workspace_size(int64_t num_tokens, int64_t n, int64_t k,
                                                      int device) {
  using namespace pace;
  if (num_tokens <= 0 || n <= 0 || k <= 0 || n % HEAD != 0) return 0;
  if (gemv_path(num_tokens, k)) return 0;  // the CUDA-core kernel needs none
  return qkv_shape(num_tokens, k, (int)(n / HEAD), sm_count(device)).workspace_bytes;
}

extern "C" int pace_linear_residual(void* residual, const void* input, const void* weight,
                                    float* row_sumsq, int64_t num_tokens, int64_t n, int64_t k,
                                    int64_t input_row_stride, int64_t residual_row_stride,
                                    int dtype, void* workspace, size_t workspace_bytes,
                                    int32_t* fault_flags, cudaStream_t stream) {
  using namespace pace;
  const char* name = "linear_residual";
  if (n % HEAD != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: n = %lld must be a multiple of %d", name,
                (long long)n, HEAD);
  // at most kGemvTokens tokens: the CUDA-core kernel, no workspace
  const bool gemv = gemv_path(num_tokens, k);
  int st = check_gemm_args(name, num_tokens, n, k, input_row_stride, residual_row_stride, dtype,
                           residual, input, weight, workspace, !gemv);
  if (st != PACE_OK || num_tokens == 0) return st;
  StreamDeviceGuard guard(stream);
  const int dev = guard.device();
  const QkvShape sh = qkv_shape(num_tokens, k, (int)(n / HEAD), sm_count(dev));
  if (!gemv && workspace_bytes < sh.workspace_bytes)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes, %zu needed", name,
                workspace_bytes, sh.workspace_bytes);
  const bool bf16 = dtype == PACE_BF16;
  if (gemv) {
    // the new rows, then their sums of squares per 32 columns (the same
    // partials the tensor-core epilogue writes) by pace_row_sumsq
    EpiParams ep = {};
    ep.n_cols = (int)n;
    const cudaError_t err =
        bf16 ? launch_gemv_t<__nv_bfloat16, __nv_bfloat16, EPI_RESIDUAL, false>(
                   input, input_row_stride, weight, k, residual, residual_row_stride, num_tokens,
                   ep, fault_flags, dev, stream)
             : launch_gemv_t<__half, __half, EPI_RESIDUAL, false>(
                   input, input_row_stride, weight, k, residual, residual_row_stride, num_tokens,
                   ep, fault_flags, dev, stream);
    if (err != cudaSuccess) return cuda_fail(err, name);
    if (!row_sumsq) return PACE_OK;
    return pace_row_sumsq(row_sumsq, residual, num_tokens, n, residual_row_stride, dtype, stream);
  }
  CUtensorMap ma, mb;
  st = tc::make_kmajor_map(&ma, input, bf16, num_tokens, k, input_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, weight, bf16, n, k, k, sh.pair ? BN / 2 : BN, name);
  if (st != PACE_OK) return st;
  EpiParams ep = {};
  ep.sumsq_out = row_sumsq;
  ep.n_cols = (int)n;
  if (bf16)
    return launch_gemm_epi<__nv_bfloat16, float, EPI_RESIDUAL, false>(
        ma, mb, residual, residual_row_stride, num_tokens, sh, ep, workspace, fault_flags, dev,
        stream, name);
  return launch_gemm_epi<__half, float, EPI_RESIDUAL, false>(ma, mb, residual,
                                                            residual_row_stride, num_tokens, sh,
                                                            ep, workspace, fault_flags, dev,
                                                            stream, name);
}

extern "C" int pace_qkv_proj_rmsnorm_rope(
    void* qkv_out, const void* hidden, const void* folded_weight, const float* row_sumsq,
    int64_t sumsq_groups, float epsilon, const int64_t* positions, int64_t num_tokens,
    int64_t hidden_size, int num_heads, int num_kv_heads, int head_size,
    int64_t hidden_row_stride, int64_t out_row_stride, const void* cos_sin_cache,
    int cache_dtype, int rot_dim, int64_t max_position, int is_neox, int dtype, void* workspace,
    size_t workspace_bytes, int32_t* fault_flags, cudaStream_t stream) {
  using namespace pace;
  const char* name = "qkv_proj_rmsnorm_rope";
  if (num_heads < 0 || num_kv_heads < 0 || num_heads + num_kv_heads <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad head counts", name);
  if (head_size != HEAD || rot_dim != head_size)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: head_size and rot_dim must both be %d (got %d, %d)", name, HEAD, head_size,
                rot_dim);
  if (cache_dtype != PACE_F32 && cache_dtype != dtype)
    return fail(PACE_ERR_UNSUPPORTED_DTYPE,
                "%s: cos_sin_cache dtype %d must be float32 or the q/k dtype %d", name,
                cache_dtype, dtype);
  if (sumsq_groups <= 0 || sumsq_groups > hidden_size)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: sumsq_groups %lld out of range", name,
                (long long)sumsq_groups);
  const int heads = num_heads + 2 * num_kv_heads;
  const int64_t n = (int64_t)heads * head_size;
  // at most kGemvTokens tokens: the CUDA-core kernel, no workspace
  const bool gemv = gemv_path(num_tokens, hidden_size);
  int st = check_gemm_args(name, num_tokens, n, hidden_size, hidden_row_stride, out_row_stride,
                           dtype, qkv_out, hidden, folded_weight, workspace, !gemv);
  if (st != PACE_OK || num_tokens == 0) return st;
  if (max_position <= 0) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: empty cos_sin_cache", name);
  if (!positions || !cos_sin_cache || !row_sumsq)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(cos_sin_cache) || (reinterpret_cast<uintptr_t>(row_sumsq) & 15u) != 0 ||
      sumsq_groups % 4 != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: cache and row_sumsq must be 16-byte aligned, sumsq_groups a multiple of 4",
                name);
  StreamDeviceGuard guard(stream);
  const int dev = guard.device();
  const QkvShape sh = qkv_shape(num_tokens, hidden_size, heads, sm_count(dev));
  if (!gemv && workspace_bytes < sh.workspace_bytes)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes, %zu needed", name,
                workspace_bytes, sh.workspace_bytes);
  EpiParams ep = rope_params(positions, cos_sin_cache, max_position, num_heads + num_kv_heads,
                             heads);
  ep.sumsq_in = row_sumsq;
  ep.sumsq_in_groups = (int)sumsq_groups;
  ep.inv_k = 1.f / (float)hidden_size;
  ep.eps = epsilon;
  if (gemv)
    return launch_gemv_rope<true>(hidden, hidden_row_stride, folded_weight, hidden_size, qkv_out,
                                  out_row_stride, num_tokens, ep, dtype, cache_dtype,
                                  is_neox != 0, fault_flags, dev, stream, name);
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  st = tc::make_kmajor_map(&ma, hidden, bf16, num_tokens, hidden_size, hidden_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, folded_weight, bf16, n, hidden_size, hidden_size,
                           sh.pair ? BN / 2 : BN, name);
  if (st != PACE_OK) return st;
#define PACE_QKV_NORM(T, C, E)                                                                  \
  launch_gemm_epi<T, C, E, true>(ma, mb, qkv_out, out_row_stride, num_tokens, sh, ep, workspace, \
                                 fault_flags, dev, stream, name)
  const int epi = is_neox ? EPI_ROPE_NEOX : EPI_ROPE_GPTJ;
  const bool f32c = cache_dtype == PACE_F32;
  if (bf16) {
    if (f32c)
      return epi == EPI_ROPE_NEOX ? PACE_QKV_NORM(__nv_bfloat16, float, EPI_ROPE_NEOX)
                                  : PACE_QKV_NORM(__nv_bfloat16, float, EPI_ROPE_GPTJ);
    return epi == EPI_ROPE_NEOX ? PACE_QKV_NORM(__nv_bfloat16, __nv_bfloat16, EPI_ROPE_NEOX)
                                : PACE_QKV_NORM(__nv_bfloat16, __nv_bfloat16, EPI_ROPE_GPTJ);
  }
  if (f32c)
    return epi == EPI_ROPE_NEOX ? PACE_QKV_NORM(__half, float, EPI_ROPE_NEOX)
                                : PACE_QKV_NORM(__half, float, EPI_ROPE_GPTJ);
  return epi == EPI_ROPE_NEOX ? PACE_QKV_NORM(__half, __half, EPI_ROPE_NEOX)
                              : PACE_QKV_NORM(__half, __half, EPI_ROPE_GPTJ);
#undef PACE_QKV_NORM
}

// ------------------------------------------------------ gate/up + SiLU --
// The MLP's first half in one GEMM: gate_up = x @ W^T with W = [gate rows;
// up rows] ([2 I, H], the layout models/llama.py:70-104 builds and loads at
// :452-469), then SiLU-and-mul (csrc/activation_kernels.cu:15-45) in the
// epilogue, so the [T, 2 I] intermediate never reaches HBM.  With row_sumsq
// the post-attention RMSNorm is applied as a per-row factor, W holding the
// norm weight folded in (see pace_qkv_proj_rmsnorm_rope).
extern "C" size_t pace_gate_up_silu_workspace_size(int64_t num_tokens, int64_t hidden_size,
                                                   int64_t intermediate_size, int device) {
  using namespace pace;
  if (num_tokens <= 0 || hidden_size <= 0 || intermediate_size <= 0 ||
      intermediate_size % HEAD != 0 || intermediate_size / HEAD > INT32_MAX / 2)
    return 0;
  if (gemv_path(num_tokens, hidden_size)) return 0;  // the CUDA-core kernel needs none
  // 2 I accumulator columns per row: one 256-column tile per 128 output columns
  return qkv_shape(num_tokens, hidden_size, (int)(2 * intermediate_size / HEAD),
                   sm_count(device))
      .workspace_bytes;
}

extern "C" int pace_gate_up_silu(void* out, const void* hidden, const void* weight,
                                 const float* row_sumsq, int64_t sumsq_groups, float epsilon,
                                 int64_t num_tokens, int64_t hidden_size,
                                 int64_t intermediate_size, int64_t hidden_row_stride,
                                 int64_t out_row_stride, int dtype, void* workspace,
                                 size_t workspace_bytes, int32_t* fault_flags,
                                 cudaStream_t stream) {
  using namespace pace;
  const char* name = "gate_up_silu";
  if (intermediate_size <= 0 || intermediate_size % HEAD != 0 ||
      intermediate_size / HEAD > INT32_MAX / 2)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: intermediate size %lld must be a multiple of %d",
                name, (long long)intermediate_size, HEAD);
  // at most kGemvTokens tokens: the CUDA-core kernel, no workspace
  const bool gemv = gemv_path(num_tokens, hidden_size);
  int st = check_gemm_args(name, num_tokens, intermediate_size, hidden_size, hidden_row_stride,
                           out_row_stride, dtype, out, hidden, weight, workspace, !gemv);
  if (st != PACE_OK || num_tokens == 0) return st;
  if (row_sumsq) {
    if (sumsq_groups <= 0 || sumsq_groups > hidden_size || sumsq_groups % 4 != 0 ||
        (reinterpret_cast<uintptr_t>(row_sumsq) & 15u) != 0)
      return fail(PACE_ERR_INVALID_ARGUMENT,
                  "%s: row_sumsq must be 16-byte aligned with a multiple of 4 groups (<= %lld)",
                  name, (long long)hidden_size);
  }
  StreamDeviceGuard guard(stream);
  const int dev = guard.device();
  const QkvShape sh =
      qkv_shape(num_tokens, hidden_size, (int)(2 * intermediate_size / HEAD), sm_count(dev));
  if (!gemv && workspace_bytes < sh.workspace_bytes)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes, %zu needed", name,
                workspace_bytes, sh.workspace_bytes);
  EpiParams ep = {};
  ep.n_cols = (int)intermediate_size;
  ep.sumsq_in = row_sumsq;
  ep.sumsq_in_groups = (int)sumsq_groups;
  ep.inv_k = 1.f / (float)hidden_size;
  ep.eps = epsilon;
  const bool bf16 = dtype == PACE_BF16;
  if (gemv) {
#define PACE_GATE_UP_GEMV(T, NORM)                                                              \
  launch_gemv_t<T, T, EPI_GATEUP_SILU, NORM>(hidden, hidden_row_stride, weight, hidden_size, out, \
                                             out_row_stride, num_tokens, ep, fault_flags, dev,    \
                                             stream)
    const cudaError_t err =
        bf16 ? (row_sumsq ? PACE_GATE_UP_GEMV(__nv_bfloat16, true)
                          : PACE_GATE_UP_GEMV(__nv_bfloat16, false))
             : (row_sumsq ? PACE_GATE_UP_GEMV(__half, true) : PACE_GATE_UP_GEMV(__half, false));
#undef PACE_GATE_UP_GEMV
    if (err != cudaSuccess) return cuda_fail(err, name);
    return PACE_OK;
  }
  CUtensorMap ma, mb;
  st = tc::make_kmajor_map(&ma, hidden, bf16, num_tokens, hidden_size, hidden_row_stride, BM,
                           name);
  if (st != PACE_OK) return st;
  // two 128-row boxes per stage: the gate rows and the up rows of the tile
  st = tc::make_kmajor_map(&mb, weight, bf16, 2 * intermediate_size, hidden_size, hidden_size,
                           HEAD, name);
  if (st != PACE_OK) return st;
#define PACE_GATE_UP(T, NORM)                                                                   \
  launch_gemm_epi<T, float, EPI_GATEUP_SILU, NORM>(ma, mb, out, out_row_stride, num_tokens, sh, \
                                                   ep, workspace, fault_flags, dev, stream, name)
  if (bf16) return row_sumsq ? PACE_GATE_UP(__nv_bfloat16, true) : PACE_GATE_UP(__nv_bfloat16, false);
  return row_sumsq ? PACE_GATE_UP(__half, true) : PACE_GATE_UP(__half, false);
#undef PACE_GATE_UP
}

// ------------------------------------------------- allocation-free variant --
// Some callers cannot allocate device memory for a workspace: a plugin host
// that hands an op only its input and output buffers, or a latency-bound
// serving loop that must not call cudaMalloc (it synchronises the device).
// pace_qkv_proj_rope_no_alloc serves them with scratch in this file-scope
// array instead: partial slots for up to kNoAllocCtas CTAs (the variant runs
// at most that many, about 43 % of a B200's SMs) and counters for up to
// kNoAllocTiles output tiles.  Every GPU that loads this code holds the array
// (15.8 MiB) until the process exits.
namespace pace {
namespace {
constexpr int kNoAllocCtas = 63;
constexpr int kNoAllocTiles = 16384;
constexpr size_t kNoAllocSlotBytes = (size_t)2 * kNoAllocCtas * SLOT_FLOATS * sizeof(float);
constexpr size_t kNoAllocBytes =
    kNoAllocSlotBytes + (size_t)(kTileCounterOffset + kNoAllocTiles) * sizeof(int);
constexpr int kMaxDevices = 64;
}  // namespace
}  // namespace pace

static __device__ __align__(256) unsigned char g_qkv_no_alloc_scratch[pace::kNoAllocBytes];

namespace pace {
namespace {
// Device address of the scratch array on the current device `dev`, looked up
// once per device (cudaGetSymbolAddress; the host-side name is not a device
// address).  nullptr on failure, with the error recorded.
void* no_alloc_scratch(int dev) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) {
    fail(PACE_ERR_INVALID_ARGUMENT, "qkv_proj_rope_no_alloc: device %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_qkv_no_alloc_scratch);
    if (err != cudaSuccess) {
      cuda_fail(err, "qkv_proj_rope_no_alloc (scratch address)");
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}
}  // namespace
}  // namespace pace

extern "C" int pace_qkv_proj_rope_no_alloc(
    void* qkv_out, const void* hidden, const void* weight, const int64_t* positions,
    int64_t num_tokens, int64_t hidden_size, int num_heads, int num_kv_heads, int head_size,
    int64_t hidden_row_stride, int64_t out_row_stride, const void* cos_sin_cache,
    int cache_dtype, int rot_dim, int64_t max_position, int is_neox, int dtype,
    int32_t* fault_flags, cudaStream_t stream) {
  using namespace pace;
  const char* name = "qkv_proj_rope_no_alloc";
  if (num_tokens < 0 || num_tokens > INT32_MAX || hidden_size <= 0 || num_heads < 0 ||
      num_kv_heads < 0 || num_heads + num_kv_heads <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad shape", name);
  if (head_size != HEAD || rot_dim != head_size)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: head_size and rot_dim must both be %d (got %d, %d)", name, HEAD, head_size,
                rot_dim);
  if (dtype != PACE_BF16 && dtype != PACE_F16)
    return fail(PACE_ERR_UNSUPPORTED_DTYPE, "%s: dtype %d must be bfloat16 or float16", name,
                dtype);
  if (cache_dtype != PACE_F32 && cache_dtype != dtype)
    return fail(PACE_ERR_UNSUPPORTED_DTYPE,
                "%s: cos_sin_cache dtype %d must be float32 or the q/k dtype %d", name,
                cache_dtype, dtype);
  const int heads = num_heads + 2 * num_kv_heads;
  const int64_t n = (int64_t)heads * head_size;
  if (hidden_row_stride < hidden_size || out_row_stride < n)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: row stride smaller than the row", name);
  if (hidden_size % 8 != 0 || hidden_row_stride % 8 != 0 || out_row_stride % 8 != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: hidden size and row strides must be multiples of 8 elements", name);
  if (hidden_size > (int64_t)INT32_MAX * BK || num_tokens > (int64_t)1 << 24)
    return fail(PACE_ERR_TOO_LARGE, "%s: shape too large", name);
  const int64_t tiles = ceil_div(num_tokens, BM) * ceil_div(n, BN);
  if (tiles > kNoAllocTiles)
    return fail(PACE_ERR_TOO_LARGE,
                "%s: %lld output tiles of %dx%d exceed the fixed scratch's %d (use "
                "pace_qkv_proj_rope with a workspace)",
                name, (long long)tiles, BM, BN, kNoAllocTiles);
  if (max_position <= 0) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: empty cos_sin_cache", name);
  if (num_tokens == 0) return PACE_OK;
  if (!qkv_out || !hidden || !weight || !positions || !cos_sin_cache)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(qkv_out) || !aligned16(hidden) || !aligned16(weight) || !aligned16(cos_sin_cache))
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: pointers must be 16-byte aligned", name);
  StreamDeviceGuard guard(stream);
  const int dev = guard.device();
  const int rot_heads = num_heads + num_kv_heads;
  if (gemv_path(num_tokens, hidden_size))  // no scratch needed
    return launch_gemv_rope<false>(
        hidden, hidden_row_stride, weight, hidden_size, qkv_out, out_row_stride, num_tokens,
        rope_params(positions, cos_sin_cache, max_position, rot_heads, heads), dtype,
        cache_dtype, is_neox != 0, fault_flags, dev, stream, name);
  void* scratch = no_alloc_scratch(dev);
  if (!scratch) return PACE_ERR_CUDA;
  QkvShape sh = qkv_shape(num_tokens, hidden_size, heads, sm_count(dev));
  // at most kNoAllocCtas CTAs have slots (an even number on CTA pairs)
  const int cap = sh.pair ? kNoAllocCtas / 2 * 2 : kNoAllocCtas;
  if (sh.ctas > cap) sh.ctas = cap;
  sh.slot_bytes = kNoAllocSlotBytes;
  // The barrier and tile counters must start at zero.  Calls leave them zero,
  // but one whose wait expired may not: clear them on the stream first (no
  // allocation).
  cudaError_t err = cudaMemsetAsync(static_cast<char*>(scratch) + kNoAllocSlotBytes, 0,
                                    (size_t)(kTileCounterOffset + tiles) * sizeof(int), stream);
  if (err != cudaSuccess) return cuda_fail(err, name);
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  int st = tc::make_kmajor_map(&ma, hidden, bf16, num_tokens, hidden_size, hidden_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, weight, bf16, n, hidden_size, hidden_size,
                           sh.pair ? BN / 2 : BN, name);
  if (st != PACE_OK) return st;
#define PACE_QKV_ROPE_NA(T, C, NX)                                                               \
  launch_qkv_rope<T, C, NX>(ma, mb, qkv_out, out_row_stride, positions, cos_sin_cache,         \
                            max_position, num_tokens, sh, rot_heads, heads, scratch,           \
                            fault_flags, dev, stream)
  const bool neox = is_neox != 0;
  const bool f32c = cache_dtype == PACE_F32;
  if (bf16) {
    if (f32c)
      return neox ? PACE_QKV_ROPE_NA(__nv_bfloat16, float, true)
                  : PACE_QKV_ROPE_NA(__nv_bfloat16, float, false);
    return neox ? PACE_QKV_ROPE_NA(__nv_bfloat16, __nv_bfloat16, true)
                : PACE_QKV_ROPE_NA(__nv_bfloat16, __nv_bfloat16, false);
  }
  if (f32c)
    return neox ? PACE_QKV_ROPE_NA(__half, float, true) : PACE_QKV_ROPE_NA(__half, float, false);
  return neox ? PACE_QKV_ROPE_NA(__half, __half, true) : PACE_QKV_ROPE_NA(__half, __half, false);
#undef PACE_QKV_ROPE_NA
}
