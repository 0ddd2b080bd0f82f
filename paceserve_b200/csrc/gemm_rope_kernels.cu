// Fused qkv projection + rotary embedding for sm_100a (tcgen05 tensor cores).
//
// Replaces the pair qkv_proj -> rotary_emb of LlamaAttention.forward
// (paceserve/model_executor/models/llama.py:176-178): the projection
// qkv = hidden @ W_qkv^T (F.linear, a library GEMM in the reference) followed
// by the in-place rotary embedding of the q and k columns
// (csrc/pos_encoding_kernels.cu:38-76, cache row = [cos(rot/2) | sin(rot/2)]).
// Here the rotation is applied to the fp32 accumulator in the GEMM's epilogue,
// so the q/k values are rounded to the storage type once (the unfused path
// rounds the GEMM output, then rotates and rounds again) and the separate rope
// launch and its 4(nq+nkv)hd bytes per token of HBM traffic disappear.
//
// Work decomposition (stream-K): the output is cut into 128 x 256 tiles (two
// heads, so both halves of every NeoX pair (i, i + 64) and every GPT-J pair
// (2i, 2i + 1) of a head sit in one tile), each tile into 64-element K blocks,
// and the (tile, K block) units are split evenly over one persistent CTA per
// SM.  A CTA whose range covers a whole tile finishes it directly; a tile
// shared by several CTAs is finished by the CTA that contributes last: every
// contributor stores its fp32 partial sum in the caller's workspace and counts
// itself in the tile's counter, and the one that completes the count adds the
// partials in segment order (so the result does not depend on which CTA came
// last), rotates and stores.  No CTA ever waits for another.  At T=512 this
// gives every SM 41.5 units instead of one or two whole tiles.
//
// Inside a CTA: a 4-stage shared-memory ring of A (128 x 64) and B (256 x 64)
// blocks filled by TMA (128-byte swizzle, no multicast; warp 4), tcgen05.mma
// (M=128, N=256, K=16, fp32) issued by one thread of warp 5 into one of two
// 256-column TMEM accumulators, and 4 epilogue warps (warp w owns TMEM lanes
// 32w..32w+31, i.e. tile rows) that drain one accumulator while the MMAs fill
// the other.  Every mbarrier wait is bounded by %globaltimer; on expiry the
// CTA records bit 30 in the caller's fault word, stops issuing, waits (bounded
// again) for its own copies and MMAs, frees TMEM and returns.
#include <mutex>

#include "tcgen05.cuh"

namespace pace {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, HEAD = 128;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter: one per head of the tile
constexpr int THREADS = (EPI_WARPS + 2) * 32;
constexpr int TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int SLOT_FLOATS = BM * BN;  // one partial tile
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait
constexpr int32_t kFaultTimeout = 1 << 30;
constexpr int kEpiBarrier = 1;  // named barrier of the 256 epilogue threads

struct Ctl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem;
  int abort;
  int last;  // epilogue: this CTA completes the current shared tile
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

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* v) {
  st_v4(p, Traits<T>::pack(v));
  st_v4(p + 8, Traits<T>::pack(v + 8));
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
// pairs), or the residual add of o_proj / down_proj.  NORM (rope kinds):
// each row of the accumulator is first scaled by its RMSNorm factor
// inv = rsqrt(sum of the row's squares / K + eps), from the sum-of-squares
// partials the producer of the input rows wrote (the residual epilogue, or
// pace_row_sumsq); the norm weight is folded into the GEMM weight by the
// caller, so x_norm @ W^T = inv * (h @ (W diag(w))^T).
constexpr int EPI_ROPE_NEOX = 0, EPI_ROPE_GPTJ = 1, EPI_RESIDUAL = 2;
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
  s.store = valid && (EPI == EPI_RESIDUAL ? head * HEAD < ep.n_cols : head < ep.total_heads);
  if (EPI != EPI_RESIDUAL && valid && head < ep.rot_heads) {
    const int64_t pos = ep.positions[m];
    if (pos >= 0 && pos < ep.max_position)
      s.cs = static_cast<const C*>(ep.cache) + pos * HEAD;
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
template <typename T, typename C, int EPI, bool NORM>
__device__ __forceinline__ float apply_step(const RowState<C>& s, int i, float* a, float* b,
                                            T* o) {
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
      float ra[16], rb[16];
      load16(o + col_a<EPI>(i), ra);
      load16(o + col_b<EPI>(i), rb);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        a[e] = Traits<T>::round(a[e] + ra[e]);
        b[e] = Traits<T>::round(b[e] + rb[e]);
        ss += a[e] * a[e] + b[e] * b[e];
      }
    }
  } else if (s.cs) {
    float cv[16], sv[16];
    load_step_cs(s.cs, i, cv, sv);
    rotate<EPI>(a, b, cv, sv);
  }
  if (s.store) {
    store16(o + col_a<EPI>(i), a);
    store16(o + col_b<EPI>(i), b);
  }
  return ss;
}

// A whole tile from TMEM: this thread's row, one head (128 columns at TMEM
// address `taddr`).  All lanes of the warp call it (TMEM loads are
// warp-wide).  ss_out: the row's sum-of-squares partials (residual), or null.
template <typename T, typename C, int EPI, bool NORM>
__device__ __forceinline__ void finish_head_tmem(uint32_t taddr, T* o, const RowState<C>& s,
                                                 float* ss_out, int head) {
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    uint32_t ra[16], rb[16];
    tc::tmem_ld16(taddr + col_a<EPI>(i), ra);
    tc::tmem_ld16(taddr + col_b<EPI>(i), rb);
    tc::tmem_wait_ld(ra);
    tc::tmem_wait_ld(rb);
    float a[16], b[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      a[e] = __uint_as_float(ra[e]);
      b[e] = __uint_as_float(rb[e]);
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

// v[0..16) += the 16 floats of (chunk, row) in a partial slot.
__device__ __forceinline__ void add16(float* v, const float* slot, int chunk, int row) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 f = ld_cg_f4(slot_q(const_cast<float*>(slot), chunk, q, row));
    v[4 * q] += f.x;
    v[4 * q + 1] += f.y;
    v[4 * q + 2] += f.z;
    v[4 * q + 3] += f.w;
  }
}

// Completion of a shared tile by the CTA that contributed last.  The 8
// epilogue warps split it by column: warp w takes step w % 4 of head w / 4
// for every valid row (lane + 32 p), so each load of a warp reads 32
// consecutive rows of one chunk.  Partials are added in segment order.
template <typename T, typename C, int EPI, bool NORM>
__device__ __forceinline__ void fixup_tile(const float* slots, const Split& sp, int64_t tile_u0,
                                           int c0, int c1, T* out_tile, int64_t out_stride,
                                           const EpiParams& ep, int m0, int valid_rows,
                                           int head0, int warp, int lane) {
  const int hh = warp / 4, i = warp % 4;
  const int head = head0 + hh;
  const int ca = hh * 8 + col_a<EPI>(i) / 16, cb = hh * 8 + col_b<EPI>(i) / 16;
  const int groups = ep.n_cols / SUMSQ_GROUP;
#pragma unroll 1
  for (int p = 0; p < BM / 32; ++p) {
    const int r = lane + 32 * p;
    if (r >= valid_rows) break;
    const RowState<C> s = row_state<C, EPI, NORM>(ep, m0 + r, true, head);
    if (!s.store) break;  // the head is past the output (odd head counts)
    float a[16], b[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) a[e] = b[e] = 0.f;
#pragma unroll 2
    for (int c = c0; c <= c1; ++c) {
      const int slot = sp.start(c) >= tile_u0 ? 2 * c : 2 * c + 1;
      const float* sl = slots + (int64_t)slot * SLOT_FLOATS;
      add16(a, sl, ca, r);
      add16(b, sl, cb, r);
    }
    T* o = out_tile + (int64_t)r * out_stride + hh * HEAD;
    const float ss = apply_step<T, C, EPI, NORM>(s, i, a, b, o);
    if (EPI == EPI_RESIDUAL && ep.sumsq_out)
      ep.sumsq_out[(int64_t)(m0 + r) * groups + head * 4 + i] = ss;
  }
}

// One persistent CTA per SM (grid = min(SMs, units)); see the file comment.
// slots: 2 partial tiles of BM x BN floats per CTA; counters: one int32 per
// tile, zero before the call and left zero by it.
template <typename T, typename C, int EPI, bool NORM>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_epi_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    T* __restrict__ out, int64_t out_stride, int num_tokens, int m_tiles,
                    int k_blocks, const EpiParams ep, int* __restrict__ counters,
                    float* __restrict__ slots, int32_t* fault) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Ctl* ctl = reinterpret_cast<Ctl*>(tiles + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int n_tiles = (ep.n_cols + BN - 1) / BN;
  const int64_t n_all = (int64_t)m_tiles * n_tiles;
  const int64_t t_stop = n_all / gridDim.x * gridDim.x;  // first stream-K tile
  Split sp;  // stream-K split of the units of tiles [t_stop, n_all)
  sp.units = (n_all - t_stop) * k_blocks;
  sp.ctas = gridDim.x;
  sp.k_blocks = k_blocks;
  const int64_t u_begin = sp.units > 0 ? sp.start(cta) : 0;
  const int64_t u_end = sp.units > 0 ? sp.start(cta + 1) : 0;
  const Walk walk0{cta, t_stop, (int64_t)gridDim.x, u_begin, u_end, k_blocks};

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&ctl->full[s], 1);
      tc::mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&ctl->tmem_full[b], 1);
      tc::mbar_init(&ctl->tmem_empty[b], EPI_WARPS);
    }
    tc::mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == EPI_WARPS && lane == 0) {
    tc::tma_prefetch_desc(&tm_a);
    tc::tma_prefetch_desc(&tm_b);
  }
  if (warp == 0) tc::tmem_alloc(&ctl->tmem, TMEM_COLS);
  tc::tc_fence_before();
  __syncthreads();
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
      while (ok && walk.next(t, kb0, kb1)) {
        const int m0 = (int)(t / n_tiles) * BM, n0 = (int)(t % n_tiles) * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++i) {
          const int s = (int)(i % STAGES);
          const uint32_t use = (uint32_t)(i / STAGES);
          if (use > 0 &&
              !tc::mbar_wait(&ctl->empty[s], (use - 1) & 1u, kWaitLimitNs, &ctl->abort)) {
            ok = false;
            break;
          }
          uint8_t* a = tiles + s * STAGE_BYTES;
          tc::mbar_arrive_expect_tx(&ctl->full[s], STAGE_BYTES);
          tc::tma_load_2d(a, &tm_a, kb * BK, m0, &ctl->full[s]);
          tc::tma_load_2d(a + A_BYTES, &tm_b, kb * BK, n0, &ctl->full[s]);
        }
      }
      if (!ok) raise_fault(ctl, fault);
      // every copy issued has landed before the CTA's shared memory is released
      // (immediate when the MMAs consumed them all)
      for (int64_t q = i > STAGES ? i - STAGES : 0; q < i; ++q)
        tc::mbar_wait(&ctl->full[q % STAGES], (uint32_t)(q / STAGES) & 1u, kWaitLimitNs,
                      nullptr);
    }
  } else if (warp == EPI_WARPS + 1) {
    // ---- MMA issuer ----------------------------------------------------
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idesc = tc::umma_idesc_f16(kBf16, BM, BN);
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
          const int s = (int)(i % STAGES);
          if (!tc::mbar_wait(&ctl->full[s], (uint32_t)(i / STAGES) & 1u, kWaitLimitNs,
                             &ctl->abort)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_addr = tc::smem_u32(tiles + s * STAGE_BYTES);
          const uint64_t ad = tc::umma_desc_sw128(a_addr);
          const uint64_t bd = tc::umma_desc_sw128(a_addr + A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc::umma_f16(d, ad + 2 * k, bd + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          tc::umma_commit(&ctl->empty[s]);
        }
        if (ok) tc::umma_commit(&ctl->tmem_full[b]);
      }
      if (!ok) raise_fault(ctl, fault);
      // every MMA issued has completed before TMEM is freed
      tc::umma_commit(&ctl->drain);
      tc::mbar_wait(&ctl->drain, 0, kWaitLimitNs, nullptr);
    }
  } else {
    // ---- epilogue: warp w drains TMEM lanes 32 (w % 4) .. +31, head w / 4 ----
    const int quarter = warp % 4, hh = warp / 4;
    const int row = quarter * 32 + lane;
    int j = 0;
    Walk walk = walk0;
    int64_t t;
    int kb0, kb1;
    for (; walk.next(t, kb0, kb1); ++j) {
      const int b = j & 1;
      const int mt = (int)(t / n_tiles), nt = (int)(t % n_tiles);
      const int m0 = mt * BM, m = m0 + row;
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
      if (whole) {
        T* o = out + (int64_t)(valid ? m : 0) * out_stride + (int64_t)head * HEAD;
        finish_head_tmem<T, C, EPI, NORM>(
            taddr, o, rs,
            EPI == EPI_RESIDUAL && ep.sumsq_out
                ? ep.sumsq_out + (int64_t)(valid ? m : 0) * (ep.n_cols / SUMSQ_GROUP)
                : nullptr,
            head);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl->tmem_empty[b]);
        continue;
      }
      // a shared tile: store this CTA's partial, then count it
      const int64_t tile_u0 = (t - t_stop) * k_blocks;  // stream-K units are relative
      const int my_slot = tile_u0 + kb0 == u_begin ? 2 * cta : 2 * cta + 1;
      store_partial(taddr, slots + (int64_t)my_slot * SLOT_FLOATS, hh, row, valid);
      // the accumulator is free for the segment after next
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl->tmem_empty[b]);
      // All epilogue threads' partial stores are ordered before thread 0's
      // fence by the barrier; the fence (cumulative) then releases them at GPU
      // scope before the count.  The CTA that completes the count fences
      // again before its threads read the other partials.
      epi_sync();
      const int c0 = sp.owner(tile_u0), c1 = sp.owner(tile_u0 + k_blocks - 1);
      if (threadIdx.x == 0) {
        __threadfence();
        const int prev = atomicAdd(&counters[t], 1);
        const int last = prev == c1 - c0;
        if (last) counters[t] = 0;  // ready for the next call
        __threadfence();
        ctl->last = last;
      }
      epi_sync();
      const bool last = *reinterpret_cast<volatile int*>(&ctl->last) != 0;
      epi_sync();  // ctl->last is rewritten by the next shared tile
      if (last)
        fixup_tile<T, C, EPI, NORM>(slots, sp, tile_u0, c0, c1,
                                    out + (int64_t)m0 * out_stride + (int64_t)nt * BN,
                                    out_stride, ep, m0, min(BM, num_tokens - m0),
                                    nt * (BN / HEAD), warp, lane);
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------- host ----
// Workspace layout: 2 partial slots per SM (a fixed size for the device),
// then one int32 counter per tile.  The counters sit at the same offset for
// every shape, so a workspace that a call of one shape left zeroed is valid
// for a call of any other shape that fits in it.
struct QkvShape {
  int m_tiles, n_tiles, k_blocks, ctas;
  size_t slot_bytes, workspace_bytes;
};

QkvShape qkv_shape(int64_t num_tokens, int64_t hidden_size, int total_heads, int sms) {
  QkvShape s;
  s.m_tiles = (int)ceil_div(num_tokens, BM);
  s.n_tiles = (int)ceil_div((int64_t)total_heads * HEAD, BN);
  s.k_blocks = (int)ceil_div(hidden_size, BK);
  const int64_t units = (int64_t)s.m_tiles * s.n_tiles * s.k_blocks;
  s.ctas = (int)(units < sms ? units : sms);
  s.slot_bytes = (size_t)2 * sms * SLOT_FLOATS * sizeof(float);
  s.workspace_bytes =
      s.slot_bytes + ((size_t)s.m_tiles * s.n_tiles * sizeof(int) + 255) / 256 * 256;
  return s;
}

template <typename T, typename C, int EPI, bool NORM>
int launch_gemm_epi(const CUtensorMap& ma, const CUtensorMap& mb, void* out, int64_t out_stride,
                    int64_t num_tokens, const QkvShape& sh, const EpiParams& ep, void* workspace,
                    int32_t* fault, int dev, cudaStream_t stream, const char* name) {
  auto kernel = gemm_epi_kernel<T, C, EPI, NORM>;
  cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), dev, SMEM_BYTES);
  if (err != cudaSuccess) return cuda_fail(err, name);
  float* slots = static_cast<float*>(workspace);
  int* counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + sh.slot_bytes);
  err = launch(kernel, dim3((unsigned)sh.ctas), dim3(THREADS), SMEM_BYTES, stream, ma, mb,
               static_cast<T*>(out), out_stride, (int)num_tokens, sh.m_tiles, sh.k_blocks, ep,
               counters, slots, fault);
  if (err != cudaSuccess) return cuda_fail(err, name);
  return PACE_OK;
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
  if (!qkv_out || !hidden || !weight || !positions || !cos_sin_cache || !workspace)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(qkv_out) || !aligned16(hidden) || !aligned16(weight) ||
      !aligned16(cos_sin_cache) || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: pointers must be 16-byte aligned (the workspace 256-byte aligned)", name);
  StreamDeviceGuard guard(stream);
  const int dev = guard.device();
  const QkvShape sh = qkv_shape(num_tokens, hidden_size, heads, sm_count(dev));
  if (workspace_bytes < sh.workspace_bytes)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes, %zu needed", name,
                workspace_bytes, sh.workspace_bytes);
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  int st = tc::make_kmajor_map(&ma, hidden, bf16, num_tokens, hidden_size, hidden_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, weight, bf16, n, hidden_size, hidden_size, BN, name);
  if (st != PACE_OK) return st;
  const int rot_heads = num_heads + num_kv_heads;
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
                    const void* workspace) {
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
  if (!out || !a || !w || !workspace) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(out) || !aligned16(a) || !aligned16(w) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
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
  return qkv_shape(num_tokens, k, (int)(n / HEAD), sm_count(device)).workspace_bytes;
}

extern "C" int pace_linear_residual(void* residual, const void* input, const void* weight,
                                    float* row_sumsq, int64_t num_tokens, int64_t n, int64_t k,
                                    int64_t input_row_stride, int64_t residual_row_stride,
                                    int dtype, void* workspace, size_t workspace_bytes,
                                    int32_t* fault_flags, cudaStream_t stream) {
  using namespace pace;
  const char* name = "linear_residual";
  int st = check_gemm_args(name, num_tokens, n, k, input_row_stride, residual_row_stride, dtype,
                           residual, input, weight, workspace);
  if (st != PACE_OK || num_tokens == 0) return st;
  if (n % HEAD != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: n = %lld must be a multiple of %d", name,
                (long long)n, HEAD);
  StreamDeviceGuard guard(stream);
  const int dev = guard.device();
  const QkvShape sh = qkv_shape(num_tokens, k, (int)(n / HEAD), sm_count(dev));
  if (workspace_bytes < sh.workspace_bytes)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes, %zu needed", name,
                workspace_bytes, sh.workspace_bytes);
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  st = tc::make_kmajor_map(&ma, input, bf16, num_tokens, k, input_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, weight, bf16, n, k, k, BN, name);
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
  int st = check_gemm_args(name, num_tokens, n, hidden_size, hidden_row_stride, out_row_stride,
                           dtype, qkv_out, hidden, folded_weight, workspace);
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
  if (workspace_bytes < sh.workspace_bytes)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes, %zu needed", name,
                workspace_bytes, sh.workspace_bytes);
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  st = tc::make_kmajor_map(&ma, hidden, bf16, num_tokens, hidden_size, hidden_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, folded_weight, bf16, n, hidden_size, hidden_size, BN, name);
  if (st != PACE_OK) return st;
  EpiParams ep = rope_params(positions, cos_sin_cache, max_position, num_heads + num_kv_heads,
                             heads);
  ep.sumsq_in = row_sumsq;
  ep.sumsq_in_groups = (int)sumsq_groups;
  ep.inv_k = 1.f / (float)hidden_size;
  ep.eps = epsilon;
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
constexpr size_t kNoAllocBytes = kNoAllocSlotBytes + (size_t)kNoAllocTiles * sizeof(int);
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
  void* scratch = no_alloc_scratch(dev);
  if (!scratch) return PACE_ERR_CUDA;
  QkvShape sh = qkv_shape(num_tokens, hidden_size, heads, sm_count(dev));
  if (sh.ctas > kNoAllocCtas) sh.ctas = kNoAllocCtas;
  sh.slot_bytes = kNoAllocSlotBytes;
  // The counters must start at zero.  Calls leave them zero, but one whose
  // wait expired may not: clear them on the stream first (no allocation).
  cudaError_t err = cudaMemsetAsync(static_cast<char*>(scratch) + kNoAllocSlotBytes, 0,
                                    (size_t)tiles * sizeof(int), stream);
  if (err != cudaSuccess) return cuda_fail(err, name);
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  int st = tc::make_kmajor_map(&ma, hidden, bf16, num_tokens, hidden_size, hidden_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, weight, bf16, n, hidden_size, hidden_size, BN, name);
  if (st != PACE_OK) return st;
  const int rot_heads = num_heads + num_kv_heads;
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
