// Mixture-of-experts grouped GEMMs for sm_100a (tcgen05 tensor cores).
//
// Replaces the expert computation of fused_experts
// (paceserve/model_executor/layers/fused_moe/fused_moe.py:411-544): the
// Triton fused_moe_kernel (:16-148) run once with w1, silu_and_mul on its
// output (:518-520), and the kernel again with w2 scaled by the routing
// weight (MUL_ROUTED_WEIGHT, :138-140).  The routed rows are ordered by
// moe_align_block_size with block 128, so every 128-row block of the sorted
// list belongs to one expert (expert_ids[block]):
//
//   pace_moe_gather_rows  a1[i]  = hidden[sorted_ids[i] / top_k]   (zero rows
//                         for the padding ids), so the GEMMs read A with TMA
//                         as a plain row-major matrix;
//   pace_moe_gemm MODE 0  out[i] = silu(a1[i] @ W1[e]_gate^T) * (a1[i] @ W1[e]_up^T)
//                         for the block's expert e, i in sorted order: one
//                         256-column tile holds 128 gate and the matching 128
//                         up columns, so SiLU-and-mul is applied to the fp32
//                         accumulator and the [*, 2I] intermediate never
//                         reaches HBM;
//   pace_moe_gemm MODE 1  out[sorted_ids[i]] = w[sorted_ids[i]] * (a2[i] @ W2[e]^T),
//                         scattered back to the flat (token, slot) rows that
//                         the reference's intermediate_cache3 uses.
//
// Tiles are 128 sorted rows x 256 columns, K in 64-element blocks through a
// 4-stage TMA ring (128-byte swizzle, no multicast), tcgen05.mma M=128 N=256
// into one of two TMEM accumulators, 8 epilogue warps; one persistent CTA per
// SM walks the tiles round-robin, m blocks fastest so that CTAs running
// together share an expert's weight tile in L2.  Only blocks below
// num_tokens_post_pad / 128 are walked.  Every mbarrier wait is bounded.
#include "tcgen05.cuh"

namespace pace {
namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = (EPI_WARPS + 2) * 32;
constexpr int TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait
constexpr int32_t kFaultTimeout = 1 << 30;
constexpr int kEpiBarrier = 1;

struct Ctl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(Ctl) <= 256, "");

__device__ __forceinline__ void raise_fault(Ctl* ctl, int32_t* fault) {
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
  if (fault) atomicOr(fault, kFaultTimeout);
}

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

// silu(x) = x / (1 + e^-x) in fp32 (csrc/activation_kernels.cu:8-12).
__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// The tiles this CTA owns, in order: t = cta, cta + grid, ... over the
// valid_blocks x n_tiles tiles that hold routed rows (m fastest).  Only the
// blocks below the padded total (read on the device) are walked, so every CTA
// gets the same number of tiles, give or take one.
struct TileWalk {
  int t, step, n_tiles, valid_blocks;
  __device__ __forceinline__ bool next(int& mb, int& nt) {
    if (t >= valid_blocks * n_tiles) return false;
    mb = t % valid_blocks;
    nt = t / valid_blocks;
    t += step;
    return true;
  }
};

// MODE 0: gate/up + SiLU-and-mul (out [EM, n] in sorted order, n = I);
// MODE 1: down projection times the routing weight, rows scattered to
// sorted_ids (out [numel, n], n = hidden).
// tm_a: [EM, K] (rows in sorted order); tm_b: the stacked expert weights as
// [E * rows_per_expert, K] (rows_per_expert = 2n for MODE 0, n for MODE 1).
template <typename T, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    T* __restrict__ out, int64_t out_stride, const int32_t* __restrict__ sorted_ids,
                    const int32_t* __restrict__ expert_ids, const int32_t* __restrict__ total_ptr,
                    const float* __restrict__ topk_weights, int m_blocks, int n, int k_blocks,
                    int num_experts, int64_t numel, int32_t* fault) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Ctl* ctl = reinterpret_cast<Ctl*>(tiles + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = MODE == 0 ? n / (BN / 2) : n / BN;

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
  // the sorted ids, expert ids, total and A are written by earlier kernels
  pdl_wait();
  const int total = *total_ptr;
  const int valid_blocks = min(m_blocks, (total + BM - 1) / BM);

  if (warp == EPI_WARPS) {
    // ---- TMA producer ----------------------------------------------------
    if (lane == 0) {
      TileWalk walk{(int)blockIdx.x, (int)gridDim.x, n_tiles, valid_blocks};
      int64_t i = 0;
      bool ok = true;
      int mb, nt;
      while (ok && walk.next(mb, nt)) {
        int e = expert_ids[mb];
        if (e < 0 || e >= num_experts) e = 0;  // cannot happen for moe_align output
        for (int kb = 0; kb < k_blocks; ++kb, ++i) {
          const int s = (int)(i % STAGES);
          const uint32_t use = (uint32_t)(i / STAGES);
          if (use > 0 &&
              !tc::mbar_wait(&ctl->empty[s], (use - 1) & 1u, kWaitLimitNs, &ctl->abort)) {
            ok = false;
            break;
          }
          uint8_t* a = tiles + s * STAGE_BYTES;
          tc::mbar_arrive_expect_tx(&ctl->full[s], STAGE_BYTES);
          tc::tma_load_2d(a, &tm_a, kb * BK, mb * BM, &ctl->full[s]);
          if (MODE == 0) {
            // gate rows [nt*128, +128) and up rows [n + nt*128, +128) of expert e
            const int g0 = e * 2 * n + nt * (BN / 2);
            tc::tma_load_2d(a + A_BYTES, &tm_b, kb * BK, g0, &ctl->full[s]);
            tc::tma_load_2d(a + A_BYTES + B_BYTES / 2, &tm_b, kb * BK, g0 + n, &ctl->full[s]);
          } else {
            tc::tma_load_2d(a + A_BYTES, &tm_b, kb * BK, e * n + nt * BN, &ctl->full[s]);
          }
        }
      }
      if (!ok) raise_fault(ctl, fault);
      for (int64_t q = i > STAGES ? i - STAGES : 0; q < i; ++q)
        tc::mbar_wait(&ctl->full[q % STAGES], (uint32_t)(q / STAGES) & 1u, kWaitLimitNs,
                      nullptr);
    }
  } else if (warp == EPI_WARPS + 1) {
    // ---- MMA issuer ------------------------------------------------------
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idesc = tc::umma_idesc_f16(kBf16, BM, BN);
      TileWalk walk{(int)blockIdx.x, (int)gridDim.x, n_tiles, valid_blocks};
      int64_t i = 0;
      int j = 0;
      bool ok = true;
      int mb, nt;
      while (ok && walk.next(mb, nt)) {
        const int b = j & 1;
        const uint32_t use_b = (uint32_t)(j >> 1);
        ++j;
        if (use_b > 0 &&
            !tc::mbar_wait(&ctl->tmem_empty[b], (use_b - 1) & 1u, kWaitLimitNs, &ctl->abort)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        for (int kb = 0; kb < k_blocks; ++kb, ++i) {
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
            tc::umma_f16(d, ad + 2 * k, bd + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          tc::umma_commit(&ctl->empty[s]);
        }
        if (ok) tc::umma_commit(&ctl->tmem_full[b]);
      }
      if (!ok) raise_fault(ctl, fault);
      tc::umma_commit(&ctl->drain);
      tc::mbar_wait(&ctl->drain, 0, kWaitLimitNs, nullptr);
    }
  } else {
    // ---- epilogue: warp w drains TMEM lanes 32 (w % 4) .. +31 -------------
    const int quarter = warp % 4, half = warp / 4;
    const int row = quarter * 32 + lane;
    TileWalk walk{(int)blockIdx.x, (int)gridDim.x, n_tiles, valid_blocks};
    int j = 0;
    int mb, nt;
    while (walk.next(mb, nt)) {
      const int b = j & 1;
      const uint32_t use = (uint32_t)(j >> 1);
      ++j;
      const int m = mb * BM + row;  // position in the sorted list
      int64_t dst = -1;             // output row, or -1 for none
      float wgt = 1.f;
      if (m < total) {
        if (MODE == 0) {
          dst = m;
        } else {
          const int id = sorted_ids[m];
          if (id >= 0 && id < numel) {
            dst = id;
            wgt = topk_weights[id];
          }
        }
      }
      bool ready = tc::mbar_wait(&ctl->tmem_full[b], use & 1u, kWaitLimitNs, &ctl->abort);
      ready = epi_all(ready);
      if (!ready) {
        raise_fault(ctl, fault);
        break;
      }
      tc::tc_fence_after();
      const uint32_t trow = tmem + (uint32_t)(b * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      if (MODE == 0) {
        // this warp: output columns [half*64, +64) = gate cols [half*64, +64)
        // and up cols [128 + half*64, +64) of the tile
        T* o = out + (dst >= 0 ? dst : 0) * out_stride + (int64_t)nt * (BN / 2) + half * 64;
#pragma unroll 1
        for (int c = 0; c < 64; c += 16) {
          uint32_t rg[16], ru[16];
          tc::tmem_ld16(trow + half * 64 + c, rg);
          tc::tmem_ld16(trow + BN / 2 + half * 64 + c, ru);
          tc::tmem_wait_ld(rg);
          tc::tmem_wait_ld(ru);
          float v[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = silu(__uint_as_float(rg[e])) * __uint_as_float(ru[e]);
          if (dst >= 0) store16(o + c, v);
        }
      } else {
        // this warp: columns [half*128, +128) of the tile
        T* o = out + (dst >= 0 ? dst : 0) * out_stride + (int64_t)nt * BN + half * 128;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t ra[16], rb[16];
          tc::tmem_ld16(trow + half * 128 + c, ra);
          tc::tmem_ld16(trow + half * 128 + c + 16, rb);
          tc::tmem_wait_ld(ra);
          tc::tmem_wait_ld(rb);
          float va[16], vb[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            va[e] = __uint_as_float(ra[e]) * wgt;
            vb[e] = __uint_as_float(rb[e]) * wgt;
          }
          if (dst >= 0) {
            store16(o + c, va);
            store16(o + c + 16, vb);
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl->tmem_empty[b]);
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
}

// a1[i] = in[sorted_ids[i] / top_k] for i < total; zero rows for the padding
// ids (>= numel).  One CTA per sorted row, 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(256)
    moe_gather_kernel(T* __restrict__ out, const T* __restrict__ in, const int32_t* __restrict__ sorted_ids,
                      const int32_t* __restrict__ total_ptr, int64_t numel, int top_k, int hidden,
                      int64_t in_stride, int64_t out_stride) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t i = blockIdx.x;
  if (i >= *total_ptr) return;
  const int id = sorted_ids[i];
  const bool pad = id < 0 || id >= numel;
  const uint4* src = reinterpret_cast<const uint4*>(in + (pad ? 0 : (int64_t)(id / top_k)) * in_stride);
  uint4* dst = reinterpret_cast<uint4*>(out + i * out_stride);
  const int nvec = hidden / 8;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x)
    dst[v] = pad ? make_uint4(0, 0, 0, 0) : ld_nc_v4(src + v);
}

}  // namespace
}  // namespace pace

extern "C" int pace_moe_gather_rows(void* out, const void* in, const int32_t* sorted_ids,
                                    int64_t num_sorted, const int32_t* num_tokens_post_pad,
                                    int64_t numel, int top_k, int64_t hidden,
                                    int64_t in_row_stride, int64_t out_row_stride, int dtype,
                                    cudaStream_t stream) {
  using namespace pace;
  const char* name = "moe_gather_rows";
  if (num_sorted < 0 || num_sorted > INT32_MAX || numel < 0 || top_k <= 0 || hidden <= 0 ||
      hidden > INT32_MAX)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad shape", name);
  if (dtype != PACE_BF16 && dtype != PACE_F16)
    return fail(PACE_ERR_UNSUPPORTED_DTYPE, "%s: dtype %d must be bfloat16 or float16", name,
                dtype);
  if (hidden % 8 != 0 || in_row_stride % 8 != 0 || out_row_stride % 8 != 0 ||
      in_row_stride < hidden || out_row_stride < hidden)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: hidden size and row strides must be multiples of 8 and >= the row", name);
  if (num_sorted == 0) return PACE_OK;
  if (!out || !in || !sorted_ids || !num_tokens_post_pad)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(out) || !aligned16(in))
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: pointers must be 16-byte aligned", name);
  StreamDeviceGuard guard(stream);
  cudaError_t err;
  if (dtype == PACE_BF16)
    err = launch(moe_gather_kernel<__nv_bfloat16>, dim3((unsigned)num_sorted), dim3(256), 0,
                 stream, static_cast<__nv_bfloat16*>(out),
                 static_cast<const __nv_bfloat16*>(in), sorted_ids, num_tokens_post_pad, numel,
                 top_k, (int)hidden, in_row_stride, out_row_stride);
  else
    err = launch(moe_gather_kernel<__half>, dim3((unsigned)num_sorted), dim3(256), 0, stream,
                 static_cast<__half*>(out), static_cast<const __half*>(in), sorted_ids,
                 num_tokens_post_pad, numel, top_k, (int)hidden, in_row_stride, out_row_stride);
  if (err != cudaSuccess) return cuda_fail(err, name);
  return PACE_OK;
}

extern "C" int pace_moe_gemm(void* out, const void* a, const void* w, int64_t num_sorted,
                             const int32_t* sorted_ids, const int32_t* expert_ids,
                             const int32_t* num_tokens_post_pad, int64_t numel,
                             const float* topk_weights, int num_experts, int64_t n, int64_t k,
                             int64_t a_row_stride, int64_t out_row_stride, int mode, int dtype,
                             int32_t* fault_flags, cudaStream_t stream) {
  using namespace pace;
  const char* name = "moe_gemm";
  if (mode != 0 && mode != 1)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: mode %d must be 0 (gate/up + SiLU) or 1 "
                "(down x routing weight)", name, mode);
  if (num_sorted < 0 || num_sorted > INT32_MAX || numel < 0 || num_experts <= 0 || n <= 0 ||
      k <= 0 || n > INT32_MAX || k > INT32_MAX)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad shape", name);
  const int n_unit = mode == 0 ? BN / 2 : BN;
  if (n % n_unit != 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: n = %lld must be a multiple of %d", name,
                (long long)n, n_unit);
  if (dtype != PACE_BF16 && dtype != PACE_F16)
    return fail(PACE_ERR_UNSUPPORTED_DTYPE, "%s: dtype %d must be bfloat16 or float16", name,
                dtype);
  if (k % 8 != 0 || a_row_stride % 8 != 0 || out_row_stride % 8 != 0 || a_row_stride < k ||
      out_row_stride < n)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: k and row strides must be multiples of 8 and >= the row", name);
  const int64_t w_rows = (int64_t)num_experts * (mode == 0 ? 2 * n : n);
  if (w_rows > INT32_MAX) return fail(PACE_ERR_TOO_LARGE, "%s: weights too large", name);
  if (num_sorted == 0) return PACE_OK;
  if (!out || !a || !w || !sorted_ids || !expert_ids || !num_tokens_post_pad ||
      (mode == 1 && !topk_weights))
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(out) || !aligned16(a) || !aligned16(w))
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: pointers must be 16-byte aligned", name);
  StreamDeviceGuard guard(stream);
  const int dev = guard.device();
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  int st = tc::make_kmajor_map(&ma, a, bf16, num_sorted, k, a_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = tc::make_kmajor_map(&mb, w, bf16, w_rows, k, k, mode == 0 ? BN / 2 : BN, name);
  if (st != PACE_OK) return st;
  const int m_blocks = (int)ceil_div(num_sorted, BM);
  const int n_tiles = (int)(n / n_unit);
  const int64_t tiles = (int64_t)m_blocks * n_tiles;
  if (tiles > INT32_MAX) return fail(PACE_ERR_TOO_LARGE, "%s: too many tiles", name);
  const int sms = sm_count(dev);
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  const int kb = (int)ceil_div(k, BK);
  auto go = [&](auto kernel, auto* outp) -> int {
    cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), dev, SMEM_BYTES);
    if (err != cudaSuccess) return cuda_fail(err, "moe_gemm (smem attribute)");
    err = launch(kernel, dim3(grid), dim3(THREADS), SMEM_BYTES, stream, ma, mb, outp,
                 out_row_stride, sorted_ids, expert_ids, num_tokens_post_pad, topk_weights,
                 m_blocks, (int)n, kb, num_experts, numel, fault_flags);
    if (err != cudaSuccess) return cuda_fail(err, name);
    return PACE_OK;
  };
  if (bf16) {
    auto* o = static_cast<__nv_bfloat16*>(out);
    return mode == 0 ? go(moe_gemm_kernel<__nv_bfloat16, 0>, o) : go(moe_gemm_kernel<__nv_bfloat16, 1>, o);
  }
  auto* o = static_cast<__half*>(out);
  return mode == 0 ? go(moe_gemm_kernel<__half, 0>, o) : go(moe_gemm_kernel<__half, 1>, o);
}
