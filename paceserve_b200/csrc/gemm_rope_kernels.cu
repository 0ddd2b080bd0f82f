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
// Tiling: one 128 x 128 output tile per CTA, 128 columns = one head, so both
// halves of every NeoX pair (i, i + 64) and every GPT-J pair (2i, 2i + 1) sit
// in the same tile.  K is consumed in 64-element (128-byte) blocks through a
// 4-stage shared-memory ring filled by TMA (128-byte swizzle, no multicast).
// Warp roles: warps 0-3 run the epilogue (warp w owns TMEM lanes 32w..32w+31,
// i.e. tile rows), warp 4 issues the TMA loads, warp 5 issues tcgen05.mma
// (M=128, N=128, K=16, fp32 accumulator in 128 TMEM columns) and commits each
// stage back to the producer.  Every mbarrier wait is bounded by %globaltimer;
// on expiry the CTA records bit 30 in the caller's fault word, stops issuing,
// waits (bounded again) for its own copies and MMAs, frees TMEM and returns.
#include "tcgen05.cuh"

namespace pace {
namespace {

constexpr int BM = 128, BN = 128, BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = (EPI_WARPS + 2) * 32;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait
constexpr int32_t kFaultTimeout = 1 << 30;

struct Ctl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t accum;
  uint64_t drain;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(Ctl) <= 256, "");

__device__ __forceinline__ void raise_fault(Ctl* ctl, int32_t* fault) {
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
  if (fault) atomicOr(fault, kFaultTimeout);
}

// 16 cache entries starting at p (16-byte aligned) as floats.
template <typename C>
__device__ __forceinline__ void load16(const C* p, float* out) {
  if constexpr (sizeof(C) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p) + i);
      out[4 * i] = v.x;
      out[4 * i + 1] = v.y;
      out[4 * i + 2] = v.z;
      out[4 * i + 3] = v.w;
    }
  } else {
    Traits<C>::unpack(__ldg(reinterpret_cast<const uint4*>(p)), out);
    Traits<C>::unpack(__ldg(reinterpret_cast<const uint4*>(p) + 1), out + 8);
  }
}

// 8 cache entries starting at p (16-byte aligned) as floats.
template <typename C>
__device__ __forceinline__ void load8(const C* p, float* out) {
  if constexpr (sizeof(C) == 4) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p) + i);
      out[4 * i] = v.x;
      out[4 * i + 1] = v.y;
      out[4 * i + 2] = v.z;
      out[4 * i + 3] = v.w;
    }
  } else {
    Traits<C>::unpack(__ldg(reinterpret_cast<const uint4*>(p)), out);
  }
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* v) {
  st_v4(p, Traits<T>::pack(v));
  st_v4(p + 8, Traits<T>::pack(v + 8));
}

template <int N>
__device__ __forceinline__ void as_float(const uint32_t (&r)[N], float* f) {
#pragma unroll
  for (int i = 0; i < N; ++i) f[i] = __uint_as_float(r[i]);
}

// grid (m tiles, heads): m fastest, so the CTAs resident together share
// weight tiles through L2 and every weight byte is fetched from HBM once.
template <typename T, typename C, bool NEOX>
__global__ void __launch_bounds__(THREADS, 1)
    qkv_rope_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    T* __restrict__ out, int64_t out_stride, const int64_t* __restrict__ positions,
                    const C* __restrict__ cache, int64_t max_position, int num_tokens,
                    int rot_heads, int k_blocks, int32_t* fault) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Ctl* ctl = reinterpret_cast<Ctl*>(tiles + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM;
  const int head = blockIdx.y;
  const int n0 = head * BN;

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&ctl->full[s], 1);
      tc::mbar_init(&ctl->empty[s], 1);
    }
    tc::mbar_init(&ctl->accum, 1);
    tc::mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == EPI_WARPS && lane == 0) {
    tc::tma_prefetch_desc(&tm_a);
    tc::tma_prefetch_desc(&tm_b);
  }
  if (warp == 0) tc::tmem_alloc(&ctl->tmem, BN);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = ctl->tmem;
  // hidden states and positions may be written by the previous kernel
  pdl_wait();

  if (warp == EPI_WARPS) {
    // ---- TMA producer --------------------------------------------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int kb = 0; kb < k_blocks; ++kb) {
        const int s = kb % STAGES;
        const uint32_t use = (uint32_t)(kb / STAGES);
        if (use > 0 && !tc::mbar_wait(&ctl->empty[s], (use - 1) & 1u, kWaitLimitNs, &ctl->abort)) {
          ok = false;
          break;
        }
        uint8_t* a = tiles + s * STAGE_BYTES;
        tc::mbar_arrive_expect_tx(&ctl->full[s], STAGE_BYTES);
        tc::tma_load_2d(a, &tm_a, kb * BK, m0, &ctl->full[s]);
        tc::tma_load_2d(a + A_BYTES, &tm_b, kb * BK, n0, &ctl->full[s]);
        issued = kb + 1;
      }
      if (!ok) {
        raise_fault(ctl, fault);
        // let every copy already issued land before the CTA's memory is released
        for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; ++kb)
          tc::mbar_wait(&ctl->full[kb % STAGES], (uint32_t)(kb / STAGES) & 1u, kWaitLimitNs,
                        nullptr);
      }
    }
  } else if (warp == EPI_WARPS + 1) {
    // ---- MMA issuer ----------------------------------------------------
    if (lane == 0) {
      constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
      constexpr uint32_t idesc = tc::umma_idesc_f16(kBf16, BM, BN);
      bool ok = true;
      for (int kb = 0; kb < k_blocks; ++kb) {
        const int s = kb % STAGES;
        if (!tc::mbar_wait(&ctl->full[s], (uint32_t)(kb / STAGES) & 1u, kWaitLimitNs,
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
          tc::umma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
        tc::umma_commit(&ctl->empty[s]);
      }
      if (ok) {
        tc::umma_commit(&ctl->accum);
      } else {
        raise_fault(ctl, fault);
        tc::umma_commit(&ctl->drain);
        tc::mbar_wait(&ctl->drain, 0, kWaitLimitNs, nullptr);
      }
    }
  } else {
    // ---- epilogue: TMEM -> rotate -> global ----------------------------
    bool ready = tc::mbar_wait(&ctl->accum, 0, kWaitLimitNs, &ctl->abort);
    ready = __all_sync(0xffffffffu, ready);
    if (ready) {
      tc::tc_fence_after();
      const int r = warp * 32 + lane;
      const int m = m0 + r;
      const bool row_ok = m < num_tokens;
      const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
      T* orow = out + (int64_t)(row_ok ? m : 0) * out_stride + n0;
      bool rot = false;
      const C* cs = cache;
      if (row_ok && head < rot_heads) {
        const int64_t pos = positions[m];
        rot = pos >= 0 && pos < max_position;
        if (rot) cs = cache + pos * BN;
      }
      if (NEOX) {
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 16) {
          uint32_t xr[16], yr[16];
          tc::tmem_ld16(trow + c, xr);
          tc::tmem_ld16(trow + BN / 2 + c, yr);
          tc::tmem_wait_ld(xr);
          tc::tmem_wait_ld(yr);
          float x[16], y[16];
          as_float(xr, x);
          as_float(yr, y);
          if (rot) {
            float cv[16], sv[16], xo[16], yo[16];
            load16(cs + c, cv);
            load16(cs + BN / 2 + c, sv);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              xo[e] = x[e] * cv[e] - y[e] * sv[e];
              yo[e] = y[e] * cv[e] + x[e] * sv[e];
            }
            if (row_ok) {
              store16(orow + c, xo);
              store16(orow + BN / 2 + c, yo);
            }
          } else if (row_ok) {
            store16(orow + c, x);
            store16(orow + BN / 2 + c, y);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          uint32_t ar[16];
          tc::tmem_ld16(trow + c, ar);
          tc::tmem_wait_ld(ar);
          float a[16];
          as_float(ar, a);
          if (rot) {
            // pairs (c + 2p, c + 2p + 1) use cache entries c/2 + p
            float cv[8], sv[8], o[16];
            load8(cs + c / 2, cv);
            load8(cs + BN / 2 + c / 2, sv);
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              o[2 * p] = a[2 * p] * cv[p] - a[2 * p + 1] * sv[p];
              o[2 * p + 1] = a[2 * p + 1] * cv[p] + a[2 * p] * sv[p];
            }
            if (row_ok) store16(orow + c, o);
          } else if (row_ok) {
            store16(orow + c, a);
          }
        }
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, BN);
}

// ---------------------------------------------------------------- host ----
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver, looked up once (no link-time
// dependency on libcuda).
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// K-major [rows, cols] 16-bit matrix with a row stride, boxes of
// box_rows x 64 elements, 128-byte swizzle.  Rows and columns past the end
// read as zero.
int make_kmajor_map(CUtensorMap* map, const void* base, bool bf16, int64_t rows, int64_t cols,
                    int64_t row_stride, int box_rows, const char* name) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(PACE_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", name);
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: tensor map rejected (CUresult %d)", name, (int)r);
  return PACE_OK;
}

template <typename T, typename C, bool NEOX>
int launch_qkv_rope(const CUtensorMap& ma, const CUtensorMap& mb, void* out, int64_t out_stride,
                    const int64_t* positions, const void* cache, int64_t max_position,
                    int64_t num_tokens, int heads, int rot_heads, int k_blocks, int32_t* fault,
                    int dev, cudaStream_t stream) {
  auto kernel = qkv_rope_kernel<T, C, NEOX>;
  cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), dev, SMEM_BYTES);
  if (err != cudaSuccess) return cuda_fail(err, "qkv_proj_rope (smem attribute)");
  const dim3 grid((unsigned)ceil_div(num_tokens, BM), (unsigned)heads);
  err = launch(kernel, grid, dim3(THREADS), SMEM_BYTES, stream, ma, mb, static_cast<T*>(out),
               out_stride, positions, static_cast<const C*>(cache), max_position,
               (int)num_tokens, rot_heads, k_blocks, fault);
  if (err != cudaSuccess) return cuda_fail(err, "qkv_proj_rope");
  return PACE_OK;
}

}  // namespace
}  // namespace pace

extern "C" int pace_qkv_proj_rope(void* qkv_out, const void* hidden, const void* weight,
                                  const int64_t* positions, int64_t num_tokens,
                                  int64_t hidden_size, int num_heads, int num_kv_heads,
                                  int head_size, int64_t hidden_row_stride,
                                  int64_t out_row_stride, const void* cos_sin_cache,
                                  int cache_dtype, int rot_dim, int64_t max_position, int is_neox,
                                  int dtype, int32_t* fault_flags, cudaStream_t stream) {
  using namespace pace;
  const char* name = "qkv_proj_rope";
  if (num_tokens < 0 || num_tokens > INT32_MAX || hidden_size <= 0 || num_heads < 0 ||
      num_kv_heads < 0 || num_heads + num_kv_heads <= 0)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: bad shape", name);
  if (head_size != BN || rot_dim != head_size)
    return fail(PACE_ERR_INVALID_ARGUMENT,
                "%s: head_size and rot_dim must both be %d (got %d, %d)", name, BN, head_size,
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
  if (max_position <= 0) return fail(PACE_ERR_INVALID_ARGUMENT, "%s: empty cos_sin_cache", name);
  if (num_tokens == 0) return PACE_OK;
  if (!qkv_out || !hidden || !weight || !positions || !cos_sin_cache)
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(qkv_out) || !aligned16(hidden) || !aligned16(weight) || !aligned16(cos_sin_cache))
    return fail(PACE_ERR_INVALID_ARGUMENT, "%s: pointers must be 16-byte aligned", name);
  if (ceil_div(hidden_size, BK) > INT32_MAX)
    return fail(PACE_ERR_TOO_LARGE, "%s: hidden size too large", name);
  StreamDeviceGuard guard(stream);
  const bool bf16 = dtype == PACE_BF16;
  CUtensorMap ma, mb;
  int st = make_kmajor_map(&ma, hidden, bf16, num_tokens, hidden_size, hidden_row_stride, BM, name);
  if (st != PACE_OK) return st;
  st = make_kmajor_map(&mb, weight, bf16, n, hidden_size, hidden_size, BN, name);
  if (st != PACE_OK) return st;
  const int rot_heads = num_heads + num_kv_heads;
  const int kb = (int)ceil_div(hidden_size, BK);
  const int dev = guard.device();
#define PACE_QKV_ROPE(T, C, NX)                                                                  \
  launch_qkv_rope<T, C, NX>(ma, mb, qkv_out, out_row_stride, positions, cos_sin_cache,          \
                            max_position, num_tokens, heads, rot_heads, kb, fault_flags, dev, \
                            stream)
  const bool neox = is_neox != 0;
  const bool f32c = cache_dtype == PACE_F32;
  if (bf16) {
    if (f32c) return neox ? PACE_QKV_ROPE(__nv_bfloat16, float, true) : PACE_QKV_ROPE(__nv_bfloat16, float, false);
    return neox ? PACE_QKV_ROPE(__nv_bfloat16, __nv_bfloat16, true)
                : PACE_QKV_ROPE(__nv_bfloat16, __nv_bfloat16, false);
  }
  if (f32c) return neox ? PACE_QKV_ROPE(__half, float, true) : PACE_QKV_ROPE(__half, float, false);
  return neox ? PACE_QKV_ROPE(__half, __half, true) : PACE_QKV_ROPE(__half, __half, false);
#undef PACE_QKV_ROPE
}
