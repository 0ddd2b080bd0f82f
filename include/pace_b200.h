/*
 * pace_b200.h — C ABI of the B200 (sm_100a) kernels behind PaceServe's
 * per-layer custom ops and its KV-transfer path.
 *
 * Every entry point takes plain device pointers, element counts and strides,
 * a dtype code and a cudaStream_t, launches on that stream, never allocates
 * device memory, never synchronises, and returns a PACE_* status code.  The
 * stream must belong to the calling thread's current device (the launch goes
 * to that device).  Launches may be captured into a CUDA graph.  On a
 * non-zero status, pace_last_error() returns a message for the calling thread.
 * Row strides are in ELEMENTS of the row's dtype.
 *
 * Each declaration names the reference interface it replaces
 * (paths inside the PaceServe project).
 */
#ifndef PACE_B200_H_
#define PACE_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define PACE_OK 0
#define PACE_ERR_INVALID_ARGUMENT 1 /* bad shape, stride, null pointer, k > E ... */
#define PACE_ERR_UNSUPPORTED_DTYPE 2
#define PACE_ERR_CUDA 3             /* a CUDA runtime call or launch failed     */
#define PACE_ERR_PEER_ACCESS 4      /* P2P / IPC mapping unavailable            */
#define PACE_ERR_TOO_LARGE 5        /* a size beyond what the kernel supports   */

/* ---- dtype codes ------------------------------------------------------- */
#define PACE_F32 0
#define PACE_F16 1
#define PACE_BF16 2
#define PACE_U8 3
#define PACE_I8 4
#define PACE_I16 5
#define PACE_I32 6
#define PACE_I64 7

/* Message describing the last non-zero status returned on this thread. */
const char* pace_last_error(void);
/* Static name of a status code. */
const char* pace_status_string(int status);
/* Library version as (major << 16) | (minor << 8) | patch. */
int pace_version(void);
/* Programmatic dependent launch (PDL) for the per-layer ops: 1 = on
 * (default), 0 = plain launches.  Process-wide. */
void pace_set_pdl(int enable);
int pace_get_pdl(void);

/* ---- normalisation ------------------------------------------------------
 * out[t,i] = (T)((T)(x[t,i] * rsqrt(mean_i(x[t,:]^2) + eps)) * w[i]),
 * fp32 accumulation.  dtype in {F32, F16, BF16}; weight has the same dtype.
 * Replaces rms_norm (csrc/layernorm.cpp:3-7, csrc/layernorm_kernels.cu:39-62)
 * called from RMSNorm.forward (paceserve/model_executor/layers/layernorm.py:31-40). */
int pace_rms_norm(void* out, const void* input, const void* weight, float epsilon,
                  int64_t num_tokens, int64_t hidden_size, int64_t input_row_stride,
                  int64_t out_row_stride, int dtype, cudaStream_t stream);

/* In place: residual <- (T)(input + residual); input <- rms_norm(residual).
 * Replaces the PyTorch add + RMSNorm pair at
 * paceserve/model_executor/models/llama.py:240-254 (no reference kernel). */
int pace_fused_add_rms_norm(void* input, void* residual, const void* weight, float epsilon,
                            int64_t num_tokens, int64_t hidden_size,
                            int64_t input_row_stride, int64_t residual_row_stride, int dtype,
                            cudaStream_t stream);

/* ---- rotary embedding ---------------------------------------------------
 * In place on query [T, num_heads*head_size] and key [T, num_kv_heads*head_size]
 * (row strides may exceed the row width: q/k views of a fused qkv tensor).
 * cos_sin_cache is [max_position, rot_dim] = [cos(rot_dim/2) | sin(rot_dim/2)],
 * of dtype cache_dtype (F32, or the same dtype as q/k).  is_neox: rotate pairs
 * (i, i + rot_dim/2); otherwise (2i, 2i+1).  Math in fp32.  Tokens whose
 * position lies outside [0, max_position) are left unchanged.  key may be NULL
 * when num_kv_heads == 0.
 * Replaces rotary_embedding (csrc/pos_encoding.cpp:3-9,
 * csrc/pos_encoding_kernels.cu:80-127) called from RotaryEmbedding.forward
 * (paceserve/model_executor/layers/rotary_embedding.py:87-103). */
int pace_rotary_embedding(const int64_t* positions, void* query, void* key, int64_t num_tokens,
                          int num_heads, int num_kv_heads, int head_size,
                          int64_t query_row_stride, int64_t key_row_stride,
                          const void* cos_sin_cache, int cache_dtype, int rot_dim,
                          int64_t max_position, int is_neox, int dtype, cudaStream_t stream);

/* ---- qkv projection with the rotary embedding in its epilogue ----------
 * qkv_out[T, (nq + 2 nkv) * head_size] = hidden[T, hidden_size] @ weight^T on
 * the tcgen05 tensor cores (fp32 accumulation), with heads 0 .. nq + nkv - 1
 * (q, then k) rotated as pace_rotary_embedding does (NeoX or GPT-J pairs,
 * cache [max_position, rot_dim] of cache_dtype F32 or dtype) before the one
 * rounding to dtype; v heads are stored as computed.  weight is the
 * contiguous [(nq + 2 nkv) * head_size, hidden_size] projection matrix
 * (row-major, as torch.nn.Linear holds it).  dtype in {F16, BF16}; head_size =
 * rot_dim = 128; hidden_size and both row strides multiples of 8 elements;
 * qkv_out, hidden, weight and the cache 16-byte aligned.  Tokens whose
 * position lies outside [0, max_position) are stored unrotated.
 * For one token, or two with hidden_size <= 8192 (decode batches), the
 * projection runs on the CUDA cores
 * instead: a stream of the weight through shared memory, one warp per
 * rotation pair of output columns over the whole K, the same epilogue; it
 * needs no workspace (pace_qkv_proj_rope_workspace_size returns 0, and
 * workspace may be NULL).
 * workspace: device memory of at least pace_qkv_proj_rope_workspace_size()
 * bytes (for this shape and device), 256-byte aligned, ZERO-FILLED before its
 * first use; every call leaves it valid for the next (its grid-barrier count
 * and per-tile counters back at zero, at offsets that do not depend on the
 * shape), so one zeroed workspace serves any number of stream-ordered calls
 * of any shapes that fit in it.  Calls that may run concurrently need
 * separate workspaces.  Above 32 tokens the kernel's CTAs (at most one per
 * SM) may meet at one grid-wide barrier, so they must all be resident
 * together: the call sizes its grid by the device's SM count (clusters of
 * two above 128 tokens, by cudaOccupancyMaxActiveClusters), and a context
 * limited to fewer SMs (an MPS share, a green context) sees the bounded wait
 * expire instead.
 * fault_flags (optional device int32, may be NULL): bit 30 is OR-ed in when a
 * bounded device wait expires (the output is then incomplete and the
 * workspace must be zero-filled again before reuse).
 * Replaces qkv_proj followed by rotary_emb in LlamaAttention.forward
 * (paceserve/model_executor/models/llama.py:176-178): F.linear, then
 * rotary_embedding (csrc/pos_encoding.cpp:3-9). */
size_t pace_qkv_proj_rope_workspace_size(int64_t num_tokens, int64_t hidden_size, int num_heads,
                                         int num_kv_heads, int device);
int pace_qkv_proj_rope(void* qkv_out, const void* hidden, const void* weight,
                       const int64_t* positions, int64_t num_tokens, int64_t hidden_size,
                       int num_heads, int num_kv_heads, int head_size,
                       int64_t hidden_row_stride, int64_t out_row_stride,
                       const void* cos_sin_cache, int cache_dtype, int rot_dim,
                       int64_t max_position, int is_neox, int dtype, void* workspace,
                       size_t workspace_bytes, int32_t* fault_flags, cudaStream_t stream);

/* ---- RMSNorm folded into the GEMMs around it ----------------------------
 * The decoder layer's "residual + x, then RMSNorm" (fused_add_rms_norm; in the
 * reference the add and RMSNorm.forward at paceserve/model_executor/models/
 * llama.py:240-254) split over the GEMMs that produce and consume it:
 *
 * pace_linear_residual: residual[t, :n] = (T)(residual[t] + input[t] @ weight^T)
 *   (o_proj / down_proj with the residual add in the epilogue; weight
 *   [n, k] row-major, n % 128 == 0), and, when row_sumsq is not NULL,
 *   row_sumsq[t, g] = sum of the new residual's squares over columns
 *   [32g, 32g + 32) (fp32, [T, n / 32]).  Workspace as for
 *   pace_qkv_proj_rope (pace_linear_residual_workspace_size; zero-filled
 *   before first use, left valid by every call).  For one token, or two with
 *   k <= 8192, it runs on the CUDA cores with no workspace (size 0, workspace
 *   may be NULL), and the partials come from pace_row_sumsq on the new rows,
 *   launched after it.
 * pace_row_sumsq: the same partials for rows no GEMM produced (layer 0).
 * pace_qkv_proj_rmsnorm_rope: pace_qkv_proj_rope on un-normalised rows
 *   `hidden`, with the RMSNorm applied as a per-row factor in the epilogue:
 *   qkv = rope(inv[t] * (hidden[t] @ folded_weight^T)),
 *   inv[t] = rsqrt(sum_g row_sumsq[t, g] / hidden_size + epsilon), where
 *   folded_weight[n, c] = (T)(w_qkv[n, c] * norm_weight[c]) is prepared once by
 *   the caller.  Equal to rms_norm then the projection up to the rounding of
 *   the normalised rows (the reference rounds them to T before its GEMM).
 *   row_sumsq 16-byte aligned, sumsq_groups (= hidden_size / 32) a multiple
 *   of 4.  At decode sizes it runs on the CUDA cores without a workspace, as
 *   pace_qkv_proj_rope does.
 * Replace fused_add_rms_norm + qkv_proj (llama.py:176, 240-254) and the
 * residual add after o_proj / the MLP.  No reference kernel. */
size_t pace_linear_residual_workspace_size(int64_t num_tokens, int64_t n, int64_t k, int device);
int pace_linear_residual(void* residual, const void* input, const void* weight, float* row_sumsq,
                         int64_t num_tokens, int64_t n, int64_t k, int64_t input_row_stride,
                         int64_t residual_row_stride, int dtype, void* workspace,
                         size_t workspace_bytes, int32_t* fault_flags, cudaStream_t stream);
int pace_row_sumsq(float* row_sumsq, const void* input, int64_t num_tokens, int64_t hidden_size,
                   int64_t input_row_stride, int dtype, cudaStream_t stream);
int pace_qkv_proj_rmsnorm_rope(void* qkv_out, const void* hidden, const void* folded_weight,
                               const float* row_sumsq, int64_t sumsq_groups, float epsilon,
                               const int64_t* positions, int64_t num_tokens,
                               int64_t hidden_size, int num_heads, int num_kv_heads,
                               int head_size, int64_t hidden_row_stride, int64_t out_row_stride,
                               const void* cos_sin_cache, int cache_dtype, int rot_dim,
                               int64_t max_position, int is_neox, int dtype, void* workspace,
                               size_t workspace_bytes, int32_t* fault_flags, cudaStream_t stream);

/* pace_gate_up_silu: the MLP's gate_up_proj and SiLU-and-mul in one
 * tensor-core GEMM (llama.py:70-104, activation_kernels.cu:15-45):
 *   out[t, i] = silu(g) * u,  g = s[t] * (hidden[t] @ weight[i]^T),
 *   u = s[t] * (hidden[t] @ weight[I + i]^T),
 * weight = [gate rows; up rows] ([2 I, hidden_size], the layout of the
 * reference's merged gate_up_proj, llama.py:452-469), out [T, I].  With
 * row_sumsq null s = 1 (gate_up_proj on normalised rows); with row_sumsq the
 * post-attention RMSNorm is a per-row factor s[t] = rsqrt(sum_g row_sumsq[t,
 * g] / hidden_size + epsilon) and weight holds the norm weight folded in, as
 * in pace_qkv_proj_rmsnorm_rope.  The [T, 2 I] gate_up activations are never
 * written: gate and up stay in fp32 through the activation, where the
 * reference rounds them to T first.  intermediate_size a multiple of 128;
 * workspace as pace_qkv_proj_rope (zero-filled, left zeroed, size from
 * pace_gate_up_silu_workspace_size).  For one token, or two with
 * hidden_size <= 8192, it runs on the CUDA cores (gate row i and up row I + i
 * streamed together by one warp) with no workspace: the size function
 * returns 0 and workspace may be NULL.
 * Replaces gate_up_proj + silu_and_mul
 * (llama.py:102-104).  No reference kernel. */
size_t pace_gate_up_silu_workspace_size(int64_t num_tokens, int64_t hidden_size,
                                        int64_t intermediate_size, int device);
int pace_gate_up_silu(void* out, const void* hidden, const void* weight, const float* row_sumsq,
                      int64_t sumsq_groups, float epsilon, int64_t num_tokens,
                      int64_t hidden_size, int64_t intermediate_size,
                      int64_t hidden_row_stride, int64_t out_row_stride, int dtype,
                      void* workspace, size_t workspace_bytes, int32_t* fault_flags,
                      cudaStream_t stream);

/* Allocation-free variant of pace_qkv_proj_rope.  No counterpart in the
 * reference.  For callers that cannot allocate device memory: a plugin host
 * that hands an op only its input and output buffers, or a latency-bound
 * serving loop that must not call cudaMalloc (it synchronises the device).
 * Same arguments and results as pace_qkv_proj_rope, without the workspace:
 * its scratch is a fixed array inside this library (15.8 MiB, held by every
 * GPU that loads the library until the process exits), so it runs at most 63
 * CTAs (slower than the workspace version) and rejects shapes of more than
 * 16384 output tiles of 128 x 256 (PACE_ERR_TOO_LARGE).  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture.  Every call shares the array:
 * calls that may overlap on the GPU (other streams, other host threads) race
 * and must be serialised by the caller.  Each call clears the tile counters
 * it uses on its stream (cudaMemsetAsync) before the kernel; it allocates
 * nothing.  At decode sizes (one token, or two with hidden_size <= 8192) it
 * runs the same CUDA-core kernel as pace_qkv_proj_rope, which needs no
 * scratch: no memset, no shared array, no CTA limit. */
int pace_qkv_proj_rope_no_alloc(void* qkv_out, const void* hidden, const void* weight,
                                const int64_t* positions, int64_t num_tokens,
                                int64_t hidden_size, int num_heads, int num_kv_heads,
                                int head_size, int64_t hidden_row_stride,
                                int64_t out_row_stride, const void* cos_sin_cache,
                                int cache_dtype, int rot_dim, int64_t max_position, int is_neox,
                                int dtype, int32_t* fault_flags, cudaStream_t stream);

/* ---- gated and element-wise activations ---------------------------------
 * *_and_mul: input [T, 2d] -> out [T, d], out = act(x[:, :d]) * x[:, d:].
 * Replaces silu_and_mul (csrc/activation.cpp:3-13,
 * csrc/activation_kernels.cu:29-48) called from SiluAndMul.forward
 * (paceserve/model_executor/layers/activation.py:19-24) and
 * paceserve/model_executor/layers/fused_moe/fused_moe.py:518-520.
 * gelu_and_mul (erf GELU) and gelu_tanh_and_mul have no reference kernel. */
int pace_silu_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                      int64_t input_row_stride, int64_t out_row_stride, int dtype,
                      cudaStream_t stream);
int pace_gelu_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                      int64_t input_row_stride, int64_t out_row_stride, int dtype,
                      cudaStream_t stream);
int pace_gelu_tanh_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                           int64_t input_row_stride, int64_t out_row_stride, int dtype,
                           cudaStream_t stream);
/* Element-wise [T, d] -> [T, d] tanh GELUs with the reference's rounding.
 * Replace gelu_new / gelu_fast (csrc/activation_kernels.cu:86-114, wrappers
 * paceserve/model_executor/layers/activation.py:27-43). */
int pace_gelu_new(void* out, const void* input, int64_t num_tokens, int64_t d,
                  int64_t input_row_stride, int64_t out_row_stride, int dtype,
                  cudaStream_t stream);
int pace_gelu_fast(void* out, const void* input, int64_t num_tokens, int64_t d,
                   int64_t input_row_stride, int64_t out_row_stride, int dtype,
                   cudaStream_t stream);

/* ---- MoE routing --------------------------------------------------------
 * Per row of gating_output [T, E] (fp32): softmax, then top-k by repeated
 * argmax, ties to the lowest expert index.  topk_weights/topk_indices/
 * token_expert_indices are [T, k]; token_expert_indices[t, j] = j*T + t.
 * renormalize != 0 additionally divides each row's k weights by their sum
 * (the reference does that in Python, fused_moe.py:371-372).  Needs no
 * workspace for any E.
 * Replaces topk_softmax (csrc/moe.cpp:3-8, csrc/moe_topk_softmax_kernels.cu:476-503)
 * called from fused_topk (paceserve/model_executor/layers/fused_moe/fused_moe.py:346-373). */
int pace_topk_softmax(float* topk_weights, int32_t* topk_indices,
                      int32_t* token_expert_indices, const float* gating_output,
                      int64_t num_tokens, int num_experts, int topk, int renormalize,
                      cudaStream_t stream);

/* Counting sort of the flat topk_ids [numel] (dtype U8/I8/I16/I32/I64) by
 * expert, each expert's segment padded to a multiple of block_size:
 *   sorted_token_ids[cumsum[e] + r] = i for the r-th (ascending i) entry of e,
 *   expert_ids[b] = e for b in [cumsum[e]/bs, cumsum[e+1]/bs),
 *   *num_tokens_post_pad = cumsum[E].
 * Slots not written keep their contents (the reference's caller pre-fills them
 * with numel) unless fill_padding != 0, in which case every padding slot of
 * sorted_token_ids up to sorted_capacity is set to numel.  Entries whose id is
 * outside [0, E) are skipped.  sorted_capacity must be >= numel + E*(bs-1),
 * expert_ids_capacity >= ceil(sorted_capacity / bs).
 * Replaces moe_align_block_size (csrc/moe.cpp:10-17,
 * csrc/moe_align_block_size_kernels.cu:112-135) called from
 * paceserve/model_executor/layers/fused_moe/fused_moe.py:151-204. */
int pace_moe_align_block_size(const void* topk_ids, int ids_dtype, int64_t numel,
                              int num_experts, int block_size, int32_t* sorted_token_ids,
                              int64_t sorted_capacity, int32_t* expert_ids,
                              int64_t expert_ids_capacity, int32_t* num_tokens_post_pad,
                              int fill_padding, cudaStream_t stream);

/* ---- MoE expert GEMMs (tcgen05) -----------------------------------------
 * The expert computation of fused_experts
 * (paceserve/model_executor/layers/fused_moe/fused_moe.py:411-544: the Triton
 * fused_moe_kernel at :16-148 with w1, silu_and_mul, then with w2 and
 * MUL_ROUTED_WEIGHT), over the routing of pace_moe_align_block_size with
 * block_size 128: sorted_token_ids [num_sorted] (padding id = numel =
 * T * top_k), expert_ids [num_sorted / 128], num_tokens_post_pad [1], all on
 * the device.  dtype in {F16, BF16}; rows 16-byte aligned, widths and row
 * strides multiples of 8 elements.
 *
 * pace_moe_gather_rows: out[i] = in[sorted_token_ids[i] / top_k] for
 * i < num_tokens_post_pad, zero rows for padding ids; rows past the padded
 * total are left untouched. */
int pace_moe_gather_rows(void* out, const void* in, const int32_t* sorted_token_ids,
                         int64_t num_sorted, const int32_t* num_tokens_post_pad, int64_t numel,
                         int top_k, int64_t hidden, int64_t in_row_stride,
                         int64_t out_row_stride, int dtype, cudaStream_t stream);
/* pace_moe_gemm, mode 0: out[i, :n] = silu(a[i] @ w[e, :n]^T) * (a[i] @ w[e, n:2n]^T)
 *   for the sorted rows i < num_tokens_post_pad, e = expert_ids[i / 128]; w is
 *   the contiguous [E, 2n, k] gate/up weight (w1), out is [num_sorted, n].
 *   SiLU in fp32 on the fp32 accumulator, one rounding.  n % 128 == 0.
 * mode 1: out[id, :n] = topk_weights[id] * (a[i] @ w[e]^T) with id =
 *   sorted_token_ids[i] < numel; w is the contiguous [E, n, k] weight (w2), out
 *   is [numel, n] (the reference's intermediate_cache3).  n % 256 == 0.
 * a is [num_sorted, k] in sorted order (mode 0: pace_moe_gather_rows output;
 * mode 1: the mode 0 output).  fault_flags (optional device int32): bit 30 is
 * OR-ed in when a bounded device wait expires. */
int pace_moe_gemm(void* out, const void* a, const void* w, int64_t num_sorted,
                  const int32_t* sorted_token_ids, const int32_t* expert_ids,
                  const int32_t* num_tokens_post_pad, int64_t numel, const float* topk_weights,
                  int num_experts, int64_t n, int64_t k, int64_t a_row_stride,
                  int64_t out_row_stride, int mode, int dtype, int32_t* fault_flags,
                  cudaStream_t stream);

/* ---- paged-KV block transfer --------------------------------------------
 * A KV cache is one tensor per layer, [num_blocks, 2, block_size, kv_heads,
 * head_dim], so block b of layer l is the contiguous slab of block_bytes
 * bytes at layer_ptr[l] + b * block_bytes.
 *
 * Copy, for every layer l < num_layers and pair j < num_pairs, the slab
 * src_block_ids[j] of src_layers[l] onto slab dst_block_ids[j] of dst_layers[l].
 * src_layers / dst_layers are HOST arrays of num_layers device pointers (each
 * may be a peer device's memory, reachable after pace_enable_peer_access or
 * through pace_ipc_open_handle); the two id arrays are DEVICE int32 arrays.
 * The kernel runs on the current device (the stream's): the destination's device pulls over
 * NVLink, the source's device pushes.  Pairs with an id outside
 * [0, src_num_blocks) / [0, dst_num_blocks) are skipped and counted into
 * *bad_pairs (device int32; the caller zeroes it).  Destination slabs must not
 * overlap source slabs.  method: 0 = automatic, 1 = SIMT 16-byte vector copy,
 * 2 = bulk-async (TMA engine) copy staged through shared memory.  bad_pairs
 * may be NULL for methods 0 and 1; method 2 requires it, because its bounded
 * waits report a timeout only there: PACE_KV_TIMEOUT_FLAG is OR-ed into
 * *bad_pairs when a wait expired (that CTA stops copying, so the copy is
 * incomplete), and PACE_KV_DRAIN_TIMEOUT_FLAG as well when a load was still
 * in flight after a second wait -- it may then land in shared memory after
 * the kernel exits, and the device must not be trusted further.  The return
 * value only reports the launch.  block_bytes must be a multiple of 16 and
 * every layer pointer 16-byte aligned.
 * Replaces the GPU->CPU->GPU move of KVhelper.get_kv_cache/insert_kv_cache
 * (paceserve/kv_transfer/kv_utils.py:33-56) used by BaseWorker._get_kv_cache/
 * _insert_kv_cache (paceserve/worker/base_worker.py:236-281). */
int pace_kv_copy_blocks(void* const* src_layers, void* const* dst_layers, int num_layers,
                        const int32_t* src_block_ids, const int32_t* dst_block_ids,
                        int64_t num_pairs, int64_t block_bytes, int64_t src_num_blocks,
                        int64_t dst_num_blocks, int32_t* bad_pairs, int method,
                        cudaStream_t stream);

/* Flags OR-ed into *bad_pairs by the bulk method (see pace_kv_copy_blocks). */
#define PACE_KV_TIMEOUT_FLAG (1 << 30)
#define PACE_KV_DRAIN_TIMEOUT_FLAG (1 << 29)

/* Options of pace_kv_copy_blocks_ex.  Zero-initialise, then set fields. */
typedef struct pace_kv_copy_opts {
  int method;             /* as pace_kv_copy_blocks */
  int max_ctas;           /* > 0: at most this many CTAs (a budget of SMs left to
                             other work on the device); 0: no cap */
  uint64_t wait_limit_ns; /* bulk method: bound of every wait; 0 = 2 s */
  int test_overarm_bytes; /* TESTS ONLY, must be 0 otherwise: with method 2, the
                             first load of CTA 0 tells its barrier to expect this
                             many bytes (a multiple of 16) more than it copies, so
                             that wait expires -- how the timeout path is tested
                             without a GPU fault */
} pace_kv_copy_opts;

/* pace_kv_copy_blocks with options: a CTA budget and the bulk method's wait
 * bound.  New: no reference counterpart (the reference moves KV through the
 * host, paceserve/kv_transfer/kv_utils.py:33-56). */
int pace_kv_copy_blocks_ex(void* const* src_layers, void* const* dst_layers, int num_layers,
                           const int32_t* src_block_ids, const int32_t* dst_block_ids,
                           int64_t num_pairs, int64_t block_bytes, int64_t src_num_blocks,
                           int64_t dst_num_blocks, int32_t* bad_pairs,
                           const pace_kv_copy_opts* opts, cudaStream_t stream);

/* The same block copy on the copy engines: no kernel, no SM.  Block ids are
 * HOST int32 arrays (the block manager's tables).  Pairs are ordered by source
 * id; each run of pairs whose source and destination ids are both consecutive
 * becomes one cudaMemcpyAsync per layer, or one cudaMemcpy2DAsync covering all
 * layers when both layer tables are evenly spaced.  Invalid pairs are skipped
 * and their number stored in *bad_pairs (host, may be NULL); *copies_issued
 * (host, may be NULL) receives the number of copies queued on `stream`.  The
 * host cost grows with the number of runs, so fragmented block tables make
 * this path slower to issue than the kernel.  Duplicate destination ids leave
 * that block with one of their sources, unspecified which.
 * Replaces, like pace_kv_copy_blocks, the host round trip of
 * paceserve/kv_transfer/kv_utils.py:33-56. */
int pace_kv_copy_blocks_ce(void* const* src_layers, void* const* dst_layers, int num_layers,
                           const int32_t* src_block_ids, const int32_t* dst_block_ids,
                           int64_t num_pairs, int64_t block_bytes, int64_t src_num_blocks,
                           int64_t dst_num_blocks, int64_t* bad_pairs, int64_t* copies_issued,
                           cudaStream_t stream);

/* Gather blocks block_ids[0..n) of every layer into out, laid out
 * [num_layers, n, block_bytes] contiguous.  out may be device memory or
 * page-locked host memory mapped into the device (zero-copy).
 * Replaces KVhelper.get_kv_cache's per-layer fancy-index gather
 * (paceserve/kv_transfer/kv_utils.py:44-46). */
int pace_kv_gather_blocks(void* const* layers, int num_layers, const int32_t* block_ids,
                          int64_t n, int64_t block_bytes, int64_t num_blocks, void* out,
                          int32_t* bad_ids, cudaStream_t stream);

/* Scatter in = [num_layers, n, block_bytes] onto blocks block_ids[0..n) of every
 * layer (inverse of pace_kv_gather_blocks).
 * Replaces KVhelper.insert_kv_cache (paceserve/kv_transfer/kv_utils.py:49-56). */
int pace_kv_scatter_blocks(const void* in, void* const* layers, int num_layers,
                           const int32_t* block_ids, int64_t n, int64_t block_bytes,
                           int64_t num_blocks, int32_t* bad_ids, cudaStream_t stream);

/* ---- paged-KV append -----------------------------------------------------
 * Write nnz new tokens' K and V rows ([kv_heads * head_dim] each, row strides
 * in elements: the k/v views of a fused qkv tensor) into the paged cache
 * [num_pages, 2, page_size, kv_heads, head_dim] (K at index 0, V at 1).  Token
 * i belongs to request b = batch_indices[i] at sequence position
 * p = positions[i] and lands on page kv_indices[kv_indptr[b] + p / page_size],
 * slot p % page_size.  kv_indptr has batch_size + 1 entries, kv_indices
 * num_kv_indices; a request's length is (pages - 1) * page_size +
 * kv_last_page_len[b].  Tokens whose request, position or page is out of range
 * are skipped and counted into *bad_tokens (device int32, may be NULL).
 * Replaces flashinfer.page.append_paged_kv_cache (FlashInfer 0.2.0, pinned in
 * PaceServe's requirements.txt:40), called at
 * paceserve/model_executor/attention/flashinfer_attention_wrapper.py:245-255. */
int pace_append_paged_kv_cache(const void* key, const void* value, int64_t nnz,
                               int num_kv_heads, int head_dim, int64_t key_row_stride,
                               int64_t value_row_stride, const int32_t* batch_indices,
                               const int32_t* positions, void* paged_cache, int64_t num_pages,
                               int page_size, const int32_t* kv_indices, int64_t num_kv_indices,
                               const int32_t* kv_indptr, const int32_t* kv_last_page_len,
                               int64_t batch_size, int32_t* bad_tokens, int dtype,
                               cudaStream_t stream);

/* Same, with each token's request and position derived in the kernel from
 * append_indptr [batch_size + 1]: request b's tokens are the last
 * append_indptr[b+1] - append_indptr[b] tokens of its sequence.  Replaces
 * the get_seq_lens + get_batch_indices_positions + append_paged_kv_cache
 * sequence at flashinfer_attention_wrapper.py:239-255 with one launch. */
int pace_append_paged_kv_cache_by_indptr(const void* key, const void* value, int64_t nnz,
                                         int num_kv_heads, int head_dim,
                                         int64_t key_row_stride, int64_t value_row_stride,
                                         const int32_t* append_indptr, void* paged_cache,
                                         int64_t num_pages, int page_size,
                                         const int32_t* kv_indices, int64_t num_kv_indices,
                                         const int32_t* kv_indptr,
                                         const int32_t* kv_last_page_len, int64_t batch_size,
                                         int32_t* bad_tokens, int dtype, cudaStream_t stream);

/* ---- peer access and CUDA IPC (KV promotion across processes) ----------- */
#define PACE_IPC_HANDLE_BYTES 64
/* Make `peer`'s memory addressable from `device` (idempotent).  New: the
 * reference moves KV through the Ray object store instead. */
int pace_enable_peer_access(int device, int peer);
/* *can = 1 if `device` can address `peer`'s memory directly. */
int pace_can_access_peer(int device, int peer, int* can);
/* Export the allocation holding dev_ptr: writes PACE_IPC_HANDLE_BYTES bytes to
 * handle_out and the byte offset of dev_ptr inside that allocation. */
int pace_ipc_get_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out);
/* Map an exported allocation into this process on `device`; *base_out is the
 * allocation's base (add the exporter's offset). */
int pace_ipc_open_handle(const void* handle, int device, void** base_out);
/* Unmap a base returned by pace_ipc_open_handle.  The caller must first make
 * sure no launched copy still reads or writes the mapping (synchronise the
 * streams that used it). */
int pace_ipc_close_handle(void* base);

#ifdef __cplusplus
}
#endif

#endif /* PACE_B200_H_ */
