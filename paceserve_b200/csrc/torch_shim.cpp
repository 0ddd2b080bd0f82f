// Thin torch extension over the C ABI (include/pace_b200.h).  It recreates
// the reference's four pybind modules with their exact signatures
// (csrc/layernorm.cpp:3-14, csrc/pos_encoding.cpp:3-16,
// csrc/activation.cpp:3-28, csrc/moe.cpp:3-28) as submodules
// layernorm_ops / pos_encoding_ops / activation_ops / moe_ops of
// paceserve_b200._C, adds the new ops (fused_add_rms_norm, gelu_and_mul,
// gelu_tanh_and_mul) in the same style, and a kv_transfer_ops submodule for
// the paged-KV block copy.  Tensors are validated here; every launch goes
// through the C ABI on the current stream of the tensors' device, and a
// non-zero status becomes a RuntimeError carrying pace_last_error().
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "pace_b200.h"

namespace {

using torch::Tensor;

int pace_dtype(const Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return PACE_F32;
    case at::kHalf: return PACE_F16;
    case at::kBFloat16: return PACE_BF16;
    case at::kByte: return PACE_U8;
    case at::kChar: return PACE_I8;
    case at::kShort: return PACE_I16;
    case at::kInt: return PACE_I32;
    case at::kLong: return PACE_I64;
    default: return -1;
  }
}

void check_status(int rc, const char* op) {
  TORCH_CHECK(rc == PACE_OK, op, " failed (", pace_status_string(rc), "): ", pace_last_error());
}

cudaStream_t stream_of(const Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

void check_cuda(const Tensor& t, const char* op, const char* name) {
  TORCH_CHECK(t.is_cuda(), op, ": ", name, " must be a CUDA tensor");
}

void check_same_device(const Tensor& a, const Tensor& b, const char* op) {
  TORCH_CHECK(a.device() == b.device(), op, ": tensors on different devices (", a.device(), " vs ",
              b.device(), ")");
}

// Device pointer of an optional int32 counter the kernel adds to, or null.  It
// must live on the launching device: a host pointer would reach the kernel.
int32_t* counter_ptr(const c10::optional<Tensor>& t, const at::Device& dev, const char* op,
                     const char* name) {
  if (!t.has_value()) return nullptr;
  TORCH_CHECK(t->is_cuda() && t->device() == dev && t->scalar_type() == at::kInt &&
                  t->numel() >= 1,
              op, ": ", name, " must be an int32 tensor with at least one element on ", dev);
  return t->data_ptr<int32_t>();
}

bool is_float_type(const Tensor& t) {
  return t.scalar_type() == at::kFloat || t.scalar_type() == at::kHalf ||
         t.scalar_type() == at::kBFloat16;
}

// Row view of a tensor whose last dimension is contiguous: (rows, width,
// row_stride).  2-D tensors may have any row stride; higher ranks must be
// collapsible into rows with a single stride.
struct Rows {
  int64_t rows, width, stride;
};

Rows rows_of(const Tensor& t, const char* op, const char* name) {
  TORCH_CHECK(t.dim() >= 1, op, ": ", name, " must have at least one dimension");
  const int64_t w = t.size(-1);
  TORCH_CHECK(t.numel() == 0 || w == 1 || t.stride(-1) == 1, op, ": ", name,
              " must be contiguous in its last dimension");
  if (t.dim() == 1) return {1, w, w};
  if (t.dim() == 2) return {t.size(0), w, t.size(0) <= 1 ? w : t.stride(0)};
  TORCH_CHECK(t.is_contiguous(), op, ": ", name, " of rank > 2 must be contiguous");
  return {w == 0 ? 0 : t.numel() / w, w, w};
}

// ------------------------------------------------------------- layernorm --
void rms_norm(Tensor& out, Tensor& input, Tensor& weight, double epsilon) {
  const char* op = "rms_norm";
  check_cuda(input, op, "input");
  check_same_device(out, input, op);
  check_same_device(weight, input, op);
  TORCH_CHECK(is_float_type(input), op, ": input dtype must be float32, float16 or bfloat16");
  TORCH_CHECK(out.scalar_type() == input.scalar_type() && weight.scalar_type() == input.scalar_type(),
              op, ": out, input and weight must share a dtype");
  const Rows in = rows_of(input, op, "input");
  const Rows o = rows_of(out, op, "out");
  TORCH_CHECK(o.rows == in.rows && o.width == in.width, op, ": out shape ", out.sizes(),
              " does not match input ", input.sizes());
  TORCH_CHECK(weight.is_contiguous() && weight.numel() == in.width, op, ": weight must be [",
              in.width, "] and contiguous");
  const at::cuda::CUDAGuard guard(input.device());
  check_status(pace_rms_norm(out.data_ptr(), input.data_ptr(), weight.data_ptr(), (float)epsilon,
                             in.rows, in.width, in.stride, o.stride, pace_dtype(input),
                             stream_of(input)),
               op);
}

void fused_add_rms_norm(Tensor& input, Tensor& residual, Tensor& weight, double epsilon) {
  const char* op = "fused_add_rms_norm";
  check_cuda(input, op, "input");
  check_same_device(residual, input, op);
  check_same_device(weight, input, op);
  TORCH_CHECK(is_float_type(input), op, ": input dtype must be float32, float16 or bfloat16");
  TORCH_CHECK(residual.scalar_type() == input.scalar_type() &&
                  weight.scalar_type() == input.scalar_type(),
              op, ": input, residual and weight must share a dtype");
  const Rows in = rows_of(input, op, "input");
  const Rows r = rows_of(residual, op, "residual");
  TORCH_CHECK(r.rows == in.rows && r.width == in.width, op, ": residual shape ", residual.sizes(),
              " does not match input ", input.sizes());
  TORCH_CHECK(weight.is_contiguous() && weight.numel() == in.width, op, ": weight must be [",
              in.width, "] and contiguous");
  const at::cuda::CUDAGuard guard(input.device());
  check_status(pace_fused_add_rms_norm(input.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                                       (float)epsilon, in.rows, in.width, in.stride, r.stride,
                                       pace_dtype(input), stream_of(input)),
               op);
}

// ---------------------------------------------------------- pos encoding --
// q/k as [T, heads * head_size] (any row stride) or [T, heads, head_size].
Rows qk_rows(const Tensor& t, int64_t head_size, const char* op, const char* name) {
  TORCH_CHECK(t.dim() == 2 || t.dim() == 3, op, ": ", name, " must be 2-D or 3-D");
  TORCH_CHECK(t.size(-1) <= 1 || t.stride(-1) == 1, op, ": ", name,
              " must be contiguous in its last dimension");
  if (t.dim() == 3) {
    TORCH_CHECK(t.size(2) == head_size, op, ": ", name, " last dim must equal head_size");
    TORCH_CHECK(t.size(1) <= 1 || t.stride(1) == head_size, op, ": ", name,
                " heads must be contiguous");
    return {t.size(0), t.size(1) * head_size, t.size(0) <= 1 ? t.size(1) * head_size : t.stride(0)};
  }
  TORCH_CHECK(t.size(1) % head_size == 0, op, ": ", name, " width ", t.size(1),
              " is not a multiple of head_size ", head_size);
  return {t.size(0), t.size(1), t.size(0) <= 1 ? t.size(1) : t.stride(0)};
}

void rotary_embedding(Tensor& positions, Tensor& query, Tensor& key, int64_t head_size,
                      Tensor& cos_sin_cache, bool is_neox) {
  const char* op = "rotary_embedding";
  check_cuda(query, op, "query");
  check_same_device(positions, query, op);
  check_same_device(key, query, op);
  check_same_device(cos_sin_cache, query, op);
  TORCH_CHECK(head_size > 0, op, ": head_size must be positive");
  TORCH_CHECK(is_float_type(query) && key.scalar_type() == query.scalar_type(), op,
              ": query and key must share a float dtype");
  TORCH_CHECK(positions.scalar_type() == at::kLong && positions.is_contiguous(), op,
              ": positions must be a contiguous int64 tensor");
  TORCH_CHECK(cos_sin_cache.dim() == 2 && cos_sin_cache.is_contiguous(), op,
              ": cos_sin_cache must be a contiguous [max_position, rot_dim] tensor");
  TORCH_CHECK(cos_sin_cache.scalar_type() == at::kFloat ||
                  cos_sin_cache.scalar_type() == query.scalar_type(),
              op, ": cos_sin_cache must be float32 or the query dtype");
  const Rows q = qk_rows(query, head_size, op, "query");
  const Rows k = qk_rows(key, head_size, op, "key");
  TORCH_CHECK(k.rows == q.rows, op, ": query and key token counts differ");
  TORCH_CHECK(positions.numel() >= q.rows, op, ": positions has ", positions.numel(),
              " entries for ", q.rows, " tokens");
  const at::cuda::CUDAGuard guard(query.device());
  check_status(pace_rotary_embedding(
                   positions.data_ptr<int64_t>(), query.data_ptr(), key.data_ptr(), q.rows,
                   (int)(q.width / head_size), (int)(k.width / head_size), (int)head_size,
                   q.stride, k.stride, cos_sin_cache.data_ptr(), pace_dtype(cos_sin_cache),
                   (int)cos_sin_cache.size(1), cos_sin_cache.size(0), is_neox ? 1 : 0,
                   pace_dtype(query), stream_of(query)),
               op);
}

// qkv = hidden @ weight^T with the rotary embedding of the q and k heads
// applied before the output is rounded (tcgen05 GEMM + rope epilogue).  It
// replaces qkv_proj followed by rotary_embedding
// (paceserve/model_executor/models/llama.py:176-178); `qkv` is the [T, (nq +
// 2 nkv) * head_size] output the split into q, k, v views reads.
// The stream-K workspace of the fused projection, kept per (device, stream):
// zero-filled once on that stream, and left zeroed by every call, so calls on
// one stream can share it; calls on different streams never do.
Tensor qkv_workspace(const at::Device& dev, cudaStream_t stream, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, Tensor> cache;
  std::lock_guard<std::mutex> lock(mu);
  Tensor& ws = cache[{dev.index(), stream}];
  if (!ws.defined() || (size_t)ws.numel() < bytes)
    ws = at::zeros({(int64_t)bytes}, at::TensorOptions().dtype(at::kByte).device(dev));
  return ws;
}

// A workspace tensor as the C ABI takes it (an undefined tensor: none).
void* ws_ptr(const Tensor& ws) { return ws.defined() ? ws.data_ptr() : nullptr; }
size_t ws_bytes(const Tensor& ws) { return ws.defined() ? (size_t)ws.nbytes() : 0; }

void qkv_proj_rotary_embedding(Tensor& qkv, Tensor& hidden, Tensor& weight, Tensor& positions,
                               int64_t head_size, int64_t num_heads, int64_t num_kv_heads,
                               Tensor& cos_sin_cache, bool is_neox,
                               const c10::optional<Tensor>& fault_flags,
                               const c10::optional<Tensor>& workspace) {
  const char* op = "qkv_proj_rotary_embedding";
  check_cuda(hidden, op, "hidden");
  check_same_device(qkv, hidden, op);
  check_same_device(weight, hidden, op);
  check_same_device(positions, hidden, op);
  check_same_device(cos_sin_cache, hidden, op);
  TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 || hidden.scalar_type() == at::kHalf, op,
              ": hidden must be bfloat16 or float16");
  TORCH_CHECK(qkv.scalar_type() == hidden.scalar_type() &&
                  weight.scalar_type() == hidden.scalar_type(),
              op, ": qkv, hidden and weight must share a dtype");
  TORCH_CHECK(positions.scalar_type() == at::kLong && positions.is_contiguous(), op,
              ": positions must be a contiguous int64 tensor");
  TORCH_CHECK(cos_sin_cache.dim() == 2 && cos_sin_cache.is_contiguous(), op,
              ": cos_sin_cache must be a contiguous [max_position, rot_dim] tensor");
  TORCH_CHECK(num_heads >= 0 && num_kv_heads >= 0 && head_size > 0, op, ": bad head counts");
  const Rows h = rows_of(hidden, op, "hidden");
  TORCH_CHECK(hidden.dim() == 2, op, ": hidden must be [T, hidden_size]");
  TORCH_CHECK(qkv.dim() == 2 && qkv.size(0) == h.rows, op, ": qkv must be [T, ",
              (num_heads + 2 * num_kv_heads) * head_size, "]");
  const Rows o = rows_of(qkv, op, "qkv");
  const int64_t n = (num_heads + 2 * num_kv_heads) * head_size;
  TORCH_CHECK(o.width == n, op, ": qkv width ", o.width, " != (num_heads + 2 * num_kv_heads) * head_size = ", n);
  TORCH_CHECK(weight.dim() == 2 && weight.is_contiguous() && weight.size(0) == n &&
                  weight.size(1) == h.width,
              op, ": weight must be a contiguous [", n, ", ", h.width, "] tensor");
  TORCH_CHECK(positions.numel() >= h.rows, op, ": positions has ", positions.numel(),
              " entries for ", h.rows, " tokens");
  const at::cuda::CUDAGuard guard(hidden.device());
  int32_t* fault = counter_ptr(fault_flags, hidden.device(), op, "fault_flags");
  if (h.rows == 0) return;
  const cudaStream_t stream = stream_of(hidden);
  const size_t need = pace_qkv_proj_rope_workspace_size(h.rows, h.width, (int)num_heads,
                                                        (int)num_kv_heads, hidden.device().index());
  Tensor ws;
  if (workspace.has_value()) {
    ws = *workspace;
    TORCH_CHECK(ws.is_cuda() && ws.device() == hidden.device() && ws.is_contiguous() &&
                    (size_t)ws.nbytes() >= need,
                op, ": workspace must be a contiguous tensor of at least ", need, " bytes on ",
                hidden.device());
  } else if (need > 0) {  // none at decode sizes
    ws = qkv_workspace(hidden.device(), stream, need);
  }
  check_status(pace_qkv_proj_rope(qkv.data_ptr(), hidden.data_ptr(), weight.data_ptr(),
                                  positions.data_ptr<int64_t>(), h.rows, h.width, (int)num_heads,
                                  (int)num_kv_heads, (int)head_size, h.stride, o.stride,
                                  cos_sin_cache.data_ptr(), pace_dtype(cos_sin_cache),
                                  (int)cos_sin_cache.size(1), cos_sin_cache.size(0),
                                  is_neox ? 1 : 0, pace_dtype(hidden), ws_ptr(ws),
                                  ws_bytes(ws), fault, stream),
               op);
}

// Workspace for the tensor-core GEMMs (caller's, or the per-stream cache).
Tensor gemm_workspace(const c10::optional<Tensor>& workspace, const at::Device& dev,
                      cudaStream_t stream, size_t need, const char* op) {
  if (workspace.has_value()) {
    const Tensor& ws = *workspace;
    TORCH_CHECK(ws.is_cuda() && ws.device() == dev && ws.is_contiguous() &&
                    (size_t)ws.nbytes() >= need,
                op, ": workspace must be a contiguous tensor of at least ", need, " bytes on ",
                dev);
    return ws;
  }
  if (need == 0) return Tensor();  // the call needs none
  return qkv_workspace(dev, stream, need);
}


// residual <- residual + input @ weight^T (o_proj / down_proj with the residual
// add in the epilogue); row_sumsq (optional, float32 [T, n / 32]) receives the
// new residual's sum-of-squares partials for the next RMSNorm.
void linear_residual(Tensor& residual, Tensor& input, Tensor& weight,
                     const c10::optional<Tensor>& row_sumsq,
                     const c10::optional<Tensor>& workspace,
                     const c10::optional<Tensor>& fault_flags) {
  const char* op = "linear_residual";
  check_cuda(input, op, "input");
  check_same_device(residual, input, op);
  check_same_device(weight, input, op);
  TORCH_CHECK(input.scalar_type() == at::kBFloat16 || input.scalar_type() == at::kHalf, op,
              ": input must be bfloat16 or float16");
  TORCH_CHECK(residual.scalar_type() == input.scalar_type() &&
                  weight.scalar_type() == input.scalar_type(),
              op, ": residual, input and weight must share a dtype");
  TORCH_CHECK(input.dim() == 2 && residual.dim() == 2 && weight.dim() == 2 &&
                  weight.is_contiguous(),
              op, ": input [T, k], residual [T, n] and a contiguous weight [n, k] expected");
  const Rows a = rows_of(input, op, "input");
  const Rows r = rows_of(residual, op, "residual");
  TORCH_CHECK(r.rows == a.rows && weight.size(0) == r.width && weight.size(1) == a.width, op,
              ": shapes do not match: input ", input.sizes(), ", residual ", residual.sizes(),
              ", weight ", weight.sizes());
  float* ss = nullptr;
  if (row_sumsq.has_value()) {
    const Tensor& t = *row_sumsq;
    check_same_device(t, input, op);
    TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous() &&
                    t.numel() >= a.rows * (r.width / 32),
                op, ": row_sumsq must be a contiguous float32 tensor of T * n / 32 entries");
    ss = t.data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(input.device());
  if (a.rows == 0) return;
  const cudaStream_t stream = stream_of(input);
  const size_t need = pace_linear_residual_workspace_size(a.rows, r.width, a.width,
                                                          input.device().index());
  Tensor ws = gemm_workspace(workspace, input.device(), stream, need, op);
  int32_t* fault = counter_ptr(fault_flags, input.device(), op, "fault_flags");
  check_status(pace_linear_residual(residual.data_ptr(), input.data_ptr(), weight.data_ptr(), ss,
                                    a.rows, r.width, a.width, a.stride, r.stride,
                                    pace_dtype(input), ws_ptr(ws), ws_bytes(ws), fault,
                                    stream),
               op);
}

void row_sumsq(Tensor& out, Tensor& input) {
  const char* op = "row_sumsq";
  check_cuda(input, op, "input");
  check_same_device(out, input, op);
  const Rows a = rows_of(input, op, "input");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() &&
                  out.numel() >= a.rows * (a.width / 32),
              op, ": out must be a contiguous float32 tensor of T * hidden / 32 entries");
  const at::cuda::CUDAGuard guard(input.device());
  check_status(pace_row_sumsq(out.data_ptr<float>(), input.data_ptr(), a.rows, a.width,
                              a.stride, pace_dtype(input), stream_of(input)),
               op);
}

// qkv = rope(inv * (hidden @ folded_weight^T)), inv the rows' RMSNorm factor
// from row_sumsq: input RMSNorm + qkv_proj + rotary_embedding in one GEMM.
void qkv_proj_rmsnorm_rotary_embedding(Tensor& qkv, Tensor& hidden, Tensor& folded_weight,
                                       Tensor& row_sumsq, double epsilon, Tensor& positions,
                                       int64_t head_size, int64_t num_heads,
                                       int64_t num_kv_heads, Tensor& cos_sin_cache,
                                       bool is_neox, const c10::optional<Tensor>& fault_flags,
                                       const c10::optional<Tensor>& workspace) {
  const char* op = "qkv_proj_rmsnorm_rotary_embedding";
  check_cuda(hidden, op, "hidden");
  for (const Tensor* t : {&qkv, &folded_weight, &row_sumsq, &positions, &cos_sin_cache})
    check_same_device(*t, hidden, op);
  TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 || hidden.scalar_type() == at::kHalf, op,
              ": hidden must be bfloat16 or float16");
  TORCH_CHECK(qkv.scalar_type() == hidden.scalar_type() &&
                  folded_weight.scalar_type() == hidden.scalar_type(),
              op, ": qkv, hidden and weight must share a dtype");
  TORCH_CHECK(positions.scalar_type() == at::kLong && positions.is_contiguous(), op,
              ": positions must be a contiguous int64 tensor");
  TORCH_CHECK(cos_sin_cache.dim() == 2 && cos_sin_cache.is_contiguous(), op,
              ": cos_sin_cache must be a contiguous [max_position, rot_dim] tensor");
  TORCH_CHECK(hidden.dim() == 2 && qkv.dim() == 2, op, ": hidden and qkv must be 2-D");
  const Rows h = rows_of(hidden, op, "hidden");
  const Rows o = rows_of(qkv, op, "qkv");
  const int64_t n = (num_heads + 2 * num_kv_heads) * head_size;
  TORCH_CHECK(o.rows == h.rows && o.width == n, op, ": qkv must be [T, ", n, "]");
  TORCH_CHECK(folded_weight.dim() == 2 && folded_weight.is_contiguous() &&
                  folded_weight.size(0) == n && folded_weight.size(1) == h.width,
              op, ": weight must be a contiguous [", n, ", ", h.width, "] tensor");
  TORCH_CHECK(row_sumsq.scalar_type() == at::kFloat && row_sumsq.is_contiguous() &&
                  row_sumsq.numel() >= h.rows * (h.width / 32),
              op, ": row_sumsq must be a contiguous float32 tensor of T * hidden / 32 entries");
  TORCH_CHECK(positions.numel() >= h.rows, op, ": positions has too few entries");
  const at::cuda::CUDAGuard guard(hidden.device());
  if (h.rows == 0) return;
  const cudaStream_t stream = stream_of(hidden);
  const size_t need = pace_qkv_proj_rope_workspace_size(h.rows, h.width, (int)num_heads,
                                                        (int)num_kv_heads, hidden.device().index());
  Tensor ws = gemm_workspace(workspace, hidden.device(), stream, need, op);
  int32_t* fault = counter_ptr(fault_flags, hidden.device(), op, "fault_flags");
  check_status(pace_qkv_proj_rmsnorm_rope(
                   qkv.data_ptr(), hidden.data_ptr(), folded_weight.data_ptr(),
                   row_sumsq.data_ptr<float>(), h.width / 32, (float)epsilon,
                   positions.data_ptr<int64_t>(), h.rows, h.width, (int)num_heads,
                   (int)num_kv_heads, (int)head_size, h.stride, o.stride,
                   cos_sin_cache.data_ptr(), pace_dtype(cos_sin_cache),
                   (int)cos_sin_cache.size(1), cos_sin_cache.size(0), is_neox ? 1 : 0,
                   pace_dtype(hidden), ws_ptr(ws), ws_bytes(ws), fault, stream),
               op);
}

// out = silu(gate) * up with [gate | up] = hidden @ weight^T, weight =
// [gate rows; up rows]: gate_up_proj + silu_and_mul in one GEMM.  With
// row_sumsq the rows are RMS-normalised by a per-row factor (the norm weight
// folded into `weight`).
void gate_up_silu(Tensor& out, Tensor& hidden, Tensor& weight,
                  const c10::optional<Tensor>& row_sumsq, double epsilon,
                  const c10::optional<Tensor>& workspace,
                  const c10::optional<Tensor>& fault_flags) {
  const char* op = "gate_up_silu";
  check_cuda(hidden, op, "hidden");
  check_same_device(out, hidden, op);
  check_same_device(weight, hidden, op);
  TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 || hidden.scalar_type() == at::kHalf, op,
              ": hidden must be bfloat16 or float16");
  TORCH_CHECK(out.scalar_type() == hidden.scalar_type() &&
                  weight.scalar_type() == hidden.scalar_type(),
              op, ": out, hidden and weight must share a dtype");
  TORCH_CHECK(hidden.dim() == 2 && out.dim() == 2 && weight.dim() == 2 && weight.is_contiguous(),
              op, ": hidden [T, H], out [T, I] and a contiguous weight [2 I, H] expected");
  const Rows h = rows_of(hidden, op, "hidden");
  const Rows o = rows_of(out, op, "out");
  TORCH_CHECK(o.rows == h.rows && weight.size(0) == 2 * o.width && weight.size(1) == h.width, op,
              ": shapes do not match: hidden ", hidden.sizes(), ", out ", out.sizes(),
              ", weight ", weight.sizes());
  const float* ss = nullptr;
  if (row_sumsq.has_value()) {
    const Tensor& t = *row_sumsq;
    check_same_device(t, hidden, op);
    TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous() &&
                    t.numel() >= h.rows * (h.width / 32),
                op, ": row_sumsq must be a contiguous float32 tensor of T * hidden / 32 entries");
    ss = t.data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(hidden.device());
  if (h.rows == 0) return;
  const cudaStream_t stream = stream_of(hidden);
  const size_t need = pace_gate_up_silu_workspace_size(h.rows, h.width, o.width,
                                                       hidden.device().index());
  // 0: none needed (decode sizes) or a shape the entry point rejects
  Tensor ws = gemm_workspace(workspace, hidden.device(), stream, need, op);
  int32_t* fault = counter_ptr(fault_flags, hidden.device(), op, "fault_flags");
  check_status(pace_gate_up_silu(out.data_ptr(), hidden.data_ptr(), weight.data_ptr(), ss,
                                 h.width / 32, (float)epsilon, h.rows, h.width, o.width, h.stride,
                                 o.stride, pace_dtype(hidden), ws_ptr(ws), ws_bytes(ws),
                                 fault, stream),
               op);
}

// ------------------------------------------------------------ activation --
using ActFn = int (*)(void*, const void*, int64_t, int64_t, int64_t, int64_t, int, cudaStream_t);

void activation(Tensor& out, Tensor& input, ActFn fn, bool gated, const char* op) {
  check_cuda(input, op, "input");
  check_same_device(out, input, op);
  TORCH_CHECK(is_float_type(input) && out.scalar_type() == input.scalar_type(), op,
              ": out and input must share a float dtype");
  const Rows in = rows_of(input, op, "input");
  const Rows o = rows_of(out, op, "out");
  const int64_t d = gated ? in.width / 2 : in.width;
  TORCH_CHECK(!gated || in.width % 2 == 0, op, ": input width must be even");
  TORCH_CHECK(o.rows == in.rows && o.width == d, op, ": out shape ", out.sizes(),
              " does not match input ", input.sizes());
  const at::cuda::CUDAGuard guard(input.device());
  check_status(fn(out.data_ptr(), input.data_ptr(), in.rows, d, in.stride, o.stride,
                  pace_dtype(input), stream_of(input)),
               op);
}

void silu_and_mul(Tensor& out, Tensor& input) {
  activation(out, input, pace_silu_and_mul, true, "silu_and_mul");
}
void gelu_and_mul(Tensor& out, Tensor& input) {
  activation(out, input, pace_gelu_and_mul, true, "gelu_and_mul");
}
void gelu_tanh_and_mul(Tensor& out, Tensor& input) {
  activation(out, input, pace_gelu_tanh_and_mul, true, "gelu_tanh_and_mul");
}
void gelu_new(Tensor& out, Tensor& input) {
  activation(out, input, pace_gelu_new, false, "gelu_new");
}
void gelu_fast(Tensor& out, Tensor& input) {
  activation(out, input, pace_gelu_fast, false, "gelu_fast");
}

// ------------------------------------------------------------------- moe --
void topk_softmax(Tensor& topk_weights, Tensor& topk_indices, Tensor& token_expert_indices,
                  Tensor& gating_output, bool renormalize) {
  const char* op = "topk_softmax";
  check_cuda(gating_output, op, "gating_output");
  check_same_device(topk_weights, gating_output, op);
  check_same_device(topk_indices, gating_output, op);
  check_same_device(token_expert_indices, gating_output, op);
  TORCH_CHECK(gating_output.scalar_type() == at::kFloat && gating_output.is_contiguous(), op,
              ": gating_output must be a contiguous float32 tensor");
  TORCH_CHECK(topk_weights.scalar_type() == at::kFloat && topk_weights.is_contiguous(), op,
              ": topk_weights must be a contiguous float32 tensor");
  TORCH_CHECK(topk_indices.scalar_type() == at::kInt && topk_indices.is_contiguous() &&
                  token_expert_indices.scalar_type() == at::kInt &&
                  token_expert_indices.is_contiguous(),
              op, ": topk_indices and token_expert_indices must be contiguous int32 tensors");
  const int64_t E = gating_output.size(-1);
  TORCH_CHECK(E > 0, op, ": no experts");
  const int64_t T = gating_output.numel() / E;
  const int64_t k = topk_weights.size(-1);
  TORCH_CHECK(topk_weights.numel() == T * k && topk_indices.numel() == T * k &&
                  token_expert_indices.numel() == T * k,
              op, ": outputs must hold [", T, ", ", k, "]");
  const at::cuda::CUDAGuard guard(gating_output.device());
  check_status(pace_topk_softmax(topk_weights.data_ptr<float>(), topk_indices.data_ptr<int32_t>(),
                                 token_expert_indices.data_ptr<int32_t>(),
                                 gating_output.data_ptr<float>(), T, (int)E, (int)k,
                                 renormalize ? 1 : 0, stream_of(gating_output)),
               op);
}

void moe_align_block_size(Tensor topk_ids, int64_t num_experts, int64_t block_size,
                          Tensor sorted_token_ids, Tensor experts_ids, Tensor num_tokens_post_pad,
                          bool fill_padding) {
  const char* op = "moe_align_block_size";
  check_cuda(topk_ids, op, "topk_ids");
  check_same_device(sorted_token_ids, topk_ids, op);
  check_same_device(experts_ids, topk_ids, op);
  check_same_device(num_tokens_post_pad, topk_ids, op);
  const int dt = pace_dtype(topk_ids);
  TORCH_CHECK(dt >= PACE_U8 && dt <= PACE_I64, op, ": topk_ids must have an integral dtype");
  TORCH_CHECK(topk_ids.is_contiguous(), op, ": topk_ids must be contiguous");
  for (const Tensor* t : {&sorted_token_ids, &experts_ids, &num_tokens_post_pad})
    TORCH_CHECK(t->scalar_type() == at::kInt && t->is_contiguous(), op,
                ": outputs must be contiguous int32 tensors");
  TORCH_CHECK(num_tokens_post_pad.numel() >= 1, op, ": num_tokens_post_pad is empty");
  TORCH_CHECK(num_experts > 0 && num_experts <= INT32_MAX && block_size > 0 &&
                  block_size <= INT32_MAX,
              op, ": num_experts and block_size must be positive int32 values");
  const at::cuda::CUDAGuard guard(topk_ids.device());
  check_status(pace_moe_align_block_size(
                   topk_ids.data_ptr(), dt, topk_ids.numel(), (int)num_experts, (int)block_size,
                   sorted_token_ids.data_ptr<int32_t>(), sorted_token_ids.numel(),
                   experts_ids.data_ptr<int32_t>(), experts_ids.numel(),
                   num_tokens_post_pad.data_ptr<int32_t>(), fill_padding ? 1 : 0,
                   stream_of(topk_ids)),
               op);
}

// Rows of the routed tokens in moe_align order (block 128): out[i] =
// input[sorted_token_ids[i] / top_k], zero for padding ids (>= numel).
void moe_gather_rows(Tensor& out, Tensor& input, Tensor& sorted_token_ids,
                     Tensor& num_tokens_post_pad, int64_t numel, int64_t top_k) {
  const char* op = "moe_gather_rows";
  check_cuda(input, op, "input");
  for (const Tensor* t : {&out, &sorted_token_ids, &num_tokens_post_pad})
    check_same_device(*t, input, op);
  TORCH_CHECK(input.scalar_type() == at::kBFloat16 || input.scalar_type() == at::kHalf, op,
              ": input must be bfloat16 or float16");
  TORCH_CHECK(out.scalar_type() == input.scalar_type(), op, ": out and input dtypes differ");
  TORCH_CHECK(sorted_token_ids.scalar_type() == at::kInt && sorted_token_ids.is_contiguous() &&
                  num_tokens_post_pad.scalar_type() == at::kInt,
              op, ": sorted_token_ids and num_tokens_post_pad must be contiguous int32");
  TORCH_CHECK(input.dim() == 2 && out.dim() == 2 && out.size(1) == input.size(1), op,
              ": input [T, H] and out [num_sorted, H] expected");
  TORCH_CHECK(out.size(0) <= sorted_token_ids.numel(), op,
              ": out has more rows than sorted_token_ids");
  const Rows in = rows_of(input, op, "input");
  const Rows o = rows_of(out, op, "out");
  TORCH_CHECK(numel <= in.rows * top_k && top_k > 0, op, ": numel exceeds the input's rows");
  const at::cuda::CUDAGuard guard(input.device());
  check_status(pace_moe_gather_rows(out.data_ptr(), input.data_ptr(),
                                    sorted_token_ids.data_ptr<int32_t>(), o.rows,
                                    num_tokens_post_pad.data_ptr<int32_t>(), numel, (int)top_k,
                                    in.width, in.stride, o.stride, pace_dtype(input),
                                    stream_of(input)),
               op);
}

// One expert GEMM of fused_experts on the tensor cores.  mode 0: out
// [num_sorted, I] = silu(a @ w1[e, :I]^T) * (a @ w1[e, I:]^T), w = w1 [E, 2I, K];
// mode 1: out [numel, H] rows sorted_token_ids[i] = topk_weights * (a @ w2[e]^T),
// w = w2 [E, H, K].
void moe_expert_gemm(Tensor& out, Tensor& a, Tensor& w, Tensor& sorted_token_ids,
                     Tensor& expert_ids, Tensor& num_tokens_post_pad, int64_t numel,
                     const c10::optional<Tensor>& topk_weights, int64_t mode,
                     const c10::optional<Tensor>& fault_flags) {
  const char* op = "moe_expert_gemm";
  check_cuda(a, op, "a");
  for (const Tensor* t : {&out, &w, &sorted_token_ids, &expert_ids, &num_tokens_post_pad})
    check_same_device(*t, a, op);
  TORCH_CHECK(mode == 0 || mode == 1, op, ": mode must be 0 (gate/up + SiLU) or 1 (down)");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 || a.scalar_type() == at::kHalf, op,
              ": a must be bfloat16 or float16");
  TORCH_CHECK(out.scalar_type() == a.scalar_type() && w.scalar_type() == a.scalar_type(), op,
              ": out, a and w must share a dtype");
  for (const Tensor* t : {&sorted_token_ids, &expert_ids, &num_tokens_post_pad})
    TORCH_CHECK(t->scalar_type() == at::kInt && t->is_contiguous(), op,
                ": routing tensors must be contiguous int32");
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous(), op, ": w must be a contiguous [E, N, K] tensor");
  TORCH_CHECK(a.dim() == 2 && out.dim() == 2, op, ": a and out must be 2-D");
  const Rows ar = rows_of(a, op, "a");
  const Rows orow = rows_of(out, op, "out");
  const int64_t E = w.size(0), k = w.size(2);
  TORCH_CHECK(ar.width == k, op, ": a width ", ar.width, " != w's K ", k);
  const int64_t n = mode == 0 ? w.size(1) / 2 : w.size(1);
  TORCH_CHECK(mode == 1 || w.size(1) % 2 == 0, op, ": w1 rows must be 2 * I");
  TORCH_CHECK(orow.width == n, op, ": out width ", orow.width, " != ", n);
  TORCH_CHECK(ar.rows <= sorted_token_ids.numel(), op, ": a has more rows than sorted_token_ids");
  TORCH_CHECK(expert_ids.numel() * 128 >= ar.rows, op,
              ": expert_ids must hold one entry per 128 sorted rows (moe_align with block 128)");
  const float* tw = nullptr;
  if (mode == 0) {
    TORCH_CHECK(orow.rows >= ar.rows, op, ": out needs a row per sorted row");
  } else {
    TORCH_CHECK(topk_weights.has_value(), op, ": mode 1 needs topk_weights");
    const Tensor& twt = *topk_weights;
    check_same_device(twt, a, op);
    TORCH_CHECK(twt.scalar_type() == at::kFloat && twt.is_contiguous() && twt.numel() >= numel,
                op, ": topk_weights must be a contiguous float32 tensor of >= numel entries");
    TORCH_CHECK(orow.rows >= numel, op, ": out needs numel rows");
    tw = twt.data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(a.device());
  int32_t* fault = counter_ptr(fault_flags, a.device(), op, "fault_flags");
  check_status(pace_moe_gemm(out.data_ptr(), a.data_ptr(), w.data_ptr(), ar.rows,
                            sorted_token_ids.data_ptr<int32_t>(), expert_ids.data_ptr<int32_t>(),
                            num_tokens_post_pad.data_ptr<int32_t>(), numel, tw, (int)E, n, k,
                            ar.stride, orow.stride, (int)mode, pace_dtype(a), fault,
                            stream_of(a)),
               op);
}

// ------------------------------------------------------------ kv transfer --
struct CacheSet {
  std::vector<void*> ptrs;
  int64_t num_blocks = 0;
  int64_t block_bytes = 0;
  c10::Device device = c10::Device(c10::kCPU);
};

CacheSet cache_set(const std::vector<Tensor>& caches, const char* op, const char* name) {
  TORCH_CHECK(!caches.empty(), op, ": ", name, " is empty");
  CacheSet s;
  s.device = caches[0].device();
  for (const Tensor& c : caches) {
    TORCH_CHECK(c.is_cuda() && c.device() == s.device, op, ": ", name,
                " must be CUDA tensors on one device");
    TORCH_CHECK(c.is_contiguous() && c.dim() >= 1, op, ": ", name, " must be contiguous");
    const int64_t nb = c.size(0);
    const int64_t bb = nb == 0 ? 0 : (int64_t)(c.numel() / nb) * (int64_t)c.element_size();
    if (s.ptrs.empty()) {
      s.num_blocks = nb;
      s.block_bytes = bb;
    }
    TORCH_CHECK(nb == s.num_blocks && bb == s.block_bytes, op, ": ", name,
                " layers differ in shape");
    s.ptrs.push_back(c.data_ptr());
  }
  return s;
}

// Block ids as a contiguous int32 tensor on `dev`.  int64 ids outside
// [0, INT32_MAX] become -1 before narrowing (on the device, no synchronisation),
// so the kernel skips and counts them instead of a wrapped id selecting a
// valid block.
Tensor ids_on(const Tensor& ids, const c10::Device& dev, const char* op, const char* name) {
  TORCH_CHECK(ids.dim() == 1, op, ": ", name, " must be 1-D");
  TORCH_CHECK(ids.scalar_type() == at::kInt || ids.scalar_type() == at::kLong, op, ": ", name,
              " must be int32 or int64");
  if (ids.scalar_type() == at::kLong) {
    Tensor t = ids.to(dev, /*non_blocking=*/false, /*copy=*/false);
    t = at::where(t.lt(0).logical_or(t.gt((int64_t)INT32_MAX)), at::full_like(t, -1), t);
    return t.to(at::kInt).contiguous();
  }
  return ids.to(dev, at::kInt, /*non_blocking=*/false, /*copy=*/false).contiguous();
}

// Method 3 of the Python-facing copies: the copy engines (pace_kv_copy_blocks_ce).
constexpr int64_t kMethodCopyEngine = 3;

// Host int32 copy of a 1-D id tensor (a device tensor is copied to the host,
// which synchronises with its stream).  int64 ids outside int32 become -1.
std::vector<int32_t> host_ids(const Tensor& ids, const char* op, const char* name) {
  TORCH_CHECK(ids.dim() == 1, op, ": ", name, " must be 1-D");
  TORCH_CHECK(ids.scalar_type() == at::kInt || ids.scalar_type() == at::kLong, op, ": ", name,
              " must be int32 or int64");
  Tensor t = ids.to(at::kCPU).to(at::kLong).contiguous();
  const int64_t* p = t.data_ptr<int64_t>();
  std::vector<int32_t> out((size_t)t.numel());
  for (int64_t i = 0; i < t.numel(); ++i)
    out[(size_t)i] = (p[i] < 0 || p[i] > (int64_t)INT32_MAX) ? -1 : (int32_t)p[i];
  return out;
}

void run_kv_copy(const std::vector<void*>& src, const std::vector<void*>& dst,
                 int64_t src_blocks, int64_t dst_blocks, int64_t block_bytes,
                 const c10::Device& exec, const Tensor& src_ids, const Tensor& dst_ids,
                 int64_t method, const c10::optional<Tensor>& bad_pairs, int64_t max_ctas,
                 int64_t wait_limit_ns, const char* op) {
  TORCH_CHECK(src.size() == dst.size(), op, ": source and destination layer counts differ (",
              src.size(), " vs ", dst.size(), ")");
  const at::cuda::CUDAGuard guard(exec);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(exec.index()).stream();
  if (method == kMethodCopyEngine) {
    std::vector<int32_t> s = host_ids(src_ids, op, "src_block_ids");
    std::vector<int32_t> d = host_ids(dst_ids, op, "dst_block_ids");
    TORCH_CHECK(s.size() == d.size(), op, ": block id lists differ in length");
    counter_ptr(bad_pairs, exec, op, "bad_pairs");  // validates the counter before any copy
    int64_t nbad = 0, issued = 0;
    int rc;
    {
      // One copy call per run of blocks can take milliseconds of host time for
      // fragmented tables: let other Python threads (the serving loop) run.
      py::gil_scoped_release no_gil;
      rc = pace_kv_copy_blocks_ce(src.data(), dst.data(), (int)src.size(), s.data(), d.data(),
                                  (int64_t)s.size(), block_bytes, src_blocks, dst_blocks, &nbad,
                                  &issued, stream);
    }
    check_status(rc, op);
    if (bad_pairs.has_value() && nbad > 0) bad_pairs->add_(nbad);  // stream-ordered, as the kernels count
    return;
  }
  Tensor s = ids_on(src_ids, exec, op, "src_block_ids");
  Tensor d = ids_on(dst_ids, exec, op, "dst_block_ids");
  TORCH_CHECK(s.numel() == d.numel(), op, ": block id lists differ in length");
  int32_t* bad = counter_ptr(bad_pairs, exec, op, "bad_pairs");
  TORCH_CHECK(method != 2 || bad != nullptr, op,
              ": method 2 reports wait timeouts through bad_pairs; pass an int32 counter");
  pace_kv_copy_opts opts = {};
  opts.method = (int)method;
  opts.max_ctas = (int)max_ctas;
  opts.wait_limit_ns = (uint64_t)wait_limit_ns;
  check_status(pace_kv_copy_blocks_ex(src.data(), dst.data(), (int)src.size(),
                                      s.data_ptr<int32_t>(), d.data_ptr<int32_t>(), s.numel(),
                                      block_bytes, src_blocks, dst_blocks, bad, &opts, stream),
               op);
  // Device copies of the ids were allocated on this same stream, so the
  // caching allocator cannot hand their memory out before the kernel ran.
}

// Copy blocks between two lists of per-layer caches (same or different GPUs).
// Runs on the destination device (pull) unless push=True.
void copy_blocks_p2p(const std::vector<Tensor>& src_caches, const std::vector<Tensor>& dst_caches,
                     const Tensor& src_block_ids, const Tensor& dst_block_ids, int64_t method,
                     bool push, const c10::optional<Tensor>& bad_pairs, int64_t max_ctas,
                     int64_t wait_limit_ns) {
  const char* op = "copy_blocks_p2p";
  CacheSet s = cache_set(src_caches, op, "src_caches");
  CacheSet d = cache_set(dst_caches, op, "dst_caches");
  TORCH_CHECK(s.block_bytes == d.block_bytes, op, ": source and destination block sizes differ");
  const c10::Device exec = push ? s.device : d.device;
  const c10::Device other = push ? d.device : s.device;
  if (exec != other)
    check_status(pace_enable_peer_access(exec.index(), other.index()), op);
  run_kv_copy(s.ptrs, d.ptrs, s.num_blocks, d.num_blocks, s.block_bytes, exec, src_block_ids,
              dst_block_ids, method, bad_pairs, max_ctas, wait_limit_ns, op);
}

// Same, with the source given as raw per-layer pointers (e.g. mapped from
// another process with ipc_open_handle) of src_num_blocks blocks each.
void copy_blocks_from_ptrs(const std::vector<int64_t>& src_ptrs, int64_t src_num_blocks,
                           const std::vector<Tensor>& dst_caches, const Tensor& src_block_ids,
                           const Tensor& dst_block_ids, int64_t method,
                           const c10::optional<Tensor>& bad_pairs, int64_t max_ctas,
                           int64_t wait_limit_ns) {
  const char* op = "copy_blocks_from_ptrs";
  CacheSet d = cache_set(dst_caches, op, "dst_caches");
  std::vector<void*> s;
  for (int64_t p : src_ptrs) s.push_back(reinterpret_cast<void*>(p));
  run_kv_copy(s, d.ptrs, src_num_blocks, d.num_blocks, d.block_bytes, d.device, src_block_ids,
              dst_block_ids, method, bad_pairs, max_ctas, wait_limit_ns, op);
}

// Destination given as raw pointers (push into another process's cache).
void copy_blocks_to_ptrs(const std::vector<Tensor>& src_caches, const std::vector<int64_t>& dst_ptrs,
                         int64_t dst_num_blocks, const Tensor& src_block_ids,
                         const Tensor& dst_block_ids, int64_t method,
                         const c10::optional<Tensor>& bad_pairs, int64_t max_ctas,
                         int64_t wait_limit_ns) {
  const char* op = "copy_blocks_to_ptrs";
  CacheSet s = cache_set(src_caches, op, "src_caches");
  std::vector<void*> d;
  for (int64_t p : dst_ptrs) d.push_back(reinterpret_cast<void*>(p));
  run_kv_copy(s.ptrs, d, s.num_blocks, dst_num_blocks, s.block_bytes, s.device, src_block_ids,
              dst_block_ids, method, bad_pairs, max_ctas, wait_limit_ns, op);
}

// out[l, j] = caches[l][block_ids[j]]; out is [L, n, ...] on the caches'
// device or pinned host memory.
void gather_blocks(const std::vector<Tensor>& caches, const Tensor& block_ids, Tensor& out,
                   const c10::optional<Tensor>& bad_ids) {
  const char* op = "gather_blocks";
  CacheSet c = cache_set(caches, op, "caches");
  const at::cuda::CUDAGuard guard(c.device);
  Tensor ids = ids_on(block_ids, c.device, op, "block_ids");
  TORCH_CHECK(out.is_contiguous(), op, ": out must be contiguous");
  TORCH_CHECK(out.is_cuda() ? out.device() == c.device : out.is_pinned(), op,
              ": out must live on the caches' device or in pinned host memory");
  TORCH_CHECK((int64_t)out.numel() * out.element_size() ==
                  (int64_t)c.ptrs.size() * ids.numel() * c.block_bytes,
              op, ": out must hold num_layers * len(block_ids) blocks");
  int32_t* bad = counter_ptr(bad_ids, c.device, op, "bad_ids");
  cudaStream_t st = at::cuda::getCurrentCUDAStream(c.device.index()).stream();
  check_status(pace_kv_gather_blocks(c.ptrs.data(), (int)c.ptrs.size(), ids.data_ptr<int32_t>(),
                                     ids.numel(), c.block_bytes, c.num_blocks, out.data_ptr(), bad,
                                     st),
               op);
}

// caches[l][block_ids[j]] = src[l, j]
void scatter_blocks(const Tensor& src, const std::vector<Tensor>& caches, const Tensor& block_ids,
                    const c10::optional<Tensor>& bad_ids) {
  const char* op = "scatter_blocks";
  CacheSet c = cache_set(caches, op, "caches");
  const at::cuda::CUDAGuard guard(c.device);
  Tensor ids = ids_on(block_ids, c.device, op, "block_ids");
  TORCH_CHECK(src.is_contiguous(), op, ": src must be contiguous");
  TORCH_CHECK(src.is_cuda() ? src.device() == c.device : src.is_pinned(), op,
              ": src must live on the caches' device or in pinned host memory");
  TORCH_CHECK((int64_t)src.numel() * src.element_size() ==
                  (int64_t)c.ptrs.size() * ids.numel() * c.block_bytes,
              op, ": src must hold num_layers * len(block_ids) blocks");
  int32_t* bad = counter_ptr(bad_ids, c.device, op, "bad_ids");
  cudaStream_t st = at::cuda::getCurrentCUDAStream(c.device.index()).stream();
  check_status(pace_kv_scatter_blocks(src.data_ptr(), c.ptrs.data(), (int)c.ptrs.size(),
                                      ids.data_ptr<int32_t>(), ids.numel(), c.block_bytes,
                                      c.num_blocks, bad, st),
               op);
}

// ------------------------------------------------------- paged-KV append --
// K or V rows of nnz tokens: [nnz, heads, hd] (heads contiguous) or [nnz, heads*hd].
int64_t kv_row_stride(const Tensor& t, int64_t heads, int64_t hd, const char* op, const char* name) {
  TORCH_CHECK(t.is_cuda(), op, ": ", name, " must be a CUDA tensor");
  if (t.dim() == 3) {
    TORCH_CHECK(t.size(1) == heads && t.size(2) == hd, op, ": ", name, " must be [nnz, ", heads,
                ", ", hd, "]");
    TORCH_CHECK((hd <= 1 || t.stride(2) == 1) && (heads <= 1 || t.stride(1) == hd), op, ": ", name,
                " heads must be contiguous");
    return t.size(0) <= 1 ? heads * hd : t.stride(0);
  }
  TORCH_CHECK(t.dim() == 2 && t.size(1) == heads * hd, op, ": ", name, " must be [nnz, ",
              heads * hd, "] or [nnz, ", heads, ", ", hd, "]");
  TORCH_CHECK(t.size(1) <= 1 || t.stride(1) == 1, op, ": ", name, " rows must be contiguous");
  return t.size(0) <= 1 ? heads * hd : t.stride(0);
}

struct PagedCache {
  int64_t pages, page_size, heads, hd;
};

PagedCache paged_cache_of(const Tensor& c, const std::string& layout, const char* op) {
  TORCH_CHECK(layout == "NHD", op, ": only the NHD layout [pages, 2, page_size, kv_heads, head_dim] "
              "(PaceServe's, flashinfer_attention_wrapper.py:63-73) is supported");
  TORCH_CHECK(c.is_cuda() && c.dim() == 5 && c.size(1) == 2 && c.is_contiguous(), op,
              ": paged_kv_cache must be a contiguous CUDA tensor [pages, 2, page_size, kv_heads, "
              "head_dim]");
  return {c.size(0), c.size(2), c.size(3), c.size(4)};
}

Tensor int32_on(const Tensor& t, const Tensor& like, const char* op, const char* name) {
  TORCH_CHECK(t.device() == like.device(), op, ": ", name, " must be on the cache's device");
  TORCH_CHECK(t.scalar_type() == at::kInt && t.dim() == 1, op, ": ", name,
              " must be a 1-D int32 tensor");
  return t.contiguous();
}

// flashinfer.page.append_paged_kv_cache's signature (FlashInfer 0.2.0).
void append_paged_kv_cache(const Tensor& append_key, const Tensor& append_value,
                           const Tensor& batch_indices, const Tensor& positions,
                           Tensor& paged_kv_cache, const Tensor& kv_indices,
                           const Tensor& kv_indptr, const Tensor& kv_last_page_len,
                           const std::string& kv_layout, const c10::optional<Tensor>& bad_tokens) {
  const char* op = "append_paged_kv_cache";
  const PagedCache pc = paged_cache_of(paged_kv_cache, kv_layout, op);
  TORCH_CHECK(append_key.scalar_type() == paged_kv_cache.scalar_type() &&
                  append_value.scalar_type() == paged_kv_cache.scalar_type(),
              op, ": key, value and cache must share a dtype");
  check_same_device(append_key, paged_kv_cache, op);
  check_same_device(append_value, paged_kv_cache, op);
  const int64_t ks = kv_row_stride(append_key, pc.heads, pc.hd, op, "append_key");
  const int64_t vs = kv_row_stride(append_value, pc.heads, pc.hd, op, "append_value");
  const int64_t nnz = append_key.size(0);
  TORCH_CHECK(append_value.size(0) == nnz, op, ": key and value token counts differ");
  Tensor bi = int32_on(batch_indices, paged_kv_cache, op, "batch_indices");
  Tensor po = int32_on(positions, paged_kv_cache, op, "positions");
  Tensor ki = int32_on(kv_indices, paged_kv_cache, op, "kv_indices");
  Tensor kp = int32_on(kv_indptr, paged_kv_cache, op, "kv_indptr");
  Tensor kl = int32_on(kv_last_page_len, paged_kv_cache, op, "kv_last_page_len");
  TORCH_CHECK(bi.numel() >= nnz && po.numel() >= nnz, op,
              ": batch_indices and positions need one entry per token");
  TORCH_CHECK(kp.numel() >= 1 && kl.numel() >= kp.numel() - 1, op,
              ": kv_indptr needs batch + 1 entries and kv_last_page_len batch entries");
  int32_t* bad = counter_ptr(bad_tokens, paged_kv_cache.device(), op, "bad_tokens");
  const at::cuda::CUDAGuard guard(paged_kv_cache.device());
  check_status(pace_append_paged_kv_cache(
                   append_key.data_ptr(), append_value.data_ptr(), nnz, (int)pc.heads, (int)pc.hd,
                   ks, vs, bi.data_ptr<int32_t>(), po.data_ptr<int32_t>(),
                   paged_kv_cache.data_ptr(), pc.pages, (int)pc.page_size, ki.data_ptr<int32_t>(),
                   ki.numel(), kp.data_ptr<int32_t>(), kl.data_ptr<int32_t>(), kp.numel() - 1, bad,
                   pace_dtype(paged_kv_cache), stream_of(paged_kv_cache)),
               op);
}

// One launch for get_seq_lens + get_batch_indices_positions + append.
void append_paged_kv_cache_by_indptr(const Tensor& append_key, const Tensor& append_value,
                                     const Tensor& append_indptr, Tensor& paged_kv_cache,
                                     const Tensor& kv_indices, const Tensor& kv_indptr,
                                     const Tensor& kv_last_page_len,
                                     const c10::optional<Tensor>& bad_tokens) {
  const char* op = "append_paged_kv_cache_by_indptr";
  const PagedCache pc = paged_cache_of(paged_kv_cache, "NHD", op);
  TORCH_CHECK(append_key.scalar_type() == paged_kv_cache.scalar_type() &&
                  append_value.scalar_type() == paged_kv_cache.scalar_type(),
              op, ": key, value and cache must share a dtype");
  check_same_device(append_key, paged_kv_cache, op);
  check_same_device(append_value, paged_kv_cache, op);
  const int64_t ks = kv_row_stride(append_key, pc.heads, pc.hd, op, "append_key");
  const int64_t vs = kv_row_stride(append_value, pc.heads, pc.hd, op, "append_value");
  const int64_t nnz = append_key.size(0);
  TORCH_CHECK(append_value.size(0) == nnz, op, ": key and value token counts differ");
  Tensor ai = int32_on(append_indptr, paged_kv_cache, op, "append_indptr");
  Tensor ki = int32_on(kv_indices, paged_kv_cache, op, "kv_indices");
  Tensor kp = int32_on(kv_indptr, paged_kv_cache, op, "kv_indptr");
  Tensor kl = int32_on(kv_last_page_len, paged_kv_cache, op, "kv_last_page_len");
  TORCH_CHECK(ai.numel() == kp.numel() && kl.numel() >= kp.numel() - 1 && kp.numel() >= 1, op,
              ": append_indptr and kv_indptr need batch + 1 entries, kv_last_page_len batch");
  int32_t* bad = counter_ptr(bad_tokens, paged_kv_cache.device(), op, "bad_tokens");
  const at::cuda::CUDAGuard guard(paged_kv_cache.device());
  check_status(pace_append_paged_kv_cache_by_indptr(
                   append_key.data_ptr(), append_value.data_ptr(), nnz, (int)pc.heads,
                   (int)pc.hd, ks, vs, ai.data_ptr<int32_t>(), paged_kv_cache.data_ptr(), pc.pages,
                   (int)pc.page_size, ki.data_ptr<int32_t>(), ki.numel(), kp.data_ptr<int32_t>(),
                   kl.data_ptr<int32_t>(), kp.numel() - 1, bad, pace_dtype(paged_kv_cache),
                   stream_of(paged_kv_cache)),
               op);
}

py::tuple ipc_get_handle(const Tensor& t) {
  TORCH_CHECK(t.is_cuda(), "ipc_get_handle: tensor must be on a CUDA device");
  const at::cuda::CUDAGuard guard(t.device());
  char h[PACE_IPC_HANDLE_BYTES];
  int64_t off = 0;
  check_status(pace_ipc_get_handle(t.data_ptr(), h, &off), "ipc_get_handle");
  return py::make_tuple(py::bytes(h, PACE_IPC_HANDLE_BYTES), off);
}

int64_t ipc_open_handle(const py::bytes& handle, int64_t device) {
  std::string h = handle;
  TORCH_CHECK(h.size() == PACE_IPC_HANDLE_BYTES, "ipc_open_handle: handle must be ",
              PACE_IPC_HANDLE_BYTES, " bytes");
  void* base = nullptr;
  check_status(pace_ipc_open_handle(h.data(), (int)device, &base), "ipc_open_handle");
  return reinterpret_cast<int64_t>(base);
}

void ipc_close_handle(int64_t base) {
  check_status(pace_ipc_close_handle(reinterpret_cast<void*>(base)), "ipc_close_handle");
}

void enable_peer_access(int64_t device, int64_t peer) {
  check_status(pace_enable_peer_access((int)device, (int)peer), "enable_peer_access");
}

bool can_access_peer(int64_t device, int64_t peer) {
  int can = 0;
  check_status(pace_can_access_peer((int)device, (int)peer, &can), "can_access_peer");
  return can != 0;
}

}  // namespace

PYBIND11_MODULE(_C, m) {
  m.doc() = "PaceServe per-layer ops and KV transfer on B200 (sm_100a)";
  m.def("version", &pace_version);
  m.def("set_pdl", [](bool on) { pace_set_pdl(on ? 1 : 0); },
        "Enable/disable programmatic dependent launch for the per-layer ops.");
  m.def("get_pdl", []() { return pace_get_pdl() != 0; });

  auto ln = m.def_submodule("layernorm_ops");
  ln.def("rms_norm", &rms_norm, "Apply Root Mean Square (RMS) Normalization to the input tensor.",
         py::arg("out"), py::arg("input"), py::arg("weight"), py::arg("epsilon"));
  ln.def("linear_residual", &linear_residual,
         "residual += input @ weight^T on the tensor cores (o_proj / down_proj with the residual "
         "add in the epilogue); row_sumsq receives the new rows' sum-of-squares partials.",
         py::arg("residual"), py::arg("input"), py::arg("weight"),
         py::arg("row_sumsq") = py::none(), py::arg("workspace") = py::none(),
         py::arg("fault_flags") = py::none());
  ln.def("row_sumsq", &row_sumsq, "out[t, g] = sum of input[t, 32g:32g+32]^2 (float32).",
         py::arg("out"), py::arg("input"));
  ln.def("fused_add_rms_norm", &fused_add_rms_norm,
         "In place: residual += input; input = rms_norm(residual) * weight.", py::arg("input"),
         py::arg("residual"), py::arg("weight"), py::arg("epsilon"));

  auto pe = m.def_submodule("pos_encoding_ops");
  pe.def("rotary_embedding", &rotary_embedding,
         "Apply GPT-NeoX or GPT-J style rotary embedding to query and key", py::arg("positions"),
         py::arg("query"), py::arg("key"), py::arg("head_size"), py::arg("cos_sin_cache"),
         py::arg("is_neox"));
  pe.def("qkv_proj_rotary_embedding", &qkv_proj_rotary_embedding,
         "qkv = hidden @ weight^T on the tensor cores with the rotary embedding applied to the "
         "q and k heads before rounding (fused qkv_proj + rotary_embedding).",
         py::arg("qkv"), py::arg("hidden"), py::arg("weight"), py::arg("positions"),
         py::arg("head_size"), py::arg("num_heads"), py::arg("num_kv_heads"),
         py::arg("cos_sin_cache"), py::arg("is_neox"), py::arg("fault_flags") = py::none(),
         py::arg("workspace") = py::none());
  pe.def("qkv_proj_rmsnorm_rotary_embedding", &qkv_proj_rmsnorm_rotary_embedding,
         "qkv = rope(inv * (hidden @ folded_weight^T)): input RMSNorm (weight folded into the "
         "projection, per-row factor from row_sumsq), qkv projection and rotary embedding in "
         "one tensor-core GEMM.",
         py::arg("qkv"), py::arg("hidden"), py::arg("folded_weight"), py::arg("row_sumsq"),
         py::arg("epsilon"), py::arg("positions"), py::arg("head_size"), py::arg("num_heads"),
         py::arg("num_kv_heads"), py::arg("cos_sin_cache"), py::arg("is_neox"),
         py::arg("fault_flags") = py::none(), py::arg("workspace") = py::none());
  pe.def("qkv_proj_rope_workspace_size",
         [](int64_t num_tokens, int64_t hidden_size, int64_t num_heads, int64_t num_kv_heads,
            int64_t device) {
           return pace_qkv_proj_rope_workspace_size(num_tokens, hidden_size, (int)num_heads,
                                                    (int)num_kv_heads, (int)device);
         },
         "Bytes of zero-filled workspace qkv_proj_rotary_embedding needs for this shape.",
         py::arg("num_tokens"), py::arg("hidden_size"), py::arg("num_heads"),
         py::arg("num_kv_heads"), py::arg("device"));

  auto act = m.def_submodule("activation_ops");
  act.def("silu_and_mul", &silu_and_mul, "Activation function used in SwiGLU.", py::arg("out"),
          py::arg("input"));
  act.def("gate_up_silu", &gate_up_silu,
          "out = silu(gate) * up, [gate | up] = hidden @ weight^T on the tensor cores "
          "(gate_up_proj + silu_and_mul in one GEMM); with row_sumsq the post-attention "
          "RMSNorm is a per-row factor and weight holds the norm weight folded in.",
          py::arg("out"), py::arg("hidden"), py::arg("weight"),
          py::arg("row_sumsq") = py::none(), py::arg("epsilon") = 1e-6,
          py::arg("workspace") = py::none(), py::arg("fault_flags") = py::none());
  act.def("gelu_and_mul", &gelu_and_mul, "GeGLU: gelu(x[:, :d]) * x[:, d:] (erf GELU).",
          py::arg("out"), py::arg("input"));
  act.def("gelu_tanh_and_mul", &gelu_tanh_and_mul,
          "GeGLU with the tanh-approximated GELU.", py::arg("out"), py::arg("input"));
  act.def("gelu_new", &gelu_new, "GELU implementation used in GPT-2.", py::arg("out"),
          py::arg("input"));
  act.def("gelu_fast", &gelu_fast, "Approximate GELU implementation.", py::arg("out"),
          py::arg("input"));

  auto moe = m.def_submodule("moe_ops");
  moe.def("topk_softmax", &topk_softmax, "Apply topk softmax to the gating outputs.",
          py::arg("topk_weights"), py::arg("topk_indices"), py::arg("token_expert_indices"),
          py::arg("gating_output"), py::arg("renormalize") = false);
  moe.def("moe_align_block_size", &moe_align_block_size,
          "Aligning the number of tokens to be processed by each expert such that it is "
          "divisible by the block size.",
          py::arg("topk_ids"), py::arg("num_experts"), py::arg("block_size"),
          py::arg("sorted_token_ids"), py::arg("experts_ids"), py::arg("num_tokens_post_pad"),
          py::arg("fill_padding") = false);
  moe.def("moe_gather_rows", &moe_gather_rows,
          "out[i] = input[sorted_token_ids[i] / top_k] (zero rows for padding ids).",
          py::arg("out"), py::arg("input"), py::arg("sorted_token_ids"),
          py::arg("num_tokens_post_pad"), py::arg("numel"), py::arg("top_k"));
  moe.def("moe_expert_gemm", &moe_expert_gemm,
          "Grouped expert GEMM on the tensor cores: mode 0 gate/up + SiLU-and-mul, mode 1 down "
          "projection times the routing weight (rows scattered to the token slots).",
          py::arg("out"), py::arg("a"), py::arg("w"), py::arg("sorted_token_ids"),
          py::arg("expert_ids"), py::arg("num_tokens_post_pad"), py::arg("numel"),
          py::arg("topk_weights") = py::none(), py::arg("mode") = 0,
          py::arg("fault_flags") = py::none());

  auto kv = m.def_submodule("kv_transfer_ops");
  kv.def("copy_blocks_p2p", &copy_blocks_p2p,
         "Copy KV blocks src_block_ids of src_caches onto dst_block_ids of dst_caches "
         "(per-layer caches, possibly on different GPUs; pull on the destination GPU by default). "
         "method: 0 auto, 1 SIMT, 2 bulk (needs bad_pairs), 3 copy engines (host ids, no SM); "
         "max_ctas > 0 caps the kernel's CTAs; wait_limit_ns bounds the bulk method's waits.",
         py::arg("src_caches"), py::arg("dst_caches"), py::arg("src_block_ids"),
         py::arg("dst_block_ids"), py::arg("method") = 0, py::arg("push") = false,
         py::arg("bad_pairs") = py::none(), py::arg("max_ctas") = 0, py::arg("wait_limit_ns") = 0);
  kv.def("copy_blocks_from_ptrs", &copy_blocks_from_ptrs, py::arg("src_ptrs"),
         py::arg("src_num_blocks"), py::arg("dst_caches"), py::arg("src_block_ids"),
         py::arg("dst_block_ids"), py::arg("method") = 0, py::arg("bad_pairs") = py::none(),
         py::arg("max_ctas") = 0, py::arg("wait_limit_ns") = 0);
  kv.def("copy_blocks_to_ptrs", &copy_blocks_to_ptrs, py::arg("src_caches"), py::arg("dst_ptrs"),
         py::arg("dst_num_blocks"), py::arg("src_block_ids"), py::arg("dst_block_ids"),
         py::arg("method") = 0, py::arg("bad_pairs") = py::none(), py::arg("max_ctas") = 0,
         py::arg("wait_limit_ns") = 0);
  kv.def("gather_blocks", &gather_blocks, py::arg("caches"), py::arg("block_ids"), py::arg("out"),
         py::arg("bad_ids") = py::none());
  kv.def("scatter_blocks", &scatter_blocks, py::arg("src"), py::arg("caches"),
         py::arg("block_ids"), py::arg("bad_ids") = py::none());
  kv.def("append_paged_kv_cache", &append_paged_kv_cache,
         "Append K/V rows of new tokens to a paged cache (flashinfer.append_paged_kv_cache).",
         py::arg("append_key"), py::arg("append_value"), py::arg("batch_indices"),
         py::arg("positions"), py::arg("paged_kv_cache"), py::arg("kv_indices"),
         py::arg("kv_indptr"), py::arg("kv_last_page_len"), py::arg("kv_layout") = "NHD",
         py::arg("bad_tokens") = py::none());
  kv.def("append_paged_kv_cache_by_indptr", &append_paged_kv_cache_by_indptr,
         "Append, deriving each token's request and position from append_indptr in the kernel.",
         py::arg("append_key"), py::arg("append_value"), py::arg("append_indptr"),
         py::arg("paged_kv_cache"), py::arg("kv_indices"), py::arg("kv_indptr"),
         py::arg("kv_last_page_len"), py::arg("bad_tokens") = py::none());
  kv.def("ipc_get_handle", &ipc_get_handle, py::arg("tensor"));
  kv.def("ipc_open_handle", &ipc_open_handle, py::arg("handle"), py::arg("device"));
  kv.def("ipc_close_handle", &ipc_close_handle, py::arg("base"));
  kv.def("enable_peer_access", &enable_peer_access, py::arg("device"), py::arg("peer"));
  kv.def("can_access_peer", &can_access_peer, py::arg("device"), py::arg("peer"));
}
