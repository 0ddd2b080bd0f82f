"""GPU parity of the RMSNorm folded into the GEMMs around it:
layernorm_ops.linear_residual (o_proj / down_proj with the residual add and the
next norm's sum-of-squares partials in the epilogue), layernorm_ops.row_sumsq,
and pos_encoding_ops.qkv_proj_rmsnorm_rotary_embedding (input RMSNorm as a
per-row factor, qkv projection and rope in one GEMM).  At decode sizes the
same entry points run the weight-streaming CUDA-core kernel (linear_residual
then computes the partials with row_sumsq).

Oracle: the reference's composition in fp32 from the same 16-bit inputs:
residual + a @ W^T (models/llama.py:248), then rms_norm (oracle/ops_ref.py),
the qkv projection and the rope rotation.  Tolerance: the float rule
max|got - ref| / max|ref| <= 1e-2, plus a per-element bound (below)."""
import pytest
import torch

import paceserve_b200 as pb
from oracle import ops_ref
from paceserve_b200 import layernorm_ops, pos_encoding_ops
from tests._util import REL_TOL, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
EPS = 1e-5


def close(got, ref, dtype, ulps=1.0, frac=1e-3):
    """max error within 1e-2 of the largest magnitude, and each element within
    `ulps` storage ulps of itself plus `frac` of the largest magnitude."""
    assert rel_err(got, ref) <= REL_TOL
    g, r = got.float().cpu(), ref.float().cpu()
    bound = ulps * torch.finfo(dtype).eps * r.abs() + frac * r.abs().max()
    assert ((g - r).abs() <= bound).all(), ((g - r).abs() - bound).max().item()


def rnd(shape, g, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


@pytest.mark.parametrize("T,K,N", [(1, 4096, 4096), (1, 14336, 4096), (2, 200, 256),
                                   (2, 14336, 4096), (37, 1024, 512), (512, 4096, 4096),
                                   (300, 14336, 4096)])
def test_linear_residual_and_row_sumsq(T, K, N):
    # one token, or two with K <= 8192: the weight-streaming CUDA-core kernel,
    # then row_sumsq on the new rows; otherwise the tensor-core GEMM with the
    # partials in its epilogue
    g = torch.Generator().manual_seed(T + K)
    a = rnd((T, K), g)
    w = rnd((N, K), g, K ** -0.5)
    res = rnd((T, N), g)
    res_d = res.to(DEV)
    ss = torch.full((T, N // 32), -1.0, device=DEV)
    layernorm_ops.linear_residual(res_d, a.to(DEV), w.to(DEV), ss)
    torch.cuda.synchronize()
    ref = res.float() + a.float() @ w.float().t()
    close(res_d, ref, torch.bfloat16)
    # the partials are the new residual's own sums of squares per 32 columns
    got = res_d.float().cpu().view(T, N // 32, 32)
    want_ss = (got.double() ** 2).sum(-1)
    assert torch.allclose(ss.cpu().double(), want_ss, rtol=1e-5, atol=1e-6)
    # row_sumsq computes the same partials from any rows
    ss2 = torch.empty_like(ss)
    layernorm_ops.row_sumsq(ss2, res_d)
    torch.cuda.synchronize()
    assert torch.allclose(ss2.cpu().double(), want_ss, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("T", [2, 20, 300])
def test_linear_residual_float16_strided_rows_without_sumsq(T):
    """fp16 rounding of the residual add; input and residual as column slices
    of wider rows; no sum-of-squares output.  T=20 finishes shared stream-K
    tiles by their last contributor, T=300 runs on CTA pairs."""
    K, N = 2048, 1024
    g = torch.Generator().manual_seed(T + 1)
    a_wide = rnd((T, K + 64), g, dtype=torch.float16).to(DEV)
    a = a_wide[:, 64:]
    w = rnd((N, K), g, K ** -0.5, dtype=torch.float16).to(DEV)
    res_wide = rnd((T, N + 128), g, dtype=torch.float16).to(DEV)
    res = res_wide[:, :N]
    tail = res_wide[:, N:].clone()
    ref = res.float().cpu() + a.float().cpu() @ w.float().cpu().t()
    layernorm_ops.linear_residual(res, a, w)
    torch.cuda.synchronize()
    close(res, ref, torch.float16)
    assert torch.equal(res_wide[:, N:], tail)  # nothing written past the row


@pytest.mark.parametrize("T", [1, 2, 3, 64, 256, 512])
@pytest.mark.parametrize("neox", [True, False])
def test_qkv_proj_rmsnorm_rope(T, neox):
    nq, nkv, hd, H = 32, 8, 128, 4096
    g = torch.Generator().manual_seed(T * 3 + neox)
    h = rnd((T, H), g)
    w_norm = (torch.randn(H, generator=g) * 0.02 + 1).to(torch.bfloat16)
    w_qkv = rnd(((nq + 2 * nkv) * hd, H), g, H ** -0.5)
    pos = torch.randint(0, 8192, (T,), generator=g)
    cache = ops_ref.cos_sin_cache(hd, 8192, 500000.0)
    folded = pb.fold_rmsnorm_weight(w_qkv.to(DEV), w_norm.to(DEV))
    h_d = h.to(DEV)
    ss = torch.empty(T, H // 32, device=DEV)
    layernorm_ops.row_sumsq(ss, h_d)
    qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, device=DEV)
    pos_encoding_ops.qkv_proj_rmsnorm_rotary_embedding(qkv, h_d, folded, ss, EPS, pos.to(DEV),
                                                       hd, nq, nkv, cache.to(DEV), neox)
    torch.cuda.synchronize()
    x = ops_ref.rms_norm_fp32(h, w_norm, EPS)
    p = x @ w_qkv.float().t()
    q, k = ops_ref.rotary_embedding_fp32(pos, p[:, : nq * hd], p[:, nq * hd: (nq + nkv) * hd], hd,
                                         cache, neox)
    ref = torch.cat([q, k, p[:, (nq + nkv) * hd:]], dim=1)
    # the folded weight is rounded to bf16 where the reference rounds the
    # normalised rows: a few ulps per product, averaged over K
    close(qkv, ref, torch.bfloat16, ulps=2.0, frac=3e-3)


def test_fused_layer_boundary_matches_unfused_ops():
    """Two layer boundaries, fused: down_proj + residual (linear_residual) ->
    input RMSNorm + qkv + rope (one GEMM); against the unfused path of this
    package: torch matmul, fused_add_rms_norm, torch matmul, rotary_embedding."""
    T, H, I, nq, nkv, hd = 200, 1024, 2048, 8, 2, 128
    g = torch.Generator().manual_seed(9)
    act = rnd((T, I), g).to(DEV)
    w_down = rnd((H, I), g, I ** -0.5).to(DEV)
    w_norm = (torch.randn(H, generator=g) * 0.02 + 1).to(torch.bfloat16).to(DEV)
    w_qkv = rnd(((nq + 2 * nkv) * hd, H), g, H ** -0.5).to(DEV)
    res0 = rnd((T, H), g).to(DEV)
    pos = torch.randint(0, 8192, (T,), generator=g).to(DEV)
    cache = ops_ref.cos_sin_cache(hd, 8192, 500000.0).to(DEV)
    n = (nq + 2 * nkv) * hd
    # fused
    res_f = res0.clone()
    ss = torch.empty(T, H // 32, device=DEV)
    layernorm_ops.linear_residual(res_f, act, w_down, ss)
    qkv_f = torch.empty(T, n, dtype=torch.bfloat16, device=DEV)
    pos_encoding_ops.qkv_proj_rmsnorm_rotary_embedding(
        qkv_f, res_f, pb.fold_rmsnorm_weight(w_qkv, w_norm), ss, EPS, pos, hd, nq, nkv, cache,
        True)
    # unfused
    x = act @ w_down.t()
    res_u = res0.clone()
    layernorm_ops.fused_add_rms_norm(x, res_u, w_norm, EPS)
    qkv_u = x @ w_qkv.t()
    pos_encoding_ops.rotary_embedding(pos, qkv_u[:, : nq * hd], qkv_u[:, nq * hd: (nq + nkv) * hd],
                                      hd, cache, True)
    torch.cuda.synchronize()
    assert rel_err(res_f, res_u) <= REL_TOL
    assert rel_err(qkv_f, qkv_u) <= REL_TOL


def test_rejected_inputs():
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        layernorm_ops.linear_residual(torch.zeros(4, 200, dtype=torch.bfloat16, device=DEV), x,
                                      torch.zeros(200, 64, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(RuntimeError, match="multiple of 32"):
        layernorm_ops.row_sumsq(torch.zeros(4, 4, device=DEV),
                                torch.zeros(4, 100, dtype=torch.bfloat16, device=DEV))
