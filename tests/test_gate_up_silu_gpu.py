"""GPU parity of activation_ops.gate_up_silu: the MLP's gate_up_proj and
SiLU-and-mul in one tensor-core GEMM, or at decode sizes one weight stream on
the CUDA cores (reference models/llama.py:102-104,
csrc/activation_kernels.cu:15-45), optionally with the post-attention RMSNorm
applied as a per-row factor (norm weight folded into the GEMM weight).

Oracle: the reference's composition in fp32 from the same 16-bit inputs,
silu(x @ Wg^T) * (x @ Wu^T) with x the rows (or rms_norm_fp32 of them,
oracle/ops_ref.py), matmuls in fp32 on the device with TF32 off.  Tolerance:
max|got - ref| / max|ref| <= 1e-2, plus a per-element bound of 2 storage ulps
of the element and 3e-3 of the largest magnitude (the fused path keeps gate
and up in fp32 where the reference rounds them to 16 bits first)."""
import pytest
import torch

import paceserve_b200 as pb
from oracle import ops_ref
from paceserve_b200 import activation_ops, layernorm_ops
from tests._util import REL_TOL, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
EPS = 1e-5


def close(got, ref, dtype, ulps=2.0, frac=3e-3):
    assert rel_err(got, ref) <= REL_TOL
    g, r = got.float().cpu(), ref.float().cpu()
    bound = ulps * torch.finfo(dtype).eps * r.abs() + frac * r.abs().max()
    assert ((g - r).abs() <= bound).all(), ((g - r).abs() - bound).max().item()


def rnd(shape, g, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def ref_gate_up(x32, w, inter):
    """silu(gate) * up in fp32; x32 fp32 rows on the device, w [2 I, H]."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        gu = x32 @ w.float().t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    gate, up = gu[:, :inter], gu[:, inter:]
    return gate * torch.sigmoid(gate) * up


@pytest.mark.parametrize("T,H,I", [(1, 4096, 14336), (2, 200, 384), (3, 1024, 256),
                                   (37, 1024, 512), (200, 1024, 384), (512, 4096, 14336),
                                   (1000, 2048, 1024)])
def test_gate_up_silu(T, H, I):
    # T <= 2: the weight-streaming kernel on CUDA cores (H = 200: fewer 16-byte
    # vectors per row than lanes); from T = 3 the tensor-core GEMM
    g = torch.Generator().manual_seed(T + H + I)
    x = rnd((T, H), g).to(DEV)
    w = rnd((2 * I, H), g, H ** -0.5).to(DEV)
    out = torch.full((T, I), float("nan"), dtype=torch.bfloat16, device=DEV)
    activation_ops.gate_up_silu(out, x, w)
    torch.cuda.synchronize()
    close(out, ref_gate_up(x.float(), w, I), torch.bfloat16)


def test_gate_up_silu_fewer_leftover_units_than_ctas():
    """SMs + 2 tiles of 16 K blocks (one data-parallel round, then 32 units for
    all the CTAs), twice: counters re-armed, no fault."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    T, H, I = 3, 1024, 128 * (sms + 2)
    g = torch.Generator().manual_seed(3)
    x = rnd((T, H), g).to(DEV)
    w = rnd((2 * I, H), g, H ** -0.5).to(DEV)
    ref = ref_gate_up(x.float(), w, I)
    fault = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):
        out = torch.full((T, I), float("nan"), dtype=torch.bfloat16, device=DEV)
        activation_ops.gate_up_silu(out, x, w, fault_flags=fault)
        torch.cuda.synchronize()
        assert fault.item() == 0
        close(out, ref, torch.bfloat16)


@pytest.mark.parametrize("T", [2, 130])
def test_gate_up_silu_float16_and_strided_rows(T):
    H, I = 1024, 640
    g = torch.Generator().manual_seed(5)
    wide = rnd((T, H + 64), g, dtype=torch.float16).to(DEV)
    x = wide[:, 32:32 + H]  # row stride H + 64, 64-byte offset
    w = rnd((2 * I, H), g, H ** -0.5, dtype=torch.float16).to(DEV)
    out_wide = torch.zeros(T, I + 128, dtype=torch.float16, device=DEV)
    out = out_wide[:, :I]
    activation_ops.gate_up_silu(out, x, w)
    torch.cuda.synchronize()
    close(out, ref_gate_up(x.float(), w, I), torch.float16)
    assert (out_wide[:, I:] == 0).all()  # nothing written past the output columns


@pytest.mark.parametrize("T", [1, 2, 96, 512])
def test_gate_up_rmsnorm_silu(T):
    H, I = 4096, 14336
    g = torch.Generator().manual_seed(T * 7)
    h = rnd((T, H), g)
    w_norm = (torch.randn(H, generator=g) * 0.02 + 1).to(torch.bfloat16)
    w = rnd((2 * I, H), g, H ** -0.5).to(DEV)
    h_d = h.to(DEV)
    ss = torch.empty(T, H // 32, device=DEV)
    layernorm_ops.row_sumsq(ss, h_d)
    out = torch.empty(T, I, dtype=torch.bfloat16, device=DEV)
    activation_ops.gate_up_silu(out, h_d, pb.fold_rmsnorm_weight(w, w_norm.to(DEV)), ss, EPS)
    torch.cuda.synchronize()
    x = ops_ref.rms_norm_fp32(h, w_norm, EPS).to(DEV)
    close(out, ref_gate_up(x, w, I), torch.bfloat16)


def test_fused_mlp_matches_unfused_ops():
    """The MLP half of a layer, fused: post-attention norm factor + gate_up +
    SiLU-and-mul (gate_up_silu), then down_proj + residual add
    (linear_residual); against this package's unfused path: fused_add_rms_norm,
    torch matmul, silu_and_mul, torch matmul, add."""
    T, H, I = 300, 1024, 2816
    g = torch.Generator().manual_seed(11)
    attn = rnd((T, H), g).to(DEV)
    res0 = rnd((T, H), g).to(DEV)
    w_norm = (torch.randn(H, generator=g) * 0.02 + 1).to(torch.bfloat16).to(DEV)
    w_gu = rnd((2 * I, H), g, H ** -0.5).to(DEV)
    w_down = rnd((H, I), g, I ** -0.5).to(DEV)
    # fused: residual += attn (the o_proj epilogue's job; a plain add here),
    # partials from row_sumsq, then the two GEMMs
    res_f = res0 + attn
    ss = torch.empty(T, H // 32, device=DEV)
    layernorm_ops.row_sumsq(ss, res_f)
    act_f = torch.empty(T, I, dtype=torch.bfloat16, device=DEV)
    activation_ops.gate_up_silu(act_f, res_f, pb.fold_rmsnorm_weight(w_gu, w_norm), ss, EPS)
    layernorm_ops.linear_residual(res_f, act_f, w_down)
    # unfused
    x = attn.clone()
    res_u = res0.clone()
    layernorm_ops.fused_add_rms_norm(x, res_u, w_norm, EPS)
    gu = x @ w_gu.t()
    act_u = torch.empty(T, I, dtype=torch.bfloat16, device=DEV)
    activation_ops.silu_and_mul(act_u, gu)
    res_u = res_u + act_u @ w_down.t()
    torch.cuda.synchronize()
    assert rel_err(act_f, act_u) <= REL_TOL
    assert rel_err(res_f, res_u) <= REL_TOL


def test_gate_up_silu_rejected_inputs():
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        activation_ops.gate_up_silu(torch.zeros(4, 200, dtype=torch.bfloat16, device=DEV), x,
                                    torch.zeros(400, 64, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(RuntimeError, match="shapes do not match"):
        activation_ops.gate_up_silu(torch.zeros(4, 128, dtype=torch.bfloat16, device=DEV), x,
                                    torch.zeros(128, 64, dtype=torch.bfloat16, device=DEV))
    # no rows: nothing launched, no error
    activation_ops.gate_up_silu(torch.zeros(0, 128, dtype=torch.bfloat16, device=DEV),
                                torch.zeros(0, 64, dtype=torch.bfloat16, device=DEV),
                                torch.zeros(256, 64, dtype=torch.bfloat16, device=DEV))
