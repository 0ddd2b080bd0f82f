"""GPU parity of the MoE expert GEMMs (tcgen05) and the fused_experts /
fused_moe drop-in against the fp32 oracle (oracle/moe_ref.fused_experts_fp32,
the reference's fused_experts restated from the same 16-bit inputs).

Tolerance: the float rule of the per-layer ops, max|got - ref| / max|ref| <=
1e-2.  The B200 path rounds the SiLU-and-mul activation to the storage type
between the two GEMMs, as the reference does (intermediate_cache2), so its
error is a few storage ulps of the activation, well inside the rule."""
import numpy as np
import pytest
import torch

from oracle import moe_ref
from paceserve_b200 import fused_moe as pb_moe
from paceserve_b200 import moe_ops
from tests._util import REL_TOL, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def make(T, H, I, E, k, dtype=torch.bfloat16, seed=0, skew=False):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(T, H, generator=g).to(dtype)
    w1 = (torch.randn(E, 2 * I, H, generator=g) / H ** 0.5).to(dtype)
    w2 = (torch.randn(E, H, I, generator=g) / I ** 0.5).to(dtype)
    gating = torch.randn(T, E, generator=g)
    if skew:  # most tokens to expert 0, none to the last expert
        gating[:, 0] += 3.0
        gating[:, -1] -= 30.0
    return hidden, w1, w2, gating


def routing(gating, k):
    w, ids, _ = moe_ref.topk_softmax(gating.numpy(), k, renormalize=True)
    return torch.from_numpy(np.ascontiguousarray(w)), torch.from_numpy(np.ascontiguousarray(ids))


@pytest.mark.parametrize("T,H,I,E,k", [(64, 256, 512, 8, 2), (1, 512, 256, 8, 2),
                                       (300, 1024, 768, 8, 2), (129, 256, 384, 16, 1),
                                       (500, 512, 256, 4, 4)])
def test_fused_experts_matches_oracle(T, H, I, E, k):
    hidden, w1, w2, gating = make(T, H, I, E, k, seed=T + E)
    tw, ids = routing(gating, k)
    out = pb_moe.fused_experts(hidden.to(DEV), w1.to(DEV), w2.to(DEV), tw.to(DEV),
                               ids.to(DEV).int())
    torch.cuda.synchronize()
    ref = moe_ref.fused_experts_fp32(hidden, w1, w2, tw, ids)
    assert rel_err(out, ref) <= REL_TOL


def test_fused_moe_routing_and_skewed_experts_fp16():
    T, H, I, E, k = 700, 512, 512, 8, 2
    hidden, w1, w2, gating = make(T, H, I, E, k, dtype=torch.float16, seed=3, skew=True)
    out = pb_moe.fused_moe(hidden.to(DEV), w1.to(DEV), w2.to(DEV), gating.to(DEV), k, True)
    torch.cuda.synchronize()
    tw, ids = routing(gating, k)
    assert (ids == E - 1).sum() == 0  # one expert gets no token: its blocks are absent
    ref = moe_ref.fused_experts_fp32(hidden, w1, w2, tw, ids)
    assert rel_err(out, ref) <= REL_TOL


def test_inplace_and_mixtral_widths():
    # Mixtral-8x7B widths (hidden 4096, intermediate 14336), few tokens
    T, H, I, E, k = 48, 4096, 14336, 8, 2
    hidden, w1, w2, gating = make(T, H, I, E, k, seed=11)
    tw, ids = routing(gating, k)
    h_dev = hidden.to(DEV)
    out = pb_moe.fused_experts(h_dev, w1.to(DEV), w2.to(DEV), tw.to(DEV), ids.to(DEV).int(),
                               inplace=True)
    torch.cuda.synchronize()
    assert out.data_ptr() == h_dev.data_ptr()
    ref = moe_ref.fused_experts_fp32(hidden, w1, w2, tw, ids)
    assert rel_err(out, ref) <= REL_TOL


def test_gate_up_silu_rows_in_sorted_order():
    """Mode 0 alone: row i of the output is silu(gate) * up of sorted row i."""
    T, H, I, E, k = 200, 512, 256, 8, 2
    hidden, w1, _, gating = make(T, H, I, E, k, seed=5)
    tw, ids = routing(gating, k)
    ids_d = ids.to(DEV).int()
    sorted_ids, expert_ids, total = pb_moe._routing(ids_d, E)
    numel = ids.numel()
    cap = sorted_ids.numel()
    a1 = torch.full((cap, H), 9.0, dtype=torch.bfloat16, device=DEV)
    moe_ops.moe_gather_rows(a1, hidden.to(DEV), sorted_ids, total, numel, k)
    act = torch.zeros(cap, I, dtype=torch.bfloat16, device=DEV)
    moe_ops.moe_expert_gemm(act, a1, w1.to(DEV), sorted_ids, expert_ids, total, numel, None, 0)
    torch.cuda.synchronize()
    n = int(total.item())
    s = sorted_ids.cpu()[:n].long()
    e_of = expert_ids.cpu().long().repeat_interleave(128)[:n]
    valid = s < numel
    tok = (s[valid] // k)
    # gathered rows: the token's hidden row, zero rows for padding
    assert torch.equal(a1[:n][valid.to(DEV)].cpu(), hidden[tok])
    assert (a1[:n][(~valid).to(DEV)].float() == 0).all()
    gu = torch.einsum("rh,rnh->rn", hidden[tok].float(), w1[e_of[valid]].float())
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    assert rel_err(act[:n][valid.to(DEV)], ref) <= REL_TOL


def test_rejects_bad_shapes():
    a = torch.zeros(128, 64, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(2, 200, 64, dtype=torch.bfloat16, device=DEV)  # 2I = 200: I not a multiple of 128
    ids = torch.zeros(128, dtype=torch.int32, device=DEV)
    out = torch.zeros(128, 100, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        moe_ops.moe_expert_gemm(out, a, w, ids, ids[:1], ids[:1], 2, None, 0)
