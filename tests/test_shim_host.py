"""CPU: the torch shim keeps the reference's module names and call signatures
and rejects what it cannot run with RuntimeError, before any GPU work."""
import inspect
import re

import pytest
import torch

import paceserve_b200
from paceserve_b200 import activation_ops, kv_transfer_ops, layernorm_ops, moe_ops, pos_encoding_ops

# name -> positional parameters of the reference binding (csrc/*.cpp)
REFERENCE_SIGNATURES = {
    (layernorm_ops, "rms_norm"): ["out", "input", "weight", "epsilon"],
    (pos_encoding_ops, "rotary_embedding"): ["positions", "query", "key", "head_size",
                                             "cos_sin_cache", "is_neox"],
    (activation_ops, "silu_and_mul"): ["out", "input"],
    (activation_ops, "gelu_new"): ["out", "input"],
    (activation_ops, "gelu_fast"): ["out", "input"],
    (moe_ops, "topk_softmax"): ["topk_weights", "topk_indices", "token_expert_indices",
                                "gating_output"],
    (moe_ops, "moe_align_block_size"): ["topk_ids", "num_experts", "block_size",
                                        "sorted_token_ids", "experts_ids", "num_tokens_post_pad"],
}


def _params(fn):
    sig = fn.__doc__.splitlines()[0]
    inner = sig[sig.index("(") + 1: sig.rindex(")")]
    return [re.split(r"[:=]", p)[0].strip() for p in inner.split(",") if p.strip()]


@pytest.mark.parametrize("mod,name", list(REFERENCE_SIGNATURES), ids=lambda x: getattr(x, "__name__", x))
def test_reference_signatures_preserved(mod, name):
    got = _params(getattr(mod, name))
    want = REFERENCE_SIGNATURES[(mod, name)]
    assert got[: len(want)] == want


def test_new_ops_present():
    assert _params(layernorm_ops.fused_add_rms_norm) == ["input", "residual", "weight", "epsilon"]
    assert _params(activation_ops.gelu_and_mul) == ["out", "input"]
    assert _params(activation_ops.gelu_tanh_and_mul) == ["out", "input"]
    assert _params(kv_transfer_ops.copy_blocks_p2p)[:4] == ["src_caches", "dst_caches",
                                                            "src_block_ids", "dst_block_ids"]


def test_cpu_tensors_rejected():
    x = torch.randn(4, 16)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        layernorm_ops.rms_norm(torch.empty_like(x), x, torch.ones(16), 1e-5)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        layernorm_ops.fused_add_rms_norm(x, x.clone(), torch.ones(16), 1e-5)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        activation_ops.silu_and_mul(torch.empty(4, 8), x)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        moe_ops.topk_softmax(torch.empty(4, 2), torch.empty(4, 2, dtype=torch.int32),
                             torch.empty(4, 2, dtype=torch.int32), torch.randn(4, 8))
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        moe_ops.moe_align_block_size(torch.zeros(8, dtype=torch.int32), 8, 64,
                                     torch.empty(600, dtype=torch.int32),
                                     torch.empty(10, dtype=torch.int32),
                                     torch.empty(1, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        pos_encoding_ops.rotary_embedding(torch.zeros(4, dtype=torch.long), torch.randn(4, 256),
                                          torch.randn(4, 128), 128, torch.randn(16, 128), True)
    with pytest.raises(RuntimeError, match="CUDA tensors on one device"):
        kv_transfer_ops.copy_blocks_p2p([torch.zeros(2, 16)], [torch.zeros(2, 16)],
                                        torch.zeros(1, dtype=torch.int32),
                                        torch.zeros(1, dtype=torch.int32))


def test_install_as_paceserve_registers_modules():
    import sys

    paceserve_b200.install_as_paceserve()
    from paceserve import layernorm_ops as ln  # noqa: F401  (the reference's import form)

    assert sys.modules["paceserve.layernorm_ops"] is layernorm_ops
    assert sys.modules["paceserve.moe_ops"] is moe_ops
    assert inspect.ismodule(sys.modules["paceserve.activation_ops"])


def test_fused_moe_dropin_signatures():
    """paceserve_b200.fused_moe keeps the parameter names and order of the
    reference's fused_experts / fused_moe (fused_moe.py:411-425, :547-563)."""
    from paceserve_b200 import fused_moe as pb_moe

    assert list(inspect.signature(pb_moe.fused_experts).parameters) == [
        "hidden_states", "w1", "w2", "topk_weights", "topk_ids", "inplace", "override_config",
        "w1_scale", "w2_scale", "a1_scale", "a2_scale"]
    assert list(inspect.signature(pb_moe.fused_moe).parameters) == [
        "hidden_states", "w1", "w2", "gating_output", "topk", "renormalize", "inplace",
        "override_config", "use_grouped_topk", "num_expert_group", "topk_group", "w1_scale",
        "w2_scale", "a1_scale", "a2_scale"]


def test_new_gemm_ops_present_and_reject_cpu_tensors():
    assert _params(pos_encoding_ops.qkv_proj_rotary_embedding)[:9] == [
        "qkv", "hidden", "weight", "positions", "head_size", "num_heads", "num_kv_heads",
        "cos_sin_cache", "is_neox"]
    assert _params(moe_ops.moe_expert_gemm)[:9] == [
        "out", "a", "w", "sorted_token_ids", "expert_ids", "num_tokens_post_pad", "numel",
        "topk_weights", "mode"]
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        pos_encoding_ops.qkv_proj_rotary_embedding(torch.empty(4, 512, dtype=torch.bfloat16), x,
                                                   torch.zeros(512, 64, dtype=torch.bfloat16),
                                                   torch.zeros(4, dtype=torch.long), 128, 2, 1,
                                                   torch.zeros(16, 128), True)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        moe_ops.moe_expert_gemm(x, x, torch.zeros(2, 256, 64, dtype=torch.bfloat16),
                                torch.zeros(128, dtype=torch.int32),
                                torch.zeros(1, dtype=torch.int32),
                                torch.zeros(1, dtype=torch.int32), 4, None, 0)


def test_fused_norm_gemm_ops_present():
    assert _params(layernorm_ops.linear_residual)[:4] == ["residual", "input", "weight",
                                                          "row_sumsq"]
    assert _params(layernorm_ops.row_sumsq) == ["out", "input"]
    assert _params(pos_encoding_ops.qkv_proj_rmsnorm_rotary_embedding)[:11] == [
        "qkv", "hidden", "folded_weight", "row_sumsq", "epsilon", "positions", "head_size",
        "num_heads", "num_kv_heads", "cos_sin_cache", "is_neox"]
    w = torch.randn(6, 4).bfloat16()
    nw = torch.tensor([1.0, 2.0, 0.5, -1.0]).bfloat16()
    folded = paceserve_b200.fold_rmsnorm_weight(w, nw)
    assert torch.equal(folded, (w.float() * nw.float()).bfloat16())


def test_gate_up_silu_present_and_rejects_cpu_tensors():
    assert _params(activation_ops.gate_up_silu)[:5] == ["out", "hidden", "weight", "row_sumsq",
                                                       "epsilon"]
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        activation_ops.gate_up_silu(torch.empty(4, 128, dtype=torch.bfloat16),
                                    torch.zeros(4, 64, dtype=torch.bfloat16),
                                    torch.zeros(256, 64, dtype=torch.bfloat16))
