"""Mixture-of-experts layer on B200: the drop-in for PaceServe's
``fused_experts`` / ``fused_moe``
(paceserve/model_executor/layers/fused_moe/fused_moe.py:411-544 and :547-622),
same arguments and results, every step a kernel of this package:

1. routing: ``moe_ops.topk_softmax`` (``fused_moe`` only) and
   ``moe_ops.moe_align_block_size`` with block 128, so each 128-row block of
   the sorted token list belongs to one expert;
2. ``moe_ops.moe_gather_rows``: the routed rows of ``hidden_states`` in sorted
   order (the reference's Triton kernel gathers them inside each tile);
3. ``moe_ops.moe_expert_gemm`` mode 0: gate/up projection with SiLU-and-mul
   applied to the fp32 accumulator (replaces the first fused_moe_kernel launch
   and ``silu_and_mul`` on intermediate_cache1);
4. ``moe_ops.moe_expert_gemm`` mode 1: down projection times the routing
   weight, rows scattered to the (token, slot) rows of intermediate_cache3
   (the second launch with MUL_ROUTED_WEIGHT);
5. the sum over the top-k slots, as the reference does it (``torch.sum``).

The reference splits the tokens into chunks of 65536 to dodge a Triton issue
(:435-437); these kernels take any count up to their int32 limits, so there is
one chunk.  Quantisation scales (``w1_scale`` ...) are not supported.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import moe_ops

BLOCK_M = 128  # rows per expert block: the GEMM tile height


def _routing(topk_ids: torch.Tensor, num_experts: int):
    numel = topk_ids.numel()
    cap = numel + num_experts * (BLOCK_M - 1)
    dev = topk_ids.device
    sorted_ids = torch.empty(cap, dtype=torch.int32, device=dev)
    expert_ids = torch.empty((cap + BLOCK_M - 1) // BLOCK_M, dtype=torch.int32, device=dev)
    total = torch.empty(1, dtype=torch.int32, device=dev)
    moe_ops.moe_align_block_size(topk_ids.contiguous(), num_experts, BLOCK_M, sorted_ids,
                                 expert_ids, total, True)
    return sorted_ids, expert_ids, total


def fused_experts(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                  topk_weights: torch.Tensor, topk_ids: torch.Tensor, inplace: bool = False,
                  override_config=None, w1_scale=None, w2_scale=None, a1_scale=None,
                  a2_scale=None) -> torch.Tensor:
    """out[t] = sum_j topk_weights[t, j] * (silu(h W1g^T) * (h W1u^T)) W2^T for
    expert e = topk_ids[t, j], h = hidden_states[t]; w1 [E, 2I, H], w2 [E, H, I].
    ``override_config`` (Triton tile sizes) has no meaning here and is ignored."""
    if any(s is not None for s in (w1_scale, w2_scale, a1_scale, a2_scale)):
        raise NotImplementedError("fused_experts: quantisation scales are not supported")
    assert hidden_states.shape[1] == w1.shape[2], "Hidden size mismatch"
    assert topk_weights.shape == topk_ids.shape, "topk shape mismatch"
    assert hidden_states.is_contiguous(), "Hidden_states must be contiguous"
    assert w1.is_contiguous(), "Expert weights1 must be contiguous"
    assert w2.is_contiguous(), "Expert weights2 must be contiguous"
    num_tokens, hidden = hidden_states.shape
    num_experts, n2, _ = w1.shape
    inter = n2 // 2
    top_k = topk_ids.shape[1]
    numel = topk_ids.numel()
    out = hidden_states if inplace else torch.empty_like(hidden_states)
    if num_tokens == 0:
        return out
    dev, dtype = hidden_states.device, hidden_states.dtype
    sorted_ids, expert_ids, total = _routing(topk_ids, num_experts)
    cap = sorted_ids.numel()
    a1 = torch.empty(cap, hidden, dtype=dtype, device=dev)
    moe_ops.moe_gather_rows(a1, hidden_states, sorted_ids, total, numel, top_k)
    act = torch.empty(cap, inter, dtype=dtype, device=dev)
    moe_ops.moe_expert_gemm(act, a1, w1, sorted_ids, expert_ids, total, numel, None, 0)
    cache3 = torch.empty(num_tokens, top_k, w2.shape[1], dtype=dtype, device=dev)
    moe_ops.moe_expert_gemm(cache3.view(numel, -1), act, w2, sorted_ids, expert_ids, total,
                            numel, topk_weights.float().contiguous().view(-1), 1)
    torch.sum(cache3, dim=1, out=out)
    return out


def fused_moe(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
              gating_output: torch.Tensor, topk: int, renormalize: bool, inplace: bool = False,
              override_config=None, use_grouped_topk: bool = False,
              num_expert_group: Optional[int] = None, topk_group: Optional[int] = None,
              w1_scale=None, w2_scale=None, a1_scale=None, a2_scale=None) -> torch.Tensor:
    """Routing (softmax top-k, ties to the lowest expert index, optional
    renormalisation) followed by fused_experts; the reference's fused_moe
    (:547-622).  Grouped top-k (DeepSeek-V2) is not supported."""
    if use_grouped_topk:
        raise NotImplementedError("fused_moe: grouped top-k is not supported")
    assert hidden_states.shape[0] == gating_output.shape[0], "Number of tokens mismatch"
    t = hidden_states.shape[0]
    dev = hidden_states.device
    weights = torch.empty(t, topk, dtype=torch.float32, device=dev)
    ids = torch.empty(t, topk, dtype=torch.int32, device=dev)
    token_expert = torch.empty(t, topk, dtype=torch.int32, device=dev)
    moe_ops.topk_softmax(weights, ids, token_expert, gating_output.float(), renormalize)
    return fused_experts(hidden_states, w1, w2, weights, ids, inplace, override_config,
                         w1_scale, w2_scale, a1_scale, a2_scale)
