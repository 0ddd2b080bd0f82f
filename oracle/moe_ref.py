"""numpy restatements of the MoE routing ops (integer outputs bit-exact).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
C_SRC = os.path.join(HERE, "moe_align_ref.c")
C_LIB = os.path.join(HERE, "_build", "libmoe_align_ref.so")


# ----------------------------------------------------------- topk_softmax --
def _pow2_split(E: int):
    """Column ownership of the reference's fused kernel for power-of-two E
    (csrc/moe_topk_softmax_kernels.cu:385-394, :236-257): vectors of LDG floats,
    VECS per lane, TPR lanes per row; lane g owns columns (v*TPR+g)*LDG + j."""
    ldg = min(4, E)
    vecs = max(1, E // (ldg * 32))
    vpt = vecs * ldg
    tpr = E // vpt
    return ldg, vecs, tpr


def softmax_rows(gating: np.ndarray) -> np.ndarray:
    """fp32 softmax per row with the reference's summation association
    (csrc/moe_topk_softmax_kernels.cu:259-303): per-lane sequential sum of the
    owned columns, XOR-butterfly over the TPR lanes, one reciprocal, multiply.
    Non-power-of-two / >256 E use a plain sequential fp32 sum."""
    g = np.ascontiguousarray(gating, dtype=np.float32)
    T, E = g.shape
    mx = g.max(axis=1, keepdims=True)
    e = np.exp((g - mx).astype(np.float32)).astype(np.float32)
    if E & (E - 1) == 0 and E <= 256:
        ldg, vecs, tpr = _pow2_split(E)
        lane_sum = np.zeros((T, tpr), dtype=np.float32)
        for lane in range(tpr):
            for v in range(vecs):
                for j in range(ldg):
                    c = (v * tpr + lane) * ldg + j
                    lane_sum[:, lane] = (lane_sum[:, lane] + e[:, c]).astype(np.float32)
        m = tpr // 2
        while m > 0:
            lane_sum = (lane_sum + lane_sum[:, np.arange(tpr) ^ m]).astype(np.float32)
            m //= 2
        s = lane_sum[:, 0]
    else:
        s = np.zeros(T, dtype=np.float32)
        for c in range(E):
            s = (s + e[:, c]).astype(np.float32)
    rcp = (np.float32(1.0) / s).astype(np.float32)
    return (e * rcp[:, None]).astype(np.float32)


def topk_softmax(gating: np.ndarray, k: int, renormalize: bool = False):
    """Reference topk_softmax (csrc/moe_topk_softmax_kernels.cu:305-380): k
    rounds of argmax over the softmax row, ties to the lowest expert index;
    token_expert_indices[t, j] = j*T + t; optional renormalisation as in
    fused_topk (paceserve/model_executor/layers/fused_moe/fused_moe.py:371-372).
    Returns (weights f32 [T,k], ids i32 [T,k], token_expert_indices i32 [T,k])."""
    p = softmax_rows(gating)
    T, E = p.shape
    work = p.copy()
    w = np.zeros((T, k), dtype=np.float32)
    ids = np.zeros((T, k), dtype=np.int32)
    rows = np.arange(T)
    for j in range(k):
        best = np.argmax(work, axis=1)  # first occurrence = lowest index on ties
        w[:, j] = work[rows, best]
        ids[:, j] = best
        work[rows, best] = -np.inf
    if renormalize:
        s = np.zeros(T, dtype=np.float32)
        for j in range(k):
            s = (s + w[:, j]).astype(np.float32)
        w = (w / s[:, None]).astype(np.float32)
    tei = (np.arange(k, dtype=np.int64)[None, :] * T + rows[:, None]).astype(np.int32)
    return w, ids, tei


# --------------------------------------------------- moe_align_block_size --
def moe_align_block_size(topk_ids: np.ndarray, num_experts: int, block_size: int):
    """csrc/moe_align_block_size_kernels.cu:41-108 restated: counts per expert,
    cumsum of counts padded to block_size, expert id per block, and each
    expert's flat indices in ascending order at cumsum[e] + rank.  Padding
    slots hold numel (the wrapper's pre-fill, fused_moe.py:191-195).  Ids
    outside [0, E) are skipped.  Returns (sorted_ids [numel + E*(bs-1)],
    expert_ids [total // bs], total)."""
    ids = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    numel = ids.size
    E, bs = int(num_experts), int(block_size)
    valid = (ids >= 0) & (ids < E)
    cnt = np.bincount(ids[valid], minlength=E).astype(np.int64)
    padded = (cnt + bs - 1) // bs * bs
    cum = np.concatenate([[0], np.cumsum(padded)]).astype(np.int64)
    total = int(cum[E])
    sorted_ids = np.full(numel + E * (bs - 1), numel, dtype=np.int32)
    for e in range(E):
        where = np.nonzero(ids == e)[0]
        sorted_ids[cum[e]: cum[e] + where.size] = where.astype(np.int32)
    blocks = total // bs
    expert_ids = np.searchsorted(cum, np.arange(blocks) * bs, side="right").astype(np.int32) - 1
    return sorted_ids, expert_ids.astype(np.int32), total


def build_c(force: bool = False) -> str:
    """Compile moe_align_ref.c with gcc into oracle/_build."""
    os.makedirs(os.path.dirname(C_LIB), exist_ok=True)
    if force or not os.path.exists(C_LIB) or os.path.getmtime(C_LIB) < os.path.getmtime(C_SRC):
        subprocess.run(["gcc", "-O2", "-std=c11", "-shared", "-fPIC", C_SRC, "-o", C_LIB], check=True)
    return C_LIB


def moe_align_block_size_c(topk_ids: np.ndarray, num_experts: int, block_size: int):
    """Same contract as moe_align_block_size, computed by the C restatement."""
    lib = ctypes.CDLL(C_LIB if os.path.exists(C_LIB) else build_c())
    fn = lib.moe_align_block_size_ref
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    ids = np.ascontiguousarray(np.asarray(topk_ids).reshape(-1), dtype=np.int64)
    numel = ids.size
    cap = numel + num_experts * (block_size - 1)
    sorted_ids = np.full(cap, numel, dtype=np.int32)
    ecap = (cap + block_size - 1) // block_size
    expert_ids = np.full(ecap, -1, dtype=np.int32)
    total = np.zeros(1, dtype=np.int32)
    rc = fn(ids.ctypes.data, numel, num_experts, block_size, sorted_ids.ctypes.data, cap,
            expert_ids.ctypes.data, ecap, total.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"moe_align_block_size_ref returned {rc}")
    t = int(total[0])
    return sorted_ids, expert_ids[: t // block_size].copy(), t


# ----------------------------------------------------------- fused experts --
def fused_experts_fp32(hidden, w1, w2, topk_weights, topk_ids):
    """fp32 restatement of fused_experts
    (paceserve/model_executor/layers/fused_moe/fused_moe.py:411-544) from the
    same 16-bit inputs: for every token t and slot j with expert
    e = topk_ids[t, j], y = silu(h W1[e, :I]^T) * (h W1[e, I:]^T) (the first
    fused_moe_kernel launch, then silu_and_mul at :518-520), z = topk_weights[t, j]
    * (y W2[e]^T) (the second launch with MUL_ROUTED_WEIGHT, :138-140), and
    out[t] = sum_j z (:539-543).  torch tensors in, fp32 [T, H] out; done per
    expert over the tokens routed to it."""
    import torch

    h = hidden.float()
    w1f, w2f = w1.float(), w2.float()
    inter = w1.shape[1] // 2
    T, k = topk_ids.shape
    out = torch.zeros(T, w2.shape[1], dtype=torch.float32)
    ids = topk_ids.long()
    tw = topk_weights.float()
    for e in range(w1.shape[0]):
        tok, slot = (ids == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        x = h[tok]
        gu = x @ w1f[e].t()
        y = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
        z = (y @ w2f[e].t()) * tw[tok, slot][:, None]
        out.index_add_(0, tok, z)
    return out
