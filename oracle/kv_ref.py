"""Restatement of the reference's KV move (KVhelper, paceserve/kv_transfer/kv_utils.py:33-56).

TEST / MEASUREMENT INFRASTRUCTURE ONLY: used by the tests as a layout oracle and
by bench.py's baseline leg to time the reference mechanism on the GPU box.
PaceServe moves a sequence's blocks GPU -> CPU with one fancy-index gather
per layer into a CPU tensor (kv_utils.py:44-46), ships it through the Ray
object store, and scatters it on the other GPU with one index-put per layer
after a host-to-device copy (kv_utils.py:51-52).  The object-store hop is not
reproduced (no Ray here), so timings of this path are a lower bound.
"""
from __future__ import annotations

import torch


def get_kv_cache(gpu_cache, block_ids):
    """kv_utils.py:44-47: CPU tensor [L, n, *block] gathered layer by layer."""
    L = len(gpu_cache)
    n = len(block_ids)
    seq_cache = torch.zeros(L, n, *gpu_cache[0].shape[1:], dtype=gpu_cache[0].dtype)
    idx = torch.tensor(list(block_ids))
    for i in range(L):
        seq_cache[i] = gpu_cache[i][idx, :, :, :, :]
    return seq_cache


def insert_kv_cache(gpu_cache, cached_content, kv_indices, device):
    """kv_utils.py:51-52: per-layer index-put of the host content."""
    idx = torch.tensor(list(kv_indices))
    for i in range(len(gpu_cache)):
        gpu_cache[i][idx, :, :, :, :] = cached_content[i].to(device)
