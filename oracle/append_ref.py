"""Restatement of FlashInfer's paged-KV append, as PaceServe uses it.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

FlashInfer (PaceServe pins ``flashinfer==0.2.0+cu121torch2.3``,
requirements.txt:40; not vendored, binary) owns the append.  PaceServe's call
site (paceserve/model_executor/attention/flashinfer_attention_wrapper.py:
239-255) computes ``seq_lens = get_seq_lens(kv_indptr, kv_last_page_len,
page_size)`` and ``batch_indices, positions =
get_batch_indices_positions(append_indptr, seq_lens, nnz)``, then calls
``append_paged_kv_cache(key, value, batch_indices, positions, cache,
kv_indices, kv_indptr, kv_last_page_len, kv_layout="NHD")``.  The metadata
comes from ``begin_forward`` (:75-209).  The published semantics, restated
here in plain torch on the CPU:

* seq_len[b] = (kv_indptr[b+1] - kv_indptr[b] - 1) * page_size + kv_last_page_len[b]
* request b's appended tokens are the last append_indptr[b+1] - append_indptr[b]
  tokens of its sequence: positions seq_len[b] - n_b + j
* token (b, p) goes to page kv_indices[kv_indptr[b] + p // page_size], slot
  p % page_size; K at cache[page, 0, slot], V at cache[page, 1, slot].
"""
from __future__ import annotations

import torch


def get_seq_lens(kv_indptr: torch.Tensor, kv_last_page_len: torch.Tensor, page_size: int):
    ip = kv_indptr.long()
    return (ip[1:] - ip[:-1] - 1) * page_size + kv_last_page_len.long()


def get_batch_indices_positions(append_indptr: torch.Tensor, seq_lens: torch.Tensor, nnz: int):
    ai = append_indptr.long().tolist()
    sl = seq_lens.long().tolist()
    bi = torch.empty(nnz, dtype=torch.int32)
    pos = torch.empty(nnz, dtype=torch.int32)
    for b in range(len(ai) - 1):
        n = ai[b + 1] - ai[b]
        for j in range(n):
            bi[ai[b] + j] = b
            pos[ai[b] + j] = sl[b] - n + j
    return bi, pos


def append_paged_kv_cache(key, value, batch_indices, positions, cache, kv_indices, kv_indptr,
                          kv_last_page_len):
    """In place on the CPU tensor `cache` [pages, 2, page_size, heads, hd]."""
    page_size = cache.shape[2]
    heads, hd = cache.shape[3], cache.shape[4]
    k = key.reshape(key.shape[0], heads, hd)
    v = value.reshape(value.shape[0], heads, hd)
    ki = kv_indices.long().tolist()
    ip = kv_indptr.long().tolist()
    for i in range(k.shape[0]):
        b = int(batch_indices[i])
        p = int(positions[i])
        page = ki[ip[b] + p // page_size]
        cache[page, 0, p % page_size] = k[i]
        cache[page, 1, p % page_size] = v[i]
    return cache
