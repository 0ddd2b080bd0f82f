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


# ---------------------------------------------------------------------------
# Invalid metadata.  FlashInfer leaves the result undefined when the metadata
# does not place a token inside its request's pages (it indexes kv_indices and
# the cache without checks).  This build's kernels skip such a token and count
# it instead; the functions below restate that rule so the tests can check it.
def token_slot(b: int, p: int, kv_indices, kv_indptr, kv_last_page_len, page_size: int,
               num_pages: int):
    """(page, slot) of token (request b, position p), or None when request b
    does not exist, its page range or last-page length (outside [1, page_size])
    is inconsistent, p lies outside [0, length) or the page id is out of range."""
    batch = len(kv_indptr) - 1
    if b < 0 or b >= batch or p < 0:
        return None
    p0, p1 = int(kv_indptr[b]), int(kv_indptr[b + 1])
    n_pages = p1 - p0
    if n_pages <= 0 or p0 < 0 or p1 > len(kv_indices):
        return None
    last = int(kv_last_page_len[b])
    if last < 1 or last > page_size:
        return None
    if p >= (n_pages - 1) * page_size + last:
        return None
    page = int(kv_indices[p0 + p // page_size])
    if page < 0 or page >= num_pages:
        return None
    return page, p % page_size


def batch_indices_positions_checked(append_indptr, kv_indptr, kv_last_page_len, page_size: int,
                                    nnz: int):
    """Token -> (request, position) from append_indptr, with request -1 for a
    token that no [append_indptr[b], append_indptr[b+1]) range covers (an indptr
    that does not start at 0 or does not ascend)."""
    ai = [int(x) for x in append_indptr]
    ip = [int(x) for x in kv_indptr]
    last = [int(x) for x in kv_last_page_len]
    batch = len(ai) - 1
    bi, pos = [-1] * nnz, [0] * nnz
    for i in range(nnz):
        lo, hi = 0, batch - 1  # largest b with ai[b] <= i, as the kernel searches
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if ai[mid] <= i:
                lo = mid
            else:
                hi = mid - 1
        b = lo
        if not (ai[b] <= i < ai[b + 1]):
            continue
        seq_len = (ip[b + 1] - ip[b] - 1) * page_size + last[b]
        bi[i], pos[i] = b, seq_len - (ai[b + 1] - ai[b]) + (i - ai[b])
    return bi, pos


def append_paged_kv_cache_checked(key, value, batch_indices, positions, cache, kv_indices,
                                  kv_indptr, kv_last_page_len):
    """append_paged_kv_cache with invalid tokens skipped; returns (cache, bad)."""
    page_size, num_pages = cache.shape[2], cache.shape[0]
    heads, hd = cache.shape[3], cache.shape[4]
    k = key.reshape(key.shape[0], heads, hd)
    v = value.reshape(value.shape[0], heads, hd)
    bad = 0
    for i in range(k.shape[0]):
        where = token_slot(int(batch_indices[i]), int(positions[i]), kv_indices, kv_indptr,
                           kv_last_page_len, page_size, num_pages)
        if where is None:
            bad += 1
            continue
        page, slot = where
        cache[page, 0, slot] = k[i]
        cache[page, 1, slot] = v[i]
    return cache, bad
