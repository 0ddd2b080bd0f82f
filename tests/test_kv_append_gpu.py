"""GPU: paged-KV append (FlashInfer append_paged_kv_cache semantics, as PaceServe
calls it at flashinfer_attention_wrapper.py:239-255), byte-exact against the
CPU restatement, for a Sarathi mixed batch built like begin_forward (:75-209)."""
import numpy as np
import pytest
import torch

from oracle import append_ref
from paceserve_b200 import cabi, kv_transfer_ops as kv

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def mixed_batch(rng, page_size=16, num_pages=600, prefills=((448, 0),), decodes=64, max_ctx=2000):
    """Metadata as begin_forward builds it: prefill chunks first (chunk length,
    tokens already processed), then decode requests of random context length.
    Pages are distinct random pages of the cache."""
    free = list(rng.permutation(num_pages))
    append_indptr, kv_indptr, kv_indices, last = [0], [0], [], []
    for chunk, done in prefills:
        total = done + chunk
        n_pages = (total + page_size - 1) // page_size
        kv_indices += [free.pop() for _ in range(n_pages)]
        append_indptr.append(append_indptr[-1] + chunk)
        kv_indptr.append(kv_indptr[-1] + n_pages)
        last.append(total % page_size or page_size)
    for _ in range(decodes):
        ctx = int(rng.integers(1, max_ctx))
        n_pages = (ctx + page_size - 1) // page_size
        kv_indices += [free.pop() for _ in range(n_pages)]
        append_indptr.append(append_indptr[-1] + 1)
        kv_indptr.append(kv_indptr[-1] + n_pages)
        last.append(ctx % page_size or page_size)
    t = lambda x: torch.tensor(x, dtype=torch.int32)  # noqa: E731
    return t(append_indptr), t(kv_indptr), t(kv_indices), t(last)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("form", ["indices", "indptr"])
def test_append_mixed_batch_matches_oracle(dtype, form):
    rng = np.random.default_rng(3)
    nq, nkv, hd, P, ps = 32, 8, 128, 2000, 16
    ai, kp, ki, kl = mixed_batch(rng, ps, P, prefills=((448, 0), (37, 100)), decodes=64, max_ctx=512)
    nnz = int(ai[-1])
    g = torch.Generator().manual_seed(4)
    qkv = torch.randn(nnz, (nq + 2 * nkv) * hd, generator=g).to(dtype)
    key, value = qkv[:, nq * hd: (nq + nkv) * hd], qkv[:, (nq + nkv) * hd:]
    cache = torch.randn(P, 2, ps, nkv, hd, generator=g).to(dtype)
    seq = append_ref.get_seq_lens(kp, kl, ps)
    bi, pos = append_ref.get_batch_indices_positions(ai, seq, nnz)
    ref = append_ref.append_paged_kv_cache(key, value, bi, pos, cache.clone(), ki, kp, kl)
    got = cache.to(DEV)
    qd = qkv.to(DEV)
    kd, vd = qd[:, nq * hd: (nq + nkv) * hd], qd[:, (nq + nkv) * hd:]  # strided views
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    if form == "indices":
        kv.append_paged_kv_cache(kd, vd, bi.to(DEV), pos.to(DEV), got, ki.to(DEV), kp.to(DEV),
                                 kl.to(DEV), "NHD", bad)
    else:
        kv.append_paged_kv_cache_by_indptr(kd, vd, ai.to(DEV), got, ki.to(DEV), kp.to(DEV),
                                           kl.to(DEV), bad)
    torch.cuda.synchronize()
    assert bad.item() == 0
    assert torch.equal(got.cpu(), ref)


def test_append_3d_rows_decode_only_and_unaligned_heads():
    rng = np.random.default_rng(5)
    nkv, hd, P, ps = 2, 36, 1000, 16  # 72-element rows: not a multiple of 16 bytes in bf16 -> scalar path
    ai, kp, ki, kl = mixed_batch(rng, ps, P, prefills=(), decodes=40, max_ctx=300)
    nnz = int(ai[-1])
    key = torch.randn(nnz, nkv, hd).bfloat16()
    value = torch.randn(nnz, nkv, hd).bfloat16()
    cache = torch.zeros(P, 2, ps, nkv, hd).bfloat16()
    bi, pos = append_ref.get_batch_indices_positions(ai, append_ref.get_seq_lens(kp, kl, ps), nnz)
    ref = append_ref.append_paged_kv_cache(key, value, bi, pos, cache.clone(), ki, kp, kl)
    got = cache.to(DEV)
    kv.append_paged_kv_cache_by_indptr(key.to(DEV), value.to(DEV), ai.to(DEV), got, ki.to(DEV),
                                       kp.to(DEV), kl.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), ref)


def test_append_bad_tokens_skipped_and_counted():
    nkv, hd, P, ps = 8, 128, 8, 16
    key = torch.randn(4, nkv * hd, device=DEV).bfloat16()
    value = torch.randn(4, nkv * hd, device=DEV).bfloat16()
    cache = torch.zeros(P, 2, ps, nkv, hd, device=DEV).bfloat16()
    kp = torch.tensor([0, 2], dtype=torch.int32, device=DEV)        # one request, 2 pages
    kl = torch.tensor([5], dtype=torch.int32, device=DEV)           # length 21
    ki = torch.tensor([3, 99], dtype=torch.int32, device=DEV)       # second page out of range
    bi = torch.tensor([0, 0, 1, 0], dtype=torch.int32, device=DEV)  # token 2: no request 1
    pos = torch.tensor([0, 20, 3, 21], dtype=torch.int32, device=DEV)  # 20 -> page 99; 21 >= length
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    kv.append_paged_kv_cache(key, value, bi, pos, cache, ki, kp, kl, "NHD", bad)
    torch.cuda.synchronize()
    assert bad.item() == 3
    assert torch.equal(cache[3, 0, 0], key[0].view(nkv, hd))
    assert torch.equal(cache[3, 1, 0], value[0].view(nkv, hd))
    assert int(cache.ne(0).sum()) == 2 * nkv * hd
    with pytest.raises(RuntimeError, match="NHD"):
        kv.append_paged_kv_cache(key, value, bi, pos, cache, ki, kp, kl, "HND")
    # a counter in host memory is rejected before any launch
    with pytest.raises(RuntimeError, match="bad_tokens must be an int32 tensor"):
        kv.append_paged_kv_cache(key, value, bi, pos, cache, ki, kp, kl, "NHD",
                                 torch.zeros(1, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="bad_tokens must be an int32 tensor"):
        kv.append_paged_kv_cache_by_indptr(key, value, torch.tensor([0, 4], dtype=torch.int32,
                                                                    device=DEV),
                                           cache, ki, kp, kl, torch.zeros(1, dtype=torch.int64,
                                                                          device=DEV))


@pytest.mark.parametrize("form", ["indices", "indptr"])
@pytest.mark.parametrize("last_len", [17, 0, -3])
def test_append_inconsistent_last_page_len_is_skipped(form, last_len):
    """kv_last_page_len outside [1, page_size] makes a request's length disagree
    with its page count; its tokens must be counted, never written (in the
    unchecked case position 20 would select kv_indices[p0 + 1], the next
    request's page)."""
    nkv, hd, P, ps = 8, 128, 8, 16
    rng = np.random.default_rng(3)
    ai = torch.tensor([0, 2, 3], dtype=torch.int32)
    kp = torch.tensor([0, 1, 2], dtype=torch.int32)        # one page per request
    ki = torch.tensor([5, 6], dtype=torch.int32)
    kl = torch.tensor([last_len, 4], dtype=torch.int32)   # request 0 inconsistent
    key = torch.from_numpy(rng.standard_normal((3, nkv * hd)).astype(np.float32)).bfloat16()
    value = torch.from_numpy(rng.standard_normal((3, nkv * hd)).astype(np.float32)).bfloat16()
    cache = torch.zeros(P, 2, ps, nkv, hd).bfloat16()
    if form == "indices":
        bi = torch.tensor([0, 0, 1], dtype=torch.int32)
        pos = torch.tensor([15, 16, 3], dtype=torch.int32)
    else:
        b_, p_ = append_ref.batch_indices_positions_checked(ai, kp, kl, ps, 3)
        bi, pos = torch.tensor(b_, dtype=torch.int32), torch.tensor(p_, dtype=torch.int32)
    want, nbad = append_ref.append_paged_kv_cache_checked(key, value, bi, pos, cache.clone(), ki,
                                                          kp, kl)
    assert nbad >= 1
    got = cache.to(DEV)
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    if form == "indices":
        kv.append_paged_kv_cache(key.to(DEV), value.to(DEV), bi.to(DEV), pos.to(DEV), got,
                                 ki.to(DEV), kp.to(DEV), kl.to(DEV), "NHD", bad)
    else:
        kv.append_paged_kv_cache_by_indptr(key.to(DEV), value.to(DEV), ai.to(DEV), got, ki.to(DEV),
                                           kp.to(DEV), kl.to(DEV), bad)
    torch.cuda.synchronize()
    assert bad.item() == nbad
    assert torch.equal(got.cpu(), want)
    assert torch.equal(got[6, 0, 3].cpu(), key[2].view(nkv, hd))  # the valid request landed


def test_append_indptr_not_starting_at_zero_is_skipped():
    """append_indptr[0] > 0: tokens before it belong to no request and are
    counted; the kernel must not place them inside request 0's window."""
    nkv, hd, P, ps = 8, 128, 8, 16
    ai = torch.tensor([2, 4], dtype=torch.int32)   # tokens 0 and 1 are uncovered
    kp = torch.tensor([0, 2], dtype=torch.int32)
    ki = torch.tensor([1, 4], dtype=torch.int32)
    kl = torch.tensor([9], dtype=torch.int32)      # length 25
    key = torch.randn(4, nkv * hd).bfloat16()
    value = torch.randn(4, nkv * hd).bfloat16()
    cache = torch.zeros(P, 2, ps, nkv, hd).bfloat16()
    b_, p_ = append_ref.batch_indices_positions_checked(ai, kp, kl, ps, 4)
    assert b_ == [-1, -1, 0, 0] and p_[2:] == [23, 24]
    want, nbad = append_ref.append_paged_kv_cache_checked(
        key, value, torch.tensor(b_, dtype=torch.int32), torch.tensor(p_, dtype=torch.int32),
        cache.clone(), ki, kp, kl)
    assert nbad == 2
    got = cache.to(DEV)
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    kv.append_paged_kv_cache_by_indptr(key.to(DEV), value.to(DEV), ai.to(DEV), got, ki.to(DEV),
                                       kp.to(DEV), kl.to(DEV), bad)
    torch.cuda.synchronize()
    assert bad.item() == 2
    assert torch.equal(got.cpu(), want)


def test_append_through_c_abi():
    lib = cabi.load()
    rng = np.random.default_rng(9)
    nkv, hd, P, ps = 8, 128, 200, 16
    ai, kp, ki, kl = mixed_batch(rng, ps, P, prefills=((20, 30),), decodes=5, max_ctx=100)
    nnz = int(ai[-1])
    key = torch.randn(nnz, nkv * hd).bfloat16()
    value = torch.randn(nnz, nkv * hd).bfloat16()
    cache = torch.zeros(P, 2, ps, nkv, hd).bfloat16()
    bi, pos = append_ref.get_batch_indices_positions(ai, append_ref.get_seq_lens(kp, kl, ps), nnz)
    ref = append_ref.append_paged_kv_cache(key, value, bi, pos, cache.clone(), ki, kp, kl)
    d = {n: t.to(DEV) for n, t in dict(key=key, value=value, bi=bi, pos=pos, cache=cache, ki=ki,
                                       kp=kp, kl=kl).items()}
    st = torch.cuda.current_stream().cuda_stream
    cabi.check(lib.pace_append_paged_kv_cache(
        d["key"].data_ptr(), d["value"].data_ptr(), nnz, nkv, hd, nkv * hd, nkv * hd,
        d["bi"].data_ptr(), d["pos"].data_ptr(), d["cache"].data_ptr(), P, ps, d["ki"].data_ptr(),
        ki.numel(), d["kp"].data_ptr(), d["kl"].data_ptr(), kp.numel() - 1, None, cabi.PACE_BF16, st))
    torch.cuda.synchronize()
    assert torch.equal(d["cache"].cpu(), ref)


def test_append_matches_flashinfer_when_available():
    """Byte-equality with the dependency PaceServe calls (the image's FlashInfer;
    PaceServe pins 0.2.0), on the bench's mixed-batch metadata."""
    try:
        import flashinfer
    except Exception as exc:  # pragma: no cover
        pytest.skip(f"flashinfer not importable: {exc}")
    import bench

    ai, kp, ki, kl = (x.to(DEV) for x in bench.append_metadata())
    nnz = int(ai[-1].item())
    nkv, hd = bench.NKV, bench.HD
    g = torch.Generator(device=DEV).manual_seed(8)
    k = torch.randn(nnz, nkv, hd, generator=g, device=DEV).bfloat16()
    v = torch.randn(nnz, nkv, hd, generator=g, device=DEV).bfloat16()
    a = torch.zeros(4096, 2, 16, nkv, hd, dtype=torch.bfloat16, device=DEV)
    b = torch.zeros_like(a)
    try:
        sl = flashinfer.get_seq_lens(kp, kl, 16)
        bi, po = flashinfer.get_batch_indices_positions(ai, sl, nnz)
        flashinfer.append_paged_kv_cache(k, v, bi, po, b, ki, kp, kl, kv_layout="NHD")
        torch.cuda.synchronize()
    except Exception as exc:  # pragma: no cover - JIT build unavailable
        pytest.skip(f"flashinfer page module unavailable: {exc}")
    kv.append_paged_kv_cache_by_indptr(k, v, ai, a, ki, kp, kl)
    c = torch.zeros_like(a)
    kv.append_paged_kv_cache(k, v, bi, po, c, ki, kp, kl)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(c, b)


@pytest.mark.parametrize("form", ["indices", "indptr"])
def test_append_large_batch_unstaged(form):
    """More than 2048 requests: the per-request metadata is read from global
    memory instead of being staged in shared memory; same bytes."""
    rng = np.random.default_rng(12)
    nkv, hd, P, ps = 2, 64, 7000, 16
    ai, kp, ki, kl = mixed_batch(rng, ps, P, prefills=((30, 5),), decodes=2100, max_ctx=40)
    assert kp.numel() - 1 > 2048
    nnz = int(ai[-1])
    key = torch.randn(nnz, nkv * hd).bfloat16()
    value = torch.randn(nnz, nkv * hd).bfloat16()
    cache = torch.zeros(P, 2, ps, nkv, hd).bfloat16()
    bi, pos = append_ref.get_batch_indices_positions(ai, append_ref.get_seq_lens(kp, kl, ps), nnz)
    ref = append_ref.append_paged_kv_cache(key, value, bi, pos, cache.clone(), ki, kp, kl)
    got = cache.to(DEV)
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    if form == "indices":
        kv.append_paged_kv_cache(key.to(DEV), value.to(DEV), bi.to(DEV), pos.to(DEV), got,
                                 ki.to(DEV), kp.to(DEV), kl.to(DEV), "NHD", bad)
    else:
        kv.append_paged_kv_cache_by_indptr(key.to(DEV), value.to(DEV), ai.to(DEV), got, ki.to(DEV),
                                           kp.to(DEV), kl.to(DEV), bad)
    torch.cuda.synchronize()
    assert bad.item() == 0
    assert torch.equal(got.cpu(), ref)


@pytest.mark.parametrize("extra_block", [False, True])
def test_promoted_request_keeps_decoding(extra_block):
    """A running request moves LP -> HP mid-decode and continues there.

    The LP worker holds 37 tokens of a request (blocks of 16, 16 and 5 tokens) in random
    blocks of every layer. The HP worker allocates its table the way
    BaseWorker._insert_kv_cache does (base_worker.py:255-277); with `extra_block`
    that table is one block longer than the sender's. align_block_tables maps the
    transfer, the promotion kernel copies the blocks, and the paged-KV append writes
    decode token 38 into the HP cache. The HP cache must then hold the 38-token
    sequence exactly, as if the request had run on HP from the start.
    """
    from paceserve_b200 import kv_transfer as kvt

    L, P, ps, nkv, hd = 3, 64, 16, 8, 128
    g = torch.Generator().manual_seed(31)
    lp = [torch.randn(P, 2, ps, nkv, hd, generator=g).bfloat16().to(DEV) for _ in range(L)]
    hp = [torch.zeros(P, 2, ps, nkv, hd, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    lp_table = [41, 7, 19]                       # 37 tokens: 16 + 16 + 5
    hp_table = [3, 58, 22] + ([9] if extra_block else [])
    dst = kvt.align_block_tables(len(lp_table), hp_table)
    kvt.promote(lp, hp, lp_table, dst)
    # decode token 38 on HP: page table = the aligned blocks, last page holds 6
    k_new = torch.randn(1, nkv * hd, generator=g).bfloat16().to(DEV)
    v_new = torch.randn(1, nkv * hd, generator=g).bfloat16().to(DEV)
    ai = torch.tensor([0, 1], dtype=torch.int32, device=DEV)
    kp = torch.tensor([0, 3], dtype=torch.int32, device=DEV)
    kl = torch.tensor([6], dtype=torch.int32, device=DEV)
    ki = torch.tensor(dst, dtype=torch.int32, device=DEV)
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    for l in range(L):
        kv.append_paged_kv_cache_by_indptr(k_new, v_new, ai, hp[l], ki, kp, kl, bad)
    torch.cuda.synchronize()
    assert bad.item() == 0
    for l in range(L):
        for j, (s, d) in enumerate(zip(lp_table, dst)):
            n = 16 if j < 2 else 5
            assert torch.equal(hp[l][d, :, :n].cpu(), lp[l][s, :, :n].cpu())
        assert torch.equal(hp[l][dst[2], 0, 5].cpu(), k_new.view(nkv, hd).cpu())
        assert torch.equal(hp[l][dst[2], 1, 5].cpu(), v_new.view(nkv, hd).cpu())
        untouched = [b for b in range(P) if b not in dst]
        assert int(hp[l][untouched].ne(0).sum()) == 0
