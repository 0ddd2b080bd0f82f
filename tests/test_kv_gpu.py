"""GPU: paged-KV block copy / gather / scatter, byte-exact against torch indexing
(the reference's KVhelper path, paceserve/kv_transfer/kv_utils.py:44-52)."""
import ctypes

import pytest
import torch

from paceserve_b200 import cabi, kv_transfer_ops as kv

pytestmark = pytest.mark.gpu


def make_cache(L, nb, shape=(2, 16, 8, 128), dtype=torch.bfloat16, device="cuda:0", seed=0):
    """randn-filled per-layer caches, like the reference's get_cache_block
    (flashinfer_attention_wrapper.py:63-73)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return [torch.randn(nb, *shape, generator=g, device=device).to(dtype) for _ in range(L)]


def pick(n, nb, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(nb, generator=g)[:n].to(torch.int32)


def check_copied(src, dst, before, sids, dids):
    mask = torch.ones(dst[0].shape[0], dtype=torch.bool)
    mask[dids.long()] = False
    for s, d, b in zip(src, dst, before):
        assert torch.equal(d[dids.long().to(d.device)].cpu(), s[sids.long().to(s.device)].cpu())
        assert torch.equal(d.cpu()[mask], b.cpu()[mask])


@pytest.mark.parametrize("method", [0, 1, 2])
@pytest.mark.parametrize("shape,dtype", [((2, 16, 8, 128), torch.bfloat16),
                                         ((2, 16, 1, 8), torch.float16),
                                         ((2, 16, 8, 128), torch.float32)])
def test_copy_blocks_same_device(method, shape, dtype):
    L, n = 4, 37
    src = make_cache(L, 64, shape, dtype, seed=1)
    dst = make_cache(L, 80, shape, dtype, seed=2)
    before = [d.clone() for d in dst]
    sids, dids = pick(n, 64, 3), pick(n, 80, 4)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda:0")  # required by method 2
    kv.copy_blocks_p2p(src, dst, sids.cuda(), dids.cuda(), method=method, bad_pairs=bad)
    torch.cuda.synchronize()
    assert bad.item() == 0
    check_copied(src, dst, before, sids, dids)


def test_copy_blocks_cpu_ids_and_bad_ids_counted():
    L = 3
    src = make_cache(L, 16, seed=5)
    dst = make_cache(L, 16, seed=6)
    before = [d.clone() for d in dst]
    sids = torch.tensor([1, 99, 2, -1, 3], dtype=torch.int32)
    dids = torch.tensor([4, 5, 16, 6, 7], dtype=torch.int32)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    for method in (1, 2):
        bad.zero_()
        kv.copy_blocks_p2p(src, dst, sids, dids, method=method, bad_pairs=bad)
        torch.cuda.synchronize()
        assert bad.item() == 3  # pairs 1, 2 and 3 are out of range and skipped
    good_s, good_d = torch.tensor([1, 3]), torch.tensor([4, 7])
    check_copied(src, dst, before, good_s, good_d)


def test_int64_ids_outside_int32_are_counted_not_wrapped():
    """An int64 id of 2**32 + 1 would wrap to block 1 if narrowed to int32; it
    must be counted as out of range instead (copy, gather and scatter)."""
    L = 2
    src = make_cache(L, 16, seed=7)
    dst = make_cache(L, 16, seed=8)
    before = [d.clone() for d in dst]
    sids = torch.tensor([2**32 + 1, 3, -(2**33), 5], dtype=torch.int64)
    dids = torch.tensor([4, 2**31, 6, 7], dtype=torch.int64)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    kv.copy_blocks_p2p(src, dst, sids.cuda(), dids.cuda(), bad_pairs=bad)
    torch.cuda.synchronize()
    assert bad.item() == 3
    check_copied(src, dst, before, torch.tensor([5]), torch.tensor([7]))
    out = torch.zeros(L, 2, *src[0].shape[1:], dtype=src[0].dtype, device="cuda:0")
    bad.zero_()
    kv.gather_blocks(src, torch.tensor([2**32 + 3, 4], dtype=torch.int64), out, bad)
    torch.cuda.synchronize()
    assert bad.item() == 1
    assert torch.equal(out[:, 1], torch.stack([s[4] for s in src]))
    assert int(out[:, 0].ne(0).sum()) == 0
    bad.zero_()
    snap = [d.clone() for d in dst]
    kv.scatter_blocks(out, dst, torch.tensor([2**32 + 9, 9], dtype=torch.int64), bad)
    torch.cuda.synchronize()
    assert bad.item() == 1
    for layer, (d, b) in enumerate(zip(dst, snap)):
        assert torch.equal(d[9], out[layer, 1])
        mask = torch.ones(16, dtype=torch.bool)
        mask[9] = False
        assert torch.equal(d[mask], b[mask])


@pytest.mark.parametrize("pinned", [False, True])
def test_gather_scatter_roundtrip(pinned):
    L, n, nb = 5, 23, 50
    cache = make_cache(L, nb, seed=7)
    ids = pick(n, nb, 8)
    if pinned:
        buf = torch.empty(L, n, 2, 16, 8, 128, dtype=torch.bfloat16, pin_memory=True)
    else:
        buf = torch.empty(L, n, 2, 16, 8, 128, dtype=torch.bfloat16, device="cuda:0")
    kv.gather_blocks(cache, ids.cuda(), buf)
    torch.cuda.synchronize()
    for l in range(L):
        assert torch.equal(buf[l].cpu(), cache[l][ids.long().cuda()].cpu())
    fresh = make_cache(L, nb, seed=9)
    before = [f.clone() for f in fresh]
    dids = pick(n, nb, 10)
    kv.scatter_blocks(buf, fresh, dids.cuda())
    torch.cuda.synchronize()
    check_copied(cache, fresh, before, ids, dids)


def test_kv_copy_through_c_abi():
    lib = cabi.load()
    L, n = 2, 9
    src = make_cache(L, 32, seed=11)
    dst = make_cache(L, 32, seed=12)
    before = [d.clone() for d in dst]
    sids, dids = pick(n, 32, 13).cuda(), pick(n, 32, 14).cuda()
    st = cabi.layer_table([t.data_ptr() for t in src])
    dt = cabi.layer_table([t.data_ptr() for t in dst])
    bad = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    cabi.check(lib.pace_kv_copy_blocks(st, dt, L, sids.data_ptr(), dids.data_ptr(), n, 65536, 32, 32,
                                       bad.data_ptr(), 1, stream))
    torch.cuda.synchronize()
    assert bad.item() == 0
    check_copied(src, dst, before, sids.cpu(), dids.cpu())


def test_promotion_sized_copy_single_gpu():
    """Promotion-workload shapes (32 layers, 64 KiB slabs), 600 blocks, one GPU."""
    L, nb, n = 32, 1024, 600
    src = make_cache(L, nb, seed=15)
    dst = [torch.zeros_like(s) for s in src]
    sids, dids = pick(n, nb, 16), pick(n, nb, 17)
    for method in (1, 2):
        for d in dst:
            d.zero_()
        bad = torch.zeros(1, dtype=torch.int32, device="cuda:0")
        kv.copy_blocks_p2p(src, dst, sids.cuda(), dids.cuda(), method=method, bad_pairs=bad)
        torch.cuda.synchronize()
        assert bad.item() == 0
        for l in (0, 13, 31):
            assert torch.equal(dst[l][dids.long().cuda()], src[l][sids.long().cuda()])
        total = sum(int(d.view(torch.int16).ne(0).any(dim=(1, 2, 3, 4)).sum()) for d in dst)
        assert total == L * n


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("push", [False, True])
@pytest.mark.parametrize("method", [1, 2])
def test_copy_blocks_across_gpus(push, method):
    L, n = 8, 40
    src = make_cache(L, 128, device="cuda:0", seed=21)
    dst = make_cache(L, 96, device="cuda:1", seed=22)
    before = [d.clone() for d in dst]
    sids, dids = pick(n, 128, 23), pick(n, 96, 24)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda:0" if push else "cuda:1")
    kv.copy_blocks_p2p(src, dst, sids, dids, method=method, push=push, bad_pairs=bad)
    torch.cuda.synchronize("cuda:0")
    torch.cuda.synchronize("cuda:1")
    check_copied(src, dst, before, sids, dids)


def test_concurrent_gather_scatter_from_threads():
    """Four host threads, each on its own stream, gather different requests to
    pinned memory and scatter them into another cache at the same time (the
    reference runs 4 KV insertion threads, decode_instance.py:50-51, and
    `_get_kv_cache` concurrently from Ray threads).  Every copy is byte-exact
    and untouched blocks stay untouched."""
    import threading

    L, nb, n = 4, 512, 40
    src = make_cache(L, nb, seed=21)
    dst = make_cache(L, nb, seed=22)
    before = [d.clone() for d in dst]
    perm_s = torch.randperm(nb, generator=torch.Generator().manual_seed(23))
    perm_d = torch.randperm(nb, generator=torch.Generator().manual_seed(24))
    jobs = [(perm_s[i * n:(i + 1) * n].to(torch.int32), perm_d[i * n:(i + 1) * n].to(torch.int32))
            for i in range(4)]
    errors = []

    def worker(sids, dids):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                host = torch.empty(L, n, 2, 16, 8, 128, dtype=torch.bfloat16, pin_memory=True)
                for _ in range(3):
                    kv.gather_blocks(src, sids.cuda(non_blocking=False), host)
                    kv.scatter_blocks(host, dst, dids.cuda(non_blocking=False))
                s.synchronize()
        except Exception as exc:  # reported to the main thread
            errors.append(exc)

    ts = [threading.Thread(target=worker, args=j) for j in jobs]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    torch.cuda.synchronize()
    assert not errors, errors
    all_s = torch.cat([j[0] for j in jobs])
    all_d = torch.cat([j[1] for j in jobs])
    check_copied(src, dst, before, all_s, all_d)


def _layer_ptrs(caches):
    return cabi.layer_table([c.data_ptr() for c in caches])


def test_bulk_copy_wait_timeout_is_reported_and_device_stays_usable():
    """The bulk method's bounded wait, made to run out without a GPU fault: the
    test-only option tells CTA 0's first barrier to expect 16 bytes more than
    its copy delivers, so that wait can never complete.  With a 1 ms bound the
    kernel must flag the timeout in bad_pairs, return, and leave the context
    usable (a normal copy right after is byte-exact)."""
    lib = cabi.load()
    L, nb, n = 2, 32, 12
    src = make_cache(L, nb, seed=11)
    dst = make_cache(L, nb, seed=12)
    bb = src[0][0].numel() * src[0].element_size()
    sids = pick(n, nb, 13).cuda()
    dids = pick(n, nb, 14).cuda()
    bad = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    opts = cabi.KvCopyOpts(method=2, max_ctas=0, wait_limit_ns=1_000_000, test_overarm_bytes=16)
    cabi.check(lib.pace_kv_copy_blocks_ex(_layer_ptrs(src), _layer_ptrs(dst), L, sids.data_ptr(),
                                          dids.data_ptr(), n, bb, nb, nb, bad.data_ptr(),
                                          ctypes.byref(opts), st))
    torch.cuda.synchronize()
    v = int(bad.item())
    assert v & cabi.PACE_KV_TIMEOUT_FLAG
    # the over-armed phase never completes, so the drain's second wait runs out too
    assert v & cabi.PACE_KV_DRAIN_TIMEOUT_FLAG
    assert v & (cabi.PACE_KV_DRAIN_TIMEOUT_FLAG - 1) == 0  # no pair was out of range
    from paceserve_b200 import kv_transfer as kvt

    with pytest.raises(kvt.KVCopyError, match="wait expired"):
        kvt.check_copy_status(bad)
    # the device still works: the same copy without the option is byte-exact
    before = [d.clone() for d in dst]
    bad.zero_()
    opts = cabi.KvCopyOpts(method=2, max_ctas=0, wait_limit_ns=0, test_overarm_bytes=0)
    cabi.check(lib.pace_kv_copy_blocks_ex(_layer_ptrs(src), _layer_ptrs(dst), L, sids.data_ptr(),
                                          dids.data_ptr(), n, bb, nb, nb, bad.data_ptr(),
                                          ctypes.byref(opts), st))
    torch.cuda.synchronize()
    assert bad.item() == 0
    check_copied(src, dst, before, sids.cpu(), dids.cpu())
    # the bulk method without a counter is refused before any launch
    assert lib.pace_kv_copy_blocks(_layer_ptrs(src), _layer_ptrs(dst), L, sids.data_ptr(),
                                   dids.data_ptr(), n, bb, nb, nb, None, 2,
                                   st) == cabi.PACE_ERR_INVALID_ARGUMENT
    with pytest.raises(RuntimeError, match="bad_pairs"):
        kv.copy_blocks_p2p(src, dst, sids, dids, method=2)


@pytest.mark.parametrize("max_ctas", [1, 8])
@pytest.mark.parametrize("method", [1, 2])
def test_copy_with_cta_budget_is_byte_exact(method, max_ctas):
    L, n = 3, 29
    src = make_cache(L, 64, seed=21)
    dst = make_cache(L, 64, seed=22)
    before = [d.clone() for d in dst]
    sids, dids = pick(n, 64, 23), pick(n, 64, 24)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    kv.copy_blocks_p2p(src, dst, sids.cuda(), dids.cuda(), method=method, bad_pairs=bad,
                       max_ctas=max_ctas)
    torch.cuda.synchronize()
    assert bad.item() == 0
    check_copied(src, dst, before, sids, dids)


@pytest.mark.parametrize("layout", ["per_layer", "one_allocation"])
@pytest.mark.parametrize("ids", ["runs", "random"])
def test_copy_engine_path_is_byte_exact(layout, ids):
    """method 3: the copy engines, one copy per run of consecutive ids (per layer,
    or one 2-D copy over all layers when the layer tensors are views of one
    allocation), host ids, invalid pairs counted."""
    L, nb = 4, 64
    g = torch.Generator(device="cuda:0").manual_seed(31)
    if layout == "one_allocation":
        base = torch.randn(L, nb, 2, 16, 8, 128, generator=g, device="cuda:0").bfloat16()
        src = list(base.unbind(0))
        dbase = torch.randn(L, nb, 2, 16, 8, 128, generator=g, device="cuda:0").bfloat16()
        dst = list(dbase.unbind(0))
    else:
        src = make_cache(L, nb, seed=32)
        dst = make_cache(L, nb, seed=33)
    before = [d.clone() for d in dst]
    if ids == "runs":
        sids = torch.tensor([40, 3, 4, 5, 10, 11, 99], dtype=torch.int32)
        dids = torch.tensor([60, 20, 21, 22, 7, 8, 1], dtype=torch.int32)
        good = slice(0, 6)
    else:
        sids, dids = pick(23, nb, 34), pick(23, nb, 35)
        sids = torch.cat([sids, torch.tensor([-1], dtype=torch.int32)])
        dids = torch.cat([dids, torch.tensor([0], dtype=torch.int32)])
        good = slice(0, 23)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    kv.copy_blocks_p2p(src, dst, sids, dids, method=3, bad_pairs=bad)
    torch.cuda.synchronize()
    assert bad.item() == 1
    check_copied(src, dst, before, sids[good], dids[good])
    if ids == "runs":
        # through the C ABI: the number of copies issued follows the runs
        lib = cabi.load()
        nbad, issued = ctypes.c_int64(-1), ctypes.c_int64(-1)
        s32 = (ctypes.c_int32 * 7)(*sids.tolist())
        d32 = (ctypes.c_int32 * 7)(*dids.tolist())
        bb = src[0][0].numel() * src[0].element_size()
        cabi.check(lib.pace_kv_copy_blocks_ce(_layer_ptrs(src), _layer_ptrs(dst), L, s32, d32, 7,
                                              bb, nb, nb, ctypes.byref(nbad), ctypes.byref(issued),
                                              torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert nbad.value == 1

        def uniform(cs):
            d = [cs[i + 1].data_ptr() - cs[i].data_ptr() for i in range(len(cs) - 1)]
            return len(set(d)) == 1 and d[0] >= 3 * bb

        runs = 3
        assert issued.value == (runs if uniform(src) and uniform(dst) else runs * L)
        if layout == "one_allocation":
            assert issued.value == runs
