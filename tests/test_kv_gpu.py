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
    kv.copy_blocks_p2p(src, dst, sids.cuda(), dids.cuda(), method=method)
    torch.cuda.synchronize()
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
        kv.copy_blocks_p2p(src, dst, sids.cuda(), dids.cuda(), method=method)
        torch.cuda.synchronize()
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
    kv.copy_blocks_p2p(src, dst, sids, dids, method=method, push=push)
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
