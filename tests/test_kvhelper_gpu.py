"""GPU: the KVhelper mirror (reference kv_utils.py:8-56) and LP->HP promotion
across processes with CUDA IPC, byte-exact against torch indexing."""
import pytest
import torch
import torch.multiprocessing as mp

from paceserve_b200 import kv_transfer as kvt

pytestmark = pytest.mark.gpu
SHAPE = (2, 16, 8, 128)


class _Model:
    dtype = torch.bfloat16

    def __init__(self, layers=4):
        self.layers = layers

    def get_num_q_heads(self, p):
        return 32

    def get_num_kv_heads(self, p):
        return 8

    def get_head_size(self):
        return 128

    def get_num_layers(self, p):
        return self.layers


class _CacheCfg:
    block_size = 16


class _Wrapper:
    def __init__(self, caches):
        self.gpu_cache = caches


class _Runner:
    def __init__(self, caches):
        self.attention_backend_wrapper = _Wrapper(caches)


class _SeqMgr:
    def __init__(self, tables):
        self.tables = tables

    def _get_block_table(self, seq):
        return self.tables[seq]


def _caches(L, nb, seed, device="cuda:0"):
    g = torch.Generator(device=device).manual_seed(seed)
    return [torch.randn(nb, *SHAPE, generator=g, device=device).bfloat16() for _ in range(L)]


def _helper(caches, L=4):
    h = kvt.KVhelper(0, _Model(L), _CacheCfg(), None)
    h.add_model_runner(_Runner(caches))
    return h


def test_get_and_insert_match_reference_semantics():
    L = 4
    src = _caches(L, 64, 1)
    h = _helper(src, L)
    table = [5, 17, 3, 40, 41]
    cache, ids = h.get_kv_cache("seq", _SeqMgr({"seq": table}))
    assert ids == table and not cache.is_cuda
    assert cache.shape == (L, len(table), *SHAPE)
    for l in range(L):  # kv_utils.py:46: seq_cache[i] = gpu_cache[i][indices]
        assert torch.equal(cache[l], src[l][torch.tensor(table)].cpu())
    dst = _caches(L, 64, 2)
    before = [d.clone() for d in dst]
    h2 = _helper(dst, L)
    dst_ids = [1, 2, 60, 33, 9]
    assert h2.insert_kv_cache(cache, dst_ids, "cuda:0") is True
    for l in range(L):
        assert torch.equal(dst[l][torch.tensor(dst_ids)], src[l][torch.tensor(table)])
        keep = torch.ones(64, dtype=torch.bool)
        keep[dst_ids] = False
        assert torch.equal(dst[l][keep.cuda()], before[l][keep.cuda()])


def test_missing_table_and_failed_insert():
    h = _helper(_caches(2, 8, 3), 2)
    cache, ids = h.get_kv_cache("nope", _SeqMgr({}))
    assert ids == [0] and cache.shape == (2, 1, *SHAPE) and not cache.any()
    assert h.insert_kv_cache(torch.zeros(2, 3, *SHAPE, dtype=torch.bfloat16), [1, 2], "cuda:0") is False


def test_reset_kv_cache():
    caches = _caches(3, 8, 4)
    h = _helper(caches, 3)
    h.reset_kv_cache(12)
    assert len(h.gpu_cache) == 3 and h.gpu_cache[0].shape == (12, *SHAPE) and not h.gpu_cache[2].any()


def _lp_proc(q_out, q_back, device, L, nb, table):
    torch.cuda.set_device(device)
    caches = _caches(L, nb, 7, device=f"cuda:{device}")
    exp = kvt.export_caches(caches)
    gathered = torch.stack([c[torch.tensor(table, device=c.device)] for c in caches]).cpu()
    q_out.put((exp, gathered))
    q_back.get(timeout=300)  # keep the caches alive until the HP side is done


def _hp_proc(q_in, q_res, device, L, nb, table, dst_table, method):
    torch.cuda.set_device(device)
    exp, gathered = q_in.get(timeout=300)
    dst = [torch.zeros(nb, *SHAPE, dtype=torch.bfloat16, device=f"cuda:{device}") for _ in range(L)]
    with kvt.ImportedCaches(exp, device) as src:
        bad = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")
        kvt.promote(src, dst, table, dst_table, method=method, bad_pairs=bad)
        torch.cuda.synchronize()
        got = torch.stack([d[torch.tensor(dst_table, device=d.device)] for d in dst]).cpu()
        q_res.put((bool(torch.equal(got, gathered)), int(bad.item())))


@pytest.mark.parametrize("method", [1, 2])
def test_promotion_across_processes_ipc(method):
    """LP and HP as separate processes (as PaceServe's Ray workers are); on a
    one-GPU box both use cuda:0, otherwise cuda:0 -> cuda:1 over NVLink."""
    hp_dev = 1 if torch.cuda.device_count() > 1 else 0
    L, nb = 8, 96
    table = [3, 50, 51, 52, 90, 7]
    dst_table = [10, 11, 12, 80, 81, 0]
    ctx = mp.get_context("spawn")
    q1, q2, q3 = ctx.Queue(), ctx.Queue(), ctx.Queue()
    lp = ctx.Process(target=_lp_proc, args=(q1, q2, 0, L, nb, table))
    hp = ctx.Process(target=_hp_proc, args=(q1, q3, hp_dev, L, nb, table, dst_table, method))
    lp.start()
    hp.start()
    try:
        ok, bad = q3.get(timeout=300)
    finally:
        q2.put("done")
        hp.join(timeout=120)
        lp.join(timeout=120)
    assert hp.exitcode == 0 and lp.exitcode == 0
    assert ok and bad == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_promote_in_process_two_gpus():
    L = 4
    src = _caches(L, 64, 11, device="cuda:0")
    dst = [torch.zeros(64, *SHAPE, dtype=torch.bfloat16, device="cuda:1") for _ in range(L)]
    h = _helper(dst, L)
    h.promote_from(src, [1, 2, 3], [60, 61, 62])
    torch.cuda.synchronize("cuda:1")
    for l in range(L):
        assert torch.equal(dst[l][[60, 61, 62]].cpu(), src[l][[1, 2, 3]].cpu())
