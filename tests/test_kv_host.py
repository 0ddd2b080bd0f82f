"""CPU: host-side logic of the KV promotion -- block-table alignment, planning,
LP->HP rank pairing, and the CacheExport exchange across gloo ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from paceserve_b200.kv_transfer import (CacheExport, KVhelper, align_block_tables,
                                        exchange_exports, pair_ranks, plan_promotion)


def test_align_block_tables():
    assert align_block_tables(3, [7, 8, 9]) == [7, 8, 9]
    assert align_block_tables(3, [7, 8, 9, 10]) == [7, 8, 9]  # extra logical-token block
    with pytest.raises(ValueError):
        align_block_tables(3, [7, 8])
    with pytest.raises(ValueError):
        align_block_tables(1, [1, 2, 3])


def test_plan_promotion():
    src, dst, tables = plan_promotion([[5, 9], [3]], [100, 101, 102, 103])
    assert src == [5, 9, 3] and dst == [100, 101, 102] and tables == [[100, 101], [102]]
    with pytest.raises(ValueError, match="not enough free"):
        plan_promotion([[1, 2, 3]], [7, 8])
    with pytest.raises(ValueError, match="twice"):
        plan_promotion([[1, 2], [2]], [7, 8, 9])


def test_pair_ranks():
    assert pair_ranks(1) == []
    assert pair_ranks(2) == [(0, 1)]
    assert pair_ranks(8) == [(0, 1), (2, 3), (4, 5), (6, 7)]
    assert pair_ranks(5) == [(0, 1), (2, 3)]


class _Model:
    dtype = torch.bfloat16

    def get_num_q_heads(self, p):
        return 32

    def get_num_kv_heads(self, p):
        return 8

    def get_head_size(self):
        return 128

    def get_num_layers(self, p):
        return 32


class _Cache:
    block_size = 16


def test_kvhelper_reads_reference_configs():
    h = KVhelper(3, _Model(), _Cache(), None)
    assert (h.rank, h.num_q_heads, h.num_kv_heads, h.head_dim, h.block_size, h.num_layers) == \
        (3, 32, 8, 128, 16, 32)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _exchange_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        exp = None
        lp, hp = pair_ranks(world)[0]
        if rank == lp:
            exp = CacheExport([bytes([i]) * 64 for i in range(32)], [0] * 32, 8192, 65536, 0,
                              (8192, 2, 16, 8, 128), "torch.bfloat16")
        got = exchange_exports(exp)
        q.put((rank, got[lp].num_layers, got[lp].handles[5], got[hp]))
    finally:
        dist.destroy_process_group()


def test_exchange_exports_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, nl, h5, hp_export in res:
        assert nl == 32 and h5 == bytes([5]) * 64 and hp_export is None
