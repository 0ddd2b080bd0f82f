"""GPU parity of MoE routing: topk_softmax and moe_align_block_size.

Integer outputs are compared bit-exact with the C/numpy oracle and with the
reference's own CUDA ops (when built).  Tie rule: the lowest expert index wins.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import moe_ref
from paceserve_b200 import moe_ops
from tests._util import ref_ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def run_topk(gating: torch.Tensor, k: int, renormalize=False):
    T = gating.shape[0]
    w = torch.empty(T, k, dtype=torch.float32, device=DEV)
    ids = torch.empty(T, k, dtype=torch.int32, device=DEV)
    tei = torch.empty(T, k, dtype=torch.int32, device=DEV)
    moe_ops.topk_softmax(w, ids, tei, gating.to(DEV), renormalize)
    return w.cpu(), ids.cpu(), tei.cpu()


@pytest.mark.parametrize("E,k", [(8, 2), (8, 1), (16, 4), (64, 6), (128, 8), (256, 8), (4, 2),
                                 (2, 1), (1, 1), (60, 4), (160, 6), (7, 2)])
@pytest.mark.parametrize("T", [1, 64, 512, 4096, 16384])
def test_topk_softmax(T, E, k):
    g = torch.randn(T, E, generator=torch.Generator().manual_seed(T * 31 + E))
    w, ids, tei = run_topk(g, k)
    ow, oids, otei = moe_ref.topk_softmax(g.numpy(), k)
    np.testing.assert_array_equal(ids.numpy(), oids)
    np.testing.assert_array_equal(tei.numpy(), otei)
    np.testing.assert_allclose(w.numpy(), ow, rtol=1e-5, atol=1e-7)
    ref = ref_ops("moe_ops")
    if ref is not None:
        rw = torch.empty(T, k, dtype=torch.float32, device=DEV)
        ri = torch.empty(T, k, dtype=torch.int32, device=DEV)
        rt = torch.empty(T, k, dtype=torch.int32, device=DEV)
        ref.topk_softmax(rw, ri, rt, g.to(DEV))
        assert torch.equal(ids, ri.cpu()) and torch.equal(tei, rt.cpu())
        if E & (E - 1) == 0 and E <= 256:
            assert torch.equal(w, rw.cpu())  # same summation order -> bit-identical
        else:
            torch.testing.assert_close(w, rw.cpu(), rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("E", [8, 16, 60, 256])
def test_topk_softmax_ties_pick_lowest_index(E):
    T, k = 6, 3
    g = torch.zeros(T, E)
    g[1, [3, E - 1]] = 2.0
    g[2, :] = -1.0
    g[3, [E - 1, E - 2, 1]] = 5.0
    g[4, 0] = -3.0
    g[5] = torch.arange(E).flip(0).float() * 0.0 + 1.0
    w, ids, _ = run_topk(g, k)
    _, oids, _ = moe_ref.topk_softmax(g.numpy(), k)
    np.testing.assert_array_equal(ids.numpy(), oids)
    assert ids[0].tolist() == [0, 1, 2]
    assert ids[1].tolist() == [3, E - 1, 0]
    assert ids[3].tolist() == [1, E - 2, E - 1]
    assert ids[4].tolist() == [1, 2, 3]


@pytest.mark.parametrize("T,E,k", [(4096, 8, 2), (512, 16, 4), (64, 60, 4)])
def test_topk_softmax_renormalize_matches_python(T, E, k):
    g = torch.randn(T, E, generator=torch.Generator().manual_seed(5)).to(DEV)
    w0, ids0, _ = run_topk(g, k, renormalize=False)
    w1, ids1, _ = run_topk(g, k, renormalize=True)
    assert torch.equal(ids0, ids1)
    composed = (w0.to(DEV) / w0.to(DEV).sum(dim=-1, keepdim=True)).cpu()  # fused_moe.py:371-372
    if k == 2:
        assert torch.equal(w1, composed)
    else:
        torch.testing.assert_close(w1, composed, rtol=1e-6, atol=1e-7)


def test_topk_softmax_strided_rows_rejected_and_misaligned_ok():
    g = torch.randn(33, 9, device=DEV)[:, 1:]  # non-contiguous
    w = torch.empty(33, 2, device=DEV)
    i = torch.empty(33, 2, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="contiguous"):
        moe_ops.topk_softmax(w, i, i.clone(), g)
    base = torch.randn(33 * 8 + 1, device=DEV)
    g2 = base[1:].view(33, 8)  # 4-byte aligned only
    t = torch.empty(33, 2, dtype=torch.int32, device=DEV)
    moe_ops.topk_softmax(w, i, t, g2)
    _, oids, _ = moe_ref.topk_softmax(g2.cpu().numpy(), 2)
    np.testing.assert_array_equal(i.cpu().numpy(), oids)
    with pytest.raises(RuntimeError, match="exceeds num_experts"):
        moe_ops.topk_softmax(torch.empty(33, 9, device=DEV), torch.empty(33, 9, dtype=torch.int32, device=DEV),
                             torch.empty(33, 9, dtype=torch.int32, device=DEV), g2)


def run_align(topk_ids: torch.Tensor, E: int, bs: int, fill_padding=False, prefill=None):
    numel = topk_ids.numel()
    cap = numel + E * (bs - 1)
    fill = numel if prefill is None else prefill
    sorted_ids = torch.full((cap,), fill, dtype=torch.int32, device=DEV)
    expert_ids = torch.full(((cap + bs - 1) // bs,), -7, dtype=torch.int32, device=DEV)
    total = torch.empty(1, dtype=torch.int32, device=DEV)
    moe_ops.moe_align_block_size(topk_ids.to(DEV), E, bs, sorted_ids, expert_ids, total, fill_padding)
    t = int(total.item())
    return sorted_ids.cpu().numpy(), expert_ids.cpu().numpy(), t


def test_moe_align_known_answer():
    with open(os.path.join(GOLDEN, "moe_align_kat.json")) as f:
        kat = json.load(f)
    s, e, t = run_align(torch.tensor(kat["topk_ids"], dtype=torch.int32), kat["num_experts"],
                        kat["block_size"])
    assert t == kat["num_tokens_post_pad"]
    assert s[:t].tolist() == kat["sorted_token_ids"]
    assert e[: t // kat["block_size"]].tolist() == kat["expert_ids"]


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64, torch.int16, torch.uint8])
@pytest.mark.parametrize("numel,E,bs", [(0, 8, 64), (1, 8, 64), (128, 8, 64), (1024, 8, 64),
                                        (8192, 8, 64), (32768, 8, 64), (777, 5, 4),
                                        (4096, 64, 16), (3000, 200, 128), (50000, 8, 16)])
def test_moe_align_block_size(numel, E, bs, dtype):
    rng = np.random.default_rng(numel + E)
    ids = torch.from_numpy(rng.integers(0, E, size=numel)).to(dtype)
    s, e, t = run_align(ids, E, bs)
    os_, oe, ot = moe_ref.moe_align_block_size_c(ids.numpy(), E, bs)
    assert t == ot
    np.testing.assert_array_equal(s, os_)
    np.testing.assert_array_equal(e[: t // bs], oe)
    ref = ref_ops("moe_ops")
    if ref is not None and numel > 0 and E <= 1024:
        cap = numel + E * (bs - 1)
        rs = torch.full((cap,), numel, dtype=torch.int32, device=DEV)
        re_ = torch.empty(((cap + bs - 1) // bs,), dtype=torch.int32, device=DEV)
        rt = torch.empty(1, dtype=torch.int32, device=DEV)
        ref.moe_align_block_size(ids.to(DEV), E, bs, rs, re_, rt)
        assert int(rt.item()) == t
        np.testing.assert_array_equal(rs.cpu().numpy(), s)
        np.testing.assert_array_equal(re_.cpu().numpy()[: t // bs], e[: t // bs])


@pytest.mark.parametrize("numel,E,bs", [(4097, 1, 16), (20000, 32, 64), (65536, 8, 64),
                                        (6000, 3, 7), (131072, 16, 128)])
@pytest.mark.parametrize("fill", [False, True])
def test_moe_align_large_inputs(numel, E, bs, fill):
    """The multi-CTA (thread-block cluster) path, with ids outside [0, E) mixed in."""
    rng = np.random.default_rng(numel + 7 * E)
    ids = rng.integers(-1, E + 1, size=numel)
    t_ids = torch.from_numpy(ids).to(torch.int32)
    s, e, t = run_align(t_ids, E, bs, fill_padding=fill, prefill=None if not fill else -3)
    os_, oe, ot = moe_ref.moe_align_block_size_c(ids, E, bs)
    assert t == ot
    np.testing.assert_array_equal(s, os_)
    np.testing.assert_array_equal(e[: t // bs], oe)


@pytest.mark.parametrize("numel", [2, 31, 32, 33, 200, 255, 256, 257])
@pytest.mark.parametrize("E,bs", [(1, 16), (8, 64), (32, 4), (7, 3)])
@pytest.mark.parametrize("fill", [False, True])
def test_moe_align_small_sizes(numel, E, bs, fill):
    """Decode-sized inputs around warp multiples, ids outside [0, E) mixed in,
    with and without in-kernel padding."""
    rng = np.random.default_rng(numel * 31 + E)
    ids = rng.integers(-1, E + 1, size=numel)
    t_ids = torch.from_numpy(ids).to(torch.int32)
    s, e, t = run_align(t_ids, E, bs, fill_padding=fill, prefill=None if not fill else -3)
    os_, oe, ot = moe_ref.moe_align_block_size_c(ids, E, bs)
    assert t == ot
    np.testing.assert_array_equal(s, os_)
    np.testing.assert_array_equal(e[: t // bs], oe)


def test_moe_align_fill_padding_and_invalid_ids():
    ids = torch.tensor([0, 9, 1, -1, 1, 3, 3, 3], dtype=torch.int64)
    s, e, t = run_align(ids, 4, 2, fill_padding=True, prefill=-5)
    os_, oe, ot = moe_ref.moe_align_block_size_c(ids.numpy(), 4, 2)
    assert t == ot
    np.testing.assert_array_equal(s, os_)  # every padding slot rewritten to numel
    np.testing.assert_array_equal(e[: t // 2], oe)
    s2, _, _ = run_align(ids, 4, 2, fill_padding=False, prefill=-5)
    assert (s2[s2 != os_] == -5).all()  # without the flag, padding keeps the caller's fill


def test_moe_align_small_output_rejected():
    ids = torch.zeros(16, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="sorted_token_ids holds"):
        moe_ops.moe_align_block_size(ids, 8, 64, torch.empty(16, dtype=torch.int32, device=DEV),
                                     torch.empty(16, dtype=torch.int32, device=DEV),
                                     torch.empty(1, dtype=torch.int32, device=DEV))


def test_mixtral_routing_chain():
    """fused_topk then moe_align_block_size, as fused_moe.py:346-373, 497-499 chain them."""
    T, E, k, bs = 4096, 8, 2, 64
    g = torch.randn(T, E, generator=torch.Generator().manual_seed(1))
    w, ids, _ = run_topk(g, k, renormalize=True)
    s, e, t = run_align(ids, E, bs)
    _, oids, _ = moe_ref.topk_softmax(g.numpy(), k, renormalize=True)
    os_, oe, ot = moe_ref.moe_align_block_size_c(oids, E, bs)
    assert t == ot
    np.testing.assert_array_equal(s, os_)
    np.testing.assert_array_equal(e[: t // bs], oe)
