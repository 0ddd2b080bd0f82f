"""CPU: the oracle against the reference's known answers and golden vectors.

The golden ``.npz`` fixtures hold outputs of the reference's own CUDA ops
(built from its sources, run on a B200 by ``tests/golden/make_golden.py``).
"""
import glob
import json
import os

import numpy as np
import pytest
import torch

from oracle import moe_ref, ops_ref
from tests._util import assert_matches_rounded

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _kat():
    with open(os.path.join(GOLDEN, "moe_align_kat.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_moe_align_known_answer(impl):
    kat = _kat()
    fn = moe_ref.moe_align_block_size if impl == "numpy" else moe_ref.moe_align_block_size_c
    sorted_ids, expert_ids, total = fn(np.array(kat["topk_ids"]), kat["num_experts"], kat["block_size"])
    assert total == kat["num_tokens_post_pad"]
    assert sorted_ids[: total].tolist() == kat["sorted_token_ids"]
    assert expert_ids.tolist() == kat["expert_ids"]


@pytest.mark.parametrize("seed,numel,E,bs", [(0, 1, 8, 64), (1, 128, 8, 64), (2, 8192, 8, 64),
                                             (3, 777, 5, 4), (4, 4096, 64, 16), (5, 0, 8, 64),
                                             (6, 3000, 256, 128)])
def test_moe_align_c_matches_numpy(seed, numel, E, bs):
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, E, size=numel)
    a = moe_ref.moe_align_block_size(ids, E, bs)
    b = moe_ref.moe_align_block_size_c(ids, E, bs)
    assert a[2] == b[2]
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])


def test_moe_align_invalid_ids_skipped():
    ids = np.array([0, 9, 1, -1, 1])
    s, e, t = moe_ref.moe_align_block_size(ids, 2, 2)
    assert t == 4
    assert s[:4].tolist() == [0, 5, 2, 4]
    s2, e2, t2 = moe_ref.moe_align_block_size_c(ids, 2, 2)
    assert t2 == t and s2.tolist() == s.tolist() and e2.tolist() == e.tolist()


def test_topk_tie_rule_lowest_index():
    g = np.zeros((3, 8), dtype=np.float32)
    g[1, [2, 5]] = 3.0
    g[2, 7] = 1.0
    w, ids, tei = moe_ref.topk_softmax(g, 2)
    assert ids[0].tolist() == [0, 1]  # all equal: lowest indices first
    assert ids[1].tolist() == [2, 5]
    assert ids[2].tolist() == [7, 0]
    assert tei.tolist() == [[0, 3], [1, 4], [2, 5]]


def test_topk_softmax_renormalize():
    rng = np.random.default_rng(0)
    g = rng.standard_normal((64, 8)).astype(np.float32)
    w, ids, _ = moe_ref.topk_softmax(g, 2, renormalize=True)
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)
    p = torch.softmax(torch.from_numpy(g), -1)
    tw, ti = torch.topk(p, 2, dim=-1)
    np.testing.assert_array_equal(ids, ti.numpy())


def test_rope_cache_and_rotation_consistent():
    cache = ops_ref.cos_sin_cache(128, 64, 500000.0)
    assert cache.shape == (64, 128)
    torch.testing.assert_close(cache[:, :64] ** 2 + cache[:, 64:] ** 2, torch.ones(64, 64))
    q = torch.randn(5, 2 * 128)
    k = torch.randn(5, 128)
    pos = torch.tensor([0, 1, 63, 64, -1])  # the last two are out of range: unchanged
    q2, k2 = ops_ref.rotary_embedding_fp32(pos, q, k, 128, cache, True)
    torch.testing.assert_close(q2[0], q[0])  # position 0 is the identity rotation
    torch.testing.assert_close(q2[3:], q[3:])
    # rotation preserves each pair's norm
    a, b = q.view(5, 2, 128)[:, :, :64], q.view(5, 2, 128)[:, :, 64:]
    a2, b2 = q2.view(5, 2, 128)[:, :, :64], q2.view(5, 2, 128)[:, :, 64:]
    torch.testing.assert_close(a * a + b * b, a2 * a2 + b2 * b2, rtol=1e-5, atol=1e-5)


def test_llama3_scaling_matches_unscaled_for_high_freqs():
    inv = ops_ref.rope_inv_freq(128, 500000.0)
    sc = ops_ref.llama3_inv_freq(inv, 8.0, 1.0, 4.0, 8192)
    assert torch.equal(sc[:8], inv[:8])  # short wavelengths are not scaled
    torch.testing.assert_close(sc[-1], inv[-1] / 8.0)


def test_fused_add_matches_composition():
    torch.manual_seed(0)
    x = torch.randn(4, 64, dtype=torch.bfloat16)
    r = torch.randn(4, 64, dtype=torch.bfloat16)
    w = torch.randn(64, dtype=torch.bfloat16)
    out, res = ops_ref.fused_add_rms_norm_rounded(x, r, w, 1e-5)
    assert torch.equal(res, x + r)  # torch's bf16 add rounds the fp32 sum once
    assert torch.equal(out, ops_ref.rms_norm_rounded(x + r, w, 1e-5))


def _golden_files():
    """Fixtures produced by the reference's CUDA ops (make_golden.py); the
    wrapper-call recording (wrapper_calls.npz) has its own tests."""
    return sorted(p for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
                  if os.path.basename(p) != "wrapper_calls.npz")


@pytest.mark.skipif(not _golden_files(), reason="no golden vectors committed yet")
@pytest.mark.parametrize("path", _golden_files(), ids=os.path.basename)
def test_oracle_against_reference_golden(path):
    """Each fixture: inputs + the reference CUDA op's outputs on a B200."""
    g = dict(np.load(path, allow_pickle=False))
    op = str(g["op"])
    t = lambda a: torch.from_numpy(np.asarray(a))  # noqa: E731

    def dt(name):
        return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[name]

    if op == "topk_softmax":
        w, ids, tei = moe_ref.topk_softmax(g["gating"], int(g["k"]))
        np.testing.assert_array_equal(ids, g["ref_ids"])
        np.testing.assert_array_equal(tei, g["ref_tei"])
        np.testing.assert_allclose(w, g["ref_weights"], rtol=2e-6, atol=1e-7)
    elif op == "moe_align_block_size":
        s, e, total = moe_ref.moe_align_block_size_c(g["topk_ids"], int(g["E"]), int(g["bs"]))
        assert total == int(g["ref_total"])
        np.testing.assert_array_equal(s, g["ref_sorted"])
        np.testing.assert_array_equal(e, g["ref_expert_ids"][: total // int(g["bs"])])
    else:
        dtype = dt(str(g["dtype"]))
        # inputs are stored as fp32 values exactly representable in `dtype`
        if op == "rms_norm":
            ref = t(g["ref_out"]).to(dtype)
            got = ops_ref.rms_norm_rounded(t(g["x"]).to(dtype), t(g["w"]).to(dtype), float(g["eps"]))
        elif op in ("silu_and_mul", "gelu_new", "gelu_fast"):
            fn = {"silu_and_mul": ops_ref.silu_and_mul_rounded, "gelu_new": ops_ref.gelu_new_rounded,
                  "gelu_fast": ops_ref.gelu_fast_rounded}[op]
            ref = t(g["ref_out"]).to(dtype)
            got = fn(t(g["x"]).to(dtype))
        elif op == "rotary_embedding":
            q2, k2 = ops_ref.rotary_embedding_fp32(t(g["positions"]), t(g["q"]).to(dtype),
                                                   t(g["k"]).to(dtype), int(g["head_size"]),
                                                   t(g["cache"]).to(dtype), bool(g["is_neox"]))
            got = torch.cat([q2, k2], 1)
            ref = torch.cat([t(g["ref_q"]), t(g["ref_k"])], 1)
            # the reference rounds each product to the storage type; the oracle does not
            err = (got.float() - ref.float()).abs().max() / ref.float().abs().max().clamp_min(1e-6)
            assert err < 1e-2, f"rope max rel err {err}"
            return
        else:
            pytest.fail(f"unknown golden op {op}")
        # 16-bit: >= 98% bit-equal, the rest within 2 ulps at the largest output;
        # fp32: within 1e-5 (CPU and GPU exp/tanh differ in the last ulps)
        assert_matches_rounded(got, ref, dtype)


def test_config1_chain_properties():
    """The fp32 single-layer chain: residual = x + r exactly; the normalised row
    divided by the weight has unit RMS; rope preserves every rotated pair's
    norm; silu_and_mul matches a float64 evaluation."""
    c = ops_ref.CONFIG1
    inp = ops_ref.config1_inputs(seed=0)
    out = ops_ref.config1_chain(inp)
    assert torch.equal(out["residual"], inp["x"] + inp["residual"])
    rms = (out["x"] / inp["w"]).pow(2).mean(-1).sqrt()
    assert torch.allclose(rms, torch.ones_like(rms), atol=1e-4)
    hd, half = c["HD"], c["HD"] // 2
    for name, heads in (("q", c["NQ"]), ("k", c["NKV"])):
        a = inp[name].reshape(c["T"], heads, hd)
        b = out[name].reshape(c["T"], heads, hd)
        na = a[..., :half] ** 2 + a[..., half:] ** 2
        nb = b[..., :half] ** 2 + b[..., half:] ** 2
        assert torch.allclose(na, nb, rtol=1e-4, atol=1e-5)
    g = inp["gate_up"].double()
    a64, b64 = g[:, : c["I"]], g[:, c["I"]:]
    act64 = a64 / (1 + torch.exp(-a64)) * b64
    assert (out["act"].double() - act64).abs().max().item() <= 1e-5 * act64.abs().max().item()
    assert ops_ref.CONFIG1_BYTES_PER_TOKEN == 279048


def test_append_checked_rule_rejects_inconsistent_metadata():
    """The invalid-metadata rule of the append (skip and count): a last-page
    length of page_size + 1, an uncovered token (append_indptr[0] > 0) and an
    out-of-range page are counted and leave the cache untouched."""
    from oracle import append_ref

    ps, heads, hd = 16, 2, 8
    cache = torch.zeros(6, 2, ps, heads, hd)
    key = torch.randn(3, heads * hd)
    value = torch.randn(3, heads * hd)
    kp = torch.tensor([0, 1, 3])
    ki = torch.tensor([2, 4, 9])          # request 1's second page (9) is out of range
    kl = torch.tensor([ps + 1, 5])        # request 0 inconsistent: 1 page, length 17
    assert append_ref.token_slot(0, 16, ki, kp, kl, ps, 6) is None
    assert append_ref.token_slot(1, 3, ki, kp, kl, ps, 6) == (4, 3)
    assert append_ref.token_slot(1, 20, ki, kp, kl, ps, 6) is None  # page 9
    got, bad = append_ref.append_paged_kv_cache_checked(
        key, value, torch.tensor([0, 1, 1]), torch.tensor([16, 3, 20]), cache.clone(), ki, kp, kl)
    assert bad == 2
    assert torch.equal(got[4, 0, 3], key[1].view(heads, hd))
    assert int(got.ne(0).sum()) == 2 * heads * hd
    bi, pos = append_ref.batch_indices_positions_checked(torch.tensor([1, 2, 3]), kp,
                                                         torch.tensor([4, 5]), ps, 3)
    assert bi == [-1, 0, 1] and pos[1:] == [3, 20]
