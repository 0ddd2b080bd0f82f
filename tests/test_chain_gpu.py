"""GPU parity of the headline configuration itself.

bench.py times one CUDA graph of the Llama-3-8B 32-layer op chain over the
Sarathi mixed batch (448 prefill tokens at positions 0..447 plus 64 decode
tokens at positions uniform in [1, 8191], bf16, fp32 cos/sin cache).  These
tests build that exact batch with bench.build_chain, replay bench's captured
graph once, and check layers 0, 1 and 31 against the CPU oracle's layer
(oracle.ops_ref.chain_layer) on snapshots of the same inputs:
  * every bf16 output within REL_TOL (1e-2) of the fp32 formula;
  * the fused norm's residual (x + r rounded to bf16) bit-exact;
  * the normed outputs and SwiGLU almost everywhere bit-equal to the
    restatement of the reference kernels' rounding points.
"""
import pytest
import torch

import bench
from oracle import ops_ref
from tests._util import REL_TOL, assert_matches_rounded, ref_ops, rel_err

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
CHECK_LAYERS = (0, 1, bench.L - 1)
INPUT_KEYS = ("hidden", "residual", "w_in", "qkv", "attn", "residual2", "w_post", "gate_up")


def _ops():
    import paceserve_b200 as pb

    return pb.layernorm_ops, pb.pos_encoding_ops, pb.activation_ops


def _snapshot(ch, layer):
    b = ch["layers"][layer]
    return {k: b[k].cpu().clone() for k in INPUT_KEYS if k in b}


def _check_layer(ch, layer, snap, pos, cache):
    b = ch["layers"][layer]
    want = {k: v.clone() for k, v in snap.items()}
    ops_ref.chain_layer(layer, want, cache, pos, bench.EPS, bench.NQ, bench.NKV, bench.HD)
    nq, nkv, hd = bench.NQ, bench.NKV, bench.HD
    # fp32 formulas (the parity rule) on the same inputs
    if layer == 0:
        exact = ops_ref.rms_norm_fp32(snap["hidden"], snap["w_in"], bench.EPS)
        assert rel_err(b["normed"], exact) <= REL_TOL
        assert_matches_rounded(b["normed"].cpu(), want["normed"], torch.bfloat16)
    else:
        exact, res = ops_ref.fused_add_rms_norm_fp32(snap["hidden"], snap["residual"],
                                                     snap["w_in"], bench.EPS)
        assert torch.equal(b["residual"].cpu(), want["residual"])
        assert rel_err(b["hidden"], exact) <= REL_TOL
        assert_matches_rounded(b["hidden"].cpu(), want["hidden"], torch.bfloat16)
    q = snap["qkv"][:, : nq * hd]
    k = snap["qkv"][:, nq * hd: (nq + nkv) * hd]
    rq, rk = ops_ref.rotary_embedding_fp32(pos, q, k, hd, cache, True)
    got = b["qkv"].cpu()
    assert rel_err(got[:, : nq * hd], rq) <= REL_TOL
    assert rel_err(got[:, nq * hd: (nq + nkv) * hd], rk) <= REL_TOL
    assert torch.equal(got[:, (nq + nkv) * hd:], snap["qkv"][:, (nq + nkv) * hd:])  # v untouched
    exact, _ = ops_ref.fused_add_rms_norm_fp32(snap["attn"], snap["residual2"], snap["w_post"],
                                               bench.EPS)
    assert torch.equal(b["residual2"].cpu(), want["residual2"])
    assert rel_err(b["attn"], exact) <= REL_TOL
    assert rel_err(b["act"], ops_ref.silu_and_mul_fp32(snap["gate_up"])) <= REL_TOL
    assert_matches_rounded(b["act"].cpu(), want["act"], torch.bfloat16, min_equal=0.999)


def test_headline_chain_graph_matches_oracle():
    """bench.py's timed object: the captured 32-layer graph over the Sarathi batch."""
    ch = bench.build_chain(DEV, seed=1234)
    g = bench.capture(lambda: bench.run_chain(ch, _ops()))  # runs the chain twice (in place)
    snaps = {layer: _snapshot(ch, layer) for layer in CHECK_LAYERS}
    pos, cache = ch["positions"].cpu(), ch["cache"].cpu()
    assert pos[: bench.T_PREFILL].tolist() == list(range(bench.T_PREFILL))
    dec = pos[bench.T_PREFILL:]
    assert len(dec) == bench.T_DECODE and int(dec.min()) >= 1 and int(dec.max()) < bench.MAX_POS
    g.replay()
    torch.cuda.synchronize()
    for layer in CHECK_LAYERS:
        _check_layer(ch, layer, snaps[layer], pos, cache)
    del g


def test_headline_chain_eager_matches_reference_ops():
    """The same batch through the reference's own CUDA ops (built from its sources)
    on layer 0: rms_norm and silu_and_mul agree to the bit in almost all
    elements, rope (bf16 cache, the reference's only form) within 1e-2."""
    ln_ref = ref_ops("layernorm_ops")
    act_ref = ref_ops("activation_ops")
    pe_ref = ref_ops("pos_encoding_ops")
    ln, pe, act = _ops()
    ch = bench.build_chain(DEV, seed=99)
    b = ch["layers"][0]
    out_ref = torch.empty_like(b["normed"])
    ln_ref.rms_norm(out_ref, b["hidden"], b["w_in"], bench.EPS)
    ln.rms_norm(b["normed"], b["hidden"], b["w_in"], bench.EPS)
    assert_matches_rounded(b["normed"].cpu(), out_ref.cpu(), torch.bfloat16, min_equal=0.99)
    a_ref = torch.empty_like(b["act"])
    act_ref.silu_and_mul(a_ref, b["gate_up"])
    act.silu_and_mul(b["act"], b["gate_up"])
    assert_matches_rounded(b["act"].cpu(), a_ref.cpu(), torch.bfloat16, min_equal=0.999)
    nq, nkv, hd = bench.NQ, bench.NKV, bench.HD
    qkv_ref = b["qkv"].clone()
    cache16 = ch["cache"].to(torch.bfloat16)
    pe_ref.rotary_embedding(ch["positions"], qkv_ref[:, : nq * hd],
                            qkv_ref[:, nq * hd: (nq + nkv) * hd], hd, cache16, True)
    pe.rotary_embedding(ch["positions"], b["q"], b["k"], hd, ch["cache"], True)
    assert rel_err(b["qkv"], qkv_ref) <= REL_TOL
