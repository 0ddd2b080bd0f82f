"""GPU parity of the per-layer ops (norms, rope, activations) through the shim
and the C ABI, against the fp32 oracle and the reference's own CUDA ops."""
import ctypes

import pytest
import torch

from oracle import ops_ref
from paceserve_b200 import activation_ops, cabi, layernorm_ops, pos_encoding_ops
from tests._util import REL_TOL, assert_matches_rounded, ref_ops, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def _gen(seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


def randn(*shape, dtype=torch.bfloat16, seed=0, mean=0.0, std=1.0):
    return (torch.randn(*shape, generator=_gen(seed)) * std + mean).to(dtype)


# ------------------------------------------------------------------ norms --
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("T,H", [(1, 4096), (3, 4096), (17, 8192), (512, 4096), (5, 100),
                                 (2, 20000), (64, 5120), (4, 8)])
def test_rms_norm(T, H, dtype):
    x = randn(T, H, dtype=dtype, seed=T * 7 + H)
    w = randn(H, dtype=dtype, seed=1, mean=1.0, std=0.02)
    out = torch.empty(T, H, dtype=dtype, device=DEV)
    layernorm_ops.rms_norm(out, x.to(DEV), w.to(DEV), 1e-5)
    assert rel_err(out, ops_ref.rms_norm_fp32(x, w, 1e-5)) <= REL_TOL
    # the reference's own rounding points: equal up to the fp32 sum order
    assert_matches_rounded(out, ops_ref.rms_norm_rounded(x, w, 1e-5), dtype)
    ref = ref_ops("layernorm_ops")
    if ref is not None and T > 0:
        ro = torch.empty_like(out)
        ref.rms_norm(ro, x.to(DEV).contiguous(), w.to(DEV), 1e-5)
        assert_matches_rounded(out, ro, dtype, min_equal=0.99)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("T,H", [(8193, 4096), (8192, 8192), (8195, 1024), (1024, 4096),
                                 (3001, 4096), (2048, 1024)])
def test_rms_norm_large_batch_shapes(T, H, dtype):
    """Large-batch launch shapes of the plain norm: T >= 8192 runs two rows per
    CTA (odd T leaves the last CTA one row); 1024 <= T < 8192 runs 128-thread
    CTAs with up to 4 vectors per thread."""
    x = randn(T, H, dtype=dtype, seed=T + H)
    w = randn(H, dtype=dtype, seed=2, mean=1.0, std=0.02)
    out = torch.full((T + 1, H), 7.0, dtype=dtype, device=DEV)  # one guard row
    layernorm_ops.rms_norm(out[:T], x.to(DEV), w.to(DEV), 1e-5)
    assert rel_err(out[:T], ops_ref.rms_norm_fp32(x, w, 1e-5)) <= REL_TOL
    assert_matches_rounded(out[:T], ops_ref.rms_norm_rounded(x, w, 1e-5), dtype)
    assert bool((out[T] == 7.0).all())


def test_rms_norm_empty_and_strided():
    x = randn(0, 4096).to(DEV)
    layernorm_ops.rms_norm(torch.empty_like(x), x, torch.ones(4096, dtype=x.dtype, device=DEV), 1e-5)
    big = randn(9, 6144, seed=3).to(DEV)
    x = big[:, 1024:5120]  # row stride 6144
    w = randn(4096, seed=4, mean=1.0, std=0.02).to(DEV)
    out = torch.empty(9, 4096, dtype=x.dtype, device=DEV)
    layernorm_ops.rms_norm(out, x, w, 1e-6)
    assert rel_err(out, ops_ref.rms_norm_fp32(x.cpu(), w.cpu(), 1e-6)) <= REL_TOL
    with pytest.raises(RuntimeError, match="share a dtype"):
        layernorm_ops.rms_norm(out, x, w.float(), 1e-6)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("T,H", [(1, 4096), (17, 4096), (128, 4096), (129, 4096), (512, 4096),
                                 (33, 8192), (6, 200)])
def test_fused_add_rms_norm(T, H, dtype):
    x = randn(T, H, dtype=dtype, seed=T + H)
    r = randn(T, H, dtype=dtype, seed=T + H + 1)
    w = randn(H, dtype=dtype, seed=2, mean=1.0, std=0.02)
    xd, rd = x.to(DEV), r.to(DEV)
    layernorm_ops.fused_add_rms_norm(xd, rd, w.to(DEV), 1e-5)
    out_ref, res_ref = ops_ref.fused_add_rms_norm_rounded(x, r, w, 1e-5)
    assert torch.equal(rd.cpu(), res_ref)  # residual <- (T)(x + r) exactly
    assert_matches_rounded(xd, out_ref, dtype)
    out32, _ = ops_ref.fused_add_rms_norm_fp32(x, r, w, 1e-5)
    assert rel_err(xd, out32) <= REL_TOL


# ------------------------------------------------------------------- rope --
def _rope_case(T, nq, nkv, hd, rot, dtype, cache_dtype, neox, seed, max_pos=8192):
    qkv = randn(T, (nq + 2 * nkv) * hd, dtype=dtype, seed=seed).to(DEV)
    q = qkv[:, : nq * hd]
    k = qkv[:, nq * hd: (nq + nkv) * hd]
    cache = ops_ref.cos_sin_cache(rot, max_pos, 500000.0).to(cache_dtype)
    g = _gen(seed + 1)
    pos = torch.randint(0, max_pos, (T,), generator=g)
    return qkv, q, k, cache, pos


@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("dtype,cache_dtype", [(torch.bfloat16, torch.float32),
                                               (torch.bfloat16, torch.bfloat16),
                                               (torch.float16, torch.float32),
                                               (torch.float32, torch.float32)])
@pytest.mark.parametrize("T,nq,nkv,hd,rot", [(1, 32, 8, 128, 128), (512, 32, 8, 128, 128),
                                             (17, 64, 8, 128, 128), (9, 8, 2, 128, 64),
                                             (5, 4, 4, 80, 80), (3, 4, 2, 72, 24),
                                             # NeoX launch shapes: token-major parts (70B
                                             # at mid T, any model at long prefill)
                                             (300, 64, 8, 128, 128), (2049, 32, 8, 128, 128),
                                             (1500, 64, 8, 128, 128)])
def test_rotary_embedding(T, nq, nkv, hd, rot, dtype, cache_dtype, neox):
    qkv, q, k, cache, pos = _rope_case(T, nq, nkv, hd, rot, dtype, cache_dtype, neox, seed=T + nq)
    q0, k0, v0 = q.cpu().clone(), k.cpu().clone(), qkv[:, (nq + nkv) * hd:].cpu().clone()
    pos_d = pos.to(DEV)
    pos_encoding_ops.rotary_embedding(pos_d, q, k, hd, cache.to(DEV), neox)
    rq, rk = ops_ref.rotary_embedding_fp32(pos, q0, k0, hd, cache, neox)
    assert rel_err(q, rq) <= REL_TOL and rel_err(k, rk) <= REL_TOL
    assert torch.equal(qkv[:, (nq + nkv) * hd:].cpu(), v0)  # v untouched
    if rot < hd:  # tail of each head untouched
        assert torch.equal(q.cpu().view(T, nq, hd)[..., rot:], q0.view(T, nq, hd)[..., rot:])
    ref = ref_ops("pos_encoding_ops")
    if ref is not None and cache_dtype == dtype:
        qkv2 = qkv.new_empty(qkv.shape)
        qkv2.copy_(torch.cat([q0, k0, v0], 1).to(DEV))
        ref.rotary_embedding(pos_d, qkv2[:, : nq * hd], qkv2[:, nq * hd: (nq + nkv) * hd], hd,
                             cache.to(DEV), neox)
        assert rel_err(q, qkv2[:, : nq * hd]) <= REL_TOL


def test_rotary_embedding_out_of_range_positions_untouched():
    qkv, q, k, cache, pos = _rope_case(4, 4, 2, 128, 128, torch.bfloat16, torch.float32, True, 5,
                                       max_pos=64)
    pos = torch.tensor([3, 64, -1, 10])
    q0 = q.cpu().clone()
    pos_encoding_ops.rotary_embedding(pos.to(DEV), q, k, 128, cache.to(DEV), True)
    assert torch.equal(q.cpu()[1:3], q0[1:3])
    assert not torch.equal(q.cpu()[0], q0[0])


def test_rotary_embedding_3d_views_and_errors():
    T, nq, nkv, hd = 6, 4, 2, 128
    q = randn(T, nq, hd, seed=1).to(DEV)
    k = randn(T, nkv, hd, seed=2).to(DEV)
    cache = ops_ref.cos_sin_cache(hd, 128, 10000.0)
    pos = torch.arange(T)
    rq, rk = ops_ref.rotary_embedding_fp32(pos, q.cpu().reshape(T, -1), k.cpu().reshape(T, -1), hd,
                                           cache, True)
    pos_encoding_ops.rotary_embedding(pos.to(DEV), q, k, hd, cache.to(DEV), True)
    assert rel_err(q.reshape(T, -1), rq) <= REL_TOL
    with pytest.raises(RuntimeError, match="float32 or the query dtype"):
        pos_encoding_ops.rotary_embedding(pos.to(DEV), q, k, hd, cache.half().to(DEV), True)
    with pytest.raises(RuntimeError, match="int64"):
        pos_encoding_ops.rotary_embedding(pos.int().to(DEV), q, k, hd, cache.to(DEV), True)


# ------------------------------------------------------------- activations --
GATED = {
    "silu_and_mul": (activation_ops.silu_and_mul, ops_ref.silu_and_mul_fp32, ops_ref.silu_and_mul_rounded),
    "gelu_and_mul": (activation_ops.gelu_and_mul, ops_ref.gelu_and_mul_fp32, None),
    "gelu_tanh_and_mul": (activation_ops.gelu_tanh_and_mul, ops_ref.gelu_tanh_and_mul_fp32, None),
}


@pytest.mark.parametrize("name", list(GATED))
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("T,d", [(1, 14336), (7, 14336), (512, 14336), (64, 28672), (3, 100), (5, 8),
                                 (65537, 64)])  # > 65535 rows: row-major grid
def test_gated_activations(name, dtype, T, d):
    op, f32, rounded = GATED[name]
    x = randn(T, 2 * d, dtype=dtype, seed=T + d)
    out = torch.empty(T, d, dtype=dtype, device=DEV)
    op(out, x.to(DEV))
    assert rel_err(out, f32(x)) <= REL_TOL
    if rounded is not None:
        assert_matches_rounded(out, rounded(x), dtype)
    if name == "silu_and_mul" and ref_ops("activation_ops") is not None:
        ro = torch.empty_like(out)
        ref_ops("activation_ops").silu_and_mul(ro, x.to(DEV))
        assert_matches_rounded(out, ro, dtype, min_equal=0.999)
    if name != "silu_and_mul":  # matches the PyTorch composition on the GPU
        a, b = x.to(DEV)[:, :d], x.to(DEV)[:, d:]
        approx = "tanh" if name == "gelu_tanh_and_mul" else "none"
        comp = torch.nn.functional.gelu(a, approximate=approx) * b
        assert_matches_rounded(out, comp, dtype)


@pytest.mark.parametrize("name", ["gelu_new", "gelu_fast"])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("T,d", [(1, 4096), (64, 10240), (3, 77)])
def test_elementwise_gelus(name, dtype, T, d):
    op = getattr(activation_ops, name)
    f32 = getattr(ops_ref, f"{name}_fp32")
    rounded = getattr(ops_ref, f"{name}_rounded")
    x = randn(T, d, dtype=dtype, seed=d)
    out = torch.empty(T, d, dtype=dtype, device=DEV)
    op(out, x.to(DEV))
    assert rel_err(out, f32(x)) <= REL_TOL
    assert_matches_rounded(out, rounded(x), dtype)
    ref = ref_ops("activation_ops")
    if ref is not None:
        ro = torch.empty_like(out)
        getattr(ref, name)(ro, x.to(DEV))
        assert_matches_rounded(out, ro, dtype, min_equal=0.999)


def test_activation_strided_rows_and_shape_errors():
    big = randn(8, 3 * 2048, seed=9).to(DEV)
    x = big[:, :4096]  # [8, 2*2048] with row stride 6144
    out = torch.empty(8, 2048, dtype=x.dtype, device=DEV)
    activation_ops.silu_and_mul(out, x)
    assert rel_err(out, ops_ref.silu_and_mul_fp32(x.cpu())) <= REL_TOL
    with pytest.raises(RuntimeError, match="does not match"):
        activation_ops.silu_and_mul(torch.empty(8, 2047, dtype=x.dtype, device=DEV), x)


# ------------------------------------------------------ direct C-ABI calls --
def test_c_abi_direct_call_matches_shim():
    lib = cabi.load()
    x = randn(33, 4096, seed=11).to(DEV)
    w = randn(4096, seed=12, mean=1.0, std=0.02).to(DEV)
    a = torch.empty_like(x)
    b = torch.empty_like(x)
    layernorm_ops.rms_norm(a, x, w, 1e-5)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.pace_rms_norm(None, None, None, 1e-5, 0, 4096, 4096, 4096, cabi.PACE_BF16, stream) == 0
    cabi.check(lib.pace_rms_norm(b.data_ptr(), x.data_ptr(), w.data_ptr(), ctypes.c_float(1e-5), 33,
                                 4096, 4096, 4096, cabi.PACE_BF16, stream))
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    gu = randn(17, 2 * 14336, seed=13).to(DEV)
    o1 = torch.empty(17, 14336, dtype=gu.dtype, device=DEV)
    o2 = torch.empty_like(o1)
    activation_ops.silu_and_mul(o1, gu)
    cabi.check(lib.pace_silu_and_mul(o2.data_ptr(), gu.data_ptr(), 17, 14336, 2 * 14336, 14336,
                                     cabi.PACE_BF16, stream))
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


def test_pdl_on_and_off_agree():
    import paceserve_b200

    x = randn(512, 2 * 14336, seed=21).to(DEV)
    outs = []
    for pdl in (True, False):
        paceserve_b200.set_pdl(pdl)
        o = torch.empty(512, 14336, dtype=x.dtype, device=DEV)
        activation_ops.silu_and_mul(o, x)
        outs.append(o)
    paceserve_b200.set_pdl(True)
    assert torch.equal(outs[0], outs[1])


def test_graph_capture_of_op_chain():
    """The ops are stream-ordered launches and capture into a CUDA graph."""
    T, H = 64, 4096
    x = randn(T, H, seed=31).to(DEV)
    r = randn(T, H, seed=32).to(DEV)
    w = randn(H, seed=33, mean=1.0, std=0.02).to(DEV)
    x0, r0 = x.clone(), r.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layernorm_ops.fused_add_rms_norm(x, r, w, 1e-5)  # warm-up
    torch.cuda.current_stream().wait_stream(s)
    x.copy_(x0)
    r.copy_(r0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layernorm_ops.fused_add_rms_norm(x, r, w, 1e-5)
    x.copy_(x0)
    r.copy_(r0)
    g.replay()
    torch.cuda.synchronize()
    out_ref, res_ref = ops_ref.fused_add_rms_norm_rounded(x0.cpu(), r0.cpu(), w.cpu(), 1e-5)
    assert torch.equal(r.cpu(), res_ref)
    assert_matches_rounded(x, out_ref, torch.bfloat16)


def test_config1_layer_chain_fp32():
    """The CPU-runnable configuration (one Llama-3-8B layer in fp32 at T=64:
    fused_add_rms_norm -> neox rope -> silu_and_mul) on the GPU against the
    oracle's fp32 chain on the same seeded inputs; fp32 outputs within 1e-5."""
    c = ops_ref.CONFIG1
    inp = ops_ref.config1_inputs(seed=0)
    ref = ops_ref.config1_chain(inp)
    d = {k: v.to(DEV) for k, v in inp.items()}
    layernorm_ops.fused_add_rms_norm(d["x"], d["residual"], d["w"], c["EPS"])
    pos_encoding_ops.rotary_embedding(d["positions"], d["q"], d["k"], c["HD"], d["cache"], True)
    act = torch.empty(c["T"], c["I"], device=DEV)
    activation_ops.silu_and_mul(act, d["gate_up"])
    torch.cuda.synchronize()
    got = {"x": d["x"], "residual": d["residual"], "q": d["q"], "k": d["k"], "act": act}
    for name, r in ref.items():
        assert rel_err(got[name], r) <= 1e-5, name
