"""GPU parity of the fused qkv projection + rotary embedding (tcgen05 GEMM with
the rotation in its epilogue; at decode sizes the weight-streaming CUDA-core
kernel with the same epilogue) against the fp32 oracle: the GEMM of the same
bf16/fp16 inputs in fp32, then the oracle's rotation.  Tolerance: the float
rule of the per-layer ops, max|got - ref| / max|ref| <= 1e-2, plus a per-element
bound of a few storage-type ulps (the only differences are the fp32 summation
order and the one final rounding)."""
import ctypes

import pytest
import torch

from oracle import ops_ref
from paceserve_b200 import cabi, pos_encoding_ops
from tests._util import REL_TOL, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _gen(seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


def reference(hidden, weight, positions, nq, nkv, hd, cache, neox):
    """fp32 oracle: qkv = hidden @ weight^T from the same 16-bit inputs, then
    the q and k heads rotated by ops_ref.rotary_embedding_fp32."""
    qkv = hidden.float() @ weight.float().t()
    q, k = ops_ref.rotary_embedding_fp32(positions, qkv[:, : nq * hd],
                                         qkv[:, nq * hd: (nq + nkv) * hd], hd, cache, neox)
    return torch.cat([q, k, qkv[:, (nq + nkv) * hd:]], dim=1)


def make_case(T, H, nq, nkv, dtype, seed, max_pos=8192, pos_hi=None):
    g = _gen(seed)
    hd = 128
    hidden = torch.randn(T, H, generator=g).to(dtype)
    # weights scaled like a trained projection so outputs stay O(1)
    weight = (torch.randn((nq + 2 * nkv) * hd, H, generator=g) / H ** 0.5).to(dtype)
    positions = torch.randint(0, pos_hi or max_pos, (T,), generator=g)
    cache = ops_ref.cos_sin_cache(hd, max_pos, 500000.0)
    return hidden, weight, positions, cache


def check(got, ref, dtype, tight=True):
    assert rel_err(got, ref) <= REL_TOL
    if tight:
        # one rounding of the fp32 accumulator: within one storage ulp of each
        # element, plus 0.1 % of the largest magnitude for the summation order
        g, r = got.float().cpu(), ref.float().cpu()
        bound = torch.finfo(dtype).eps * r.abs() + 1e-3 * r.abs().max()
        assert ((g - r).abs() <= bound).all(), ((g - r).abs() - bound).max().item()


@pytest.mark.parametrize("T", [1, 2, 3, 17, 128, 200, 256, 300, 512])
@pytest.mark.parametrize("neox", [True, False])
def test_llama3_8b_shape(T, neox):
    # T <= 2: the weight-streaming kernel on CUDA cores; 3 <= T <= 128: single
    # CTAs on tensor cores (T = 3 and 17 finish shared tiles by their last
    # contributor); T = 200 and 256: CTA pairs, stream-K; 300 and 512: CTA
    # pairs, one data-parallel round
    nq, nkv, hd, H = 32, 8, 128, 4096
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, T)
    qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, device=DEV)
    fault = torch.zeros(1, dtype=torch.int32, device=DEV)
    pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hidden.to(DEV), weight.to(DEV),
                                               positions.to(DEV), hd, nq, nkv, cache.to(DEV),
                                               neox, fault)
    torch.cuda.synchronize()
    assert fault.item() == 0
    check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache, neox), torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cache_16bit", [False, True])
def test_dtypes_and_cache_types(dtype, cache_16bit):
    T, H, nq, nkv, hd = 130, 1024, 4, 2, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, dtype, 5)
    if cache_16bit:
        cache = cache.to(dtype)
    qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=dtype, device=DEV)
    pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hidden.to(DEV), weight.to(DEV),
                                               positions.to(DEV), hd, nq, nkv, cache.to(DEV),
                                               True)
    torch.cuda.synchronize()
    check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache.float(), True), dtype)


@pytest.mark.parametrize("H", [64, 200, 4104])
def test_hidden_not_a_multiple_of_the_k_block(H):
    # the K tail past the last full 64-element block is zero-filled by TMA
    T, nq, nkv, hd = 40, 2, 1, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, H)
    qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, device=DEV)
    pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hidden.to(DEV), weight.to(DEV),
                                               positions.to(DEV), hd, nq, nkv, cache.to(DEV),
                                               True)
    torch.cuda.synchronize()
    check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache, True), torch.bfloat16)


def test_strided_rows_and_out_of_range_positions():
    T, H, nq, nkv, hd = 200, 512, 4, 2, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, 9)
    positions[::7] = -3
    positions[3::11] = 8192  # == max_position: out of range
    big = torch.zeros(T, H + 64, dtype=torch.bfloat16)
    big[:, :H] = hidden
    n = (nq + 2 * nkv) * hd
    out_big = torch.full((T, n + 256), 7.0, dtype=torch.bfloat16, device=DEV)
    qkv = out_big[:, :n]
    pos_encoding_ops.qkv_proj_rotary_embedding(qkv, big.to(DEV)[:, :H], weight.to(DEV),
                                               positions.to(DEV), hd, nq, nkv, cache.to(DEV),
                                               True)
    torch.cuda.synchronize()
    ref = reference(hidden, weight, positions, nq, nkv, hd, cache, True)
    check(qkv, ref, torch.bfloat16)
    # tokens out of range are the plain projection
    plain = hidden.float() @ weight.float().t()
    bad = (positions < 0) | (positions >= 8192)
    check(qkv.cpu()[bad], plain[bad], torch.bfloat16)
    # the padding columns past the output row are untouched
    assert (out_big[:, n:].cpu() == 7.0).all()


@pytest.mark.parametrize("T,H,dtype,cache_16bit,neox",
                         [(1, 200, torch.float16, True, True), (2, 4104, torch.bfloat16, False, False),
                          (1, 1032, torch.float16, False, False), (2, 64, torch.bfloat16, True, True)])
def test_decode_rows_on_cuda_cores(T, H, dtype, cache_16bit, neox):
    """At most 2 rows: one warp per rotation pair streams the weight.  K that
    is not a multiple of the 256 elements a warp reads per pass (H = 200: 25
    vectors, fewer than the lanes), odd head counts, strided rows, positions
    out of range, 16-bit caches, and nothing written past the output rows."""
    nq, nkv, hd = 3, 1, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, dtype, T * 1000 + H)
    positions[0] = -1  # not rotated
    if cache_16bit:
        cache = cache.to(dtype)
    big = torch.zeros(T, H + 40, dtype=dtype)
    big[:, 8:8 + H] = hidden
    n = (nq + 2 * nkv) * hd
    out_big = torch.full((T, n + 64), 5.0, dtype=dtype, device=DEV)
    qkv = out_big[:, :n]
    pos_encoding_ops.qkv_proj_rotary_embedding(qkv, big.to(DEV)[:, 8:8 + H], weight.to(DEV),
                                               positions.to(DEV), hd, nq, nkv, cache.to(DEV),
                                               neox)
    torch.cuda.synchronize()
    check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache.float(), neox), dtype)
    plain = hidden.float() @ weight.float().t()
    check(qkv.cpu()[:1], plain[:1], dtype)
    assert (out_big[:, n:].cpu() == 5.0).all()


def test_decode_rows_graph_replay_is_deterministic():
    T, H, nq, nkv, hd = 2, 4096, 32, 8, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, 31)
    hd_, wd, pd, cd = hidden.to(DEV), weight.to(DEV), positions.to(DEV), cache.to(DEV)
    qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, device=DEV)
    pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hd_, wd, pd, hd, nq, nkv, cd, True)
    torch.cuda.synchronize()
    first = qkv.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hd_, wd, pd, hd, nq, nkv, cd, True)
    qkv.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(qkv, first)
    check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache, True), torch.bfloat16)


def test_matches_unfused_projection_then_rope():
    """The fused result against the path it replaces: a library GEMM, then the
    rotary_embedding op on the q/k views.  The unfused path rounds twice, so the
    two differ by at most a couple of bf16 ulps."""
    T, H, nq, nkv, hd = 512, 4096, 32, 8, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, 21)
    hd_, wd, pd, cd = hidden.to(DEV), weight.to(DEV), positions.to(DEV), cache.to(DEV)
    unfused = hd_ @ wd.t()
    pos_encoding_ops.rotary_embedding(pd, unfused[:, : nq * hd], unfused[:, nq * hd: (nq + nkv) * hd],
                                      hd, cd, True)
    fused = torch.empty_like(unfused)
    pos_encoding_ops.qkv_proj_rotary_embedding(fused, hd_, wd, pd, hd, nq, nkv, cd, True)
    torch.cuda.synchronize()
    ref = reference(hidden, weight, positions, nq, nkv, hd, cache, True)
    check(fused, ref, torch.bfloat16)
    check(unfused, ref, torch.bfloat16, tight=False)


def test_graph_capture_and_repeat():
    T, H, nq, nkv, hd = 256, 2048, 8, 2, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, 4)
    hd_, wd, pd, cd = hidden.to(DEV), weight.to(DEV), positions.to(DEV), cache.to(DEV)
    qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hd_, wd, pd, hd, nq, nkv, cd, True)
    torch.cuda.current_stream().wait_stream(s)
    first = qkv.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hd_, wd, pd, hd, nq, nkv, cd, True)
    qkv.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(qkv, first)  # deterministic: same bits every run
    check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache, True), torch.bfloat16)


def test_c_abi_direct_call_and_workspace_reuse():
    lib = cabi.load()
    T, H, nq, nkv, hd = 64, 256, 2, 1, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, 2)
    hd_, wd, pd, cd = hidden.to(DEV), weight.to(DEV), positions.to(DEV), cache.to(DEV)
    n = (nq + 2 * nkv) * hd
    need = lib.pace_qkv_proj_rope_workspace_size(T, H, nq, nkv, 0)
    assert need == pos_encoding_ops.qkv_proj_rope_workspace_size(T, H, nq, nkv, 0) > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ref = reference(hidden, weight, positions, nq, nkv, hd, cache, True)
    for _ in range(3):  # the workspace is left valid: reusable without clearing
        out = torch.empty(T, n, dtype=torch.bfloat16, device=DEV)
        st = lib.pace_qkv_proj_rope(out.data_ptr(), hd_.data_ptr(), wd.data_ptr(), pd.data_ptr(),
                                    T, H, nq, nkv, hd, H, n, cd.data_ptr(), cabi.PACE_F32, hd,
                                    8192, 1, cabi.PACE_BF16, ws.data_ptr(), need, None, stream)
        assert st == cabi.PACE_OK, lib.pace_last_error()
        torch.cuda.synchronize()
        check(out, ref, torch.bfloat16)
    # after the partial slots (two of 128 x 256 fp32 per SM): the grid barrier
    # (arrival count re-armed, one generation per call that needed it, none
    # when the tiles run data-parallel), then the per-tile counters, all zero
    slot_bytes = 2 * torch.cuda.get_device_properties(0).multi_processor_count * 128 * 256 * 4
    bar = ws[slot_bytes: slot_bytes + 256].view(torch.int32)
    assert bar[0].item() == 0 and bar[32].item() in (0, 3)
    assert int(bar[1:32].sum().item()) == 0 and int(bar[33:].sum().item()) == 0
    assert int(ws[slot_bytes + 256:].sum().item()) == 0
    st = lib.pace_qkv_proj_rope(out.data_ptr(), hd_.data_ptr(), wd.data_ptr(), pd.data_ptr(), T,
                                H, nq, nkv, hd, H, n, cd.data_ptr(), cabi.PACE_F32, hd, 8192, 1,
                                cabi.PACE_BF16, ws.data_ptr(), need - 1, None, stream)
    assert st == cabi.PACE_ERR_INVALID_ARGUMENT
    assert b"workspace" in lib.pace_last_error()


def test_caller_workspace_through_the_shim():
    T, H, nq, nkv, hd = 700, 1024, 8, 2, 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, 12)
    need = pos_encoding_ops.qkv_proj_rope_workspace_size(T, H, nq, nkv, 0)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, device=DEV)
    pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hidden.to(DEV), weight.to(DEV),
                                               positions.to(DEV), hd, nq, nkv, cache.to(DEV),
                                               True, None, ws)
    torch.cuda.synchronize()
    check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache, True), torch.bfloat16)
    with pytest.raises(RuntimeError, match="workspace"):
        pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hidden.to(DEV), weight.to(DEV),
                                                   positions.to(DEV), hd, nq, nkv, cache.to(DEV),
                                                   True, None, ws[: need // 2])


def test_one_workspace_across_shapes():
    """A zeroed workspace stays valid when calls of different shapes (different
    tile counts) share it, in either order."""
    nq, nkv, hd, H = 8, 2, 128, 1024
    need = max(pos_encoding_ops.qkv_proj_rope_workspace_size(T, H, nq, nkv, 0)
               for T in (1, 300, 1500))
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    for T in (1, 1500, 300, 1, 300, 1500):
        hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, T)
        qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, device=DEV)
        pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hidden.to(DEV), weight.to(DEV),
                                                   positions.to(DEV), hd, nq, nkv,
                                                   cache.to(DEV), False, None, ws)
        torch.cuda.synchronize()
        check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache, False),
              torch.bfloat16)


@pytest.mark.parametrize("T,H,nq,nkv", [(1, 8192, 64, 8), (2048, 4096, 32, 8), (333, 4096, 3, 1)])
def test_larger_and_odd_head_counts(T, H, nq, nkv):
    # 70B-wide rows at one token (every tile shared by many CTAs), a long
    # prefill, and an odd head count (the last tile's second head is absent)
    hd = 128
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, T + nq)
    qkv = torch.empty(T, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, device=DEV)
    pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hidden.to(DEV), weight.to(DEV),
                                               positions.to(DEV), hd, nq, nkv, cache.to(DEV),
                                               True)
    torch.cuda.synchronize()
    check(qkv, reference(hidden, weight, positions, nq, nkv, hd, cache, True), torch.bfloat16)


@pytest.mark.parametrize("extra", [1, 2, 9])
def test_fewer_leftover_units_than_ctas(extra):
    """SMs + extra tiles of 16 K blocks: after one data-parallel round the
    leftover 16 * extra units are fewer than the CTAs, so the stream-K split
    must use only as many CTAs as units (a tile's contributors consecutive).
    Called twice: the tile counters must be left re-armed."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    T, H, hd, nkv = 128, 1024, 128, 2
    nq = 2 * (sms + extra) - 2 * nkv  # (sms + extra) tiles of two heads
    hidden, weight, positions, cache = make_case(T, H, nq, nkv, torch.bfloat16, extra)
    ref = reference(hidden, weight, positions, nq, nkv, hd, cache, True)
    fault = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = (hidden.to(DEV), weight.to(DEV), positions.to(DEV), hd, nq, nkv, cache.to(DEV), True,
            fault)
    for _ in range(2):
        qkv = torch.full((T, (nq + 2 * nkv) * hd), float("nan"), dtype=torch.bfloat16,
                         device=DEV)
        pos_encoding_ops.qkv_proj_rotary_embedding(qkv, *args)
        torch.cuda.synchronize()
        assert fault.item() == 0
        check(qkv, ref, torch.bfloat16)


def test_rejected_shapes():
    T, H, nq, nkv = 4, 256, 2, 1
    hidden = torch.randn(T, H, device=DEV).bfloat16()
    cache = torch.randn(8192, 64, device=DEV)
    weight = torch.randn((nq + 2 * nkv) * 64, H, device=DEV).bfloat16()
    qkv = torch.empty(T, (nq + 2 * nkv) * 64, dtype=torch.bfloat16, device=DEV)
    pos = torch.zeros(T, dtype=torch.long, device=DEV)
    with pytest.raises(RuntimeError, match="head_size"):
        pos_encoding_ops.qkv_proj_rotary_embedding(qkv, hidden, weight, pos, 64, nq, nkv, cache, True)
    with pytest.raises(RuntimeError, match="bfloat16 or float16"):
        pos_encoding_ops.qkv_proj_rotary_embedding(qkv.float(), hidden.float(), weight.float(), pos,
                                                   64, nq, nkv, cache, True)
