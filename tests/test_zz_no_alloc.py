"""GPU test of the allocation-free qkv projection + rotary embedding entry
point, pace_qkv_proj_rope_no_alloc, called through the C ABI.

It exists for callers that cannot allocate device memory (a plugin host that
hands an op only its input and output buffers, or a serving loop that must
not call cudaMalloc because it synchronises the device); its scratch is a
fixed array inside the library instead of a caller workspace.  The test
checks two calls in a row against the workspace entry point
(pace_qkv_proj_rope) within the same tolerance the fused op's parity tests
use, and that shapes beyond the fixed scratch are refused.

This file is named so that pytest collects it last; it must pass alone in a
fresh process and after the other tests.
"""
import ctypes

import pytest
import torch

from oracle import ops_ref
from paceserve_b200 import cabi
from tests._util import REL_TOL, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def close(got, ref, dtype):
    """The fused op's rule: within 1e-2 of the largest magnitude, and per
    element within one storage ulp plus 0.1 % of the largest magnitude (the two
    entry points split the K sum differently, so fp32 summation order differs)."""
    assert rel_err(got, ref) <= REL_TOL
    g, r = got.float().cpu(), ref.float().cpu()
    bound = torch.finfo(dtype).eps * r.abs() + 1e-3 * r.abs().max()
    assert ((g - r).abs() <= bound).all()


@pytest.mark.parametrize("T", [512, 37, 2])
def test_no_alloc_matches_the_workspace_entry_point(T):
    lib = cabi.load()
    nq, nkv, hd, H = 32, 8, 128, 4096
    n = (nq + 2 * nkv) * hd
    g = torch.Generator().manual_seed(T)
    hidden = torch.randn(T, H, generator=g).bfloat16().to(DEV)
    weight = (torch.randn(n, H, generator=g) / H ** 0.5).bfloat16().to(DEV)
    positions = torch.randint(0, 8192, (T,), generator=g).to(DEV)
    cache = ops_ref.cos_sin_cache(hd, 8192, 500000.0).to(DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    fault = torch.zeros(1, dtype=torch.int32, device=DEV)

    need = lib.pace_qkv_proj_rope_workspace_size(T, H, nq, nkv, 0)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    ref = torch.empty(T, n, dtype=torch.bfloat16, device=DEV)
    st = lib.pace_qkv_proj_rope(ref.data_ptr(), hidden.data_ptr(), weight.data_ptr(),
                                positions.data_ptr(), T, H, nq, nkv, hd, H, n, cache.data_ptr(),
                                cabi.PACE_F32, hd, 8192, 1, cabi.PACE_BF16, ws.data_ptr(), need,
                                None, stream)
    assert st == cabi.PACE_OK, lib.pace_last_error()

    outs = []
    for _ in range(2):  # two calls in a row share the fixed scratch
        out = torch.full((T, n), 3.0, dtype=torch.bfloat16, device=DEV)
        st = lib.pace_qkv_proj_rope_no_alloc(out.data_ptr(), hidden.data_ptr(), weight.data_ptr(),
                                             positions.data_ptr(), T, H, nq, nkv, hd, H, n,
                                             cache.data_ptr(), cabi.PACE_F32, hd, 8192, 1,
                                             cabi.PACE_BF16, fault.data_ptr(), stream)
        assert st == cabi.PACE_OK, lib.pace_last_error()
        outs.append(out)
    torch.cuda.synchronize()
    assert fault.item() == 0
    for out in outs:
        close(out, ref, torch.bfloat16)
    # the same split of the work every call: the same bits
    assert torch.equal(outs[0], outs[1])


def test_no_alloc_refuses_shapes_beyond_its_scratch():
    lib = cabi.load()
    # 100000 tokens x 6144 columns = 782 x 24 tiles > 16384: refused before
    # any pointer is used
    st = lib.pace_qkv_proj_rope_no_alloc(None, None, None, None, 100000, 4096, 32, 8, 128, 4096,
                                         6144, None, cabi.PACE_F32, 128, 8192, 1,
                                         cabi.PACE_BF16, None, None)
    assert st == cabi.PACE_ERR_TOO_LARGE
    assert b"scratch" in lib.pace_last_error()
