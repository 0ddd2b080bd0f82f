"""CPU: the C-ABI library loads, exports every symbol the header declares, and
rejects bad arguments with a status and a message before touching the GPU."""
import ctypes
import os
import re

import pytest

from paceserve_b200 import cabi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pace_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pace_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ["pace_rms_norm", "pace_fused_add_rms_norm", "pace_rotary_embedding",
              "pace_silu_and_mul", "pace_gelu_and_mul", "pace_topk_softmax",
              "pace_moe_align_block_size", "pace_kv_copy_blocks"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(cabi.LIBRARY_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    assert sorted(cabi.SIGNATURES) == declared_functions()


def test_status_strings_and_version():
    lib = cabi.load()
    assert lib.pace_status_string(cabi.PACE_OK) == b"PACE_OK"
    assert lib.pace_status_string(cabi.PACE_ERR_TOO_LARGE) == b"PACE_ERR_TOO_LARGE"
    assert lib.pace_version() > 0


def _expect(status, code, needle):
    lib = cabi.load()
    assert status == code
    assert needle in lib.pace_last_error().decode()


def test_argument_errors_need_no_gpu():
    lib = cabi.load()
    _expect(lib.pace_rms_norm(None, None, None, 1e-5, -1, 8, 8, 8, cabi.PACE_BF16, None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "bad shape")
    _expect(lib.pace_rms_norm(None, None, None, 1e-5, 4, 8, 4, 8, cabi.PACE_BF16, None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "row stride")
    # zero tokens is a no-op, not an error
    assert lib.pace_rms_norm(None, None, None, 1e-5, 0, 8, 8, 8, cabi.PACE_BF16, None) == 0
    _expect(lib.pace_topk_softmax(None, None, None, None, 4, 8, 9, 0, None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "exceeds num_experts")
    _expect(lib.pace_topk_softmax(None, None, None, None, 4, 2048, 2, 0, None),
            cabi.PACE_ERR_TOO_LARGE, "exceeds 1024")
    _expect(lib.pace_moe_align_block_size(None, cabi.PACE_I32, 9, 5, 4, None, 10, None, 5, None, 0,
                                          None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "sorted_token_ids holds")
    _expect(lib.pace_rotary_embedding(None, None, None, 4, 2, 1, 128, 256, 128, None, 0, 130, 10, 1,
                                      cabi.PACE_BF16, None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "rot_dim")
    _expect(lib.pace_silu_and_mul(None, None, 4, 8, 8, 8, cabi.PACE_BF16, None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "row stride")
    # the qkv projection needs no workspace up to 2 tokens (CUDA-core kernel),
    # the stream-K workspace from 3 on; 0 also for a bad shape
    assert lib.pace_qkv_proj_rope_workspace_size(2, 4096, 32, 8, 0) == 0
    assert lib.pace_qkv_proj_rope_workspace_size(3, 4096, 32, 8, 0) > 0
    assert lib.pace_qkv_proj_rope_workspace_size(3, 4096, 0, 0, 0) == 0
    assert lib.pace_gate_up_silu_workspace_size(2, 4096, 14336, 0) == 0
    assert lib.pace_gate_up_silu_workspace_size(3, 4096, 14336, 0) > 0
    assert lib.pace_linear_residual_workspace_size(2, 4096, 4096, 0) == 0
    assert lib.pace_linear_residual_workspace_size(3, 4096, 4096, 0) > 0
    # two tokens over a long K (down_proj) stay on the tensor cores
    assert lib.pace_linear_residual_workspace_size(2, 4096, 14336, 0) > 0
    assert lib.pace_linear_residual_workspace_size(1, 4096, 14336, 0) == 0
    tab = cabi.layer_table([0])
    _expect(lib.pace_kv_copy_blocks(tab, tab, 0, None, None, 1, 65536, 1, 1, None, 0, None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "num_layers")
    _expect(lib.pace_kv_copy_blocks(tab, tab, 1, None, None, 1, 100, 1, 1, None, 0, None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "multiple of 16")
    _expect(lib.pace_kv_copy_blocks(tab, tab, 1, None, None, 1, 65536, 1, 1, None, 5, None),
            cabi.PACE_ERR_INVALID_ARGUMENT, "method")


def test_check_raises_pace_error():
    lib = cabi.load()
    rc = lib.pace_silu_and_mul(None, None, -3, 8, 16, 8, cabi.PACE_F16, None)
    with pytest.raises(cabi.PaceError, match="bad shape"):
        cabi.check(rc)


def test_last_error_is_per_thread():
    """pace_last_error() is thread-local: concurrent callers (the reference's
    KV insertion threads, decode_instance.py:50-51) each read their own message."""
    import threading

    lib = cabi.load()
    barrier = threading.Barrier(2)
    seen = {}

    def norm_caller():
        rc = lib.pace_rms_norm(None, None, None, 1e-5, -1, 8, 8, 8, cabi.PACE_BF16, None)
        barrier.wait()  # the other thread has now failed too
        barrier.wait()
        seen["norm"] = (rc, lib.pace_last_error().decode())

    def topk_caller():
        barrier.wait()
        rc = lib.pace_topk_softmax(None, None, None, None, 4, 8, 9, 0, None)
        barrier.wait()
        seen["topk"] = (rc, lib.pace_last_error().decode())

    ts = [threading.Thread(target=norm_caller), threading.Thread(target=topk_caller)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert seen["norm"][0] == cabi.PACE_ERR_INVALID_ARGUMENT and "rms_norm" in seen["norm"][1]
    assert seen["topk"][0] == cabi.PACE_ERR_INVALID_ARGUMENT and "num_experts" in seen["topk"][1]
