"""ctypes binding of the C ABI (``include/pace_b200.h``) for callers without torch.

This is the binding a Python host would add to call ``libpace_b200.so``
directly: plain integers for device pointers and streams, status codes mapped
to ``PaceError``.  ``load()`` returns the configured ``ctypes.CDLL``.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p

LIBRARY_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libpace_b200.so")

PACE_OK = 0
PACE_ERR_INVALID_ARGUMENT = 1
PACE_ERR_UNSUPPORTED_DTYPE = 2
PACE_ERR_CUDA = 3
PACE_ERR_PEER_ACCESS = 4
PACE_ERR_TOO_LARGE = 5

PACE_F32, PACE_F16, PACE_BF16 = 0, 1, 2
PACE_U8, PACE_I8, PACE_I16, PACE_I32, PACE_I64 = 3, 4, 5, 6, 7
PACE_IPC_HANDLE_BYTES = 64
PACE_KV_TIMEOUT_FLAG = 1 << 30
PACE_KV_DRAIN_TIMEOUT_FLAG = 1 << 29


class KvCopyOpts(ctypes.Structure):
    """``pace_kv_copy_opts``."""

    _fields_ = [("method", c_int), ("max_ctas", c_int), ("wait_limit_ns", c_uint64),
                ("test_overarm_bytes", c_int)]


_P = c_void_p  # device pointer / stream
_ACT = [_P, _P, c_int64, c_int64, c_int64, c_int64, c_int, _P]

# name -> (restype, argtypes); one entry per declaration in pace_b200.h
SIGNATURES: dict[str, tuple] = {
    "pace_last_error": (c_char_p, []),
    "pace_status_string": (c_char_p, [c_int]),
    "pace_version": (c_int, []),
    "pace_set_pdl": (None, [c_int]),
    "pace_get_pdl": (c_int, []),
    "pace_rms_norm": (c_int, [_P, _P, _P, c_float, c_int64, c_int64, c_int64, c_int64, c_int, _P]),
    "pace_fused_add_rms_norm": (
        c_int,
        [_P, _P, _P, c_float, c_int64, c_int64, c_int64, c_int64, c_int, _P],
    ),
    "pace_rotary_embedding": (
        c_int,
        [_P, _P, _P, c_int64, c_int, c_int, c_int, c_int64, c_int64, _P, c_int, c_int, c_int64,
         c_int, c_int, _P],
    ),
    "pace_qkv_proj_rope": (
        c_int,
        [_P, _P, _P, _P, c_int64, c_int64, c_int, c_int, c_int, c_int64, c_int64, _P, c_int,
         c_int, c_int64, c_int, c_int, _P, c_size_t, _P, _P],
    ),
    "pace_qkv_proj_rope_workspace_size": (c_size_t, [c_int64, c_int64, c_int, c_int, c_int]),
    "pace_linear_residual_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int]),
    "pace_linear_residual": (
        c_int,
        [_P, _P, _P, _P, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, _P, c_size_t, _P,
         _P],
    ),
    "pace_row_sumsq": (c_int, [_P, _P, c_int64, c_int64, c_int64, c_int, _P]),
    "pace_qkv_proj_rmsnorm_rope": (
        c_int,
        [_P, _P, _P, _P, c_int64, c_float, _P, c_int64, c_int64, c_int, c_int, c_int, c_int64,
         c_int64, _P, c_int, c_int, c_int64, c_int, c_int, _P, c_size_t, _P, _P],
    ),
    "pace_gate_up_silu_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int]),
    "pace_gate_up_silu": (
        c_int,
        [_P, _P, _P, _P, c_int64, c_float, c_int64, c_int64, c_int64, c_int64, c_int64, c_int,
         _P, c_size_t, _P, _P],
    ),
    "pace_moe_gather_rows": (
        c_int, [_P, _P, _P, c_int64, _P, c_int64, c_int, c_int64, c_int64, c_int64, c_int, _P]),
    "pace_moe_gemm": (
        c_int,
        [_P, _P, _P, c_int64, _P, _P, _P, c_int64, _P, c_int, c_int64, c_int64, c_int64, c_int64,
         c_int, c_int, _P, _P],
    ),
    "pace_qkv_proj_rope_no_alloc": (
        c_int,
        [_P, _P, _P, _P, c_int64, c_int64, c_int, c_int, c_int, c_int64, c_int64, _P, c_int,
         c_int, c_int64, c_int, c_int, _P, _P],
    ),
    "pace_silu_and_mul": (c_int, _ACT),
    "pace_gelu_and_mul": (c_int, _ACT),
    "pace_gelu_tanh_and_mul": (c_int, _ACT),
    "pace_gelu_new": (c_int, _ACT),
    "pace_gelu_fast": (c_int, _ACT),
    "pace_topk_softmax": (c_int, [_P, _P, _P, _P, c_int64, c_int, c_int, c_int, _P]),
    "pace_moe_align_block_size": (
        c_int,
        [_P, c_int, c_int64, c_int, c_int, _P, c_int64, _P, c_int64, _P, c_int, _P],
    ),
    "pace_kv_copy_blocks": (
        c_int,
        [POINTER(c_void_p), POINTER(c_void_p), c_int, _P, _P, c_int64, c_int64, c_int64, c_int64,
         _P, c_int, _P],
    ),
    "pace_kv_copy_blocks_ex": (
        c_int,
        [POINTER(c_void_p), POINTER(c_void_p), c_int, _P, _P, c_int64, c_int64, c_int64, c_int64,
         _P, POINTER(KvCopyOpts), _P],
    ),
    "pace_kv_copy_blocks_ce": (
        c_int,
        [POINTER(c_void_p), POINTER(c_void_p), c_int, POINTER(c_int32), POINTER(c_int32), c_int64,
         c_int64, c_int64, c_int64, POINTER(c_int64), POINTER(c_int64), _P],
    ),
    "pace_kv_gather_blocks": (
        c_int,
        [POINTER(c_void_p), c_int, _P, c_int64, c_int64, c_int64, _P, _P, _P],
    ),
    "pace_kv_scatter_blocks": (
        c_int,
        [_P, POINTER(c_void_p), c_int, _P, c_int64, c_int64, c_int64, _P, _P],
    ),
    "pace_append_paged_kv_cache": (
        c_int,
        [_P, _P, c_int64, c_int, c_int, c_int64, c_int64, _P, _P, _P, c_int64, c_int, _P, c_int64,
         _P, _P, c_int64, _P, c_int, _P],
    ),
    "pace_append_paged_kv_cache_by_indptr": (
        c_int,
        [_P, _P, c_int64, c_int, c_int, c_int64, c_int64, _P, _P, c_int64, c_int, _P, c_int64, _P,
         _P, c_int64, _P, c_int, _P],
    ),
    "pace_enable_peer_access": (c_int, [c_int, c_int]),
    "pace_can_access_peer": (c_int, [c_int, c_int, POINTER(c_int)]),
    "pace_ipc_get_handle": (c_int, [_P, c_void_p, POINTER(c_int64)]),
    "pace_ipc_open_handle": (c_int, [c_void_p, c_int, POINTER(c_void_p)]),
    "pace_ipc_close_handle": (c_int, [_P]),
}


class PaceError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


_lib = None


def load(path: str = LIBRARY_PATH) -> ctypes.CDLL:
    """Load the library and declare every entry point's signature."""
    global _lib
    if _lib is not None and path == LIBRARY_PATH:
        return _lib
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path == LIBRARY_PATH:
        _lib = lib
    return lib


def check(status: int) -> None:
    """Raise PaceError with the library's message for a non-zero status."""
    if status != PACE_OK:
        msg = load().pace_last_error()
        raise PaceError(status, msg.decode() if msg else "")


def layer_table(ptrs) -> ctypes.Array:
    """A host array of device pointers for the KV entry points."""
    arr = (c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = c_void_p(int(p))
    return arr
