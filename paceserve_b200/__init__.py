"""B200-native (sm_100a) implementation of PaceServe's per-layer op hot path
and its paged-KV transfer.

The ops are exposed as the same pybind modules, with the same signatures, as
PaceServe's ``csrc`` extensions (``paceserve.layernorm_ops`` ...), so the
unchanged engine can import them in their place (``install_as_paceserve()``):

    from paceserve_b200 import layernorm_ops, pos_encoding_ops, activation_ops, moe_ops
    layernorm_ops.rms_norm(out, x, weight, eps)

Every op launches a hand-written CUDA kernel through the C ABI in
``libpace_b200.so`` (``include/pace_b200.h``).  There is no fallback: importing
this package fails if the native library is missing, and every op raises
``RuntimeError`` for tensors it cannot run on the GPU.
"""
from __future__ import annotations

import os
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))

try:
    import torch  # noqa: F401  (loads libc10/libtorch that _C links against)

    from . import _C  # type: ignore[attr-defined]
except ImportError as exc:  # pragma: no cover - exercised only on a broken install
    raise ImportError(
        "paceserve_b200: the native extension is not built "
        f"({exc}); run `python paceserve_b200/build.py`"
    ) from exc

layernorm_ops = _C.layernorm_ops
pos_encoding_ops = _C.pos_encoding_ops
activation_ops = _C.activation_ops
moe_ops = _C.moe_ops
kv_transfer_ops = _C.kv_transfer_ops

for _name in ("layernorm_ops", "pos_encoding_ops", "activation_ops", "moe_ops", "kv_transfer_ops"):
    sys.modules[f"{__name__}.{_name}"] = getattr(_C, _name)

LIBRARY_PATH = os.path.join(_HERE, "libpace_b200.so")


def set_pdl(enabled: bool) -> None:
    """Programmatic dependent launch for the per-layer ops (default on)."""
    _C.set_pdl(bool(enabled))


def get_pdl() -> bool:
    return bool(_C.get_pdl())


def fold_rmsnorm_weight(linear_weight, norm_weight):
    """The projection weight with an RMSNorm weight folded into its input
    columns, W'[n, c] = W[n, c] * w[c] (rounded to W's dtype), for the GEMMs
    that apply the norm as a per-row factor in their epilogue
    (``pos_encoding_ops.qkv_proj_rmsnorm_rotary_embedding``).  Prepared once per
    model load."""
    return (linear_weight.float() * norm_weight.float()[None, :]).to(linear_weight.dtype).contiguous()


def install_as_paceserve() -> None:
    """Register these modules as ``paceserve.{layernorm,pos_encoding,activation,moe}_ops``.

    PaceServe's layer wrappers import the ops with ``from paceserve import
    layernorm_ops`` (model_executor/layers/layernorm.py:8, activation.py:6,
    rotary_embedding.py:30, fused_moe/fused_moe.py:12).  Calling this before the
    engine imports its layers makes those imports resolve to this package.
    """
    import importlib
    import types

    try:
        pkg = importlib.import_module("paceserve")
    except ImportError:
        pkg = types.ModuleType("paceserve")
        pkg.__path__ = []  # type: ignore[attr-defined]
        sys.modules["paceserve"] = pkg
    for name in ("layernorm_ops", "pos_encoding_ops", "activation_ops", "moe_ops", "kv_transfer_ops"):
        mod = getattr(_C, name)
        sys.modules[f"paceserve.{name}"] = mod
        setattr(pkg, name, mod)


__all__ = [
    "layernorm_ops",
    "pos_encoding_ops",
    "activation_ops",
    "moe_ops",
    "kv_transfer_ops",
    "install_as_paceserve",
    "fold_rmsnorm_weight",
    "set_pdl",
    "get_pdl",
    "LIBRARY_PATH",
]
