"""Shared helpers for the tests (not a test module)."""
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Parity rule for float ops: max|got - ref| / max(max|ref|, 1e-6) <= REL_TOL
# against the fp32 reference formula (bf16/fp16 outputs).
REL_TOL = 1e-2


def rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    got = got.float().cpu()
    ref = ref.float().cpu()
    if ref.numel() == 0:
        return 0.0
    return ((got - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


def max_ulps(got: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype) -> float:
    """Largest difference in units of the storage type's epsilon at the reference's magnitude."""
    got = got.float().cpu()
    ref = ref.float().cpu()
    if ref.numel() == 0:
        return 0.0
    ulp = torch.finfo(dtype).eps * ref.abs().clamp_min(torch.finfo(dtype).tiny)
    return ((got - ref).abs() / ulp).max().item()


def assert_matches_rounded(got: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype,
                           min_equal: float = 0.98) -> None:
    """`ref` reproduces the kernel's rounding points (on the CPU, or the
    reference's own kernel).  exp/tanh/erf implementations may differ in the
    last fp32 ulps, which can flip a bf16/fp16 rounding, so require: almost
    all elements bit-equal, the rest within two storage-type ulps at the
    output's largest magnitude.  fp32 outputs: within 1e-5 of the largest
    magnitude (tanh-based formulas cancel near 1 + tanh(x) = 0, so per-element
    ulps can be large)."""
    if dtype == torch.float32:
        assert rel_err(got, ref) <= 1e-5
        return
    g, r = got.float().cpu(), ref.float().cpu()
    if r.numel() == 0:
        return
    frac = (g == r).float().mean().item()
    assert frac >= min_equal, f"only {frac:.4f} of elements bit-equal"
    assert rel_err(g, r) <= 2 * torch.finfo(dtype).eps


_REF_CACHE = {}


def ref_ops(name: str):
    """The reference's own CUDA module, built from its sources into oracle/_ref.

    On a machine with a CUDA GPU the module must load: a missing or broken
    build raises, so a GPU run can never pass with the comparisons against the
    reference silently skipped.  Without a GPU (where no GPU test runs) it
    returns None when the module is unavailable."""
    if name not in _REF_CACHE:
        from oracle.build_ref import load_ref_ops

        try:
            mod = load_ref_ops(name)
            err = None if mod is not None else "not built (oracle/_ref is missing it)"
        except Exception as exc:  # noqa: BLE001 - reported below with its cause
            mod, err = None, f"{type(exc).__name__}: {exc}"
        if mod is None and torch.cuda.is_available():
            raise RuntimeError(f"reference op module {name!r} cannot be loaded: {err}; "
                               "build it with `python oracle/build_ref.py <reference root>`")
        _REF_CACHE[name] = mod
    return _REF_CACHE[name]
