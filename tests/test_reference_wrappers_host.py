"""CPU: PaceServe's own layer wrappers bind to this package's shim, unchanged.

Needs the reference checkout (argument-free: ``PACE_REFERENCE_ROOT`` or a
``reference`` directory beside this repository); skipped without it.  Each
check runs in a child process, because it installs ``paceserve.*`` modules.

* binding: with ``install_as_paceserve()`` in place, the wrapper files load
  by path and every wrapper call reaches the shim's own argument checks (on
  this GPU-less machine: "must be a CUDA tensor") -- a signature or module
  mismatch would fail earlier with ImportError/TypeError instead;
* fixture: recording the wrappers' op calls again reproduces the committed
  tests/golden/wrapper_calls.* that the GPU replay test uses.
"""
import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GEN = os.path.join(ROOT, "tests", "golden", "make_wrapper_golden.py")


def _ref_root():
    env = os.environ.get("PACE_REFERENCE_ROOT")
    return env or os.path.join(os.path.dirname(ROOT), "reference")


needs_ref = pytest.mark.skipif(
    not os.path.isdir(os.path.join(_ref_root(), "paceserve", "model_executor", "layers")),
    reason="reference checkout not present")

BIND = textwrap.dedent("""
    import importlib.util, sys, torch
    sys.path.insert(0, {root!r})
    spec = importlib.util.spec_from_file_location("mwg", {gen!r})
    mwg = importlib.util.module_from_spec(spec); spec.loader.exec_module(mwg)
    import paceserve_b200 as pb
    pb.install_as_paceserve()
    import paceserve
    assert paceserve.layernorm_ops is pb.layernorm_ops
    mwg.install_stubs({{}})            # only the timer stand-in; ops stay the shim's
    w = mwg.load_wrappers({ref!r})
    calls = []
    def expect_shim(name, fn):
        try:
            fn()
        except RuntimeError as e:
            assert "must be a CUDA tensor" in str(e), (name, str(e))
            calls.append(name)
            return
        raise AssertionError(name + ": reached no shim check")
    g = torch.Generator().manual_seed(0)
    with mwg.CudaOnCpu():
        with mwg.default_dtype(torch.bfloat16):
            norm = w["ref_layernorm"].RMSNorm(64, eps=1e-5)
            rope = w["ref_rotary_embedding"].get_rope(128, 128, 256, 500000, True,
                                                       mwg.LLAMA3_SCALING, torch.bfloat16)
        x = torch.randn(3, 64, generator=g).bfloat16()
        expect_shim("rms_norm", lambda: norm(x))
        expect_shim("silu_and_mul", lambda: w["ref_activation"].SiluAndMul()(torch.randn(3, 8).bfloat16()))
        expect_shim("gelu_new", lambda: w["ref_activation"].NewGELU()(torch.randn(3, 8).half()))
        expect_shim("gelu_fast", lambda: w["ref_activation"].FastGELU()(torch.randn(3, 8).half()))
        qkv = torch.randn(2, 4 * 128).bfloat16()
        q, k, _ = qkv.split([2 * 128, 128, 128], dim=-1)
        expect_shim("rotary_embedding", lambda: rope(torch.tensor([0, 5]), q, k))
        expect_shim("topk_softmax", lambda: w["ref_fused_moe"].fused_topk(
            torch.randn(4, 16).bfloat16(), torch.randn(4, 8).bfloat16(), 2, True))
        expect_shim("moe_align_block_size", lambda: w["ref_fused_moe"].moe_align_block_size(
            torch.randint(0, 8, (4, 2), dtype=torch.int32), 16, 8))
    print("bound:", ",".join(calls))
""")


def _run(code: str):
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT,
                          timeout=600)


@needs_ref
def test_reference_wrappers_bind_to_the_shim():
    r = _run(BIND.format(root=ROOT, gen=GEN, ref=_ref_root()))
    assert r.returncode == 0, r.stdout + r.stderr
    assert ("bound: rms_norm,silu_and_mul,gelu_new,gelu_fast,rotary_embedding,topk_softmax,"
            "moe_align_block_size") in r.stdout


@needs_ref
def test_committed_wrapper_fixture_matches_the_reference():
    r = subprocess.run([sys.executable, GEN, _ref_root(), "--check"], capture_output=True,
                       text=True, cwd=ROOT, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
