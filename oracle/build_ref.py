"""Build the reference's own CUDA ops from their sources, for use as a GPU oracle.

Test infrastructure only: nothing in the product imports this file or its
outputs.  The four reference torch extensions (``layernorm_ops``,
``pos_encoding_ops``, ``activation_ops``, ``moe_ops``; reference
``setup.py:98-134``) are compiled from the ``.cpp``/``.cu`` files where they
lie in the reference checkout, with the reference's own nvcc flags
(``setup.py:15-21``: ``-O2 -std=c++17 -D_GLIBCXX_USE_CXX11_ABI``) plus the
sm_100a target, into ``oracle/_ref/<name>/<name>.so``.  The reference's build
system (its ``setup.py``) is not run; ``torch.utils.cpp_extension.load`` only
drives nvcc/g++ with torch's include paths, which is how torch's
``BuildExtension`` would have compiled these files.

The resulting ``.so`` files are git-ignored but travel to the GPU box, where
``load_ref_ops`` imports them without the reference sources being present.

Usage: ``python oracle/build_ref.py [reference_root]`` (default: the
``PACE_REFERENCE_ROOT`` environment variable, else a ``reference`` checkout
beside this repository).  Skips modules whose ``.so`` is newer than its sources.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
DEFAULT_REF_ROOT = os.environ.get(
    "PACE_REFERENCE_ROOT",
    os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

# module name -> reference source files (paths relative to the reference root)
REF_MODULES = {
    "layernorm_ops": ["csrc/layernorm.cpp", "csrc/layernorm_kernels.cu"],
    "pos_encoding_ops": ["csrc/pos_encoding.cpp", "csrc/pos_encoding_kernels.cu"],
    "activation_ops": ["csrc/activation.cpp", "csrc/activation_kernels.cu"],
    "moe_ops": [
        "csrc/moe.cpp",
        "csrc/moe_align_block_size_kernels.cu",
        "csrc/moe_topk_softmax_kernels.cu",
    ],
}


def so_path(name: str) -> str:
    return os.path.join(REF_OUT, name, f"{name}.so")


def _build_one(name: str, ref_root: str, verbose: bool) -> str:
    from torch.utils import cpp_extension

    srcs = [os.path.join(ref_root, s) for s in REF_MODULES[name]]
    out = so_path(name)
    if os.path.exists(out) and all(os.path.getmtime(out) >= os.path.getmtime(s) for s in srcs):
        return out
    bdir = os.path.join(REF_OUT, name)
    os.makedirs(bdir, exist_ok=True)
    # The reference's NVCC_FLAGS (setup.py:15-21) with sm_100a as the target.
    nvcc = [
        "-O2",
        "-std=c++17",
        "-D_GLIBCXX_USE_CXX11_ABI=1",
        "-gencode",
        "arch=compute_100a,code=sm_100a",
    ]
    cpp_extension.load(
        name=name,
        sources=srcs,
        extra_cflags=["-O2", "-std=c++17", "-D_GLIBCXX_USE_CXX11_ABI=1"],
        extra_cuda_cflags=nvcc,
        extra_include_paths=[os.path.join(ref_root, "csrc")],
        build_directory=bdir,
        verbose=verbose,
        with_cuda=True,
        is_python_module=True,
    )
    return out


def build(ref_root: str = DEFAULT_REF_ROOT, verbose: bool = False, jobs: int = 4) -> list[str]:
    """Compile every reference module missing or stale under ``oracle/_ref``."""
    if not os.path.isdir(os.path.join(ref_root, "csrc")):
        return []
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    # a host compiler that links libstdc++ dynamically (a static copy inside
    # an extension breaks c10's std::ostream-based error messages)
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"
    os.environ.setdefault("MAX_JOBS", "4")
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(_build_one, n, ref_root, verbose) for n in REF_MODULES]
        return [f.result() for f in futs]


def load_ref_ops(name: str):
    """Import a prebuilt reference module from ``oracle/_ref`` (None if absent)."""
    path = so_path(name)
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (provides the c10/ATen symbols the module needs)

    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF_ROOT
    for p in build(root, verbose=True):
        print("built", p)
