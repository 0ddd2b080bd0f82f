"""Build recipe for the package's native code (in-tree, sm_100a only).

Outputs, next to this file:
  * ``libpace_b200.so`` -- the C-ABI library (every kernel, ``include/pace_b200.h``),
    compiled with nvcc for ``sm_100a`` and linked against the static CUDA runtime;
  * ``_C.so`` -- the torch extension (pybind modules layernorm_ops, pos_encoding_ops,
    activation_ops, moe_ops, kv_transfer_ops) that validates tensors and calls
    the C ABI; it links ``libpace_b200.so`` through ``$ORIGIN``.

Objects go to ``<repo>/_build``.  Steps whose outputs are newer than every
input are skipped.  Run ``python paceserve_b200/build.py`` (or
``__graft_entry__.build()``); the package itself cannot be imported before
the extension exists.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libpace_b200.so")
EXT = os.path.join(PKG, "_C.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CCBIN = ["-ccbin", "/usr/bin/g++"] if os.path.exists("/usr/bin/g++") else []
NVCC_FLAGS = ARCH + CCBIN + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-I" + INCLUDE,
]
CUDA_SOURCES = [
    "status.cu",
    "layernorm_kernels.cu",
    "pos_encoding_kernels.cu",
    "activation_kernels.cu",
    "moe_kernels.cu",
    "kv_transfer_kernels.cu",
    "kv_append_kernels.cu",
    "gemm_rope_kernels.cu",
    "moe_gemm_kernels.cu",
]


def _newer(out: str, inputs: list[str]) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(i) <= t for i in inputs)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def host_cxx() -> str:
    """A C++ compiler that links libstdc++ as a shared library.  A private static
    copy inside the extension would meet torch's shared copy in the same
    std::ostream (c10 error messages) and crash on an uninitialised locale."""
    for cand in ("/usr/bin/g++", os.environ.get("CXX", ""), "g++"):
        if not cand or (os.path.isabs(cand) and not os.path.exists(cand)):
            continue
        probe = subprocess.run([cand, "-print-file-name=libstdc++.so"], capture_output=True, text=True)
        if probe.returncode == 0 and os.path.isabs(probe.stdout.strip()):
            return cand
    raise RuntimeError("no C++ compiler with a shared libstdc++ found")


def check_dynamic_libstdcxx(so: str) -> None:
    out = subprocess.run(["readelf", "-d", so], capture_output=True, text=True).stdout
    if "libstdc++.so" not in out:
        raise RuntimeError(f"{so} does not link libstdc++ dynamically")


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def build_library(verbose: bool = False, jobs: int = 6) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = _headers()
    objs = []
    todo = []
    for src in CUDA_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if not _newer(o, [s] + hdrs):
            todo.append([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o])
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(lambda c: _run(c, verbose), todo))
    if not _newer(LIB, objs):
        _run([NVCC] + ARCH + CCBIN + ["-shared", "-cudart", "static", "-o", LIB] + objs, verbose)
        check_dynamic_libstdcxx(LIB)
    return LIB


def build_extension(verbose: bool = False) -> str:
    import torch  # noqa: F401
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "torch_shim.cpp")
    if _newer(EXT, [src, LIB] + _headers()):
        return EXT
    torch_lib = os.path.join(os.path.dirname(cpp_extension.__file__), "..", "lib")
    torch_lib = os.path.abspath(torch_lib)
    incs = cpp_extension.include_paths(device_type="cuda")
    py_inc = sysconfig.get_paths()["include"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cxx = host_cxx()
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", src, "-o", EXT]
    cmd += ["-I" + INCLUDE, "-I" + py_inc] + ["-isystem" + i for i in incs]
    cmd += [
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=_C",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        "-L" + PKG,
        "-lpace_b200",
        "-Wl,-rpath,$ORIGIN",
        "-L" + torch_lib,
        "-Wl,-rpath," + torch_lib,
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-ltorch_python",
    ]
    _run(cmd, verbose)
    check_dynamic_libstdcxx(EXT)
    return EXT


def build(verbose: bool = False) -> None:
    build_library(verbose)
    build_extension(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
    print(EXT)
