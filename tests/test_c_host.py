"""The C ABI from a plain C host: tests/c_host/abi_check.c is compiled with gcc
against include/pace_b200.h and linked with libpace_b200.so, as a C or C++
integration would do."""
import os
import shutil
import subprocess

import pytest

from tests._util import ROOT

PKG = os.path.join(ROOT, "paceserve_b200")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    exe = str(tmp_path / "abi_check")
    cmd = [gcc, "-O2", "-std=c11", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "c_host", "abi_check.c"),
           "-L", PKG, "-lpace_b200", "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-lm",
           "-Wl,-rpath," + PKG, "-Wl,-rpath," + os.path.join(CUDA, "lib64"), "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_host_argument_errors(tmp_path):
    exe = build(tmp_path)
    r = subprocess.run([exe, "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "abi_check cpu ok" in r.stdout


@pytest.mark.gpu
def test_c_host_runs_kernels(tmp_path):
    exe = build(tmp_path)
    r = subprocess.run([exe, "gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "abi_check gpu ok" in r.stdout
