"""The C ABI from a plain C caller (tests/c_harness/nvfp4_c_check.c): it compiles as C99
against include/nvfp4_b200.h and links against the library on any machine; on a GPU it
runs the dense and grouped GEMMs and the argument-error checks against its own
double-precision restatement of the reference's math."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = "/usr/local/cuda"
PKG = os.path.join(ROOT, "nvfp4_hackathon_b200")


def _build(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None or not os.path.exists(os.path.join(CUDA, "include", "cuda_runtime_api.h")):
        pytest.skip("gcc or the CUDA runtime headers are not available")
    if not os.path.exists(os.path.join(PKG, "libnvfp4_b200.so")):
        pytest.skip("libnvfp4_b200.so is not built")
    exe = str(tmp_path / "nvfp4_c_check")
    cmd = [gcc, "-std=c99", "-O2", "-Wall", "-Wextra", "-Werror",
           os.path.join(ROOT, "tests", "c_harness", "nvfp4_c_check.c"),
           "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(CUDA, "include"),
           "-L" + PKG, "-lnvfp4_b200", "-L" + os.path.join(CUDA, "lib64"), "-lcudart", "-lm",
           "-Wl,-rpath," + PKG, "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c_caller_builds_and_links(tmp_path):
    _build(tmp_path)


@pytest.mark.gpu
def test_c_caller_runs(tmp_path, cuda):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("OK")
