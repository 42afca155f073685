"""Register budget of the GEMM kernels, checked at compile time (no GPU needed).

The 20-warp block gets at most 96 registers per thread. A change to the epilogue that keeps
the packed accumulator tile live across a loop back-edge once pushed every plain
instantiation into local memory (up to 1.7 KB of spills per thread) and cost 10-130 % in
run time without changing any result, so only a compile-time check sees it. The plain
schedule (SK = false, fp16/bf16 or fp32 C) and the quantiser must not spill; the opt-in
stream-K instantiations are allowed to.
"""
import os
import re
import shutil
import subprocess

import pytest

from nvfp4_hackathon_b200.csrc import build as nbuild


def _ptxas_report(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    src = os.path.join(nbuild.HERE, "nvfp4_capi.cu")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-c",
           "-Xptxas", "-v", "-o", str(tmp_path / "capi.o"), src]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out, cur, spill = [], None, None
    for line in r.stderr.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            cur = m.group(1)
        m = re.search(r"(\d+) bytes spill stores", line)
        if m and cur:
            spill = int(m.group(1))
        m = re.search(r"Used (\d+) registers", line)
        if m and cur:
            out.append((cur, int(m.group(1)), spill))
            cur = None
    return out


def test_plain_kernels_do_not_spill(tmp_path):
    report = _ptxas_report(tmp_path)
    gemms = [r for r in report if "nvfp4_gemm_kernel" in r[0]]
    assert gemms, "no GEMM instantiation found in the ptxas report"
    # mangled template arguments end in ...ELb<CTA2>ELb<SK>ELb<F32>EEEv
    plain = [r for r in gemms if re.search(r"ELb[01]ELb0ELb[01]EEEv", r[0])]
    assert plain
    bad = [r for r in plain + [r for r in report if "quantize" in r[0]] if r[2] != 0]
    assert not bad, "spilling instantiations: " + "; ".join(f"{n[-48:]} {g} regs {s} B" for n, g, s in bad)
    assert all(g <= 96 for _, g, _ in gemms)
