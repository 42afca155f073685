"""The C-ABI library loads without a GPU and exports every declared symbol."""
import os
import re

from nvfp4_hackathon_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "nvfp4_b200.h")).read()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(nvfp4_\w+)\(", src, flags=re.M)))


def test_header_matches_loader_list():
    assert declared_symbols() == sorted(_native.EXPORTED)


def test_library_loads_and_exports():
    lib = _native.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.nvfp4_abi_version() == 2


def test_workspace_size_is_host_only():
    lib = _native.load()
    assert lib.nvfp4_grouped_gemm_workspace_size(0) == 0
    assert lib.nvfp4_grouped_gemm_workspace_size(64) >= 64 * 2 * 128 + 65 * 4
    assert lib.nvfp4_grouped_gemm_workspace_size(2000) == 0
