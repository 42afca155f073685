"""Generate tests/golden/to_blocked_golden.npz from the reference's own code.

Run with REF, the root of a checkout of the reference (the directory holding
``kernels/``), as the argument or in the NVFP4_REF_ROOT environment variable; it
imports ``to_blocked`` from kernels/gemm/reference.py and
kernels/group_gemm/reference.py (pure torch, runs on the CPU) and records its
outputs on seeded random scale matrices, plus torch's float8_e4m3fn decode of
all 256 byte values (the dtype the reference's scales use).

    python tests/golden/make_layout_golden.py [REF]
"""
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load(path, name):
    d = os.path.dirname(path)
    sys.path.insert(0, d)
    try:
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        sys.path.remove(d)
        for m in ("task", "utils"):
            sys.modules.pop(m, None)
    return mod


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NVFP4_REF_ROOT")
    if not ref:
        sys.exit("usage: make_layout_golden.py REF (or set NVFP4_REF_ROOT)")
    gemm_ref = load(os.path.join(ref, "kernels/gemm/reference.py"), "ref_gemm_reference")
    group_ref = load(os.path.join(ref, "kernels/group_gemm/reference.py"), "ref_group_reference")
    rng = np.random.default_rng(2024)
    out = {}
    # gemm to_blocked: rows % 128 == 0, cols % 4 == 0 (kernels/gemm/reference.py:13-24)
    for i, (r, c) in enumerate([(128, 4), (256, 32), (384, 112)]):
        m = rng.integers(0, 256, size=(r, c), dtype=np.uint8)
        out[f"gemm_in_{i}"] = m
        out[f"gemm_out_{i}"] = gemm_ref.to_blocked(torch.from_numpy(m)).numpy()
    # group to_blocked pads ragged shapes with zeros (kernels/group_gemm/reference.py:14-36)
    for i, (r, c) in enumerate([(72, 16), (130, 6), (256, 448)]):
        m = rng.integers(0, 256, size=(r, c), dtype=np.uint8)
        out[f"group_in_{i}"] = m
        out[f"group_out_{i}"] = group_ref.to_blocked(torch.from_numpy(m)).numpy()
    out["e4m3_values"] = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    np.savez_compressed(os.path.join(HERE, "to_blocked_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "to_blocked_golden.npz"))


if __name__ == "__main__":
    main()
