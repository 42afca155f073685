"""Generate tests/golden/reference_fixtures.npz with the reference's OWN input
generators and numerical path, on a B200.

It imports ``generate_input`` and ``ref_kernel`` from the reference's
kernels/gemm/reference.py (:56-158, :27-53) and kernels/group_gemm/reference.py
(:137-201, :39-74), runs them on the reference's own test cases
(kernels/gemm/run_tests.py:13-24, kernels/group_gemm/profile_group_gemm.py:76-83)
with their seed, and saves the exact input bytes and the ``ref_kernel`` output
(torch._scaled_mm, cuBLASLt).  Only the cases whose tensors are small enough for a
committed fixture are kept (every grouped test case; the dense 128 x 256 x 256 case).

    python tests/golden/make_reference_fixtures.py REF [OUT]

REF is the root of a copy of the reference (the directory holding ``kernels/``), e.g.
the pip install target of the reference; it needs a GPU (the generators allocate on
cuda) and the reference's ``utils.py``.
"""
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

DENSE_CASES = [(128, 256, 256, 1, 1111)]          # kernels/gemm/run_tests.py:14
GROUP_CASES = [                                    # kernels/group_gemm/profile_group_gemm.py:76-81
    ([96, 128], [128, 256], [256, 512], 2, 1111),
    ([256, 72], [512, 384], [256, 256], 2, 1111),
    ([128, 128], [128, 256], [512, 256], 2, 1111),
    ([80, 128, 256], [384, 256, 128], [256, 512, 256], 3, 1111),
]


def load(path, name):
    """Import one of the reference's task modules with its directory first on sys.path
    (they import ``task`` and ``utils`` by bare name)."""
    d = os.path.dirname(path)
    for m in ("task", "utils", "reference"):
        sys.modules.pop(m, None)
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


def u8(t):
    return t.contiguous().view(torch.uint8).cpu().numpy() if t.dtype != torch.uint8 else t.cpu().numpy()


def storage_u8(t):
    """All bytes of a tensor's storage, in storage order (the permuted scales are views)."""
    s = t.untyped_storage()
    return torch.empty(0, dtype=torch.uint8, device=t.device).set_(s, 0, (s.nbytes(),), (1,)).cpu().numpy()


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NVFP4_REF_ROOT")
    if not ref:
        sys.exit("usage: make_reference_fixtures.py REF [OUT]")
    out_path = sys.argv[2] if len(sys.argv) > 2 else os.path.join(HERE, "reference_fixtures.npz")
    gemm_ref = load(os.path.join(ref, "kernels/gemm/reference.py"), "ref_gemm_reference")
    out = {}
    for i, (m, n, k, l, seed) in enumerate(DENSE_CASES):
        data = gemm_ref.generate_input(m=m, n=n, k=k, l=l, seed=seed)
        a, b, sfa, sfb, sfa_p, sfb_p, c = data
        out[f"dense{i}_mnkl"] = np.array([m, n, k, l])
        # a, b: (m, k/2, l) views of (l, m, k/2) storage; stored as (l, m, k/2) bytes
        out[f"dense{i}_a"] = u8(a.view(torch.uint8).permute(2, 0, 1))
        out[f"dense{i}_b"] = u8(b.view(torch.uint8).permute(2, 0, 1))
        out[f"dense{i}_sfa"] = u8(sfa.view(torch.uint8))  # (m, k/16, l) plain
        out[f"dense{i}_sfb"] = u8(sfb.view(torch.uint8))
        out[f"dense{i}_sfa_perm"] = storage_u8(sfa_p)  # (l, rm, rk, 32, 4, 4) storage bytes
        out[f"dense{i}_sfb_perm"] = storage_u8(sfb_p)
        res = gemm_ref.ref_kernel(data)
        torch.cuda.synchronize()
        out[f"dense{i}_c_ref"] = res.permute(2, 0, 1).contiguous().cpu().numpy()  # (l, m, n) fp16
    group_ref = load(os.path.join(ref, "kernels/group_gemm/reference.py"), "ref_group_reference")
    for i, (ms, ns, ks, g, seed) in enumerate(GROUP_CASES):
        data = group_ref.generate_input(m=ms, n=ns, k=ks, g=g, seed=seed)
        abc, sf, sfp, sizes = data
        out[f"group{i}_sizes"] = np.array(sizes)
        for j, ((a, b, c), (sa, sb), (pa, pb)) in enumerate(zip(abc, sf, sfp)):
            out[f"group{i}_{j}_a"] = u8(a.view(torch.uint8)[:, :, 0])
            out[f"group{i}_{j}_b"] = u8(b.view(torch.uint8)[:, :, 0])
            out[f"group{i}_{j}_sfa"] = u8(sa.view(torch.uint8)[:, :, 0])
            out[f"group{i}_{j}_sfb"] = u8(sb.view(torch.uint8)[:, :, 0])
            out[f"group{i}_{j}_sfa_perm"] = storage_u8(pa)
            out[f"group{i}_{j}_sfb_perm"] = storage_u8(pb)
        res = group_ref.ref_kernel(data)
        torch.cuda.synchronize()
        for j, c in enumerate(res):
            out[f"group{i}_{j}_c_ref"] = c[:, :, 0].contiguous().cpu().numpy()
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()
