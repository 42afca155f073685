"""Generate tests/golden/scaled_mm_golden.npz on a B200.

The reference's numerical path is ``ref_kernel`` (kernels/gemm/reference.py:27-53):
for each batch, torch._scaled_mm(A, B^T, to_blocked(SFA), to_blocked(SFB),
out_dtype=float16) over float4_e2m1fn_x2 codes and float8_e4m3fn scales.  This
script makes exactly that call on seeded inputs created on the host (numpy), so
the fixtures pin the CPU oracle to the reference's own arithmetic (cuBLASLt
block-scaled GEMM) without a GPU at test time.

    python tests/golden/make_scaled_mm_golden.py [OUT.npz]
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CASES = [(128, 256, 256), (256, 128, 512), (128, 384, 1024)]


def to_blocked(m: np.ndarray) -> np.ndarray:
    """128x4 blocked layout of a (rows, cols) scale matrix, rows % 128 == 0, cols % 4 == 0."""
    r, c = m.shape
    return m.reshape(r // 128, 128, c // 4, 4).transpose(0, 2, 1, 3).reshape(-1, 4, 32, 4) \
        .transpose(0, 2, 1, 3).reshape(-1)


def main():
    out_path = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "scaled_mm_golden.npz")
    rng = np.random.default_rng(1111)
    out = {}
    for i, (m, n, k) in enumerate(CASES):
        a = rng.integers(0, 256, size=(m, k // 2), dtype=np.uint8)
        b = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
        # scales: the reference's generator draws e4m3 integers 0..3 (kernels/gemm/reference.py:108)
        sfa = torch.from_numpy(rng.integers(0, 4, size=(m, k // 16)).astype(np.float32)).to(torch.float8_e4m3fn)
        sfb = torch.from_numpy(rng.integers(0, 4, size=(n, k // 16)).astype(np.float32)).to(torch.float8_e4m3fn)
        sfa_u8, sfb_u8 = sfa.view(torch.uint8).numpy(), sfb.view(torch.uint8).numpy()
        A = torch.from_numpy(a).cuda().view(torch.float4_e2m1fn_x2)
        B = torch.from_numpy(b).cuda().view(torch.float4_e2m1fn_x2)
        sa = torch.from_numpy(to_blocked(sfa_u8)).cuda().view(torch.float8_e4m3fn)
        sb = torch.from_numpy(to_blocked(sfb_u8)).cuda().view(torch.float8_e4m3fn)
        c = torch._scaled_mm(A, B.transpose(0, 1), sa, sb, bias=None, out_dtype=torch.float16)
        out[f"a_{i}"], out[f"b_{i}"] = a, b
        out[f"sfa_{i}"], out[f"sfb_{i}"] = sfa_u8, sfb_u8
        out[f"c_{i}"] = c.cpu().numpy()
    out["torch_version"] = np.array(torch.__version__)
    out["device"] = np.array(torch.cuda.get_device_name(0))
    np.savez_compressed(out_path, **out)
    print("wrote", out_path)


if __name__ == "__main__":
    main()
