"""NVFP4 quantisation on the GPU (the step before the GEMM).

``quantize(x)`` turns real-valued activations or weights into exactly the tensors the
GEMM entry points take: packed e2m1 codes, plain e4m3 block scales and the same scales
in the permuted layout.  It is the reference's input generation
(kernels/gemm/reference.py:86-150 -- per-16-element amax / 6 -> e4m3 scale, nearest e2m1,
``to_blocked``) done by one HBM-bound kernel instead of a chain of torch ops; the
rounding rules are those of ``inputs.quantize_nvfp4``, bit for bit.
"""
from __future__ import annotations

import torch

from . import _native

_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def quantize(x: torch.Tensor, stream=None, plain: bool = True):
    """x: (rows, K) or (L, rows, K) CUDA tensor, fp32 / fp16 / bf16, K % 64 == 0.

    Returns ``(codes, sf, sf_perm)`` laid out like the reference's input tuple:
    codes (rows, K/2, L) float4_e2m1fn_x2, sf (rows, K/16, L) float8_e4m3fn (None when
    ``plain`` is False) and sf_perm (32, 4, ceil(rows/128), 4, K/64, L) float8_e4m3fn.
    """
    if x.dim() == 2:
        x = x.unsqueeze(0)
    if x.dim() != 3 or not x.is_cuda or x.dtype not in _DTYPES:
        raise ValueError("x must be a (rows, K) or (L, rows, K) fp32/fp16/bf16 CUDA tensor")
    l, rows, k = x.shape
    if k % 64:
        raise ValueError(f"K must be a multiple of 64 (got {k})")
    x = x.contiguous()
    rm, rk = (rows + 127) // 128, k // 64
    codes = torch.empty((l, rows, k // 2), dtype=torch.uint8, device=x.device)
    perm = torch.empty((l, rm, rk, 32, 4, 4), dtype=torch.uint8, device=x.device)
    flat = torch.empty((l, rows, k // 16), dtype=torch.uint8, device=x.device) if plain else None
    lib = _native.load()
    if stream is None:
        stream = torch.cuda.current_stream(x.device).cuda_stream
    rc = lib.nvfp4_quantize(x.data_ptr(), _DTYPES[x.dtype], rows, k, l, codes.data_ptr(),
                            perm.data_ptr(), flat.data_ptr() if plain else None, stream)
    _native.check(rc, "nvfp4_quantize")
    codes_v = codes.permute(1, 2, 0).view(torch.float4_e2m1fn_x2)
    sf_v = flat.view(torch.float8_e4m3fn).permute(1, 2, 0) if plain else None
    perm_v = perm.view(torch.float8_e4m3fn).permute(3, 4, 1, 5, 2, 0)
    return codes_v, sf_v, perm_v
