"""NVFP4 quantisation on the GPU (the step before the GEMM).

``quantize(x)`` turns real-valued activations or weights into exactly the tensors the
GEMM entry points take: packed e2m1 codes, plain e4m3 block scales and the same scales
in the permuted layout.  The quantisation rule is the one the benchmark configurations
specify for their inputs (fp32 values -> per-16-element amax / 6 -> e4m3 scale -> nearest
e2m1 code, ties to even; restated on the host by ``inputs.quantize_nvfp4``, which this
kernel matches bit for bit).  The reference itself draws random codes and small integer
scales instead of quantising values; from it comes only the permuted scale layout
(``to_blocked``, kernels/gemm/reference.py:13-24 and :113-150).
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


def _main():
    """Time the quantiser: python -m nvfp4_hackathon_b200.quantize --rows 8192 --k 8192."""
    import argparse
    import json

    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--dtype", default="bf16", choices=["f32", "f16", "bf16"])
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--graph", action="store_true", help="time the calls replayed from a CUDA graph")
    args = ap.parse_args()
    dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[args.dtype]
    # three inputs so consecutive calls do not find their input in L2
    xs = [torch.randn((args.rows, args.k), device="cuda", dtype=dt) for _ in range(3)]
    for x in xs:
        quantize(x, plain=False)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    if args.graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(args.reps):
                quantize(xs[i % 3], plain=False)
        g.replay()
        torch.cuda.synchronize()
        ev[0].record()
        g.replay()
        ev[1].record()
    else:
        ev[0].record()
        for i in range(args.reps):
            quantize(xs[i % 3], plain=False)
        ev[1].record()
    torch.cuda.synchronize()
    us = ev[0].elapsed_time(ev[1]) * 1e3 / args.reps
    nbytes = args.rows * args.k * (xs[0].element_size() + 0.5 + 1.0 / 16)
    print(json.dumps({"rows": args.rows, "k": args.k, "dtype": args.dtype, "graph": args.graph,
                      "us_per_call": round(us, 2),
                      "gb_per_s": round(nbytes / us / 1e3, 1)}))


if __name__ == "__main__":
    _main()
