"""Fused epilogue of the dense GEMM (bias per output column, relu / gelu, fp16, bf16 or fp32 C)
against the oracle's float64 product with the same epilogue applied before rounding."""
import math

import numpy as np
import pytest
import torch

from nvfp4_hackathon_b200 import _native, gemm, inputs
from oracle import nvfp4_oracle as orc
from tests.helpers import u8

pytestmark = pytest.mark.gpu


def _exact(data):
    """float64 (l, m, n) of dequant(A) @ dequant(B)^T (no rounding)."""
    a, b, sfa, sfb = data[:4]
    da = orc.dequant(u8(a.permute(2, 0, 1).contiguous()), u8(sfa.cpu().contiguous()))
    db = orc.dequant(u8(b.permute(2, 0, 1).contiguous()), u8(sfb.cpu().contiguous()))
    return np.matmul(da, np.swapaxes(db, -1, -2))


def _act(x, name):
    if name == "relu":
        return np.maximum(x, 0.0)
    if name == "gelu":
        erf = np.vectorize(math.erf)
        return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))
    return x


@pytest.mark.parametrize("m,n,k,l", [(64, 384, 1024, 1), (256, 640, 512, 2), (128, 1536, 7168, 1)])
@pytest.mark.parametrize("activation", [None, "relu", "gelu"])
@pytest.mark.parametrize("out", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("with_bias", [False, True])
def test_fused_epilogue(cuda, m, n, k, l, activation, out, with_bias):
    data = list(inputs.generate_input(m, n, k, l, seed=21))
    data[6] = torch.zeros((l, m, n), device="cuda", dtype=out).permute(1, 2, 0)
    g = torch.Generator(device="cuda").manual_seed(5)
    bias = (torch.randn(n, generator=g, device="cuda") * 4) if with_bias else None
    c = gemm.fused(tuple(data), bias=bias, activation=activation)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    exp = _exact(data)
    if bias is not None:
        exp = exp + bias.double().cpu().numpy()[None, None, :]
    exp = torch.from_numpy(_act(exp, activation)).to(out).double().numpy()
    got = c.permute(2, 0, 1).double().cpu().numpy()
    tol = 8e-3 if out == torch.bfloat16 else 1e-3  # one ulp of bf16; the reference checker's 1e-3 otherwise
    bad = np.abs(got - exp) > tol + tol * np.abs(exp)
    assert not bad.any(), f"{bad.sum()} mismatches, max err {np.abs(got - exp).max()}"


def test_bf16_output_through_custom_kernel(cuda):
    data = list(inputs.generate_input(128, 256, 512, 1, seed=2))
    data[6] = torch.zeros((1, 128, 256), device="cuda", dtype=torch.bfloat16).permute(1, 2, 0)
    c = gemm.custom_kernel(tuple(data))
    torch.cuda.synchronize()
    exp = torch.from_numpy(_exact(data)).to(torch.bfloat16).double().numpy()
    got = c.permute(2, 0, 1).double().cpu().numpy()
    assert np.allclose(got, exp, rtol=8e-3, atol=8e-3)


def test_grouped_rejects_fused_options(cuda):
    lib = _native.load()
    opt = _native.options(activation=1)
    import ctypes
    rc = lib.nvfp4_grouped_gemm_ex(16, 16, 16, 1, 16, 1 << 20, None, ctypes.byref(opt))
    assert rc == 3  # NVFP4_ERR_UNSUPPORTED


@pytest.mark.parametrize("m,n,k,l", [(64, 384, 1024, 1), (200, 520, 512, 2), (300, 2304, 2048, 1)])
def test_fp32_output_through_custom_kernel(cuda, m, n, k, l):
    """fp32 C: every tile config (swap for M <= 128, 256-wide tiles for N >= 2048), ragged
    edges, batches; compared with the exact product at the reference checker's tolerance."""
    data = list(inputs.generate_input(m, n, k, l, seed=4))
    data[6] = torch.full((l, m, n), float("nan"), device="cuda", dtype=torch.float32).permute(1, 2, 0)
    c = gemm.custom_kernel(tuple(data))
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    exp = _exact(data)
    got = c.permute(2, 0, 1).double().cpu().numpy()
    assert np.isfinite(got).all()
    assert np.allclose(got, exp, rtol=1e-3, atol=1e-3)
    # fp32 keeps what fp16 rounds away
    assert np.abs(got - exp).max() < np.abs(exp.astype(np.float16).astype(np.float64) - exp).max()


def test_fp32_output_rejects_stream_k(cuda):
    data = list(inputs.generate_input(128, 256, 512, 1, seed=2))
    data[6] = torch.zeros((1, 128, 256), device="cuda", dtype=torch.float32).permute(1, 2, 0)
    with pytest.raises(RuntimeError):
        gemm.custom_kernel(tuple(data), opt=_native.options(out_dtype=2, stream_k=2))
