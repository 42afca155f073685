"""The CUDA quantiser (nvfp4_quantize) against the torch restatement of the reference's
input generation (inputs.quantize_nvfp4, kernels/gemm/reference.py:86-150): bit-exact
codes and scales, the permuted layout byte for byte, and a quantise -> GEMM round trip."""
import numpy as np
import pytest
import torch

from nvfp4_hackathon_b200 import gemm, inputs, layout
from nvfp4_hackathon_b200.quantize import quantize
from oracle import nvfp4_oracle as orc
from tests.helpers import assert_close, dense_expected, u8


def _reference(x3):
    """Per batch: torch quantiser -> (codes (l, rows, K/2), plain (l, rows, K/16), permuted)."""
    codes, scales = [], []
    for b in range(x3.shape[0]):
        c, s = inputs.quantize_nvfp4(x3[b].float())
        codes.append(c)
        scales.append(s)
    codes = torch.stack(codes, 0)
    plain = torch.stack(scales, 0)  # (l, rows, K/16)
    perm = layout.permute_sf(plain.permute(1, 2, 0))
    return codes, plain, perm


def _check_exact(x3):
    codes, sf, perm = quantize(x3)
    torch.cuda.synchronize()
    rc, rs, rp = _reference(x3)
    got_codes = codes.view(torch.uint8).permute(2, 0, 1)
    assert torch.equal(got_codes, rc), "codes differ"
    assert torch.equal(sf.view(torch.uint8).permute(2, 0, 1), rs.view(torch.uint8)), "scales differ"
    assert torch.equal(perm.view(torch.uint8), rp.view(torch.uint8)), "permuted scales differ"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("l,rows,k", [(1, 128, 64), (1, 200, 512), (2, 77, 1024), (1, 1, 64)])
def test_quantize_bit_exact(cuda, dtype, l, rows, k):
    g = torch.Generator(device="cuda").manual_seed(rows * 131 + k)
    x = torch.randn((l, rows, k), generator=g, device="cuda", dtype=torch.float32)
    # magnitudes from subnormal e4m3 scales (amax / 6 < 2^-6) to large ones
    mag = torch.logspace(-4, 2, rows, device="cuda").reshape(1, rows, 1)
    x = (x * mag).to(dtype)
    _check_exact(x)


@pytest.mark.gpu
def test_quantize_ties_zeros_and_signs(cuda):
    # block 0: amax 6 -> scale 1, exact e2m1 midpoints (ties) of both signs
    row = [6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0]
    blocks = [row, [0.0] * 16, [-0.0] * 15 + [1e-30], [3.0] * 16]
    x = torch.tensor(blocks * 4, device="cuda").reshape(1, 4, 64)
    _check_exact(x)


def _boundary_rows():
    """Rows of 64 values: per block, amax = 6 s (so the block's scale is exactly s) and 15
    values at and within two fp32 ulps of s times each e2m1 decision threshold, both signs,
    for every positive finite e4m3 scale s (normal and subnormal)."""
    s_vals = torch.arange(1, 127, dtype=torch.uint8).view(torch.float8_e4m3fn).float().tolist()
    thresholds = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    blocks = []
    for sv in s_vals:
        vals = []
        for t in thresholds:
            base = torch.tensor(t * sv, dtype=torch.float32)
            around = [base]
            lo = hi = base
            for _ in range(2):
                lo = torch.nextafter(lo, torch.tensor(-float("inf")))
                hi = torch.nextafter(hi, torch.tensor(float("inf")))
                around += [lo, hi]
            for v in around:
                vals += [float(v), -float(v)]
        for i in range(0, len(vals), 15):
            chunk = vals[i:i + 15]
            blocks.append([6.0 * sv] + chunk + [0.0] * (15 - len(chunk)))
    while len(blocks) % 4:
        blocks.append([0.0] * 16)
    return torch.tensor(blocks, dtype=torch.float32).reshape(1, -1, 64)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_rounding_boundaries(cuda, dtype):
    x = _boundary_rows().to("cuda")
    _check_exact(x.to(dtype))


@pytest.mark.gpu
def test_quantize_feeds_the_gemm(cuda):
    m, n, k = 192, 384, 1024
    g = torch.Generator(device="cuda").manual_seed(7)
    xa = torch.randn((m, k), generator=g, device="cuda", dtype=torch.bfloat16)
    xb = torch.randn((n, k), generator=g, device="cuda", dtype=torch.bfloat16)
    a, sfa, sfa_p = quantize(xa)
    b, sfb, sfb_p = quantize(xb)
    c = torch.zeros((1, m, n), device="cuda", dtype=torch.float16).permute(1, 2, 0)
    data = (a, b, sfa, sfb, sfa_p, sfb_p, c)
    out = gemm.custom_kernel(data)
    torch.cuda.synchronize()
    assert_close(out.permute(2, 0, 1).cpu().numpy(), dense_expected(data), "quantise -> gemm")
    # and the quantised GEMM tracks the bf16 product within the fp4 quantisation error
    ref = (xa.float() @ xb.float().T).cpu().numpy()
    err = np.abs(out[:, :, 0].float().cpu().numpy() - ref) / np.sqrt(k)
    assert err.mean() < 0.25


def test_quantize_argument_errors():
    with pytest.raises(ValueError):
        quantize(torch.zeros(2, 64))  # not a CUDA tensor
    with pytest.raises(ValueError):
        quantize(torch.zeros(2, 64, dtype=torch.int32))
