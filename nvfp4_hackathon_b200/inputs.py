"""Seeded input generators for the two entry points (torch, any device).

Two families:

* ``generate_input`` / ``generate_group_input`` follow the reference's own
  generators (kernels/gemm/reference.py:56-158, kernels/group_gemm/reference.py:
  126-201): uniformly random e2m1 bytes (the grouped variant masks every
  nibble to sign + 2 LSBs), small integer e4m3 scales, random (non-zero)
  filler in the padding of the permuted scale tensors, and a random fp16 C
  that the kernel must overwrite.  The random streams differ from the
  reference's CUDA RNG; the value distributions and layouts are the same.
* ``quantize_nvfp4`` / ``generate_quantized_input`` implement the BASELINE
  generation: fp32 N(0, 1) values, per 16-element block along K the scale
  e4m3(amax / 6), values rounded to the nearest e2m1 code (ties to even).
"""
from __future__ import annotations

import math

import torch

from .layout import SF_VEC, ceil_div, permute_sf

E2M1_MAGS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
# midpoints between neighbouring magnitudes; ties go to the even code
_MIDS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)
_TIES_UP = (0.75, 1.75, 3.5)


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _perm_filler(l: int, mn: int, sf_k: int, lo: int, hi: int, g, device) -> torch.Tensor:
    per = ceil_div(mn, 128) * ceil_div(sf_k, 4) * 512
    return torch.randint(lo, hi, (l * per,), generator=g, device=device, dtype=torch.int64) \
        .to(torch.float8_e4m3fn).view(torch.uint8)


def generate_input(m: int, n: int, k: int, l: int, seed: int, device="cuda"):
    """7-tuple ``(a, b, sfa, sfb, sfa_permuted, sfb_permuted, c)`` with the reference's
    shapes, dtypes and strides (kernels/gemm/reference.py:56-158)."""
    g = _gen(device, seed)
    a = torch.randint(-128, 128, (l, m, k // 2), generator=g, device=device, dtype=torch.int8)
    b = torch.randint(-128, 128, (l, n, k // 2), generator=g, device=device, dtype=torch.int8)
    a = a.permute(1, 2, 0).view(torch.float4_e2m1fn_x2)
    b = b.permute(1, 2, 0).view(torch.float4_e2m1fn_x2)
    c = torch.randn((l, m, n), generator=g, device=device, dtype=torch.float16).permute(1, 2, 0)
    sf_k = ceil_div(k, SF_VEC)

    def scales(mn):
        plain = torch.randint(0, 4, (l, mn, sf_k), generator=g, device=device, dtype=torch.int64)
        plain = plain.to(torch.float8_e4m3fn).permute(1, 2, 0)
        perm = permute_sf(plain, _perm_filler(l, mn, sf_k, 0, 4, g, device))
        return plain, perm

    sfa, sfa_p = scales(m)
    sfb, sfb_p = scales(n)
    return (a, b, sfa, sfb, sfa_p, sfb_p, c)


def generate_group_input(m, n, k, g: int, seed: int, device="cuda"):
    """4-tuple of lists ``([(a, b, c)], [(sfa, sfb)], [(sfa_p, sfb_p)], [(m, n, k, 1)])``
    as kernels/group_gemm/reference.py:137-201 builds it (plain scales on the host)."""
    gen = _gen(device, seed)
    abc, sf, sfp, sizes = [], [], [], []
    for i in range(g):
        mi, ni, ki = int(m[i]), int(n[i]), int(k[i])

        def fp4(rows):
            raw = torch.randint(0, 255, (1, rows, ki // 2), generator=gen, device=device,
                                dtype=torch.int64).to(torch.uint8)
            return (raw & 0b1011_1011).permute(1, 2, 0).view(torch.float4_e2m1fn_x2)

        a, b = fp4(mi), fp4(ni)
        c = torch.randn((1, mi, ni), generator=gen, device=device, dtype=torch.float16).permute(1, 2, 0)
        sf_k = ceil_div(ki, SF_VEC)

        def scales(mn):
            plain = torch.randint(1, 3, (1, mn, sf_k), generator=gen, device=device,
                                  dtype=torch.int64).to(torch.float8_e4m3fn).permute(1, 2, 0)
            perm = permute_sf(plain, _perm_filler(1, mn, sf_k, 1, 3, gen, device))
            return plain, perm

        sfa, sfa_p = scales(mi)
        sfb, sfb_p = scales(ni)
        abc.append((a, b, c))
        sf.append((sfa.cpu(), sfb.cpu()))
        sfp.append((sfa_p, sfb_p))
        sizes.append((mi, ni, ki, 1))
    return (abc, sf, sfp, sizes)


# ----------------------------------------------------------------------------- quantiser
def quantize_nvfp4(x: torch.Tensor):
    """fp32 (rows, K) -> (codes (rows, K/2) uint8, scales (rows, K/16) float8_e4m3fn).

    scale = e4m3(amax_16 / 6); code = nearest e2m1 of x / scale (ties to even);
    element 2i in the low nibble.
    """
    rows, kk = x.shape
    assert kk % SF_VEC == 0
    blk = x.float().reshape(rows, kk // SF_VEC, SF_VEC)
    amax = blk.abs().amax(dim=-1)
    scale = (amax / 6.0).to(torch.float8_e4m3fn)
    s32 = scale.float().unsqueeze(-1)
    v = torch.where(s32 > 0, blk / torch.where(s32 > 0, s32, torch.ones_like(s32)),
                    torch.zeros_like(blk))
    mag = v.abs().clamp(max=6.0)
    mids = torch.tensor(_MIDS, device=x.device, dtype=torch.float32)
    code = torch.bucketize(mag, mids, right=False)
    for t in _TIES_UP:
        code = code + (mag == t).to(code.dtype)
    code = code | ((v < 0) & (code > 0)).to(code.dtype) << 3
    code = code.reshape(rows, kk).to(torch.uint8)
    packed = code[:, 0::2] | (code[:, 1::2] << 4)
    return packed, scale


def _quantized_operand(rows: int, k: int, l: int, g, device):
    codes, scales = [], []
    for _ in range(l):
        x = torch.randn((rows, k), generator=g, device=device, dtype=torch.float32)
        c, s = quantize_nvfp4(x)
        codes.append(c)
        scales.append(s)
    packed = torch.stack(codes, 0)                  # (l, rows, K/2)
    plain = torch.stack(scales, 0).permute(1, 2, 0)  # (rows, K/16, l)
    return packed.permute(1, 2, 0).view(torch.float4_e2m1fn_x2), plain


def generate_quantized_input(m: int, n: int, k: int, l: int, seed: int, device="cuda"):
    """BASELINE-style 7-tuple: N(0, 1) -> e4m3 per-16 scale -> e2m1, C zero-initialised."""
    g = _gen(device, seed)
    a, sfa = _quantized_operand(m, k, l, g, device)
    b, sfb = _quantized_operand(n, k, l, g, device)
    c = torch.zeros((l, m, n), device=device, dtype=torch.float16).permute(1, 2, 0)
    return (a, b, sfa, sfb, permute_sf(sfa), permute_sf(sfb), c)


def generate_quantized_group_input(m_list, n: int, k: int, seed: int, device="cuda"):
    """BASELINE-style grouped 4-tuple (one B_g per group; C_g zero-initialised)."""
    g = _gen(device, seed)
    abc, sf, sfp, sizes = [], [], [], []
    for mi in m_list:
        mi = int(mi)
        a, sfa = _quantized_operand(mi, k, 1, g, device)
        b, sfb = _quantized_operand(n, k, 1, g, device)
        c = torch.zeros((1, mi, n), device=device, dtype=torch.float16).permute(1, 2, 0)
        abc.append((a, b, c))
        sf.append((sfa, sfb))
        sfp.append((permute_sf(sfa), permute_sf(sfb)))
        sizes.append((mi, n, k, 1))
    return (abc, sf, sfp, sizes)


# ----------------------------------------------------------------------------- group sizes
def uniform_group_sizes(g: int, seed: int, lo=64, hi=1024, step=64) -> list[int]:
    """M_g drawn uniformly from {lo, lo+step, ..., hi}."""
    gen = torch.Generator().manual_seed(seed)
    choices = (hi - lo) // step + 1
    return [lo + step * int(v) for v in torch.randint(0, choices, (g,), generator=gen)]


def zipf_group_sizes(g: int, total: int, s: float = 1.1, multiple: int = 16) -> list[int]:
    """configs[4a]: counts proportional to rank^-s, rounded to multiples of ``multiple``;
    the rounding remainder goes to the largest fractional parts so the sum is ``total``."""
    w = [1.0 / (r + 1) ** s for r in range(g)]
    tot_w = sum(w)
    units = total // multiple
    raw = [units * x / tot_w for x in w]
    base = [int(math.floor(v)) for v in raw]
    rem = units - sum(base)
    order = sorted(range(g), key=lambda i: (-(raw[i] - base[i]), i))
    for i in order[:rem]:
        base[i] += 1
    return [b * multiple for b in base]
