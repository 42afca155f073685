"""Scale-factor layout helpers (torch, any device).

The permuted ("blocked") layout is the one the reference's generators build
(kernels/gemm/reference.py:113-150): logical shape (32, 4, rest_mn, 4, rest_k, l)
over storage (l, rest_mn, rest_k, 32, 4, 4); scale (i, j, b) lives at byte
((((b*rest_mn + i//128)*rest_k + j//4)*32 + i%32)*16 + ((i%128)//32)*4 + j%4.
"""
from __future__ import annotations

import torch

SF_VEC = 16


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def permuted_shape(mn: int, sf_k: int, l: int) -> tuple[int, ...]:
    return (32, 4, ceil_div(mn, 128), 4, ceil_div(sf_k, 4), l)


def permuted_strides(mn: int, sf_k: int, l: int) -> tuple[int, ...]:
    rm, rk = ceil_div(mn, 128), ceil_div(sf_k, 4)
    return (16, 4, rk * 512, 1, 512, rm * rk * 512)


def blocked_index(mn: int, sf_k: int, device) -> torch.Tensor:
    """(mn, sf_k) int64 byte offsets inside one batch of the permuted storage."""
    rk = ceil_div(sf_k, 4)
    i = torch.arange(mn, device=device, dtype=torch.int64)[:, None]
    j = torch.arange(sf_k, device=device, dtype=torch.int64)[None, :]
    return (((i // 128) * rk + j // 4) * 32 + i % 32) * 16 + ((i % 128) // 32) * 4 + j % 4


def permute_sf(plain: torch.Tensor, filler: torch.Tensor | None = None) -> torch.Tensor:
    """Plain scales (mn, sf_k, l) float8_e4m3fn -> permuted view (32, 4, rm, 4, rk, l).

    Padding bytes (rows past mn, K-vectors past sf_k) take ``filler`` (a flat
    uint8 tensor of the storage size) or zero.
    """
    mn, sf_k, l = plain.shape
    rm, rk = ceil_div(mn, 128), ceil_div(sf_k, 4)
    per = rm * rk * 512
    if filler is None:
        store = torch.zeros((l, per), dtype=torch.uint8, device=plain.device)
    else:
        store = filler.to(torch.uint8).reshape(l, per).clone()
    idx = blocked_index(mn, sf_k, plain.device).reshape(-1)
    src = plain.view(torch.uint8).permute(2, 0, 1).reshape(l, -1)
    store.scatter_(1, idx.unsqueeze(0).expand(l, -1), src)
    view = store.view(torch.float8_e4m3fn).reshape(l, rm, rk, 32, 4, 4)
    return view.permute(3, 4, 1, 5, 2, 0)


def is_permuted_layout(t: torch.Tensor, mn: int, sf_k: int, l: int) -> bool:
    """True when ``t`` has the reference's permuted shape and storage order
    (strides of size-1 dimensions are ignored)."""
    if tuple(t.shape) != permuted_shape(mn, sf_k, l):
        return False
    want = permuted_strides(mn, sf_k, l)
    return all(sz == 1 or st == w for sz, st, w in zip(t.shape, t.stride(), want))
