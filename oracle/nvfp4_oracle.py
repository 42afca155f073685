"""CPU oracle for the NVFP4 GEMM and grouped-GEMM hot paths.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the parity tests,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg compare the CUDA
path against.  The product path (``nvfp4_hackathon_b200``) never imports it.

It restates, in numpy, what the reference computes on the GPU:

* ``ref_kernel`` (kernels/gemm/reference.py:27-53): for every batch l,
  ``C[:, :, l] = fp16(_scaled_mm(A[:, :, l], B[:, :, l].T, blocked(SFA), blocked(SFB)))``,
  i.e. dequantise e2m1 codes times their e4m3 block scale (one scale per 16
  elements along K), multiply with fp32-or-better accumulation, round to fp16.
* grouped ``ref_kernel`` (kernels/group_gemm/reference.py:39-74): the same per group.
* the permuted ("blocked") scale-factor layout: the scatter at
  kernels/gemm/reference.py:143-150 (== group_gemm/reference.py:114-121) and
  ``to_blocked`` (kernels/gemm/reference.py:13-24, group_gemm/reference.py:14-36).

Number formats (the torch dtypes the reference uses):
* ``float4_e2m1fn_x2``: two e2m1 codes per byte, element 2i in the low nibble.
  e2m1 = sign bit 3, exponent bits 2..1 (bias 1), mantissa bit 0;
  magnitudes {0, 0.5, 1, 1.5, 2, 3, 4, 6}.
* ``float8_e4m3fn``: sign bit 7, exponent bits 6..3 (bias 7), mantissa bits 2..0,
  subnormals for exponent 0, 0x7F / 0xFF = NaN, no infinities.

Parity pin: the layout functions are checked against fixtures produced by the
reference's own ``to_blocked`` (tests/golden/make_layout_golden.py); the GEMM
semantics against ``torch._scaled_mm`` outputs (tests/golden/make_scaled_mm_golden.py,
and live on the GPU in tests/test_gpu_parity.py::test_oracle_matches_scaled_mm), and
against the reference's own ``generate_input`` + ``ref_kernel`` run on a B200
(tests/golden/make_reference_fixtures.py).
"""
from __future__ import annotations

import numpy as np

SF_VEC = 16  # elements per scale factor (kernels/gemm/reference.py:6)

# e2m1 code -> value, built from the bit fields (not a copied table).
def _e2m1_table() -> np.ndarray:
    vals = np.zeros(16, dtype=np.float64)
    for code in range(16):
        sign = -1.0 if code & 0x8 else 1.0
        e = (code >> 1) & 0x3
        m = code & 0x1
        mag = (m * 0.5) if e == 0 else (1.0 + 0.5 * m) * 2.0 ** (e - 1)
        vals[code] = sign * mag
    return vals


def _e4m3_table() -> np.ndarray:
    vals = np.zeros(256, dtype=np.float64)
    for b in range(256):
        sign = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            vals[b] = np.nan
        elif e == 0:
            vals[b] = sign * (m / 8.0) * 2.0 ** (-6)
        else:
            vals[b] = sign * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E2M1 = _e2m1_table()
E4M3 = _e4m3_table()


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


# ----------------------------------------------------------------------------- decode
def decode_e2m1(packed: np.ndarray) -> np.ndarray:
    """(…, K/2) uint8 -> (…, K) float64; low nibble is element 2i."""
    packed = np.asarray(packed, dtype=np.uint8)
    lo = E2M1[packed & 0x0F]
    hi = E2M1[packed >> 4]
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.float64)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def decode_e4m3(raw: np.ndarray) -> np.ndarray:
    return E4M3[np.asarray(raw, dtype=np.uint8)]


# ----------------------------------------------------------------------------- SF layout
def blocked_offset(i: np.ndarray, j: np.ndarray, rest_k: int) -> np.ndarray:
    """Byte offset of scale (row i, K-vector j) inside one batch of the permuted tensor.

    Storage order (rest_mn, rest_k, 32, 4, 4): atom (i // 128, j // 4) is 512 bytes;
    inside it row i sits at (i % 32) * 16 + ((i % 128) // 32) * 4 and vector j at + j % 4
    (kernels/gemm/reference.py:143-150).
    """
    i = np.asarray(i, dtype=np.int64)
    j = np.asarray(j, dtype=np.int64)
    return (((i // 128) * rest_k + j // 4) * 32 + i % 32) * 16 + ((i % 128) // 32) * 4 + j % 4


def permute_sf(plain: np.ndarray, fill: np.ndarray | None = None) -> np.ndarray:
    """Plain scales (mn, sf_k, l) uint8 -> permuted storage, flat (l, rest_mn*rest_k*512).

    Padding bytes take ``fill`` (flat array of the same size) or zero.
    """
    mn, sf_k, l = plain.shape
    rm, rk = ceil_div(mn, 128), ceil_div(sf_k, 4)
    per = rm * rk * 512
    out = np.zeros((l, per), dtype=np.uint8) if fill is None else fill.reshape(l, per).copy()
    ii, jj = np.meshgrid(np.arange(mn), np.arange(sf_k), indexing="ij")
    off = blocked_offset(ii, jj, rk)
    for b in range(l):
        out[b, off] = plain[:, :, b]
    return out


def unpermute_sf(perm: np.ndarray, mn: int, sf_k: int, l: int) -> np.ndarray:
    """Permuted storage (any shape, l * rest_mn * rest_k * 512 bytes) -> plain (mn, sf_k, l)."""
    rm, rk = ceil_div(mn, 128), ceil_div(sf_k, 4)
    flat = np.asarray(perm, dtype=np.uint8).reshape(l, rm * rk * 512)
    ii, jj = np.meshgrid(np.arange(mn), np.arange(sf_k), indexing="ij")
    off = blocked_offset(ii, jj, rk)
    return np.stack([flat[b][off] for b in range(l)], axis=-1)


def to_blocked(mat: np.ndarray) -> np.ndarray:
    """Restatement of ``to_blocked`` (kernels/group_gemm/reference.py:14-36):
    (rows, cols) -> flat blocked layout, zero-padded to 128 rows x 4 cols."""
    rows, cols = mat.shape
    rb, cb = ceil_div(rows, 128), ceil_div(cols, 4)
    padded = np.zeros((rb * 128, cb * 4), dtype=mat.dtype)
    padded[:rows, :cols] = mat
    blocks = padded.reshape(rb, 128, cb, 4).transpose(0, 2, 1, 3)          # (rb, cb, 128, 4)
    return blocks.reshape(-1, 4, 32, 4).transpose(0, 2, 1, 3).reshape(-1)  # 128 rows -> (4, 32)


# ----------------------------------------------------------------------------- GEMM
def dequant(packed_lmk: np.ndarray, sf_plain_mkl: np.ndarray) -> np.ndarray:
    """packed (l, mn, K/2) uint8 and plain scales (mn, K/16, l) uint8 -> (l, mn, K) float64."""
    vals = decode_e2m1(packed_lmk)
    sf = decode_e4m3(np.transpose(sf_plain_mkl, (2, 0, 1)))  # (l, mn, K/16)
    k = vals.shape[-1]
    sf_full = np.repeat(sf, SF_VEC, axis=-1)[..., :k]
    return vals * sf_full


def gemm_ref(a_lmk: np.ndarray, b_lnk: np.ndarray, sfa: np.ndarray, sfb: np.ndarray,
             dtype=np.float64) -> np.ndarray:
    """C (l, m, n) fp16 = fp16(dequant(A) @ dequant(B)^T), accumulation in ``dtype``.

    a_lmk: (l, m, K/2) uint8; b_lnk: (l, n, K/2) uint8; sfa: (m, K/16, l); sfb: (n, K/16, l).
    """
    da = dequant(a_lmk, sfa).astype(dtype)
    db = dequant(b_lnk, sfb).astype(dtype)
    c = np.matmul(da, np.swapaxes(db, -1, -2))
    with np.errstate(over="ignore"):
        return c.astype(np.float16)


def grouped_gemm_ref(groups, dtype=np.float64):
    """groups: iterable of (a (m, K/2) u8, b (n, K/2) u8, sfa (m, K/16) u8, sfb (n, K/16) u8)
    -> list of (m, n) fp16 (kernels/group_gemm/reference.py:39-74 with l = 1)."""
    out = []
    for a, b, sfa, sfb in groups:
        c = gemm_ref(a[None], b[None], sfa[..., None], sfb[..., None], dtype=dtype)
        out.append(c[0])
    return out


def allclose_report(received: np.ndarray, expected: np.ndarray, rtol=1e-3, atol=1e-3,
                    max_print=5) -> list[str]:
    """Restatement of ``verbose_allclose`` (kernels/gemm/utils.py:30-91): element-wise
    |r - e| <= atol + rtol*|e|, plus NaN / +inf / -inf must match."""
    r = np.asarray(received, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    if r.shape != e.shape:
        return ["SIZE MISMATCH"]
    with np.errstate(invalid="ignore"):
        bad = np.abs(r - e) > atol + rtol * np.abs(e)
    bad |= np.isnan(r) ^ np.isnan(e)
    bad |= np.isposinf(r) ^ np.isposinf(e)
    bad |= np.isneginf(r) ^ np.isneginf(e)
    idx = np.argwhere(bad)
    if len(idx) == 0:
        return []
    msgs = [f"Number of mismatched elements: {len(idx)}"]
    for ix in idx[:max_print]:
        t = tuple(int(v) for v in ix)
        msgs.append(f"ERROR AT {t}: {r[t]} {e[t]}")
    if len(idx) > max_print:
        msgs.append(f"... and {len(idx) - max_print} more mismatched elements.")
    return msgs


# ----------------------------------------------------------------------------- quantiser
def quantize_ref(x: np.ndarray):
    """fp32 (rows, K) -> (codes (rows, K/2) uint8, scales (rows, K/16) uint8 e4m3 bytes).

    The input generation the benchmark configurations specify:
    per 16-element block along K, scale = e4m3(amax / 6) rounded to nearest, ties to the even
    code; each value becomes the nearest e2m1 code of x / scale (magnitude clamped to 6), ties
    to the even code, -0 written as +0; element 2i in the low nibble.  Restated here by
    exhaustive nearest-value search over the two code tables (the product's host version,
    nvfp4_hackathon_b200.inputs.quantize_nvfp4, uses bucketize and torch's fp8 cast; the GPU
    kernel uses the hardware cvt), so the three are independent.  Scales of 480 or more
    (amax >= 2880) fall outside e4m3 and are not covered.
    """
    x = np.asarray(x, dtype=np.float32)
    rows, kk = x.shape
    blk = x.reshape(rows, kk // SF_VEC, SF_VEC)
    amax = np.abs(blk).max(axis=-1).astype(np.float32)
    target = (amax / np.float32(6.0)).astype(np.float32)
    e4m3 = _e4m3_table().astype(np.float64)
    pos = np.arange(0, 0x7F)                    # +0 .. 448, byte order = value order
    vals = e4m3[pos]
    d = np.abs(target[..., None].astype(np.float64) - vals)
    best = d.min(axis=-1, keepdims=True)
    cand = d == best
    # ties: the even code (the larger of two tied neighbours is odd iff the smaller is even)
    idx = np.where(cand & (pos % 2 == 0), pos, 10_000).min(axis=-1)
    idx = np.where(idx == 10_000, np.argmax(cand, axis=-1), idx)
    scale_b = pos[idx].astype(np.uint8)
    s32 = vals[idx].astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = np.where(s32[..., None] > 0, blk / np.where(s32 > 0, s32, 1)[..., None], 0).astype(np.float32)
    mag = np.minimum(np.abs(v), np.float32(6.0)).astype(np.float64)
    table = _e2m1_table()[:8].astype(np.float64)   # magnitudes of codes 0..7
    dd = np.abs(mag[..., None] - table)
    bb = dd.min(axis=-1, keepdims=True)
    c = dd == bb
    code = np.where(c & (np.arange(8) % 2 == 0), np.arange(8), 99).min(axis=-1)
    code = np.where(code == 99, np.argmax(c, axis=-1), code).astype(np.uint8)
    code = code | (((v < 0) & (code > 0)).astype(np.uint8) << 3)
    code = code.reshape(rows, kk)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    return packed, scale_b
