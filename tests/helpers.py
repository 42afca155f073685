"""Shared test helpers: run the oracle on the tensors a CUDA call consumed."""
import numpy as np
import torch

from oracle import nvfp4_oracle as orc

RTOL = 1e-3  # tolerance of the reference checker (kernels/gemm/reference.py:161)
ATOL = 1e-3


def u8(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.uint8).cpu().numpy() if t.dtype != torch.uint8 else t.cpu().numpy()


def dense_expected(data, rows=None, dtype=None) -> np.ndarray:
    """Oracle C as (l, m, n) fp16 for a 7-tuple; ``rows`` restricts to a subset of M."""
    a, b, sfa, sfb = data[:4]
    a_lmk = u8(a.permute(2, 0, 1).contiguous())
    b_lnk = u8(b.permute(2, 0, 1).contiguous())
    sa = u8(sfa.cpu().contiguous())
    sb = u8(sfb.cpu().contiguous())
    if rows is not None:
        a_lmk = a_lmk[:, rows]
        sa = sa[rows]
    m, n, k = a_lmk.shape[1], b_lnk.shape[1], a_lmk.shape[2] * 2
    if dtype is None:
        dtype = np.float64 if m * n * k <= 4e9 else np.float32
    return orc.gemm_ref(a_lmk, b_lnk, sa, sb, dtype=dtype)


def assert_close(got: np.ndarray, exp: np.ndarray, what=""):
    bad = orc.allclose_report(got, exp, rtol=RTOL, atol=ATOL)
    assert not bad, f"{what}: " + " ".join(bad)


def spread_rows(m: int, block: int = 128, salt: int = 37) -> np.ndarray:
    """One row in every ``block``-row block of M at a varying offset, plus the first and
    last rows: a sample that touches every M-tile row block of the kernel's raster."""
    nb = (m + block - 1) // block
    rows = {0, m - 1}
    for b in range(nb):
        r = b * block + (b * salt + 11) % block
        rows.add(min(m - 1, r))
    return np.array(sorted(rows), dtype=np.int64)
