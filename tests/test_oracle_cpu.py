"""The CPU oracle against known answers and against fixtures made by the
reference's own code (tests/golden/)."""
import os

import numpy as np
import pytest
import torch

from nvfp4_hackathon_b200 import inputs, layout
from oracle import nvfp4_oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_e2m1_known_values_and_nibble_order():
    assert list(orc.E2M1[:8]) == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert list(orc.E2M1[8:]) == [-0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    # byte 0x21: low nibble (code 1 = 0.5) is element 0, high nibble (code 2 = 1.0) element 1
    assert list(orc.decode_e2m1(np.array([[0x21, 0xF7]], dtype=np.uint8))[0]) == [0.5, 1.0, 6.0, -6.0]


def test_e4m3_table_matches_torch_float8():
    g = np.load(os.path.join(GOLDEN, "to_blocked_golden.npz"))
    ref = g["e4m3_values"]
    mine = orc.E4M3.astype(np.float32)
    assert np.array_equal(np.isnan(ref), np.isnan(mine))
    assert np.array_equal(ref[~np.isnan(ref)], mine[~np.isnan(mine)])
    assert orc.E4M3[0x7E] == 448.0 and orc.E4M3[0x01] == 2.0 ** -9


@pytest.mark.parametrize("i", range(3))
def test_to_blocked_matches_reference_gemm(i):
    g = np.load(os.path.join(GOLDEN, "to_blocked_golden.npz"))
    assert np.array_equal(orc.to_blocked(g[f"gemm_in_{i}"]), g[f"gemm_out_{i}"])


@pytest.mark.parametrize("i", range(3))
def test_to_blocked_matches_reference_group_padding(i):
    g = np.load(os.path.join(GOLDEN, "to_blocked_golden.npz"))
    assert np.array_equal(orc.to_blocked(g[f"group_in_{i}"]), g[f"group_out_{i}"])


@pytest.mark.parametrize("mn,sf_k,l", [(128, 4, 1), (200, 12, 2), (72, 16, 1), (384, 36, 3)])
def test_permuted_layout_round_trip_and_blocked_equivalence(mn, sf_k, l):
    rng = np.random.default_rng(mn * 31 + sf_k)
    plain = rng.integers(0, 256, size=(mn, sf_k, l), dtype=np.uint8)
    t = torch.from_numpy(plain).view(torch.float8_e4m3fn)
    perm = layout.permute_sf(t)
    assert layout.is_permuted_layout(perm, mn, sf_k, l)
    flat = perm.permute(5, 2, 4, 0, 1, 3).contiguous().view(torch.uint8).numpy().reshape(l, -1)
    assert np.array_equal(orc.unpermute_sf(flat, mn, sf_k, l), plain)
    assert np.array_equal(orc.permute_sf(plain), flat)
    for b in range(l):  # the permuted storage of one batch is the blocked layout
        assert np.array_equal(flat[b], orc.to_blocked(plain[:, :, b]))


def test_oracle_matches_scaled_mm_fixtures():
    path = os.path.join(GOLDEN, "scaled_mm_golden.npz")
    if not os.path.exists(path):
        pytest.skip("scaled_mm fixtures not generated (tests/golden/make_scaled_mm_golden.py, on a GPU)")
    g = np.load(path)
    i = 0
    while f"a_{i}" in g:
        exp = g[f"c_{i}"]
        got = orc.gemm_ref(g[f"a_{i}"][None], g[f"b_{i}"][None], g[f"sfa_{i}"][..., None],
                           g[f"sfb_{i}"][..., None])[0]
        assert not orc.allclose_report(got, exp, rtol=1e-3, atol=1e-3), f"case {i}"
        i += 1
    assert i >= 3


def test_quantizer_bounds_and_ties():
    torch.manual_seed(0)
    x = torch.randn(32, 512) * 3
    packed, scale = inputs.quantize_nvfp4(x)
    deq = orc.dequant(packed.numpy()[None], scale.view(torch.uint8).numpy()[..., None])[0]
    s = np.repeat(scale.float().numpy(), 16, axis=1)
    # each value within half a code step (<= 1.0 * scale for the widest gap 4 -> 6) or clamped at 6*s
    assert np.all(np.abs(deq - x.numpy()) <= np.maximum(1.0 * s, np.abs(x.numpy()) - 6 * s) + 1e-6)
    # ties go to the even code: 0.25->0, 0.75->1, 1.25->1, 1.75->2, 2.5->2, 3.5->4, 5->4
    row = torch.tensor([[6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0] + [0.0] * 8])
    p, sc = inputs.quantize_nvfp4(row)
    assert float(sc.float()[0, 0]) == 1.0
    vals = orc.decode_e2m1(p.numpy())[0][:8]
    assert list(vals) == [6.0, 0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0]
    z, zs = inputs.quantize_nvfp4(torch.zeros(1, 16))
    assert int(z.sum()) == 0 and float(zs.float().sum()) == 0.0


def test_allclose_report_semantics():
    e = np.array([1.0, np.nan, np.inf, -np.inf, 100.0])
    assert orc.allclose_report(e.copy(), e) == []
    r = e.copy()
    r[4] = 100.2  # 0.2 > 1e-3 + 1e-3 * 100
    assert "mismatched elements: 1" in orc.allclose_report(r, e)[0]
    r = e.copy()
    r[1] = 0.0
    assert orc.allclose_report(r, e)


def test_small_gemm_against_explicit_sum():
    rng = np.random.default_rng(5)
    a = rng.integers(0, 256, size=(1, 4, 32), dtype=np.uint8)
    b = rng.integers(0, 256, size=(1, 3, 32), dtype=np.uint8)
    sa = rng.integers(0, 4, size=(4, 4, 1)).astype(np.float32)
    sb = rng.integers(0, 4, size=(3, 4, 1)).astype(np.float32)
    sa8 = torch.from_numpy(sa).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    sb8 = torch.from_numpy(sb).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    c = orc.gemm_ref(a, b, sa8, sb8)
    A = orc.decode_e2m1(a[0])
    B = orc.decode_e2m1(b[0])
    for i in range(4):
        for j in range(3):
            exp = sum(A[i, kk] * sa[i, kk // 16, 0] * B[j, kk] * sb[j, kk // 16, 0] for kk in range(64))
            assert c[0, i, j] == np.float16(exp)


def test_quantiser_restatements_agree():
    """The oracle's quantiser (exhaustive nearest-value search) and the host generator used for
    the benchmark inputs (bucketize + torch's fp8 cast) give the same codes and scales, on
    N(0, 1) data over a wide range of magnitudes and on values placed exactly on the e2m1
    rounding midpoints of many scales (the ties)."""
    import torch
    from nvfp4_hackathon_b200.inputs import quantize_nvfp4
    rng = np.random.default_rng(5)
    x = rng.standard_normal((96, 512)).astype(np.float32)
    x *= (2.0 ** rng.integers(-12, 8, size=(96, 1))).astype(np.float32)
    # ties: blocks whose amax is 6 * s (scale exactly s) holding the midpoints * s
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.75, -2.5, 0.0, 6.0, -5.0,
                     1.0, 3.0, 4.0, -6.0], dtype=np.float32)
    scales = _e4m3_vals_for_test()
    ties = np.stack([mids * s for s in scales]).astype(np.float32)  # each row: one block of 16
    ties = ties.reshape(-1, 64) if ties.shape[0] % 4 == 0 else ties[: ties.shape[0] // 4 * 4].reshape(-1, 64)
    for arr in (x, ties):
        c_ref, s_ref = orc.quantize_ref(arr)
        c_t, s_t = quantize_nvfp4(torch.from_numpy(arr))
        assert np.array_equal(s_ref, s_t.view(torch.uint8).numpy())
        assert np.array_equal(c_ref, c_t.numpy())


def _e4m3_vals_for_test():
    # positive normal e4m3 values from 2^-6 to 448 whose 6x stays finite in fp32
    vals = [v for v in orc.E4M3[1:0x7F] if v >= 2.0 ** -6]
    return np.array(vals, dtype=np.float32)
