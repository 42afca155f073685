"""Parity on the reference's OWN inputs and numerical path.

tests/golden/reference_fixtures.npz holds inputs drawn by the reference's own
``generate_input`` (kernels/gemm/reference.py:56-158, kernels/group_gemm/reference.py:
137-201) on its own test cases and seed, and the output of its ``ref_kernel``
(torch._scaled_mm, kernels/gemm/reference.py:27-53), recorded on a B200 by
tests/golden/make_reference_fixtures.py.  The CPU test pins the oracle to those
outputs; the GPU test feeds the exact same tensors, in the reference's layouts, to the
drop-in ``custom_kernel`` entry points and applies the reference checker's tolerance
(rtol = atol = 1e-3, kernels/gemm/reference.py:161).
"""
import os

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as orc
from tests.helpers import assert_close

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_fixtures.npz")


def _fixture():
    if not os.path.exists(PATH):
        pytest.skip("reference fixtures not generated")
    return np.load(PATH)


def _dense_ids(fx):
    return sorted({k.split("_")[0] for k in fx.files if k.startswith("dense")})


def _group_ids(fx):
    return sorted({k.split("_")[0] for k in fx.files if k.startswith("group") and k.endswith("_sizes")})


def test_oracle_matches_reference_ref_kernel():
    fx = _fixture()
    for d in _dense_ids(fx):
        got = orc.gemm_ref(fx[f"{d}_a"], fx[f"{d}_b"], fx[f"{d}_sfa"], fx[f"{d}_sfb"])
        assert_close(got, fx[f"{d}_c_ref"], f"oracle {d}")
        # the permuted bytes the reference built hold the plain scales at the documented offsets
        m, n, k, l = (int(v) for v in fx[f"{d}_mnkl"])
        for plain, perm, mn in ((fx[f"{d}_sfa"], fx[f"{d}_sfa_perm"], m), (fx[f"{d}_sfb"], fx[f"{d}_sfb_perm"], n)):
            assert np.array_equal(orc.unpermute_sf(perm, mn, k // 16, l), plain)
    for gname in _group_ids(fx):
        sizes = fx[f"{gname}_sizes"]
        groups = [(fx[f"{gname}_{j}_a"], fx[f"{gname}_{j}_b"], fx[f"{gname}_{j}_sfa"], fx[f"{gname}_{j}_sfb"])
                  for j in range(len(sizes))]
        for j, c in enumerate(orc.grouped_gemm_ref(groups)):
            assert_close(c, fx[f"{gname}_{j}_c_ref"], f"oracle {gname} group {j}")


def _perm_tensor(storage: np.ndarray, mn: int, sf_k: int, l: int) -> torch.Tensor:
    rm, rk = -(-mn // 128), -(-sf_k // 4)
    t = torch.from_numpy(storage.copy()).cuda().view(torch.float8_e4m3fn).reshape(l, rm, rk, 32, 4, 4)
    return t.permute(3, 4, 1, 5, 2, 0)


def _codes(arr_lmk: np.ndarray) -> torch.Tensor:
    """(l, mn, k/2) bytes -> (mn, k/2, l) float4_e2m1fn_x2 view, the reference's layout."""
    return torch.from_numpy(arr_lmk.copy()).cuda().permute(1, 2, 0).view(torch.float4_e2m1fn_x2)


@pytest.mark.gpu
def test_custom_kernels_on_reference_inputs(cuda):
    from nvfp4_hackathon_b200 import _native, gemm, group_gemm
    fx = _fixture()
    for d in _dense_ids(fx):
        m, n, k, l = (int(v) for v in fx[f"{d}_mnkl"])
        a, b = _codes(fx[f"{d}_a"]), _codes(fx[f"{d}_b"])
        sfa = torch.from_numpy(fx[f"{d}_sfa"]).cuda().view(torch.float8_e4m3fn)
        sfb = torch.from_numpy(fx[f"{d}_sfb"]).cuda().view(torch.float8_e4m3fn)
        c = torch.randn((l, m, n), dtype=torch.float16, device="cuda").permute(1, 2, 0)
        data = (a, b, sfa, sfb, _perm_tensor(fx[f"{d}_sfa_perm"], m, k // 16, l),
                _perm_tensor(fx[f"{d}_sfb_perm"], n, k // 16, l), c)
        out = gemm.custom_kernel(data)
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        assert out is c
        assert_close(out.permute(2, 0, 1).cpu().numpy(), fx[f"{d}_c_ref"], f"custom_kernel {d}")
    for gname in _group_ids(fx):
        sizes = [tuple(int(v) for v in s) for s in fx[f"{gname}_sizes"]]
        abc, sf, sfp = [], [], []
        for j, (m, n, k, l) in enumerate(sizes):
            a = _codes(fx[f"{gname}_{j}_a"][None])
            b = _codes(fx[f"{gname}_{j}_b"][None])
            c = torch.randn((1, m, n), dtype=torch.float16, device="cuda").permute(1, 2, 0)
            abc.append((a, b, c))
            sf.append((torch.from_numpy(fx[f"{gname}_{j}_sfa"][..., None].copy()).view(torch.float8_e4m3fn),
                       torch.from_numpy(fx[f"{gname}_{j}_sfb"][..., None].copy()).view(torch.float8_e4m3fn)))
            sfp.append((_perm_tensor(fx[f"{gname}_{j}_sfa_perm"], m, k // 16, 1),
                        _perm_tensor(fx[f"{gname}_{j}_sfb_perm"], n, k // 16, 1)))
        outs = group_gemm.custom_kernel((abc, sf, sfp, sizes))
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        for j, c in enumerate(outs):
            assert_close(c[:, :, 0].cpu().numpy(), fx[f"{gname}_{j}_c_ref"], f"custom_kernel {gname} group {j}")
