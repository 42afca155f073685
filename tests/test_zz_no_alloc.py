"""GPU test of nvfp4_grouped_gemm_noalloc, the grouped GEMM entry point that
allocates nothing (its scratch is a fixed array inside the library).  It exists
for callers that cannot allocate device memory while they run, e.g. code that
works from a pre-planned pool.  This file is collected last on purpose: if it
fails, a run that stops at the first failure has already run everything else.

The test calls the entry point through the C ABI twice in a row, on two
different problems, and compares each result with the ordinary entry point
(which uses a caller-provided workspace) and with the CPU oracle, with the
tolerance of the other parity tests.
"""
import numpy as np
import pytest
import torch

from nvfp4_hackathon_b200 import _native, group_gemm, inputs
from oracle import nvfp4_oracle as orc
from tests.helpers import assert_close, u8

pytestmark = pytest.mark.gpu

CASES = [
    ([80, 176, 0, 72, 248], [1024] * 5, [1024] * 5),
    ([192, 320, 40], [384, 256, 512], [512, 256, 768]),
]


def _clone_outputs(gdata):
    abc, sf, sfp, sizes = gdata
    abc2 = [(a, b, torch.full_like(c, float("nan"))) for a, b, c in abc]
    return (abc2, sf, sfp, sizes)


@pytest.mark.parametrize("first", [0, 1])
def test_noalloc_matches_workspace_entry_point_two_calls(cuda, first):
    lib = _native.load()
    order = [CASES[first], CASES[1 - first]]
    for i, (m, n, k) in enumerate(order):
        gdata = inputs.generate_group_input(m, n, k, len(m), seed=100 + i)
        # ordinary entry point (caller-provided workspace)
        expected = [c[:, :, 0].cpu().numpy() for c in group_gemm.custom_kernel(gdata)]
        torch.cuda.synchronize()
        # no-allocation entry point on the same inputs, fresh outputs
        g2 = _clone_outputs(gdata)
        table = group_gemm._table(g2[0], g2[2], g2[3], g2[0][0][0].device)
        G = len(m)
        p = table.data_ptr()
        rc = lib.nvfp4_grouped_gemm_noalloc(p, p + 16 * G, p + 40 * G, G,
                                            torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "nvfp4_grouped_gemm_noalloc")
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        for g, ((a, b, c), (sa, sb), e) in enumerate(zip(g2[0], g2[1], expected)):
            got = c[:, :, 0].cpu().numpy()
            assert_close(got, e, f"call {i} group {g} vs workspace entry point")
            ref = orc.grouped_gemm_ref([(u8(a[:, :, 0].contiguous()), u8(b[:, :, 0].contiguous()),
                                         u8(sa[:, :, 0].contiguous()), u8(sb[:, :, 0].contiguous()))])[0]
            assert_close(got, ref, f"call {i} group {g} vs oracle")


def test_noalloc_rejects_too_many_groups(cuda):
    lib = _native.load()
    rc = lib.nvfp4_grouped_gemm_noalloc(16, 16, 16, 257, None)
    assert rc == 3
    assert b"256" in lib.nvfp4_last_error()
