"""CUDA path vs the CPU oracle (parity tests proper; they call the C ABI
through the drop-in modules)."""
import ctypes

import numpy as np
import pytest
import torch

from nvfp4_hackathon_b200 import _native, gemm, group_gemm, inputs
from oracle import nvfp4_oracle as orc
from tests.helpers import assert_close, dense_expected, spread_rows, u8

pytestmark = pytest.mark.gpu

# kernels/gemm/run_tests.py:13-30 (test + benchmark shapes), all seed 1111
REF_GEMM_CASES = [
    (128, 256, 256, 1), (128, 1536, 7168, 1), (128, 3072, 1536, 1), (256, 7168, 256, 1),
    (256, 7168, 2048, 1), (2304, 4608, 7168, 1), (384, 7168, 2304, 1), (512, 512, 7168, 1),
    (512, 4096, 512, 1), (512, 1536, 7168, 1),
    (128, 7168, 16384, 1), (128, 4096, 7168, 1), (128, 7168, 2048, 1),
]


def _run_dense(data, opt=None):
    out = gemm.custom_kernel(data, opt=opt)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return out.permute(2, 0, 1).cpu().numpy()


@pytest.mark.parametrize("m,n,k,l", REF_GEMM_CASES)
def test_reference_gemm_cases(cuda, m, n, k, l):
    data = inputs.generate_input(m, n, k, l, seed=1111)
    got = _run_dense(data)
    assert_close(got, dense_expected(data), f"{m}x{n}x{k}")


@pytest.mark.parametrize("m,n,k", [(128, 256, 512), (64, 14336, 4096)])
def test_baseline_configs_full(cuda, m, n, k):
    data = inputs.generate_quantized_input(m, n, k, 1, seed=1111)
    got = _run_dense(data)
    assert_close(got, dense_expected(data), f"c {m}x{n}x{k}")


def test_baseline_8192_cubed_sampled_rows(cuda):
    m = n = k = 8192
    data = inputs.generate_quantized_input(m, n, k, 1, seed=1111)
    got = _run_dense(data)
    rows = spread_rows(m)  # one row in every 128-row M block
    exp = dense_expected(data, rows=rows, dtype=np.float32)
    assert_close(got[:, rows], exp, "8192^3 sampled rows")


# every tile shape and operand order, with ragged M/N, short K and batches
SHAPES = [(72, 136, 64, 1), (200, 100, 192, 2), (129, 257, 320, 1), (64, 512, 1024, 3),
          (256, 512, 768, 1), (1, 64, 128, 1)]
CONFIGS = [(1, 64), (1, 128), (1, 256), (2, 64), (2, 128), (2, 256)]


CONFIGS += [(2, 64, 128), (2, 128, 128), (1, 128, 128), (1, 256, 128)]  # 128-wide K stages
CONFIGS += [(2, 64, 0, 2), (2, 128, 0, 2), (1, 128, 0, 2), (1, 256, 0, 2)]  # CTA-pair (M=256) tiles


@pytest.mark.parametrize("cfg", CONFIGS)
@pytest.mark.parametrize("m,n,k,l", SHAPES)
def test_tile_configs_ragged(cuda, cfg, m, n, k, l):
    order, bn = cfg[0], cfg[1]
    stage_k = cfg[2] if len(cfg) > 2 else 0
    pair = cfg[3] if len(cfg) > 3 else 0
    data = inputs.generate_input(m, n, k, l, seed=7)
    got = _run_dense(data, opt=_native.options(operand_order=order, tile_n=bn, stage_k=stage_k,
                                               cta_pair=pair))
    assert_close(got, dense_expected(data), f"order={order} bn={bn} {m}x{n}x{k}x{l}")


# stream-K (fp32 partials of split tiles reduced by the CTA holding k-step 0): forced on and
# off, down to one tile over many CTAs, ragged edges, a partial last k-stage, batches
SK_SHAPES = [(64, 128, 2048, 1), (100, 300, 1088, 1), (128, 4096, 7168, 1), (64, 14336, 4096, 1),
             (200, 100, 1280, 2), (1, 64, 4096, 1)]


@pytest.mark.parametrize("bn", [64, 128])
@pytest.mark.parametrize("sk", [1, 2])
@pytest.mark.parametrize("m,n,k,l", SK_SHAPES)
def test_stream_k(cuda, bn, sk, m, n, k, l):
    data = inputs.generate_input(m, n, k, l, seed=11)
    got = _run_dense(data, opt=_native.options(operand_order=2, tile_n=bn, stream_k=sk))
    assert_close(got, dense_expected(data), f"stream_k={sk} bn={bn} {m}x{n}x{k}x{l}")


def test_stream_k_max_ctas_and_repeat(cuda):
    data = inputs.generate_input(128, 512, 4096, 1, seed=13)
    exp = dense_expected(data)
    for ctas in (5, 37, 148):
        opt = _native.options(operand_order=2, tile_n=128, stream_k=2, max_ctas=ctas)
        first = _run_dense(data, opt=opt).copy()
        assert_close(first, exp, f"max_ctas={ctas}")
        assert np.array_equal(first.view(np.uint16), _run_dense(data, opt=opt).view(np.uint16))


def test_guard_bands_untouched(cuda):
    m, n, k = 200, 264, 512
    data = list(inputs.generate_input(m, n, k, 1, seed=3))
    pad = 4096
    buf = torch.full((m * n + 2 * pad,), 12345.0, dtype=torch.float16, device="cuda")
    c = buf[pad:pad + m * n].view(m, n, 1)
    data[6] = c
    got = _run_dense(tuple(data))
    assert_close(got, dense_expected(data), "guard")
    assert torch.all(buf[:pad] == 12345.0) and torch.all(buf[pad + m * n:] == 12345.0)


def test_overwrites_c_and_repeats_bitwise(cuda):
    data = inputs.generate_input(256, 1024, 2048, 1, seed=5)
    first = _run_dense(data).copy()
    data[6].fill_(float("nan"))
    second = _run_dense(data)
    assert np.array_equal(first.view(np.uint16), second.view(np.uint16))


def test_timeout_sets_status_and_context_survives(cuda):
    data = inputs.generate_input(128, 256, 512, 1, seed=1)
    a, b, _, _, sfa, sfb, c = data
    _native.status_reset()
    opt = _native.options(timeout_ns=50_000_000, debug=1)
    gemm.launch(a, b, sfa, sfb, c, 128, 256, 512, 1, opt=opt)
    torch.cuda.synchronize()
    st = _native.status()
    assert st in (2, 3), st
    _native.status_reset()
    got = _run_dense(data)
    assert_close(got, dense_expected(data), "after timeout")


def test_timeout_in_callers_status_word(cuda):
    """opt.dev_status: the call's device-side error lands in the caller's own word and the
    per-device word stays clear."""
    data = inputs.generate_input(128, 256, 512, 1, seed=1)
    a, b, _, _, sfa, sfb, c = data
    _native.status_reset()
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    opt = _native.options(timeout_ns=50_000_000, debug=1, dev_status=word.data_ptr())
    gemm.launch(a, b, sfa, sfb, c, 128, 256, 512, 1, opt=opt)
    torch.cuda.synchronize()
    assert int(word.item()) in (2, 3)
    assert _native.status() == 0
    got = _run_dense(data)
    assert_close(got, dense_expected(data), "after timeout")


def _grouped_expected(gdata, rows=None):
    outs = []
    for i, ((a, b, _), (sa, sb)) in enumerate(zip(gdata[0], gdata[1])):
        a_u, b_u = u8(a[:, :, 0].contiguous()), u8(b[:, :, 0].contiguous())
        sa_u, sb_u = u8(sa[:, :, 0].cpu().contiguous()), u8(sb[:, :, 0].cpu().contiguous())
        if rows is not None:
            a_u, sa_u = a_u[:rows], sa_u[:rows]
        outs.append(orc.grouped_gemm_ref([(a_u, b_u, sa_u, sb_u)], dtype=np.float32)[0])
    return outs


def _run_grouped(gdata, opt=None):
    outs = group_gemm.custom_kernel(gdata, opt=opt)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return [c[:, :, 0].cpu().numpy() for c in outs]


# kernels/group_gemm/profile_group_gemm.py:42-83
REF_GROUP_CASES = [
    ([96, 128], [128, 256], [256, 512]),
    ([256, 72], [512, 384], [256, 256]),
    ([128, 128], [128, 256], [512, 256]),
    ([80, 128, 256], [384, 256, 128], [256, 512, 256]),
    ([80, 176, 128, 72, 64, 248, 96, 160], [4096] * 8, [7168] * 8),
    ([40, 76, 168, 72, 164, 148, 196, 160], [7168] * 8, [2048] * 8),
    ([192, 320], [3072] * 2, [4096] * 2),
    ([128, 384], [4096] * 2, [1536] * 2),
]


@pytest.mark.parametrize("bn,stage_k,pair", [(64, 0, 0), (128, 0, 0), (192, 0, 0), (256, 0, 0),
                                             (128, 128, 0), (128, 0, 2), (256, 0, 2)])
@pytest.mark.parametrize("order", [0, 1])
@pytest.mark.parametrize("case", range(len(REF_GROUP_CASES)))
def test_reference_group_cases(cuda, case, order, bn, stage_k, pair):
    if order == 1 and not ((bn == 256 and stage_k == 0) or (bn == 128 and stage_k == 0 and pair == 0)):
        pytest.skip("tokens-on-M grouped kernel is built for tile_n 128 and 256 (pair: 256)")
    m, n, k = REF_GROUP_CASES[case]
    gdata = inputs.generate_group_input(m, n, k, len(m), seed=1111)
    got = _run_grouped(gdata, opt=_native.options(tile_n=bn, stage_k=stage_k, cta_pair=pair,
                                                  operand_order=order))
    for g, (x, e) in enumerate(zip(got, _grouped_expected(gdata))):
        assert_close(x, e, f"case {case} group {g}")


@pytest.mark.parametrize("pair,order", [(0, 0), (2, 0), (0, 1), (2, 1)])
def test_grouped_config3(cuda, pair, order):
    ms = inputs.uniform_group_sizes(8, seed=1111)
    gdata = inputs.generate_quantized_group_input(ms, 4096, 7168, seed=1111)
    got = _run_grouped(gdata, opt=_native.options(cta_pair=pair, tile_n=256 if (pair or order) else 0,
                                                  operand_order=order))
    for g, (x, e) in enumerate(zip(got, _grouped_expected(gdata))):
        assert_close(x, e, f"c3 group {g}")


def test_grouped_config4a_sampled(cuda):
    ms = inputs.zipf_group_sizes(64, 32768)
    gdata = inputs.generate_quantized_group_input(ms, 2048, 7168, seed=1111)
    got = _run_grouped(gdata)
    for g, ((a, b, _), (sa, sb)) in enumerate(zip(gdata[0], gdata[1])):
        if ms[g] == 0:
            continue
        rows = spread_rows(ms[g], block=128)
        e = orc.grouped_gemm_ref([(u8(a[:, :, 0])[rows], u8(b[:, :, 0]),
                                   u8(sa[:, :, 0].contiguous())[rows],
                                   u8(sb[:, :, 0].contiguous()))], dtype=np.float32)[0]
        assert_close(got[g][rows], e, f"c4a group {g}")


@pytest.mark.parametrize("order", [0, 1])
def test_grouped_pairs_past_the_edge(cuda, order):
    """CTA pairs whose second CTA lies wholly past the 128-row side: groups of 16..128 tokens
    (tokens on that side) and B_g of 384 rows (B_g on that side)."""
    ms = [16, 48, 128, 130, 0, 272]
    gdata = inputs.generate_group_input(ms, [384] * 6, [512] * 6, 6, seed=21)
    got = _run_grouped(gdata, opt=_native.options(tile_n=256, cta_pair=2, operand_order=order))
    for g, (x, e) in enumerate(zip(got, _grouped_expected(gdata))):
        assert_close(x, e, f"order {order} group {g}")


def test_grouped_empty_groups_and_reuse(cuda):
    ms = [0, 64, 0, 130]
    gdata = inputs.generate_group_input(ms, [256, 256, 256, 384], [512] * 4, 4, seed=9)
    got1 = _run_grouped(gdata)
    got2 = _run_grouped(gdata)  # cached device table
    for g, (x, y, e) in enumerate(zip(got1, got2, _grouped_expected(gdata))):
        assert_close(x, e, f"group {g}")
        assert np.array_equal(x.view(np.uint16), y.view(np.uint16))


def test_oracle_matches_scaled_mm(cuda):
    """Pins the oracle (and nibble order) to the reference's own ref_kernel call:
    torch._scaled_mm on to_blocked scales (kernels/gemm/reference.py:44-51)."""
    m, n, k = 256, 384, 1024
    data = inputs.generate_input(m, n, k, 1, seed=1111)
    a, b, sfa, sfb = data[:4]
    sa = torch.from_numpy(orc.to_blocked(u8(sfa[:, :, 0].contiguous()))).cuda().view(torch.float8_e4m3fn)
    sb = torch.from_numpy(orc.to_blocked(u8(sfb[:, :, 0].contiguous()))).cuda().view(torch.float8_e4m3fn)
    try:
        ref = torch._scaled_mm(a[:, :, 0], b[:, :, 0].transpose(0, 1), sa, sb, bias=None,
                               out_dtype=torch.float16)
    except Exception as e:  # pragma: no cover
        pytest.skip(f"torch._scaled_mm fp4 unavailable: {e}")
    ref = ref.cpu().numpy()[None]
    assert_close(dense_expected(data), ref, "oracle vs _scaled_mm")
    assert_close(_run_dense(data), ref, "kernel vs _scaled_mm")
