"""CUDA-graph capture of every entry point (the way bench.py and a serving loop use them):
capture once, rewrite the inputs in place, replay, and compare with an eager call on the
same inputs.  The grouped call is also captured cold (its device table built inside the
capture), which replays a copy from the table's pinned host buffer."""
import pytest
import torch

from nvfp4_hackathon_b200 import _native, gemm, group_gemm, inputs
from nvfp4_hackathon_b200.quantize import quantize

pytestmark = pytest.mark.gpu


def _refill(dst_tuple, src_tuple):
    for d, s in zip(dst_tuple, src_tuple):
        if isinstance(d, torch.Tensor) and d.dtype != torch.float16 and d.dtype != torch.float32:
            d.view(torch.uint8).copy_(s.view(torch.uint8))


def _capture(fn, warm=True):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        if warm:
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


@pytest.mark.parametrize("m,n,k,opt", [
    (64, 1536, 2048, {}),
    (512, 2304, 1024, {}),
    (128, 1024, 4096, {"stream_k": 2}),
    (200, 640, 1024, {"out_dtype": 2}),
])
def test_dense_capture_replay(cuda, m, n, k, opt):
    data = list(inputs.generate_quantized_input(m, n, k, 1, seed=1))
    if opt.get("out_dtype") == 2:
        data[6] = torch.zeros((1, m, n), device="cuda", dtype=torch.float32).permute(1, 2, 0)
    data = tuple(data)
    o = _native.options(**opt) if opt else None
    g = _capture(lambda: gemm.custom_kernel(data, opt=o))
    fresh = inputs.generate_quantized_input(m, n, k, 1, seed=2)
    _refill(data, fresh)
    data[6].zero_()
    g.replay()
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    got = data[6].clone()
    data[6].zero_()
    gemm.custom_kernel(data, opt=o)
    torch.cuda.synchronize()
    assert torch.equal(got, data[6]), "replay differs from the eager call on the same inputs"


@pytest.mark.parametrize("warm", [True, False])
def test_grouped_capture_replay(cuda, warm):
    ms = [64, 320, 0, 128, 1024]
    data = inputs.generate_quantized_group_input(ms, 1024, 2048, seed=3)
    g = _capture(lambda: group_gemm.custom_kernel(data), warm=warm)
    fresh = inputs.generate_quantized_group_input(ms, 1024, 2048, seed=4)
    for (a, b, c), (fa, fb, _) in zip(data[0], fresh[0]):
        a.view(torch.uint8).copy_(fa.view(torch.uint8))
        b.view(torch.uint8).copy_(fb.view(torch.uint8))
        c.zero_()
    for (sa, sb), (fsa, fsb) in zip(data[2], fresh[2]):
        sa.view(torch.uint8).copy_(fsa.view(torch.uint8))
        sb.view(torch.uint8).copy_(fsb.view(torch.uint8))
    # churn the pinned host allocator: a freed table source would be handed out here
    junk = [torch.full((7 * len(ms),), -1, dtype=torch.int64).pin_memory() for _ in range(8)]
    g.replay()
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    got = [c.clone() for _, _, c in data[0]]
    for _, _, c in data[0]:
        c.zero_()
    group_gemm.custom_kernel(data)
    torch.cuda.synchronize()
    for i, (x, (_, _, c)) in enumerate(zip(got, data[0])):
        assert torch.equal(x, c), f"group {i}: replay differs from the eager call"
    del junk


def test_quantize_capture_replay(cuda):
    x = torch.randn((300, 1024), device="cuda", dtype=torch.bfloat16)
    out = {}

    def fn():
        out["r"] = quantize(x)
    g = _capture(fn)
    x.copy_(torch.randn_like(x) * 3)
    g.replay()
    torch.cuda.synchronize()
    codes, sf, perm = out["r"]
    e_codes, e_sf, e_perm = quantize(x)
    torch.cuda.synchronize()
    assert torch.equal(codes.view(torch.uint8), e_codes.view(torch.uint8))
    assert torch.equal(sf.view(torch.uint8), e_sf.view(torch.uint8))
    assert torch.equal(perm.view(torch.uint8), e_perm.view(torch.uint8))
