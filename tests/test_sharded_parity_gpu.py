"""Parity of the multi-GPU partitions, run on ONE GPU: every rank's shard is computed in
turn on cuda:0 and the reassembled output is compared with the CPU oracle.

* configs[4b]: the dense GEMM M=16384, N=28672, K=8192 split into P column shards
  (``sharding.column_shard``, P = 2, 4, 8); shard r computes C[:, lo:hi] from B[lo:hi]
  and its scales, and ``assemble_columns`` puts the shards back in column order.
* configs[4a]: the G=64 Zipf expert GEMM split by ``sharding.plan_expert_shards``
  (P = 2, 4, 8); a split expert's row pieces write straight into that expert's C.

The oracle (``oracle/nvfp4_oracle.py``: the reference's ref_kernel semantics,
kernels/gemm/reference.py:27-53) runs on sampled rows spread over every 128-row
M block (all of it would take minutes on the host).
"""
import numpy as np
import pytest
import torch

from nvfp4_hackathon_b200 import _native, gemm, group_gemm, inputs, sharding
from nvfp4_hackathon_b200.layout import permute_sf
from oracle import nvfp4_oracle as orc
from tests.helpers import assert_close, spread_rows, u8

pytestmark = pytest.mark.gpu


def _dense_shard(data, lo, hi):
    a, b, sfa, sfb, sfa_p, _, c = data
    m = a.shape[0]
    sfb_s = sfb[lo:hi]
    c_s = torch.full((m, hi - lo, 1), float("nan"), dtype=torch.float16, device=c.device)
    return (a, b[lo:hi], sfa, sfb_s, sfa_p, permute_sf(sfb_s), c_s)


def test_config4b_column_shards_reassembled(cuda):
    m, n, k = 16384, 28672, 8192
    data = inputs.generate_quantized_input(m, n, k, 1, seed=4242)
    rows = spread_rows(m)
    a, b, sfa, sfb = data[:4]
    exp = orc.gemm_ref(u8(a[:, :, 0])[rows][None], u8(b[:, :, 0])[None],
                       u8(sfa.cpu().contiguous())[rows], u8(sfb.cpu().contiguous()), dtype=np.float32)
    rows_t = torch.from_numpy(rows).to(a.device)
    for world in (2, 4, 8):
        lo0, hi0 = sharding.column_shard(n, world, 0)
        gathered = torch.zeros((world, len(rows), hi0 - lo0), dtype=torch.float16, device=a.device)
        for r in range(world):
            lo, hi = sharding.column_shard(n, world, r)
            shard = _dense_shard(data, lo, hi)
            c_s = gemm.custom_kernel(shard)
            torch.cuda.synchronize()
            _native.raise_on_device_error()
            gathered[r, :, : hi - lo] = c_s[rows_t, :, 0]
            del shard, c_s
        full = sharding.assemble_columns(gathered, n, world)
        assert tuple(full.shape) == (len(rows), n)
        assert_close(full.cpu().numpy()[None], exp, f"c4b P={world}")


def test_config4a_expert_plan_reassembled(cuda):
    n, k = 2048, 7168
    ms = inputs.zipf_group_sizes(64, 32768)
    gdata = inputs.generate_quantized_group_input(ms, n, k, seed=4343)
    abc, sf, sfp, sizes = gdata
    samples, exp = {}, {}
    for e, m in enumerate(ms):
        if m == 0:
            continue
        a, b, _ = abc[e]
        sa, sb = sf[e]
        rows = spread_rows(m, block=128)
        samples[e] = rows
        exp[e] = orc.grouped_gemm_ref([(u8(a[:, :, 0])[rows], u8(b[:, :, 0]),
                                        u8(sa[:, :, 0].contiguous())[rows],
                                        u8(sb[:, :, 0].contiguous()))], dtype=np.float32)[0]
    for world in (2, 4, 8):
        plan = sharding.plan_expert_shards(ms, world, n=n, k=k)
        covered = {e: 0 for e in samples}
        for (a, b, c) in abc:
            c.fill_(float("nan"))
        for r in range(world):
            g_abc, g_sf, g_sfp, g_sizes = [], [], [], []
            for (e, lo, hi) in plan[r]:
                a, b, c = abc[e]
                sa, sb = sf[e]
                g_abc.append((a[lo:hi], b, c[lo:hi]))
                g_sf.append((sa[lo:hi], sb))
                g_sfp.append((permute_sf(sa[lo:hi]), sfp[e][1]))
                g_sizes.append((hi - lo, n, k, 1))
                covered[e] += hi - lo
            if g_abc:
                group_gemm.custom_kernel((g_abc, g_sf, g_sfp, g_sizes))
                torch.cuda.synchronize()
                _native.raise_on_device_error()
        assert all(covered[e] == ms[e] for e in samples)
        for e, rows in samples.items():
            got = abc[e][2][:, :, 0].cpu().numpy()[rows]
            assert_close(got, exp[e], f"c4a P={world} expert {e}")
