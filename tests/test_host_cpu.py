"""Host-side logic without a GPU: group sizes, the multi-GPU shard planner and the
NCCL-free parts of the column gather (run with gloo ranks on the CPU)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nvfp4_hackathon_b200 import inputs, sharding


def test_zipf_sizes_sum_and_alignment():
    ms = inputs.zipf_group_sizes(64, 32768)
    assert sum(ms) == 32768 and all(m % 16 == 0 for m in ms)
    assert ms == sorted(ms, reverse=True) and ms[0] > 8 * ms[-1]


def test_uniform_sizes_range():
    ms = inputs.uniform_group_sizes(8, 1111)
    assert len(ms) == 8 and all(64 <= m <= 1024 and m % 64 == 0 for m in ms)
    assert ms == inputs.uniform_group_sizes(8, 1111)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_expert_plan_covers_every_token_once_and_balances(world):
    ms = inputs.zipf_group_sizes(64, 32768)
    plan = sharding.plan_expert_shards(ms, world)
    cover = {}
    for shard in plan:
        for e, lo, hi in shard:
            assert lo % 16 == 0 and hi > lo
            cover.setdefault(e, []).append((lo, hi))
    for e, m in enumerate(ms):
        ranges = sorted(cover.get(e, []))
        assert sum(hi - lo for lo, hi in ranges) == m
        pos = 0
        for lo, hi in ranges:
            assert lo == pos
            pos = hi
    costs = sharding.plan_costs(plan)
    assert max(costs) / min(costs) < 1.1


def test_column_shards_partition_n():
    for n, world in [(28672, 8), (28672, 3), (1000, 4)]:
        cols = []
        for r in range(world):
            lo, hi = sharding.column_shard(n, world, r)
            cols += list(range(lo, hi))
        assert cols == list(range(n))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, n, m):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = sharding.column_shard(n, world, rank)
    full = torch.arange(m * n, dtype=torch.float32).reshape(m, n)
    shard = full[:, lo:hi].contiguous()
    lo0, hi0 = sharding.column_shard(n, world, 0)
    gathered = torch.empty((world, m, hi0 - lo0), dtype=torch.float32)
    sharding.gather_columns(shard, gathered, dist)
    assert torch.equal(sharding.assemble_columns(gathered, n, world), full)
    dist.destroy_process_group()


def test_column_gather_two_ranks_gloo():
    mp.spawn(_gather_worker, args=(2, _free_port(), 1000, 3), nprocs=2, join=True)


def test_grouped_tile_choice():
    from nvfp4_hackathon_b200 import group_gemm
    c3 = [(m, 4096, 7168, 1) for m in inputs.uniform_group_sizes(8, 1111)]
    c4a = [(m, 2048, 7168, 1) for m in inputs.zipf_group_sizes(64, 32768)]
    assert group_gemm.choose_tile_n(c3, 148) == 192
    assert group_gemm.choose_tile_n(c4a, 148) == 256
    assert group_gemm.choose_tile_n([(0, 4096, 7168, 1)], 148) in (128, 192, 256)
