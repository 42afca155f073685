"""Multi-GPU partitioning for configs[4] of the benchmark (one process per GPU).

* Grouped GEMM (configs[4a]): experts are independent, so they are split across
  ranks with no collective on the compute path.  ``plan_expert_shards`` cuts
  experts larger than the per-rank token share into row ranges (rows of A_g are
  independent; the B_g of a split expert is read by every rank that holds a
  piece) and assigns pieces longest-processing-time-first under a cost model of
  MMA time per token plus weight-load time per expert.
* Dense GEMM (configs[4b]): each rank owns a contiguous block of N columns of B
  and C; A is replicated.  ``gather_columns`` assembles the column shards on
  every rank with one NCCL all-gather over NVLink when the caller wants them.

The reference has no multi-GPU code; this module is the B200 build's own.
"""
from __future__ import annotations

import math

# cost model (B200): fp4 MMA throughput and HBM bandwidth, used only for balancing
_FP4_FLOPS = 6.0e15
_HBM_BYTES = 6.5e12


def column_shard(n: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """[lo, hi) of the N columns owned by ``rank``: equal blocks rounded to ``align``."""
    per = math.ceil(n / world / align) * align
    lo = min(n, rank * per)
    hi = min(n, lo + per)
    return lo, hi


def expert_cost(tokens: int, n: int, k: int) -> float:
    """Seconds for one expert piece: MMA time of its tokens + load of B_g, A rows and C."""
    if tokens <= 0:
        return 0.0
    flops = 2.0 * tokens * n * k
    b_bytes = n * k // 2 + n * (k // 16)
    a_bytes = tokens * (k // 2 + k // 16 + 2 * n)
    return flops / _FP4_FLOPS + (b_bytes + a_bytes) / _HBM_BYTES


def plan_expert_shards(tokens_per_expert, world: int, n: int = 2048, k: int = 7168,
                       row_align: int = 16):
    """Assign experts (or row ranges of experts) to ranks.

    Returns ``plan[rank] = [(expert, row_lo, row_hi), ...]`` covering every token
    exactly once.  Empty experts are dropped.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    total = sum(int(t) for t in tokens_per_expert)
    share = max(row_align, math.ceil(total / world / row_align) * row_align)
    pieces = []
    for e, t in enumerate(tokens_per_expert):
        t = int(t)
        if t <= 0:
            continue
        n_pieces = max(1, math.ceil(t / share))
        step = math.ceil(t / n_pieces / row_align) * row_align
        lo = 0
        while lo < t:
            hi = min(t, lo + step)
            pieces.append((e, lo, hi))
            lo = hi
    pieces.sort(key=lambda p: (-expert_cost(p[2] - p[1], n, k), p[0], p[1]))
    load = [0.0] * world
    plan = [[] for _ in range(world)]
    for e, lo, hi in pieces:
        r = min(range(world), key=lambda i: (load[i], i))
        plan[r].append((e, lo, hi))
        load[r] += expert_cost(hi - lo, n, k)
    for r in range(world):
        plan[r].sort()
    return plan


def plan_costs(plan, n: int = 2048, k: int = 7168):
    return [sum(expert_cost(hi - lo, n, k) for _, lo, hi in shard) for shard in plan]


def gather_columns(c_shard, gathered, dist) -> None:
    """All-gather the (M, n_local) fp16 column shards into ``gathered`` (world, M, n_pad).

    Shards are zero-padded to equal width for the collective; rank r's columns
    are gathered[r, :, :hi - lo] (see ``assemble_columns``).
    """
    m, w = c_shard.shape
    n_pad = gathered.shape[2]
    if w == n_pad and c_shard.is_contiguous():
        src = c_shard
    else:
        import torch
        src = torch.zeros((m, n_pad), dtype=c_shard.dtype, device=c_shard.device)
        src[:, :w] = c_shard
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(gathered, src)  # one NCCL collective over NVLink
    else:  # gloo (CPU tests) has no all_gather_into_tensor
        dist.all_gather(list(gathered.unbind(0)), src)


def assemble_columns(gathered, n: int, world: int):
    """(world, M, n_pad) gathered shards -> (M, N) tensor in column order."""
    import torch
    parts = []
    for r in range(world):
        lo, hi = column_shard(n, world, r)
        if hi > lo:
            parts.append(gathered[r, :, : hi - lo])
    return torch.cat(parts, dim=1)
