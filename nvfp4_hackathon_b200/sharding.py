"""Multi-GPU partitioning for configs[4] of the benchmark (one process per GPU).

* Grouped GEMM (configs[4a]): experts are independent, so they are split across
  ranks with no collective on the compute path.  ``plan_expert_shards`` cuts
  experts larger than the per-rank token share into row ranges (rows of A_g are
  independent; the B_g of a split expert is read by every rank that holds a
  piece) and assigns pieces longest-processing-time-first under a cost model of
  MMA time per token plus weight-load time per expert.
* Dense GEMM (configs[4b]): each rank owns a contiguous block of N columns of B
  and C; A is replicated.  When every rank wants the whole C, ``gemm_allgather``
  fuses the all-gather into the GEMM: each rank's epilogue stores its tiles into
  every rank's full C (opened through CUDA IPC, ``PeerBuffers``) over NVLink, and
  one tiny all-reduce orders the reads after all ranks' kernels.
  ``gather_columns`` is the unfused alternative (one NCCL all-gather + re-interleave).

The reference has no multi-GPU code; this module is the B200 build's own.
"""
from __future__ import annotations

import ctypes
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


class PeerBuffers:
    """Every rank's copy of one full-size buffer, usable from this process.

    ``ptrs[r]`` is the device address of rank r's buffer (this rank's own tensor for r ==
    rank, a CUDA IPC mapping of the peer's allocation otherwise).  Collective: every rank
    constructs it with a tensor of the same shape, in the same order.
    """

    def __init__(self, tensor, dist):
        from . import _native
        self._lib = lib = _native.load()
        rank, world = dist.get_rank(), dist.get_world_size()
        hsize = lib.nvfp4_ipc_handle_size()
        buf = ctypes.create_string_buffer(hsize)
        off = ctypes.c_ulonglong()
        _native.check(lib.nvfp4_ipc_get_handle(tensor.data_ptr(), buf, ctypes.byref(off)),
                      "nvfp4_ipc_get_handle")
        handles = [None] * world
        dist.all_gather_object(handles, (buf.raw, off.value))
        self.tensor = tensor
        self.ptrs, self._opened = [], []
        for r, (h, o) in enumerate(handles):
            if r == rank:
                self.ptrs.append(tensor.data_ptr())
                continue
            p = ctypes.c_void_p()
            _native.check(lib.nvfp4_ipc_open_handle(ctypes.create_string_buffer(h, hsize), ctypes.byref(p)),
                          "nvfp4_ipc_open_handle")
            self._opened.append(p.value)
            self.ptrs.append(p.value + o)

    def close(self):
        for p in self._opened:
            self._lib.nvfp4_ipc_close(p)
        self._opened = []


def gemm_allgather(data, peers: PeerBuffers, col_lo: int, n_full: int, stream=None) -> None:
    """C[:, col_lo : col_lo + n] of every rank's full (M, n_full) fp16 buffer = this rank's
    A @ B_shard^T, in one kernel: the epilogue stores each tile to all ranks' buffers.

    ``data`` is this rank's 7-tuple (L = 1; B holds the rank's n columns); its c is unused.
    The peers may read their buffers only after every rank's kernel: follow with a
    stream-ordered collective (``dist.all_reduce`` of a 1-element tensor) or a barrier.
    The kernel also writes into every peer's buffer, so when peers read their C between
    two calls, order each call after those reads as well (the same collective or barrier
    before the call): otherwise the next call's stores race with a peer still reading.
    """
    import torch
    from . import _native
    a, b, _, _, sfa_p, sfb_p, _ = data
    m, kb, l = a.shape
    if l != 1:
        raise ValueError("gemm_allgather needs L == 1")
    n = b.shape[0]
    outs = (ctypes.c_void_p * len(peers.ptrs))(*[p + 2 * col_lo for p in peers.ptrs])
    s = torch.cuda.current_stream().cuda_stream if stream is None else stream
    rc = peers._lib.nvfp4_gemm_multi(a.data_ptr(), b.data_ptr(), sfa_p.data_ptr(), sfb_p.data_ptr(),
                                     outs, len(peers.ptrs), n_full, m, n, 2 * kb, s)
    _native.check(rc, "nvfp4_gemm_multi")
