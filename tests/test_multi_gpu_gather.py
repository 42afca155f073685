"""Fused N-sharded GEMM + all-gather over NVLink (nvfp4_gemm_multi with peer buffers opened
through CUDA IPC) on 2 GPUs: every rank's full C must equal the single-GPU GEMM of the whole
problem.  Skipped on boxes with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, m, n, k, q):
    import torch.distributed as dist
    from nvfp4_hackathon_b200 import gemm, inputs, sharding
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        full = inputs.generate_quantized_input(m, n, k, 1, seed=17, device="cuda")
        ref = gemm.custom_kernel(full)[:, :, 0].clone()
        lo, hi = sharding.column_shard(n, world, rank)
        a, b, sfa, sfb, _, _, _ = full
        b_r, sfb_r = b[lo:hi].contiguous(), sfb[lo:hi].contiguous()
        from nvfp4_hackathon_b200.layout import permute_sf
        shard = (a, b_r, sfa, sfb_r, full[4], permute_sf(sfb_r), None)
        c_full = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
        peers = sharding.PeerBuffers(c_full, dist)
        for _ in range(2):  # twice: the second call overwrites in place
            sharding.gemm_allgather(shard, peers, lo, n)
            token = torch.zeros(1, device="cuda")
            dist.all_reduce(token)
        torch.cuda.synchronize()
        ok = torch.equal(c_full, ref)
        peers.close()
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gemm_allgather_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    m, n, k = 256, 1024, 512
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, m, n, k, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}
