"""Multi-GPU partitioning on real GPUs (NCCL): every rank computes its
contiguous (b*H+h, q-tile) unit range and the optional all-gather assembles
the output, which must equal the single-GPU result bit for bit (each unit's
arithmetic does not depend on the partition).  Needs 2 B200s; skipped
otherwise (the partition logic itself is covered by gloo tests on CPU).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPE = (1, 6, 1000, 128)


def _inputs():
    g = torch.Generator().manual_seed(5)
    q = torch.randn(SHAPE, generator=g).to(torch.bfloat16)
    k = (torch.randn(SHAPE, generator=g) + torch.randn(SHAPE[-1], generator=g) * 1.7).to(torch.bfloat16)
    v = torch.randn(SHAPE, generator=g).to(torch.bfloat16)
    return q, k, v


def _worker(rank, world, port, smooth, out_q):
    import torch.distributed as dist
    from datetime import timedelta
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from vc_b200 import parallel as P
        B, H, S, D = SHAPE
        q, k, v = (x.to(dev) for x in _inputs())
        s = P.shard(B, H, S, world, rank)
        local = P.sharded_attention(q, k, v, s, v_smooth=smooth)
        full = P.gather_rows(local, s, B, H, S)
        torch.cuda.synchronize()
        if rank == 0:
            from sageattention_local import sageattn_vc
            ref = sageattn_vc(q, k, v, v_smooth=smooth)
            out_q.put((rank, bool(torch.equal(full, ref)), float((full.float() - ref.float()).abs().max())))
        else:
            out_q.put((rank, True, 0.0))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:   # report instead of leaving the parent waiting
        out_q.put((rank, False, repr(e)))


@pytest.mark.parametrize("smooth", [False, True])
def test_two_gpu_shards_gather_to_the_single_gpu_result(smooth):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, smooth, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, ok, info = q.get(timeout=300)
        results[r] = (ok, info)
    for p in procs:
        p.join(timeout=120)
    assert all(ok for ok, _ in results.values()), results
