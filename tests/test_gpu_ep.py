"""Expert parallelism on the CUDA path (NCCL).  One rank: dispatch to itself
must reproduce moe_block bit for bit (the same float32 slot-order sum, one
rounding).  Two ranks (when two GPUs are present): each rank's output within
the block tolerance of the single-GPU block on the full weights."""
from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import traceback

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _weights(dev, E=64, d=512, I=256):
    import vxmoe
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    return vxmoe.MoEWeights.random(E, d, I, I, 8, device=dev, generator=g)


def test_ep_single_rank_equals_block():
    import torch.distributed as dist
    import vxmoe
    from vxmoe.ep import ExpertParallelMoE, shard_weights
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = "29653"
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        w = _weights(dev)
        ep = ExpertParallelMoE(shard_weights(w, 0, 1), w.num_experts)
        for T in (1, 5, 64):
            x = torch.randn((T, w.hidden), device=dev).to(torch.bfloat16)
            y = ep(x)
            ref = vxmoe.moe_block(x, w)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(y.view(torch.int16).cpu().numpy(),
                                          ref.view(torch.int16).cpu().numpy())
    finally:
        dist.destroy_process_group()


def _worker(rank, port, q):
    try:
        import torch.distributed as dist
        import vxmoe
        from vxmoe.ep import ExpertParallelMoE, shard_weights
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", rank=rank, world_size=2,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        w = _weights(dev)
        ep = ExpertParallelMoE(shard_weights(w, rank, 2), w.num_experts)
        g = torch.Generator(device=dev)
        g.manual_seed(100 + rank)
        x = torch.randn((32, w.hidden), device=dev, generator=g).to(torch.bfloat16)
        y = ep(x)
        ref = vxmoe.moe_block(x, w)
        torch.cuda.synchronize()
        yn, rn = y.float().cpu().numpy(), ref.float().cpu().numpy()
        err = float(np.max(np.abs(yn - rn)) / np.max(np.abs(rn)))
        same = float(np.mean(y.view(torch.int16).cpu().numpy() == ref.view(torch.int16).cpu().numpy()))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", err, same))
    except Exception as exc:
        q.put((rank, "error", repr(exc), traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_ep_two_gpus_match_single_gpu_block():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 29663, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, status, a, b in res:
        assert status == "ok", b
        assert a < 1e-2, f"rank {rank} normwise error {a}"
        assert b > 0.95, f"rank {rank} only {b:.3f} identical"
