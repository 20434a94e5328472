"""Expert parallelism on the CUDA path.  One rank: dispatch to itself must
reproduce moe_block bit for bit (the same float32 slot-order sum, one
rounding), over the peer-memory transport and over NCCL, eagerly and as a
replayed CUDA graph; a dispatch wait that nothing satisfies runs out and
reports it instead of hanging.  Two ranks (when two GPUs are present): the
two transports agree bit for bit, and each rank's output is within the block
tolerance of the single-GPU block on the full weights."""
from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import traceback

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _weights(dev, E=64, d=512, I=256, top_k=8):
    import vxmoe
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    return vxmoe.MoEWeights.random(E, d, I, I, top_k, device=dev, generator=g)


def _bits(t):
    return t.view(torch.int16).cpu().numpy()


def _init_single(port):
    import torch.distributed as dist
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    return dist, dev


@pytest.mark.parametrize("transport,packed", [("p2p", False), ("p2p", True),
                                              ("collective", False)])
def test_ep_single_rank_equals_block(transport, packed):
    import vxmoe
    from vxmoe import ep as E
    dist, dev = _init_single(29653)
    try:
        w = _weights(dev)
        shard = E.shard_weights(w, 0, 1)
        if packed:
            w.pack()
            shard.pack()
        layer = E.ExpertParallelMoE(shard, w.num_experts, transport=transport)
        for T in (1, 5, 64, 256):
            x = torch.randn((T, w.hidden), device=dev).to(torch.bfloat16)
            y = layer(x)
            # the expert-parallel step runs the multi-kernel pipeline; the block
            # runs batches of at most four tokens as the single cooperative
            # launch (another float32 summation order), so its reference here
            # is the block with the grouped GEMV kernels forced
            old = w.expert_path
            if T <= 4:
                w.expert_path = vxmoe._lib.PATH_GEMV
            try:
                ref = vxmoe.moe_block(x, w)
            finally:
                w.expert_path = old
            torch.cuda.synchronize()
            np.testing.assert_array_equal(_bits(y), _bits(ref))
        if layer.exchange is not None:
            assert layer.exchange.errors() == 0
    finally:
        E.close_exchanges()
        dist.destroy_process_group()


def test_ep_p2p_prefill_capacity_equals_block():
    """A capacity above the decode default carries a prefill-sized batch over
    the peer transport (the tcgen05 GEMM pipeline on the received rows)."""
    import vxmoe
    from vxmoe import ep as E
    dist, dev = _init_single(29656)
    try:
        w = _weights(dev)
        shard = E.shard_weights(w, 0, 1)
        w.pack()
        shard.pack()
        layer = E.ExpertParallelMoE(shard, w.num_experts, transport="p2p", capacity=1024)
        for T in (300, 700):
            x = torch.randn((T, w.hidden), device=dev).to(torch.bfloat16)
            y = layer(x)
            ref = vxmoe.moe_block(x, w)
            torch.cuda.synchronize()
            assert layer.last_stats["mode"] == "p2p"
            np.testing.assert_array_equal(_bits(y), _bits(ref))
        assert layer.exchange.errors() == 0
    finally:
        E.close_exchanges()
        dist.destroy_process_group()


def test_ep_p2p_graph_replay_equals_eager():
    from vxmoe import ep as E
    dist, dev = _init_single(29654)
    try:
        w = _weights(dev)
        layer = E.ExpertParallelMoE(E.shard_weights(w, 0, 1), w.num_experts, transport="p2p")
        g = E.GraphedExpertParallel(layer, 24)
        for seed in (1, 2, 3):
            torch.manual_seed(seed)
            x = torch.randn((24, w.hidden), device=dev).to(torch.bfloat16)
            ref = layer(x).clone()
            y = g(x).clone()
            torch.cuda.synchronize()
            np.testing.assert_array_equal(_bits(y), _bits(ref))
        assert layer.exchange.errors() == 0
        del g
    finally:
        E.close_exchanges()
        dist.destroy_process_group()


def test_ep_p2p_wait_without_dispatch_runs_out():
    """The experts' wait for a dispatch that never comes gives up after the
    exchange's bound and sets bit 0 of the error word; the GPU stays usable."""
    from vxmoe import ep as E
    dist, dev = _init_single(29655)
    try:
        w = _weights(dev)
        shard = E.shard_weights(w, 0, 1)
        ex = E.PeerExchange(None, 16, w.hidden, w.top_k, w.num_experts, dev, wait_ns=20_000_000)
        ex.experts(8, shard)          # no dispatch: flag_dispatch stays at 0
        torch.cuda.synchronize()
        assert ex.errors() & 1
        x = torch.ones(4, device=dev)
        assert float((x * 2).sum().item()) == 8.0
        ex.close()
    finally:
        dist.destroy_process_group()


def _worker(rank, port, q):
    try:
        import torch.distributed as dist
        import vxmoe
        from vxmoe import ep as E
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", rank=rank, world_size=2,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        w = _weights(dev)
        shard = E.shard_weights(w, rank, 2)
        p2p = E.ExpertParallelMoE(shard, w.num_experts, transport="p2p")
        coll = E.ExpertParallelMoE(shard, w.num_experts, transport="collective")
        g = torch.Generator(device=dev)
        g.manual_seed(100 + rank)
        worst, same_min, agree = 0.0, 1.0, True
        for T in (1, 32, 200):
            x = torch.randn((T, w.hidden), device=dev, generator=g).to(torch.bfloat16)
            y = p2p(x)
            yc = coll(x)
            ref = vxmoe.moe_block(x, w)
            torch.cuda.synchronize()
            agree &= bool(np.array_equal(_bits(y), _bits(yc)))
            yn, rn = y.float().cpu().numpy(), ref.float().cpu().numpy()
            worst = max(worst, float(np.max(np.abs(yn - rn)) / np.max(np.abs(rn))))
            same_min = min(same_min, float(np.mean(_bits(y) == _bits(ref))))
        graphed = E.GraphedExpertParallel(p2p, 32)
        x = torch.randn((32, w.hidden), device=dev, generator=g).to(torch.bfloat16)
        eager = p2p(x).clone()
        replay = graphed(x).clone()
        torch.cuda.synchronize()
        agree &= bool(np.array_equal(_bits(eager), _bits(replay)))
        errors = p2p.exchange.errors()
        del graphed
        E.close_exchanges()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", (worst, same_min, agree, errors), ""))
    except Exception as exc:
        q.put((rank, "error", repr(exc), traceback.format_exc()))


def _worker_c4(rank, port, q):
    """The C4 shape on two ranks: production width (512 experts, d = 2048,
    I = 512, top-10) on the packed pool, 2,048 tokens per rank, so each
    shard's experts run the tcgen05 GEMM; the peer transport sized for the
    whole batch.  Compared with the single-GPU block on the full weights."""
    try:
        import torch.distributed as dist
        import vxmoe
        from vxmoe import ep as E
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", rank=rank, world_size=2,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        w = _weights(dev, E=512, d=2048, I=512, top_k=10)
        w.pack()
        shard = E.shard_weights(w, rank, 2)
        shard.pack()
        ep = E.ExpertParallelMoE(shard, w.num_experts, transport="p2p", capacity=2048)
        g = torch.Generator(device=dev)
        g.manual_seed(300 + rank)
        x = torch.randn((2048, w.hidden), device=dev, generator=g).to(torch.bfloat16)
        y = ep(x)
        ref = vxmoe.moe_block(x, w)
        torch.cuda.synchronize()
        yn, rn = y.float().cpu().numpy(), ref.float().cpu().numpy()
        worst = float(np.linalg.norm(yn - rn) / np.linalg.norm(rn))
        same = float(np.mean(_bits(y) == _bits(ref)))
        errors = ep.exchange.errors()
        E.close_exchanges()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", (worst, same, errors), ""))
    except Exception as exc:
        q.put((rank, "error", repr(exc), traceback.format_exc()))


def _run_two(target, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_ep_two_gpus_c4_shape_match_single_gpu_block():
    for rank, status, a, b in _run_two(_worker_c4, 29671):
        assert status == "ok", b
        worst, same, errors = a
        assert errors == 0, f"rank {rank}: a wait ran out ({errors})"
        # the same per-expert GEMMs and the same slot-order combine: almost every bit
        assert worst < 1e-3, f"rank {rank} normwise difference {worst}"
        assert same > 0.95, f"rank {rank} only {same:.3f} identical"


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
        worst, same, agree, errors = a
        assert errors == 0, f"rank {rank}: a wait ran out ({errors})"
        assert agree, f"rank {rank}: p2p and NCCL transports (or graph replay) differ"
        assert worst < 1e-2, f"rank {rank} normwise error {worst}"
        assert same > 0.95, f"rank {rank} only {same:.3f} identical"
