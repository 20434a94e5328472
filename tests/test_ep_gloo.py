"""Expert parallelism over gloo ranks on the CPU: the dispatch / combine
exchange of vxmoe.ep with the CPU oracle as the compute backend.  Checks the
block output of every rank against the single-process oracle, and that a rank
which fails mid-step ends its peer's collective with an error (a short
process-group timeout) instead of hanging it."""
from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import traceback

import numpy as np
import pytest
import torch

import vxmoe_oracle as O

E, D, I, K = 16, 128, 64, 4


class OracleBackend:
    """The EP backend interface on the CPU oracle (bf16 values in torch
    tensors; the kernels' arithmetic restated)."""

    def __init__(self, p, rank, world, fail_in_experts=False):
        self.p, self.rank, self.El = p, rank, p.num_experts // world
        self.fail = fail_in_experts

    def route(self, x, num_experts):
        xn = x.float().numpy()
        r = O.router(xn, self.p.router_w, self.p.top_k)
        _, sg = O.shared_parts(xn, self.p)
        return (torch.from_numpy(r.inds.astype(np.int32)), torch.from_numpy(r.weights).to(torch.bfloat16),
                torch.from_numpy(sg[:, 0]).to(torch.bfloat16))

    def experts_partial(self, xr, ids, scores):
        if self.fail:
            raise RuntimeError("injected failure in the expert pass")
        xn, idn, sc = xr.float().numpy(), ids.numpy(), scores.float().numpy()
        out = np.zeros((xn.shape[0], D), np.float32)
        for r in range(xn.shape[0]):
            acc = np.zeros(D, np.float32)
            for s in range(idn.shape[1]):
                if idn[r, s] < 0:
                    continue
                e = self.rank * self.El + int(idn[r, s])
                y = O.expert_mlp_bf16(xn[r:r + 1], self.p.gate.expert(e), self.p.up.expert(e),
                                      self.p.down.expert(e))[3][0]
                acc = (acc + (y * sc[r, s]).astype(np.float32)).astype(np.float32)
            out[r] = acc
        return torch.from_numpy(out)

    def shared(self, x, num_experts):
        shared, _ = O.shared_parts(x.float().numpy(), self.p)
        return torch.from_numpy(shared).to(torch.bfloat16)


def _worker(rank, world, port, q, fail_rank, mode="capacity"):
    try:
        import torch.distributed as dist
        from vxmoe.ep import ExpertParallelMoE
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=8))
        p = O.make_params(seed=3, experts=E, hidden=D, inter=I, shared_inter=I, top_k=K)
        backend = OracleBackend(p, rank, world, fail_in_experts=(rank == fail_rank))

        class _Shard:
            top_k = K

        ep = ExpertParallelMoE(_Shard(), E, backend=backend)
        if mode == "counts":
            ep.capacity_max_tokens = 0          # force the count-based exchange
        x = O.make_x(100 + rank, 6, D)
        y = ep(torch.from_numpy(x).to(torch.bfloat16))
        q.put((rank, "ok", y.float().numpy(), x, ep.last_stats))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the test, never swallowed
        q.put((rank, "error", repr(exc), traceback.format_exc(), None))


def _run(world, port, fail_rank=-1, timeout=120, mode="capacity"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank, mode)) for r in range(world)]
    for pr in procs:
        pr.start()
    out = {}
    for _ in range(world):
        rank, status, a, b, c = q.get(timeout=timeout)
        out[rank] = (status, a, b, c)
    for pr in procs:
        pr.join(timeout=30)
        if pr.is_alive():
            pr.kill()
    return out


@pytest.mark.parametrize("mode,port", [("capacity", 29631), ("counts", 29636)])
def test_ep_two_ranks_matches_single_process_oracle(mode, port):
    out = _run(2, port, mode=mode)
    p = O.make_params(seed=3, experts=E, hidden=D, inter=I, shared_inter=I, top_k=K)
    for rank in range(2):
        status, y, x, stats = out[rank]
        assert status == "ok", x
        assert stats["mode"] == mode
        ref = O.moe_block(x, p).y
        assert O.normwise_error(y, ref) < 1e-2
        assert np.mean(O.bf16_bits(y) == O.bf16_bits(ref)) > 0.95
        if mode == "counts":
            assert sum(stats["send_counts"]) == stats["sent_rows"]
            assert stats["sent_rows"] <= 6 * 2      # one row per (token, destination)


def test_ep_exchange_modes_agree_bit_for_bit():
    a = _run(2, 29646, mode="capacity")
    b = _run(2, 29651, mode="counts")
    for rank in range(2):
        np.testing.assert_array_equal(O.bf16_bits(a[rank][1]), O.bf16_bits(b[rank][1]))


def test_ep_failing_rank_does_not_hang_its_peer():
    out = _run(2, 29641, fail_rank=1)
    assert out[1][0] == "error" and "injected failure" in out[1][1]
    assert out[0][0] == "error"      # the peer's next collective ended with an error
