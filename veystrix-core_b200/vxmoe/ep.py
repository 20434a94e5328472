"""Expert parallelism for the routed MoE block across the GPUs of one node.

Each rank holds a contiguous shard of E/P routed experts plus the router and
the shared expert (replicated).  One step on every rank, for its own tokens:

1. route: bf16 logits, top-k ids, renormalised weights, shared gate;
2. dispatch: every token goes once to each rank that owns at least one of its
   experts (deduplicated per destination), with that rank's slot ids (local,
   -1 for slots served elsewhere) and the slot weights; a count exchange
   first, then NCCL all-to-all-v of the rows;
3. local experts: the received rows through this rank's grouped kernels,
   giving float32 partial sums over the rank's slots;
4. combine: partials return to the home rank (the reverse all-to-all), which
   adds them in rank order, rounds once and adds bf16(sg * shared), the same
   float32-then-bf16 contract as the single-GPU combine
   (models/flashnext/metal_runtime.py:315-334).

The reference runs on one Apple GPU and has no collective; this is the B200
scale-out of the same block.  The compute backend is injectable: the CUDA
backend runs the library's kernels; tests substitute a CPU backend so the
exchange runs over gloo ranks without a GPU.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib, ops


class CudaBackend:
    """Router, local-expert and shared-expert compute on the CUDA library."""

    def __init__(self, shard: "ops.MoEWeights", router_w, shared_expert_gate):
        self.w = shard
        self.router_w = router_w
        self.seg = shared_expert_gate
        self.shared_w = None
        if shard.shared_gate is not None:
            self.shared_w = ops.MoEWeights(shard.shared_gate, shard.shared_up, shard.shared_down,
                                           top_k=1, device=shard.device)
            if shard.pool is not None:
                self.shared_w.pack(shard.pool.down_rows)

    def route(self, x, num_experts):
        r = ops.route(x, self.router_w, self.w.top_k, self.seg)
        return r.inds, r.weights, r.shared_gate

    def experts_partial(self, xr, ids, scores):
        return ops.moe_experts_partial(xr, ids, scores, self.w)

    def shared(self, x, num_experts):
        if self.shared_w is None:
            return None
        T = x.shape[0]
        routes = torch.zeros((T, 1), dtype=torch.int32, device=x.device)
        # the pipeline the single-GPU block would give its shared rows
        path = _lib.PATH_GEMM if T * self.w.top_k >= 4 * num_experts else _lib.PATH_GEMV
        return ops.moe_experts(x, routes, self.shared_w, path=path)[:, 0, :]


def shard_weights(w: "ops.MoEWeights", rank: int, world: int) -> "ops.MoEWeights":
    """The rank's contiguous share of the routed banks (views, no copy)."""
    E = w.num_experts
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    El = E // world
    sl = slice(rank * El, (rank + 1) * El)

    def part(p):
        return ops.Q4Projection(p.weight[sl], p.scales[sl], p.biases[sl])

    return ops.MoEWeights(part(w.gate), part(w.up), part(w.down), router_w=w.router_w,
                          shared_gate=w.shared_gate, shared_up=w.shared_up,
                          shared_down=w.shared_down, shared_expert_gate=w.shared_expert_gate,
                          top_k=w.top_k, device=w.device, check_router=False)


class ExpertParallelMoE:
    """The block with its routed experts split over the process group."""

    def __init__(self, shard: "ops.MoEWeights", num_experts: int, group=None, backend=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = int(num_experts)
        if self.E % self.world:
            raise ValueError(f"{self.E} experts do not split over {self.world} ranks")
        self.El = self.E // self.world
        self.k = shard.top_k
        if backend is None:
            backend = CudaBackend(shard, shard.router_w, shard.shared_expert_gate)
        self.backend = backend
        self.last_stats = {}

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    # Decode-sized batches take the fixed-capacity exchange: every rank sends
    # every destination a block of T rows (token order; rows of tokens with no
    # expert there carry ids -1 and cost no expert work), so no counts travel
    # to the host and the step is graph-capturable.  Larger batches exchange
    # only the rows that are needed, after a count all-to-all.
    capacity_max_tokens = 256

    def __call__(self, x):
        if int(x.shape[0]) <= self.capacity_max_tokens:
            return self._call_capacity(x)
        return self._call_counts(x)

    def _call_capacity(self, x):
        T, d = int(x.shape[0]), int(x.shape[1])
        P, El, k = self.world, self.El, self.k
        dev = x.device
        inds, wts, sg = self.backend.route(x, self.E)
        inds = inds.reshape(T, k).to(torch.int64)
        dest = inds // El                                           # [T, k]
        # per destination p: token t's slot ids local to p (-1 elsewhere)
        ranks = torch.arange(P, device=dev).view(P, 1, 1)
        ids = torch.where(dest.unsqueeze(0) == ranks, inds.unsqueeze(0) - ranks * El,
                          torch.full((P, T, k), -1, dtype=torch.int64, device=dev))
        meta = torch.cat([ids.to(torch.float32),
                          wts.reshape(1, T, k).expand(P, T, k).to(torch.float32)], 2)   # [P, T, 2k]
        xs = x.unsqueeze(0).expand(P, T, d).contiguous()
        xr = torch.empty_like(xs)
        mr = torch.empty_like(meta)
        self._a2a(xr, xs, None, None)
        self._a2a(mr, meta.contiguous(), None, None)
        rids = mr[..., :k].reshape(P * T, k).to(torch.int32).contiguous()
        rsc = mr[..., k:].reshape(P * T, k).to(torch.bfloat16).contiguous()
        part = self.backend.experts_partial(xr.reshape(P * T, d), rids, rsc)   # float32 [P*T, d]
        back = torch.empty((P, T, d), dtype=torch.float32, device=dev)
        self._a2a(back, part.reshape(P, T, d).contiguous(), None, None)
        shared = self.backend.shared(x, self.E)
        routed = back[0]
        for p in range(1, P):                                       # rank order, float32
            routed = routed + back[p]
        y = routed.to(torch.bfloat16)
        if shared is not None:
            sy = (sg.reshape(T, 1).float() * shared.float()).to(torch.bfloat16)
            y = (y.float() + sy.float()).to(torch.bfloat16)
        self.last_stats = {"mode": "capacity", "rows_per_peer": T}
        return y

    def _call_counts(self, x):
        T, d = int(x.shape[0]), int(x.shape[1])
        P, El, k = self.world, self.El, self.k
        dev = x.device
        inds, wts, sg = self.backend.route(x, self.E)
        inds = inds.reshape(T, k).to(torch.int64)
        dest = inds // El                                           # [T, k]
        member = torch.zeros((T, P), dtype=torch.bool, device=dev)
        member.scatter_(1, dest, True)
        # send rows sorted by (destination, token)
        send_dst, send_tok = member.t().nonzero(as_tuple=True)
        send_counts = member.sum(0).to(torch.int64)                # [P]
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        S, R = sum(sc), sum(rc)
        ids = inds[send_tok] - send_dst[:, None] * El
        ids = torch.where(dest[send_tok] == send_dst[:, None], ids, torch.full_like(ids, -1))
        meta = torch.cat([ids.to(torch.float32), wts.reshape(T, k)[send_tok].to(torch.float32)], 1)
        xs = x[send_tok].contiguous()
        xr = torch.empty((R, d), dtype=x.dtype, device=dev)
        mr = torch.empty((R, 2 * k), dtype=torch.float32, device=dev)
        self._a2a(xr, xs, rc, sc)
        self._a2a(mr, meta.contiguous(), rc, sc)
        rids = mr[:, :k].to(torch.int32).contiguous()
        rsc = mr[:, k:].to(torch.bfloat16).contiguous()
        part = self.backend.experts_partial(xr, rids, rsc)         # float32 [R, d]
        back = torch.empty((S, d), dtype=torch.float32, device=dev)
        self._a2a(back, part.contiguous(), sc, rc)
        shared = self.backend.shared(x, self.E)
        slots = torch.zeros((T, P, d), dtype=torch.float32, device=dev)
        slots[send_tok, send_dst] = back
        routed = slots[:, 0, :]
        for p in range(1, P):                                       # rank order, float32
            routed = routed + slots[:, p, :]
        y = routed.to(torch.bfloat16)
        if shared is not None:
            sy = (sg.reshape(T, 1).float() * shared.float()).to(torch.bfloat16)
            y = (y.float() + sy.float()).to(torch.bfloat16)
        self.last_stats = {"mode": "counts", "sent_rows": S, "received_rows": R, "send_counts": sc}
        return y
