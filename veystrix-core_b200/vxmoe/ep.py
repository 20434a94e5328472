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

Three transports carry steps 2 and 4:

* ``p2p`` (decode-sized batches on CUDA, the default there): every rank's
  exchange buffer is mapped into every rank (CUDA IPC over NVLink); dispatch
  stores rows straight into the owners' buffers, the experts' combine kernel
  stores each partial straight into its home rank, and flags in the buffers
  order the steps (vx_ep_* in the C ABI).  No library collective runs and
  nothing reaches the host, so the step captures into a CUDA graph
  (``GraphedExpertParallel``).
* ``collective``, the process group's all-to-all (NCCL on GPUs, gloo in the
  CPU tests): decode-sized batches in fixed blocks of T rows per peer
  (equal-split all-to-all, no counts on the host: mode ``capacity``), larger
  batches after a count all-to-all as all-to-all-v of only the rows needed
  (mode ``counts``; every transport uses it above ``capacity_max_tokens``).

The reference runs on one Apple GPU and has no collective; this is the B200
scale-out of the same block.  The compute backend is injectable: the CUDA
backend runs the library's kernels; tests substitute a CPU backend so the
NCCL-shaped exchange runs over gloo ranks without a GPU.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops


class PeerExchange:
    """Every rank's exchange buffer (vx_ep_buffer_bytes) mapped into every
    rank of the group through CUDA IPC.  Construction is collective: all
    ranks build it together (handles travel by all-gather; a barrier makes
    sure every buffer is zeroed before any rank stores into it).  Layers share
    one exchange, since every rank runs them in the same order; ``close``
    (also collective) unmaps the peers' buffers.  ``wait_ns`` bounds every
    wait of the step (0: the library's 20 s); a wait that runs out sets a bit
    of ``errors()`` and lets the step finish with undefined values."""

    def __init__(self, group, tokens_cap: int, hidden: int, top_k: int, num_experts: int,
                 device: torch.device, wait_ns: int = 0):
        lib = _lib.load()
        self.lib = lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        if self.world > _lib.EP_MAX_RANKS:
            raise ValueError(f"the peer exchange spans at most {_lib.EP_MAX_RANKS} ranks")
        self.tokens_cap, self.hidden, self.top_k = int(tokens_cap), int(hidden), int(top_k)
        self.num_experts = int(num_experts)
        nbytes = lib.vx_ep_buffer_bytes(self.world, self.tokens_cap, self.hidden, self.top_k)
        if nbytes == 0:
            raise ValueError("invalid exchange shape")
        self.buf = torch.zeros(int(nbytes), dtype=torch.uint8, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        handle = (ctypes.c_ubyte * _lib.EP_IPC_HANDLE_BYTES)()
        off = ctypes.c_uint64()
        _lib.check(lib.vx_ep_ipc_handle(self.buf.data_ptr(), handle, ctypes.byref(off)),
                   "vx_ep_ipc_handle")
        mine = torch.tensor(list(bytes(handle)) + list(int(off.value).to_bytes(8, "little")),
                            dtype=torch.uint8, device=device)
        every = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(every, mine, group=group)
        comm = _lib.VxEpComm()
        self._opened = []
        try:
            for p in range(self.world):
                if p == self.rank:
                    comm.buffers[p] = self.buf.data_ptr()
                    continue
                blob = bytes(every[p].cpu().tolist())
                h = (ctypes.c_ubyte * _lib.EP_IPC_HANDLE_BYTES).from_buffer_copy(
                    blob[:_lib.EP_IPC_HANDLE_BYTES])
                o = int.from_bytes(blob[_lib.EP_IPC_HANDLE_BYTES:], "little")
                ptr = ctypes.c_void_p()
                _lib.check(lib.vx_ep_ipc_open(h, o, ctypes.byref(ptr)), "vx_ep_ipc_open")
                comm.buffers[p] = ptr.value
                self._opened.append((ptr.value, o))
        except Exception:
            self._unmap()
            raise
        comm.rank, comm.world, comm.tokens_cap = self.rank, self.world, self.tokens_cap
        comm.hidden, comm.top_k, comm.num_experts = self.hidden, self.top_k, self.num_experts
        comm.err = self.err.data_ptr()
        comm.wait_ns = int(wait_ns)
        self.comm = comm
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def fits(self, tokens_cap, hidden, top_k, num_experts) -> bool:
        return (tokens_cap <= self.tokens_cap and hidden == self.hidden and top_k == self.top_k
                and num_experts == self.num_experts)

    def dispatch(self, x, inds, weights) -> None:
        _lib.check(self.lib.vx_ep_dispatch(ctypes.byref(self.comm), x.data_ptr(), int(x.shape[0]),
                                           inds.data_ptr(), weights.data_ptr(),
                                           ops._stream(self.device)), "vx_ep_dispatch")

    def experts(self, T: int, shard: "ops.MoEWeights") -> None:
        st = shard.vx(with_shared=False)
        nb = self.lib.vx_ep_experts_workspace(ctypes.byref(self.comm), int(T), ctypes.byref(st))
        if nb == 0:
            raise ValueError("the shard does not match the exchange")
        ws = ops._WS.get(nb, self.device)
        _lib.check(self.lib.vx_ep_experts(ctypes.byref(self.comm), int(T), ctypes.byref(st),
                                          ws.data_ptr(), ws.numel(), ops._stream(self.device)),
                   "vx_ep_experts")

    def combine(self, T: int, inds, shared, shared_gate, y) -> None:
        _lib.check(self.lib.vx_ep_combine(ctypes.byref(self.comm), int(T), inds.data_ptr(),
                                          ops._ptr(shared), ops._ptr(shared_gate), y.data_ptr(),
                                          ops._stream(self.device)), "vx_ep_combine")

    def errors(self) -> int:
        """Bits of the timeout word (synchronises): 1 dispatch, 2 combine."""
        return int(self.err.item())

    def _unmap(self):
        for ptr, o in self._opened:
            self.lib.vx_ep_ipc_close(ptr, o)
        self._opened = []

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)    # no rank still stores into a buffer
        self._unmap()


_EXCHANGES = {}


def peer_exchange(group, tokens_cap, hidden, top_k, num_experts, device) -> PeerExchange:
    """The group's shared exchange on this device (collective on first use)."""
    key = (id(group), torch.device(device).index)
    ex = _EXCHANGES.get(key)
    if ex is None or not ex.fits(tokens_cap, hidden, top_k, num_experts):
        if ex is not None:
            ex.close()
        ex = PeerExchange(group, tokens_cap, hidden, top_k, num_experts, torch.device(device))
        _EXCHANGES[key] = ex
    return ex


def close_exchanges() -> None:
    """Unmap every peer exchange of this process (collective); call before
    destroying the process group."""
    for ex in list(_EXCHANGES.values()):
        ex.close()
    _EXCHANGES.clear()


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
        r = ops.route(x, self.router_w, self.w.top_k, self.seg, router_bias=self.w.router_bias)
        return r.inds, r.weights, r.shared_gate

    def experts_partial(self, xr, ids, scores):
        return ops.moe_experts_partial(xr, ids, scores, self.w)

    def experts_p2p(self, exchange: PeerExchange, T: int) -> None:
        exchange.experts(T, self.w)

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
        return ops.Q4Projection(p.weight[sl], p.scales[sl], p.biases[sl], p.group_size)

    out = ops.MoEWeights(part(w.gate), part(w.up), part(w.down), router_w=w.router_w,
                         shared_gate=w.shared_gate, shared_up=w.shared_up,
                         shared_down=w.shared_down, shared_expert_gate=w.shared_expert_gate,
                         top_k=w.top_k, device=w.device, check_router=False)
    out.router_bias = w.router_bias
    return out


class ExpertParallelMoE:
    """The block with its routed experts split over the process group."""

    def __init__(self, shard: "ops.MoEWeights", num_experts: int, group=None, backend=None,
                 transport: str = "auto", capacity: int = 256):
        """``capacity``: the largest per-rank batch that takes the fixed-block
        exchange (peer stores, or the equal-split all-to-all); the peer
        transport's buffers are sized for it (about 3 * world * capacity * d * 4
        bytes per rank).  Larger batches use the count exchange."""
        self.capacity_max_tokens = int(capacity)
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
        if transport == "auto":
            transport = ("p2p" if isinstance(backend, CudaBackend) and self.world <= _lib.EP_MAX_RANKS
                         else "collective")
        if transport not in ("p2p", "collective"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.exchange = None
        self._side = None
        if transport == "p2p":
            self.exchange = peer_exchange(group, self.capacity_max_tokens, shard.hidden, self.k,
                                          self.E, shard.device)
        self.last_stats = {}
        self.exchange_events = None   # a list: record the device time of every all-to-all

    def _a2a(self, out, inp, out_splits, in_splits):
        timed = self.exchange_events is not None and torch.cuda.is_available() and out.is_cuda
        if timed:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        if timed:
            e1.record()
            self.exchange_events.append((e0, e1))

    def exchange_ms(self) -> float:
        """Milliseconds the recorded all-to-all calls took on the device
        (synchronises); recording is on while ``exchange_events`` is a list."""
        if not self.exchange_events:
            return 0.0
        torch.cuda.synchronize()
        return float(sum(a.elapsed_time(b) for a, b in self.exchange_events))

    # Batches up to the capacity take the fixed-block exchange: every rank
    # sends every destination a block of T rows (token order; rows of tokens
    # with no expert there carry ids -1 and cost no expert work, and the peer
    # transport does not even store them), so no counts travel to the host and
    # the step is graph-capturable.  Larger batches exchange only the rows
    # that are needed, after a count all-to-all.

    def __call__(self, x):
        if int(x.shape[0]) <= self.capacity_max_tokens:
            if self.transport == "p2p":
                return self._call_p2p(x)
            return self._call_capacity(x)
        return self._call_counts(x)

    def _call_p2p(self, x):
        """Every rank passes the same number of tokens.  The shared expert
        of the rank's own tokens runs on a second stream, beside the
        exchange and the routed experts."""
        x = x.contiguous()
        T, d = int(x.shape[0]), int(x.shape[1])
        inds, wts, sg = self.backend.route(x, self.E)
        inds = inds.reshape(T, self.k).contiguous()
        wts = wts.reshape(T, self.k).contiguous()
        ex = self.exchange
        main = torch.cuda.current_stream(x.device)
        if self._side is None:
            self._side = torch.cuda.Stream(x.device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            shared = self.backend.shared(x, self.E)
        ex.dispatch(x, inds, wts)
        self.backend.experts_p2p(ex, T)
        main.wait_stream(self._side)
        if shared is not None:
            shared.record_stream(main)
        y = torch.empty((T, d), dtype=torch.bfloat16, device=x.device)
        gate = sg.reshape(T).contiguous() if shared is not None else None
        ex.combine(T, inds, shared.contiguous() if shared is not None else None, gate, y)
        self.last_stats = {"mode": "p2p", "rows_per_peer": T}
        return y

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


class GraphedExpertParallel:
    """An expert-parallel layer on the peer transport for a fixed batch size,
    captured once into a CUDA graph (router, dispatch, experts, shared expert
    and combine: every launch of the step).  Construction runs one step on
    every rank (collective).  The output belongs to the graph and is
    overwritten by the next call."""

    def __init__(self, layer: ExpertParallelMoE, tokens: int):
        if layer.transport != "p2p":
            raise ValueError("graph capture needs the p2p transport")
        dev = layer.exchange.device
        self.layer = layer
        self.x = torch.zeros((int(tokens), layer.exchange.hidden), dtype=torch.bfloat16, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            layer(self.x)                         # kernel attributes, workspace
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.y = layer(self.x)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.y
