"""Benchmark of the routed sparse-MoE layer on B200 (one JSON line on rank 0).

Workload: one MoE layer, a batch of 64 independent decode
tokens per GPU, hidden 2048, 512 routed experts (top-10, renormalised) plus
one shared expert, SwiGLU experts with intermediate 512, 4-bit affine
group-32 weights; x bf16 ~N(0,1), synthetic random-init weights with the
benchmark distributions.  A step is one pass of the block over one batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl vxmoe|reference]

value      tokens/s over all ranks, inputs resident in HBM, device-timed
           (CUDA events, max over ranks); weights rotate over several pools
           so the working set is far larger than L2.
e2e        the same through the public API with x copied from pinned host
           memory and y copied back inside the timed region.
roofline   the dominant kernel's algorithmic bytes per launch over its
           CUDA-event duration against the measured HBM copy bandwidth.
c1_decode_1_token, c4_prefill_2048_tokens
           (single GPU, default run) the two north-star shapes - BASELINE
           config 1 (one decode token) and config 4 (2,048-token prefill) -
           timed in the same process on the same rotating pools: step time,
           HBM fraction and, for C4, the gate/up GEMM's tensor-pipe rate.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "veystrix-core_b200"))

METRIC = "MoE-layer tokens/s and achieved HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
HIDDEN, EXPERTS, INTER, SHARED_INTER, TOPK = 2048, 512, 512, 512, 10
EXPERT_BYTES = 3 * (INTER * HIDDEN // 2 + 2 * INTER * (HIDDEN // 32) * 2)   # 1,966,080
PROJ_BYTES = EXPERT_BYTES // 3                                               # 655,360
ROUTER_BYTES = EXPERTS * HIDDEN * 2
SHARED_GATE_BYTES = HIDDEN // 2 + 2 * (HIDDEN // 32) * 2                     # 1,280
NOMINAL_HBM_GBS = 8000.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="vxmoe", choices=("vxmoe", "reference"))
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--pools", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=1,
                    help="> 1: BASELINE config 3, a decode stack of this many distinct layers "
                         "(h += MoE(RMSNorm(h)), mixers identity)")
    ap.add_argument("--c5", action="store_true",
                    help="BASELINE config 5: 65,536-token prefill through 4 layers with 32 hot experts "
                         "(strong scaling over --gpus)")
    ap.add_argument("--ep-transport", default="p2p", choices=("p2p", "collective"),
                    help="expert-parallel exchange: peer stores over NVLink or NCCL all-to-all")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the block's kernels one by one instead of replaying a CUDA graph")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the C1 (1 token) and C4 (2,048 tokens) sub-measurements of the default run")
    ap.add_argument("--layout", default="tiled", choices=("tiled", "mlx"),
                    help="expert weights as the tiled resident pool (default) or the MLX arrays")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def block_launches(T, k=TOPK, E=EXPERTS):
    """Kernels one single-GPU block call launches (the library's dispatch):
    at most four tokens, the whole block in one cooperative launch; else the
    router - one fused launch, with the expert sort in its last token block
    while T*k <= 1024, or from 256 tokens the tiled logits, the top-k and
    the shared-expert gate (three) - then a permutation launch unless the
    router sorted (three above 16,384 routes); then the x records, gate/up,
    h records and down GEMVs (decode), or the x gather and the two tcgen05
    GEMMs (T*k >= 4E); then the combine."""
    P = T * k
    if T <= 4:
        return 1   # the single cooperative decode launch (and one memset)
    fused_sort = P <= 1024
    router = 3 if (T >= 256 and not fused_sort) else 1
    perm = 0 if fused_sort else (1 if P <= 16384 else 3)
    experts = 3 if P >= 4 * E else 4
    return router + perm + experts + 1


def layer_bytes(U, T):
    """Algorithmic bytes of one layer step: each touched expert once, the
    shared expert, the router, the shared gate row, x in and y out."""
    return U * EXPERT_BYTES + EXPERT_BYTES + ROUTER_BYTES + SHARED_GATE_BYTES + T * HIDDEN * 2 * 2


def stage_bytes(stage, U, T):
    P = T * TOPK
    if stage == "gate_up_swiglu":
        return (U + 1) * 2 * PROJ_BYTES + T * HIDDEN * 2 + (P + T) * INTER * 2
    if stage == "down":
        return (U + 1) * PROJ_BYTES + (P + T) * INTER * 2 + (P + T) * HIDDEN * 2
    if stage == "router":
        return ROUTER_BYTES + SHARED_GATE_BYTES + T * HIDDEN * 2 + T * EXPERTS * 2
    if stage == "decode":   # the whole block in one launch
        return layer_bytes(U, T)
    return None


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,"
              "utilization.gpu")

    def __init__(self, index, period_ms=50):
        self.path = tempfile.mktemp(suffix=".csv")
        self.fh = open(self.path, "w")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(period_ms), "-i", str(index)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        self.t0 = time.time()
        # nvidia-smi takes a moment to start: wait (up to 5 s) for its first
        # sample, so that the warm-up and the timed region fall inside the window
        while self.proc is not None and time.time() - self.t0 < 5.0:
            self.fh.flush()
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)

    def hold(self, fn, seconds=1.0):
        """Replay `fn` (the timed work) for `seconds` of wall time with the
        sampler running, so that the window holds enough samples under the
        same load as the timed region (which is often shorter than one
        sampling period)."""
        import torch
        t_end = time.time() + seconds
        while time.time() < t_end:
            for _ in range(8):
                fn()
            torch.cuda.synchronize()

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, busy, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                clk, top = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            sm.append(clk)
            mx.append(top)
            try:
                if float(parts[9]) >= 50.0:
                    busy.append(clk)
            except ValueError:
                pass
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        # the window also holds host-side set-up with the GPU idle: the median
        # is taken over the samples with the GPU busy (utilisation >= 50 %)
        return {"sm_mhz": statistics.median(busy or sm), "sm_max_mhz": max(mx),
                "samples": len(sm), "samples_under_load": len(busy), "reasons": sorted(reasons),
                "window": f"sampled every 50 ms from before warm-up to the end of the GPU work "
                          f"({time.time() - self.t0:.1f} s, the last second replaying the timed steps)"}


# --------------------------------------------------------------------------
# reference arm: the CPU restatement of the block on this host's cores
# --------------------------------------------------------------------------


def cpu_sample(args):
    """The CPU sample both legs time (the cpu_baseline of the vxmoe arm and the
    reference arm), fixed by the command line alone so that the two legs of
    one driver run time the same work: steps of the workload's own token
    count, at most 4,096 tokens in all (about 5-10 s of the restatement on 16
    host threads), after three untimed warm-up steps."""
    tokens = args.tokens
    steps = max(2, min(args.steps, 4096 // max(1, tokens)))
    return steps, 3, tokens


def cpu_oracle_time(steps, warmup, tokens=64, seed=0):
    """Time the CPU restatement of the block (the reference's MLX path is not
    installable here) on `steps` batches of `tokens` tokens of the benchmark
    workload.  Returns (tokens/s over the timed steps, cores, kind, sample
    description)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import vxmoe_oracle as O
    try:
        import vxmoe_cref as C   # C/OpenMP restatement
        runner, cores = C.block_runner(seed), C.threads()
        impl = f"C/OpenMP restatement of the block on {cores} host threads"
    except Exception:
        params = O.make_params(seed=seed)
        runner, cores = (lambda x: O.moe_block(x, params)), 1
        impl = "NumPy restatement of the block on 1 host thread"
    rng = np.random.default_rng(seed + 1)
    xs = [O.bf16_round(rng.normal(0, 1, size=(tokens, HIDDEN))) for _ in range(steps + warmup)]
    for i in range(warmup):
        runner(xs[i])
    per_step = []
    for i in range(steps):
        t0 = time.perf_counter()
        runner(xs[warmup + i])
        per_step.append(time.perf_counter() - t0)
    dt = sum(per_step)
    sample = (f"{impl} (MLX unavailable): {steps} timed steps of {tokens} tokens after {warmup} "
              f"warm-up steps, same layer shape and distributions; median step "
              f"{1000.0 * statistics.median(per_step):.1f} ms")
    return steps * tokens / dt, cores, "port", sample


def run_reference(args, rank, world):
    if rank != 0:
        return
    steps, warmup, tokens = cpu_sample(args)
    v, cores, kind, sample = cpu_oracle_time(steps, warmup, tokens=tokens)
    line = {
        "metric": METRIC, "value": round(v, 3), "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 * tokens / v, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "impl": "reference",
        "config": config_dict(args, world),
        "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(args, world):
    return {
        "workload": ("BASELINE config 2: one MoE layer, batched decode of %d tokens per GPU, "
                     "d=2048, 512 routed experts top-10 + 1 shared, SwiGLU I=512, Q4 affine g32"
                     % args.tokens),
        "global_batch": args.tokens * world, "tokens_per_gpu": args.tokens,
        "experts": EXPERTS, "hidden": HIDDEN, "intermediate": INTER, "top_k": TOPK,
        "parallelism": ((f"ep{world}: {EXPERTS // world} experts per GPU, dispatch/combine as "
                         + ("peer stores over NVLink (CUDA IPC buffers, flag-ordered)"
                            if args.ep_transport == "p2p" else "NCCL all-to-all"))
                        if world > 1 else "single GPU, all experts resident"),
        "l2": f"inputs larger than L2: {args.pools} rotating weight pools of {EXPERTS} experts",
        "launch": ("one CUDA graph per weight pool (x copied into the graph's input buffer each step)"
                   if not args.no_graph and (world == 1 or args.ep_transport == "p2p")
                   else "kernels launched one by one"),
        "weight_layout": ("tiled resident pool (packed once at load)" if args.layout == "tiled"
                          else "MLX arrays"),
    }


# --------------------------------------------------------------------------
# vxmoe arm
# --------------------------------------------------------------------------


def main_stack(args):
    """a decode stack of `args.layers` distinct MoE layers
    (each with its own random weights, packed into the tiled pool), the
    residual stream h += MoE(RMSNorm(h)) with gain 1.0 and eps 1e-6, mixers
    replaced by identity.  A step is one pass of T tokens through every layer,
    captured as one CUDA graph (the stack is launch-bound at T=1 otherwise)."""
    import torch
    import vxmoe
    from vxmoe import _lib
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, L = args.tokens, args.layers
    K, W = args.steps, max(3, args.warmup)
    g = torch.Generator(device=dev)
    layers = []
    for i in range(L):
        g.manual_seed(100 + i)
        layers.append(vxmoe.MoEWeights.random(EXPERTS, HIDDEN, INTER, SHARED_INTER, TOPK, device=dev,
                                              generator=g).pack())
    gain = torch.ones(HIDDEN, dtype=torch.bfloat16, device=dev)
    g.manual_seed(7)
    xs = torch.randn((K + W, T, HIDDEN), device=dev, generator=g).to(torch.bfloat16)

    def stack(h):
        for w in layers:
            h = h + vxmoe.moe_block(vxmoe.rms_norm(h, gain, 1e-6), w)
        return h

    h_in = torch.zeros((T, HIDDEN), dtype=torch.bfloat16, device=dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        stack(h_in)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        h_out = stack(h_in)

    def step(x):
        h_in.copy_(x, non_blocking=True)
        graph.replay()
        return h_out

    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(dev.index)
    for i in range(W):
        step(xs[i])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        step(xs[W + i])
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    hx = xs[W:W + K].cpu().pin_memory()
    hy = torch.empty((K, T, HIDDEN), dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(K):
        hy[i].copy_(step(hx[i].to(dev, non_blocking=True)), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    # routing statistics and stage times: one step without the graph
    h = xs[W].clone()
    Us = []
    _lib.profile_enable(True)
    for w in layers:
        n = vxmoe.rms_norm(h, gain, 1e-6)
        y, inds, _ = vxmoe.moe_block(n, w, return_routing=True)
        Us.append(int(torch.unique(inds).numel()))
        h = h + y
    stages = _lib.profile_read()
    _lib.profile_enable(False)
    torch.cuda.synchronize()
    sampler.hold(lambda: step(xs[W]))
    clocks = sampler.stop()

    hbm_gbs, _, peak_kind = peaks()
    step_bytes = sum(layer_bytes(U, T) for U in Us)
    achieved = step_bytes / (ms / K / 1000.0) / 1e9
    dom = max(stages, key=lambda k: stages[k][1]) if stages else None
    roof = None
    if dom is not None:
        b = stage_bytes(dom, sum(Us) / len(Us), T)
        ach = b / (stages[dom][1] / 1000.0) / 1e9 if b else None
        roof = {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1) if ach else None,
                "peak": hbm_gbs, "unit": "GB/s", "frac": round(ach / hbm_gbs, 4) if ach else None,
                "traffic": None, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": int(b) if b else None,
                "avg_launch_ms": round(stages[dom][1], 5)}
    cpu = None
    if not args.no_cpu_baseline:
        steps_c, warm_c, _ = cpu_sample(args)
        v, cores, kind, sample = cpu_oracle_time(steps_c, warm_c, tokens=T)
        cpu = {"value": round(v / L, 4), "unit": "tokens/s", "cores": cores, "kind": kind,
               "sample": sample + f"; one layer timed, tokens/s divided by {L} layers"}
    line = {
        "metric": METRIC, "value": round(K * T / (ms / 1000.0), 2), "unit": "tokens/s", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": round(ms / K, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": (f"BASELINE config 3: {L}-layer routed-MoE decode stack, batch {T}, "
                                "RMSNorm (gain 1, eps 1e-6) + MoE block + residual per layer, mixers identity; "
                                "d=2048, 512 experts top-10 + shared, I=512, Q4 affine g32"),
                   "global_batch": T, "layers": L, "experts": EXPERTS, "hidden": HIDDEN,
                   "intermediate": INTER, "top_k": TOPK, "parallelism": "single GPU, every layer resident",
                   "l2": f"{L} distinct layers ({L} x 1.0 GB of experts, plus the tiled pool) >> L2",
                   "launch": "the whole stack as one CUDA graph"},
        "hbm": {"achieved_gbs": round(achieved, 1), "frac_of_8tbps": round(achieved / NOMINAL_HBM_GBS, 4),
                "frac_of_measured": round(achieved / hbm_gbs, 4), "bytes_per_step": int(step_bytes),
                "distinct_experts_mean": round(sum(Us) / len(Us), 1)},
        "roofline": roof,
        "stages_ms": {k: round(v[1], 5) for k, v in stages.items()},
        "e2e": {"value": round(K * T / (e2e_ms / 1000.0), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": T * HIDDEN * 2, "d2h_bytes_per_step": T * HIDDEN * 2},
        "cpu_baseline": cpu,
        "clocks": clocks,
        "gpu_launches": (1 + block_launches(T)) * L * K,   # per layer: RMSNorm + the block's kernels
    }
    print(json.dumps(line), flush=True)


C5_TOKENS = 65536      # 8 sequences x 8,192 tokens
C5_LAYERS = 4
C5_HOT = 32            # hot experts, +2.0 on their router logits
LAYER_FLOPS_PER_TOKEN = 2 * TOPK * 3 * HIDDEN * INTER + 2 * 3 * HIDDEN * SHARED_INTER + 2 * EXPERTS * HIDDEN


def main_c5(args):
    """prefill of 8 x 8,192 = 65,536 tokens through 4
    stacked layers (h += MoE(RMSNorm(h)), distinct weights per layer), with
    +2.0 added to the router logits of 32 hot experts chosen with seed 0, so
    expert load is skewed.  The total is fixed (strong scaling): N ranks take
    65,536/N tokens each; for N > 1 the experts are split over the ranks and
    the exchange is the NCCL count transport.  Reports the load imbalance
    (max/mean routed rows per expert at N = 1, per rank for N > 1) and the
    device time of the all-to-all calls."""
    import numpy as np
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    import vxmoe
    from vxmoe.ep import ExpertParallelMoE
    T, L = C5_TOKENS // world, C5_LAYERS
    K, W = args.steps, max(3, args.warmup)
    hot = np.random.default_rng(0).choice(EXPERTS, C5_HOT, replace=False)
    bias = torch.zeros(EXPERTS, dtype=torch.bfloat16, device=dev)
    bias[torch.from_numpy(hot).to(dev)] = 2.0
    g = torch.Generator(device=dev)
    gr = torch.Generator(device=dev)
    layers, weights = [], []
    for i in range(L):
        g.manual_seed(200 + 97 * i + rank)
        gr.manual_seed(300 + i)            # router and shared expert: the same on every rank
        w = vxmoe.MoEWeights.random(EXPERTS // world, HIDDEN, INTER, SHARED_INTER, TOPK, device=dev,
                                    generator=g, router_experts=EXPERTS, router_generator=gr).pack()
        w.router_bias = bias
        weights.append(w)
        if world == 1:
            layers.append(lambda x, w=w: vxmoe.moe_block(x, w))
        else:
            # peer transport: fixed blocks of T rows per peer, stored over NVLink by the
            # kernels; collective: NCCL count exchange + all-to-all-v
            p2p = args.ep_transport == "p2p"
            layers.append(ExpertParallelMoE(w, EXPERTS, transport=args.ep_transport,
                                            capacity=T if p2p else 256))
    gain = torch.ones(HIDDEN, dtype=torch.bfloat16, device=dev)

    def step(x):
        h = x
        for f in layers:
            h = h + f(vxmoe.rms_norm(h, gain, 1e-6))
        return h

    g.manual_seed(7 + rank)
    xs = torch.randn((2, T, HIDDEN), device=dev, generator=g).to(torch.bfloat16)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(dev.index) if rank == 0 else None
    for i in range(W):
        step(xs[i % 2])
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for i in range(K):
        step(xs[i % 2])
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    clocks = sampler.stop() if sampler else None

    # end to end: pinned host x -> device -> stack -> pinned host y
    hx = xs.cpu().pin_memory()
    hy = torch.empty((T, HIDDEN), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty((T, HIDDEN), dtype=torch.bfloat16, device=dev)
    barrier()
    e0.record(stream)
    for i in range(K):
        dx.copy_(hx[i % 2], non_blocking=True)
        hy.copy_(step(dx), non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))

    # load statistics and exchange time (outside the timed regions)
    if world == 1:
        r = vxmoe.router(vxmoe.rms_norm(xs[0], gain, 1e-6), weights[0])
        counts = torch.bincount(r.inds.reshape(-1).long(), minlength=EXPERTS).float()
        imbalance = {"per": "expert", "max_over_mean": round(float(counts.max() / counts.mean()), 3),
                     "hot_share": round(float(counts[torch.from_numpy(hot).to(dev)].sum() / counts.sum()), 4)}
        exchange_ms = 0.0
    else:
        for f in layers:
            f.exchange_events = []
        step(xs[0])
        exchange_ms = sum(f.exchange_ms() for f in layers)
        # routed slots each rank's expert shard receives (first layer, all ranks' tokens)
        r = vxmoe.route(vxmoe.rms_norm(xs[0], gain, 1e-6), weights[0].router_w, TOPK,
                        router_bias=bias)
        vals = torch.bincount(r.inds.reshape(-1).long() // (EXPERTS // world), minlength=world).double()
        dist.all_reduce(vals)
        imbalance = {"per": "rank", "max_over_mean": round(float(vals.max() / vals.mean()), 3),
                     "routed_slots": [int(v) for v in vals.tolist()]}
        exchange_ms = max_over_ranks(exchange_ms)
        for f in layers:
            f.exchange_events = None
        timeouts = 0
        from vxmoe import ep as ep_mod
        for ex in ep_mod._EXCHANGES.values():
            timeouts |= ex.errors()
        layers.clear()
        ep_mod.close_exchanges()
        barrier()
        dist.destroy_process_group()
        if timeouts:
            raise RuntimeError(f"rank {rank}: an expert-parallel wait ran out (bits {timeouts})")
    if rank != 0:
        return
    _, tf_burst, peak_kind = peaks()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            tf_sus = float(json.load(fh)["bf16_tflops_sustained"])
    except Exception:
        tf_sus = tf_burst
    step_flops = float(LAYER_FLOPS_PER_TOKEN) * C5_TOKENS * L
    achieved = step_flops / (ms / K / 1000.0) / 1e12 / world     # per GPU
    line = {
        "metric": METRIC, "value": round(K * C5_TOKENS / (ms / 1000.0), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": (f"BASELINE config 5: prefill of 8 x 8,192 = {C5_TOKENS} tokens through "
                                f"{L} stacked layers (h += MoE(RMSNorm(h))), +2.0 on the router logits of "
                                f"{C5_HOT} hot experts; d=2048, 512 experts top-10 + shared, I=512, Q4 g32"),
                   "global_batch": C5_TOKENS, "tokens_per_gpu": T, "layers": L,
                   "parallelism": ((f"ep{world}: {EXPERTS // world} experts per GPU, " +
                                    ("blocks of T rows stored into the peers over NVLink by the dispatch "
                                     "and combine kernels" if args.ep_transport == "p2p"
                                     else "NCCL count exchange + all-to-all-v"))
                                   if world > 1 else "single GPU"),
                   "l2": "inputs larger than L2 (268 MB of activations per layer, 4 distinct layers)"},
        "layer_tokens_per_s": round(K * C5_TOKENS * L / (ms / 1000.0), 1),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tf_sus, "unit": "TFLOP/s",
                     "frac": round(achieved / tf_sus, 4), "traffic": None, "peak_kind": peak_kind + " sustained",
                     "algorithmic_flops_per_step": step_flops,
                     "note": "whole step: routed + shared expert + router MMA flops per GPU over the step time"},
        "load_imbalance": imbalance,
        # device time of the NCCL all-to-all calls; the peer transport's stores run inside the
        # dispatch and combine kernels and have no separate time
        "all_to_all_ms_per_step": (round(exchange_ms, 3) if world > 1 and args.ep_transport != "p2p"
                                   else None),
        "e2e": {"value": round(K * C5_TOKENS / (e2e_ms / 1000.0), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": T * HIDDEN * 2 * world, "d2h_bytes_per_step": T * HIDDEN * 2 * world},
        "cpu_baseline": None,
        "clocks": clocks,
        "gpu_launches": None,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.c5 and args.impl != "reference":
        return main_c5(args)
    if args.layers > 1 and args.impl != "reference":
        return main_stack(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # NCCL's communicator set-up lines (rank count per communicator) in the log
        os.environ["NCCL_DEBUG"] = "INFO"
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if args.impl == "reference":
        run_reference(args, rank, world)
        if dist is not None:
            dist.destroy_process_group()
        return

    import vxmoe
    from vxmoe import _lib
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T = args.tokens
    K, W = args.steps, max(3, args.warmup)
    g = torch.Generator(device=dev)
    gr = torch.Generator(device=dev)
    pools, layers, plain = [], [], []
    for i in range(args.pools):
        g.manual_seed(1000 * rank + i)
        gr.manual_seed(5000 + i)          # router and shared expert: the same on every rank
        if world == 1:
            w = vxmoe.MoEWeights.random(EXPERTS, HIDDEN, INTER, SHARED_INTER, TOPK, device=dev,
                                        generator=g)
            if args.layout == "tiled":
                w.pack()
            pools.append(w)
            plain.append(lambda x, w=w: vxmoe.moe_block(x, w))
            # one CUDA graph per weight pool: the block's launches replay as one
            layers.append(plain[-1] if args.no_graph else vxmoe.GraphedBlock(w, T))
        else:
            # expert parallel: this rank holds experts [rank*E/N, (rank+1)*E/N)
            from vxmoe.ep import ExpertParallelMoE, GraphedExpertParallel
            w = vxmoe.MoEWeights.random(EXPERTS // world, HIDDEN, INTER, SHARED_INTER, TOPK,
                                        device=dev, generator=g, router_experts=EXPERTS,
                                        router_generator=gr)
            if args.layout == "tiled":
                w.pack()
            pools.append(w)
            # the peer transport carries the whole batch (prefill sizes included) in
            # fixed blocks; the collective one switches to the count exchange above 256
            ep = ExpertParallelMoE(w, EXPERTS, transport=args.ep_transport,
                                   capacity=max(256, T) if args.ep_transport == "p2p" else 256)
            plain.append(ep)
            graphed = args.ep_transport == "p2p" and not args.no_graph
            layers.append(GraphedExpertParallel(ep, T) if graphed else ep)
    g.manual_seed(7 + rank)
    nx = K + W
    xs = (torch.randn((nx, T, HIDDEN), device=dev, generator=g)).to(torch.bfloat16)
    torch.cuda.synchronize()
    # our kernels per step on one GPU: block_launches(T); EP runs the router, the
    # shard's pass (permute, activation records, gate/up, down; plus the h records when
    # the shard's rows take the GEMV path), the shared expert's own pass (permute ..
    # unpermute) and, on the peer transport, dispatch, the dispatch wait and the combine
    shard_gemv = T * world * TOPK < 4 * (EXPERTS // max(world, 1))
    launches_per_step = (block_launches(T) if world == 1
                         else (14 if args.ep_transport == "p2p" else 11) + (1 if shard_gemv else 0))

    def step(i):
        return layers[i % len(layers)](xs[i])

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(dev.index) if rank == 0 else None
    for i in range(W):
        step(i)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for i in range(K):
        step(W + i)
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))

    # end to end: pinned host x -> device -> block -> pinned host y, every
    # step moving its own input and output; the copies run on a copy stream
    # beside the compute (step i+1's input and step i's output while step i
    # computes), ordered by events: an input buffer is refilled only after
    # the step that read it, and a layer's output buffer is read back before
    # that layer runs again
    hx = xs[W:W + K].cpu().pin_memory()
    hy = torch.empty((K, T, HIDDEN), dtype=torch.bfloat16).pin_memory()
    dxs = [torch.empty((T, HIDDEN), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    cs = torch.cuda.Stream(dev)

    def e2e_steps(n, first):
        ev_in = [torch.cuda.Event(), torch.cuda.Event()]
        used = [None, None]
        out_done = {}
        with torch.cuda.stream(cs):
            dxs[0].copy_(hx[0], non_blocking=True)
            ev_in[0].record(cs)
        for i in range(n):
            b = i % 2
            stream.wait_event(ev_in[b])
            li = (first + i) % len(layers)
            if li in out_done:
                stream.wait_event(out_done[li])
            y = layers[li](dxs[b])
            done = torch.cuda.Event()
            done.record(stream)
            used[b] = done
            with torch.cuda.stream(cs):
                if i + 1 < n:
                    nb = (i + 1) % 2
                    if used[nb] is not None:
                        cs.wait_event(used[nb])
                    dxs[nb].copy_(hx[(i + 1) % K], non_blocking=True)
                    ev_in[nb].record(cs)
                cs.wait_event(done)
                y.record_stream(cs)
                hy[i % K].copy_(y, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                out_done[li] = ev
        fin = torch.cuda.Event()
        fin.record(cs)
        stream.wait_event(fin)

    e2e_steps(W, 0)
    barrier()
    e0.record(stream)
    e2e_steps(K, W)
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    # the pipelined copies delivered the step's own output: the last step again
    again = layers[(W + K - 1) % len(layers)](hx[K - 1].to(dev)).cpu()
    if not torch.equal(again.view(torch.int16), hy[K - 1].view(torch.int16)):
        raise RuntimeError("end-to-end pass: the host output differs from a direct call")

    # spread of single steps (outside the timed regions): each of up to 200
    # steps between its own pair of events; per step the max over ranks
    n_dist = min(K, 200)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_dist)]
    barrier()
    for i, (a, b) in enumerate(evs):
        a.record(stream)
        step(W + i)
        b.record(stream)
    barrier()
    per_step = torch.tensor([a.elapsed_time(b) for a, b in evs], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(per_step, op=dist.ReduceOp.MAX)
    per_step = sorted(per_step.tolist())

    def pct(f):
        return round(per_step[min(len(per_step) - 1, int(f * (len(per_step) - 1) + 0.5))], 5)

    step_dist = {"steps": n_dist, "median": pct(0.5), "p10": pct(0.1), "p90": pct(0.9)}

    # routing statistics (outside the timed regions): distinct experts this
    # rank's weights serve per step (under expert parallelism, among the
    # tokens of all ranks routed to its shard)
    Us = []
    El = EXPERTS // world
    for i in range(K):
        w = pools[(W + i) % len(pools)]
        r = vxmoe.route(xs[W + i], w.router_w, TOPK, w.shared_expert_gate)
        inds = r.inds.reshape(-1)
        if dist is not None:
            allr = [torch.empty_like(inds) for _ in range(world)]
            dist.all_gather(allr, inds)
            inds = torch.cat(allr)
            inds = inds[(inds // El) == rank]
        Us.append(int(torch.unique(inds).numel()))
    U_mean = sum(Us) / len(Us)
    if dist is not None:
        t = torch.tensor([U_mean], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        U_mean = float(t.item()) / world
        Us = [U_mean] * K

    # per-kernel durations: the same steps again with stage events
    _lib.profile_enable(True)
    for i in range(K):
        plain[(W + i) % len(plain)](xs[W + i])
    stages = _lib.profile_read()
    _lib.profile_enable(False)
    barrier()
    # under expert parallelism every rank's stage times (its timeline: router,
    # dispatch, the wait for the other ranks' rows, the shard's kernels,
    # combine), gathered on rank 0
    per_rank_stages = None
    if dist is not None:
        mine = {k: round(v[1], 5) for k, v in stages.items()}
        per_rank_stages = [None] * world
        dist.all_gather_object(per_rank_stages, mine)

    # the two north-star shapes on the same rotating pools (single GPU)
    extra = None
    if world == 1 and T == 64 and args.layout == "tiled" and not args.no_graph and not args.no_extra:
        extra = extra_configs(pools, W, K, dev, stream)
    if world == 1 and sampler is not None:
        hold_i = [0]

        def replay():
            step(W + hold_i[0] % K)
            hold_i[0] += 1

        sampler.hold(replay)
    clocks = sampler.stop() if sampler else None

    ep_timeouts = 0
    if dist is not None:
        from vxmoe import ep as ep_mod
        for ex in ep_mod._EXCHANGES.values():
            ep_timeouts |= ex.errors()
        layers.clear()
        plain.clear()
        ep_mod.close_exchanges()
        dist.barrier()
        dist.destroy_process_group()
    if ep_timeouts:
        raise RuntimeError(f"rank {rank}: an expert-parallel wait ran out (bits {ep_timeouts})")
    if rank != 0:
        return

    hbm_gbs, bf16_tflops, peak_kind = peaks()
    value = K * T * world / (ms / 1000.0)
    total_bytes = sum(layer_bytes(U, T) for U in Us)
    achieved_layer = total_bytes / (ms / 1000.0) / 1e9
    dom = max(stages, key=lambda s: stages[s][1]) if stages else None
    roof = None
    if dom is not None:
        b = stage_bytes(dom, U_mean, T)
        avg_ms = stages[dom][1]
        ach = b / (avg_ms / 1000.0) / 1e9 if b else None
        roof = {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1) if ach else None,
                "peak": hbm_gbs, "unit": "GB/s", "frac": round(ach / hbm_gbs, 4) if ach else None,
                "traffic": traffic_for(dom, T), "peak_kind": peak_kind,
                "algorithmic_bytes_per_launch": int(b) if b else None,
                "avg_launch_ms": round(avg_ms, 5)}
    # prefill batches run the tcgen05 GEMMs: their tensor-pipe rate beside the HBM roofline
    tensor = None
    if world == 1 and T * TOPK >= 4 * EXPERTS and "gate_up_swiglu" in stages:
        flops = 2.0 * HIDDEN * 2 * (T * TOPK * INTER + T * SHARED_INTER)   # gate and up, routed + shared
        tf = flops / (stages["gate_up_swiglu"][1] / 1000.0) / 1e12
        tensor = {"kernel": "gate_up_swiglu", "achieved": round(tf, 1), "peak": bf16_tflops,
                  "unit": "TFLOP/s", "frac": round(tf / bf16_tflops, 4),
                  "peak_kind": f"{peak_kind} bf16 GEMM burst", "flops_per_launch": int(flops)}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        steps_c, warm_c, tok_c = cpu_sample(args)
        v, cores, kind, sample = cpu_oracle_time(steps_c, warm_c, tokens=tok_c)
        cpu = {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": kind,
               "sample": sample}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(ms / K, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_dict(args, world),
        # single steps timed one by one after the timed region (launch gaps included)
        "step_ms_spread": step_dist,
        "tensor_roofline": tensor,
        "hbm": {"achieved_gbs": round(achieved_layer, 1),
                "frac_of_8tbps": round(achieved_layer / NOMINAL_HBM_GBS, 4),
                "frac_of_measured": round(achieved_layer / hbm_gbs, 4),
                "bytes_per_step": int(total_bytes / K), "distinct_experts_mean": round(U_mean, 1)},
        "roofline": roof,
        "stages_ms": {k: round(v[1], 5) for k, v in stages.items()},
        "e2e": {"value": round(K * T * world / (e2e_ms / 1000.0), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": T * HIDDEN * 2, "d2h_bytes_per_step": T * HIDDEN * 2},
        "cpu_baseline": cpu,
        "clocks": clocks,
        "gpu_launches": launches_per_step * K,
    }
    if per_rank_stages is not None:
        line["stages_ms_per_rank"] = per_rank_stages
    if extra is not None:
        line.update(extra)
    print(json.dumps(line), flush=True)


def extra_configs(pools, W, K, dev, stream):
    """BASELINE config 1 (one decode token) and config 4 (a 2,048-token
    prefill) through the same resident pools as the headline, each pool's
    block captured as a CUDA graph for that batch size and the pools rotated
    per step (inputs larger than L2).  Returns the two sub-objects of the
    JSON line: step time, tokens/s, the layer's algorithmic HBM bytes over the
    step time and, for C4, the gate/up GEMM's tensor-pipe rate."""
    import torch
    import vxmoe
    from vxmoe import _lib
    hbm_gbs, tf_burst, peak_kind = peaks()
    out = {}
    for key, T, steps in (("c1_decode_1_token", 1, max(K, 100)),
                          ("c4_prefill_2048_tokens", 2048, max(3, min(K, 10)))):
        g = torch.Generator(device=dev)
        g.manual_seed(9000 + T)
        xs = torch.randn((W + steps, T, HIDDEN), device=dev, generator=g).to(torch.bfloat16)
        graphs = [vxmoe.GraphedBlock(w, T) for w in pools]
        for i in range(W):
            graphs[i % len(graphs)](xs[i])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            graphs[(W + i) % len(graphs)](xs[W + i])
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        ms_per_call = None
        if T == 1:
            # A decode stack replays its layers inside one graph, each layer
            # reading the previous one's output where it lies: all the steps
            # captured in one graph (each step's x resident in HBM, the pools
            # rotated as above) leave no per-call input copy or graph launch
            # between the blocks.  The per-call replay above stays beside it.
            ms_per_call = ms
            seq = torch.cuda.CUDAGraph()
            with torch.cuda.graph(seq):
                for i in range(steps):
                    vxmoe.moe_block(xs[W + i], pools[(W + i) % len(pools)])
            seq.replay()
            torch.cuda.synchronize()
            e0.record(stream)
            seq.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
            del seq
        Us = []
        for i in range(steps):
            w = pools[(W + i) % len(pools)]
            r = vxmoe.route(xs[W + i], w.router_w, TOPK, w.shared_expert_gate)
            Us.append(int(torch.unique(r.inds).numel()))
        n_prof = min(steps, 20)
        _lib.profile_enable(True)
        for i in range(n_prof):
            vxmoe.moe_block(xs[W + i], pools[(W + i) % len(pools)])
        stages = _lib.profile_read()
        _lib.profile_enable(False)
        torch.cuda.synchronize()
        del graphs
        step_bytes = sum(layer_bytes(U, T) for U in Us) / len(Us)
        gbs = step_bytes / (ms / 1000.0) / 1e9
        entry = {
            "tokens": T, "steps": steps, "ms_per_step": round(ms, 5),
            "tokens_per_s": round(T / (ms / 1000.0), 1),
            "hbm": {"achieved_gbs": round(gbs, 1), "frac_of_8tbps": round(gbs / NOMINAL_HBM_GBS, 4),
                    "frac_of_measured": round(gbs / hbm_gbs, 4), "bytes_per_step": int(step_bytes),
                    "distinct_experts_mean": round(sum(Us) / len(Us), 1)},
            "stages_ms": {k: round(v[1], 5) for k, v in stages.items()},
            "launch": "one CUDA graph per weight pool, pools rotated per step",
        }
        if T == 1:
            entry["north_star"] = ">= 0.70 of 8 TB/s at decode batch 1 (hbm.frac_of_8tbps)"
            entry["launch"] = ("all steps in one CUDA graph, each step's x resident in HBM, pools "
                               "rotated per step")
            entry["ms_per_step_one_graph_per_call"] = round(ms_per_call, 5)
        if "decode" in stages:
            kgbs = step_bytes / (stages["decode"][1] / 1000.0) / 1e9
            entry["kernel"] = {"name": "decode_kernel (router to combine, one cooperative launch)",
                               "avg_launch_ms": round(stages["decode"][1], 5),
                               "achieved_gbs": round(kgbs, 1), "frac_of_measured": round(kgbs / hbm_gbs, 4),
                               "frac_of_8tbps": round(kgbs / NOMINAL_HBM_GBS, 4)}
        if "gate_up_swiglu" in stages and T * TOPK >= 4 * EXPERTS:
            flops = 2.0 * HIDDEN * 2 * (T * TOPK * INTER + T * SHARED_INTER)
            tf = flops / (stages["gate_up_swiglu"][1] / 1000.0) / 1e12
            layer_tf = LAYER_FLOPS_PER_TOKEN * T / (ms / 1000.0) / 1e12
            entry["tensor_roofline"] = {
                "kernel": "gate_up_swiglu", "achieved": round(tf, 1), "peak": tf_burst,
                "unit": "TFLOP/s", "frac": round(tf / tf_burst, 4),
                "peak_kind": f"{peak_kind} bf16 GEMM burst", "flops_per_launch": int(flops),
                "layer_frac": round(layer_tf / tf_burst, 4),
                "north_star": ">= 0.60 of dense bf16 peak at 2,048-token prefill (frac)"}
        out[key] = entry
    return out


def traffic_for(kernel, tokens):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, when
    it was captured on this workload (the same tokens per step), else None."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as fh:
            d = json.load(fh).get(kernel, {})
        return d.get("dram_bytes_per_launch") if d.get("tokens") == tokens else None
    except Exception:
        return None


if __name__ == "__main__":
    main()
