#!/usr/bin/env python
"""Benchmark of the IQ3_XXS routed-expert MoE layer (BASELINE.json metric:
MoE-layer tokens/s and achieved HBM GB/s against the measured B200 peak).

Default workload (--workload decode1): BASELINE config 2, one MoE layer at
batch 1 - hidden 5120, 160 routed experts + 1 shared, intermediate 1536,
top-8, IQ3_XXS experts from the counter-based generator, fp32 router
N(0, 0.02), x bf16 N(0, 1).  One step = one token through one layer.  Steps
cycle through --layers distinct layer copies (8 x 1.45 GB) so consecutive
steps never find their 85 MB of weights in the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gpeed|reference]

Other workloads: --workload ragged64 (config 3: 64 tokens, Zipf-skewed expert
loads, quantised GEMV path), --workload prefill (config 4: 4096 tokens,
tensor-core grouped GEMMs; with --ep and N >= 2 GPUs the experts are split over
the GPUs with NCCL all-to-all dispatch and combine), --workload stack40 (config
5 on one GPU: 40 layers, decode batches 1 to 256), --workload glm5 (batch-1
decode at the reference model's default MoE shape: hidden 4096, 288 experts,
intermediate 2048).

N > 1 (launched by torchrun): expert parallelism.  Every GPU holds 1/N of
every routed expert's intermediate rows (units of 32 rows, the
tensor-parallel split of each expert; --ep-split experts instead gives each
GPU 160/N whole routed experts) plus the whole shared expert; each rank
brings one token per step (weak scaling).  A step is one persistent kernel
per rank (gpeed_moe_decode_ep): its token goes to every rank over NVLink peer
memory, each rank routes its own token and sends its picks to every rank, the
rank runs its share of every pick (its slice of each expert; or, with expert
ranges, the picks in its range) and its own token's shared expert and adds
the sums into the owning rank's output; no collective library on the data
path.  With
--ep-nccl the exchanges are an NCCL all-gather and reduce-scatter around
gpeed_moe_decode_partial instead.  Steps are captured in CUDA graphs.  value =
tokens over all ranks / the slowest rank's time.  The reference arm runs on
rank 0 only, on every host core.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "MoE-layer tokens/s (IQ3_XXS dequant-GEMM); achieved HBM GB/s vs B200 peak"
H, I, E, K_TOP = 5120, 1536, 160, 8
EXPERT_BYTES = 3 * I * (H // 256) * 98            # one expert, 3 matrices: 9,031,680 B
ROUTER_BYTES = E * H * 4
LAYER_TOKEN_BYTES = (K_TOP + 1) * EXPERT_BYTES + ROUTER_BYTES + H * 2 + H * 4   # ~84.59 MB per token-layer
GATEUP_BYTES = (K_TOP + 1) * 2 * I * (H // 256) * 98 + H * 2 + (K_TOP + 1) * I * 4  # dominant kernel, per launch


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.rows = []
        if self.proc is None:
            return
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 9:
                self.rows.append(parts)

    def summary(self, extra_rows=()):
        rows = list(getattr(self, "rows", [])) + list(extra_rows)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def traffic_from_profiles(name: str):
    """DRAM bytes per launch recorded from an ncu capture in profiles/ (or None)."""
    p = os.path.join(REPO, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


def host_layer(seed, stream0, router_seed):
    from oracle import oracle
    nb = lambda rows, inn: rows * inn // 256
    sizes = [nb(E * I, H), nb(E * I, H), nb(E * H, I), nb(I, H), nb(I, H), nb(H, I)]
    names = ("gate", "up", "down", "gate_sh", "up_sh", "down_sh")
    layer = {n: oracle.synth_iq3xxs(seed, stream0 + m, sizes[m]) for m, n in enumerate(names)}
    layer["router"] = router_for(router_seed)
    layer["corr"] = np.zeros(E, np.float32)
    return layer


def router_for(seed):
    return (np.random.default_rng(seed).standard_normal((E, H)) * 0.02).astype(np.float32)


def tokens(n, seed):
    import torch
    return torch.from_numpy(np.random.default_rng(seed).standard_normal((n, H)).astype(np.float32)).to(torch.bfloat16)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_time_layer(kind: str, budget_s: float, max_tokens: int):
    """The reference CPU expert path (oracle/_ref, or the oracle port) on this host."""
    from oracle import oracle
    chk = oracle.Checker(kind)
    chk.set_num_threads(host_cores())
    layer = host_layer(1000, 0, 0)
    shape = oracle.Shape(H, I, E, K_TOP, 2.5, 1, 10.0)
    X = tokens(max_tokens + 1, 7).float().numpy()
    chk.moe_forward(shape, layer, X[0])  # warm-up
    t0 = time.perf_counter()
    done = 0
    while done < max_tokens and time.perf_counter() - t0 < budget_s:
        chk.moe_forward(shape, layer, X[1 + done])
        done += 1
    dt = time.perf_counter() - t0
    return done / dt, done, dt, chk.num_threads()


def run_reference(args, world):
    from oracle import oracle
    kind = "reference" if oracle.available("reference") else "port"
    steps = args.steps
    # each step = one token through one layer on the host cores; the run is
    # capped at ~120 s of timed work
    budget = float(os.environ.get("GPEED_REF_BUDGET_S", "120"))
    chk = oracle.Checker(kind)
    chk.set_num_threads(host_cores())  # torchrun starts ranks with OMP_NUM_THREADS=1
    layer = host_layer(1000, 0, 0)
    shape = oracle.Shape(H, I, E, K_TOP, 2.5, 1, 10.0)
    X = tokens(args.warmup + steps, 7).float().numpy()
    for i in range(args.warmup):
        chk.moe_forward(shape, layer, X[i])
    t0 = time.perf_counter()
    done = 0
    while done < steps and time.perf_counter() - t0 < budget:
        chk.moe_forward(shape, layer, X[args.warmup + done])
        done += 1
    dt = time.perf_counter() - t0
    tps = done / dt
    sample = (f"{done} of {steps} steps (1 token x 1 layer each, H=5120 E=160+1 I=1536 top-8) "
              f"within a {budget:.0f} s cap; weights RAM-resident")
    line = {
        "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": world, "steps": done, "warmup": args.warmup,
        "ms_per_step": 1000.0 * dt / max(done, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "decode1: MoE layer decode, batch 1 (BASELINE config 2)", "hidden": H,
                   "n_experts": E, "top_k": K_TOP, "inter": I, "n_shared": 1, "quant": "IQ3_XXS"},
        "impl": "reference",
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": chk.num_threads(), "kind": kind,
                         "sample": sample},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def prefill_side_timing(ctx, layers, stream, n=4096, reps=6):
    """BASELINE config 4 timed once beside the decode workload (not the line's
    value): `reps` forwards of an n-token bf16 batch through the already
    resident layer copies, alternating, so each forward streams its experts
    from HBM; CUDA events on the launching stream, after two warm-up
    forwards.  Reports ms per layer forward, tokens/s, the grouped GEMMs'
    share (per-stage events of one more forward) and the gate/up GEMM's
    TFLOP/s.  Any failure here is reported in the dict instead of ending the
    run."""
    import torch

    from gpeed_b200 import _capi
    try:
        x = tokens(n, 4242).cuda()
        y = torch.empty(n, H, device="cuda")
        with torch.cuda.stream(stream):
            for l in range(2):
                layers[l % len(layers)].forward(x, y, stream=stream)
        stream.synchronize()
        ctx.check(stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(reps):
                layers[i % len(layers)].forward(x, y, stream=stream)
            e1.record(stream)
        stream.synchronize()
        ctx.check(stream)
        ms = e0.elapsed_time(e1) / reps
        _capi.call("gpeed_ctx_profile", ctx.handle, 1)
        try:
            with torch.cuda.stream(stream):
                layers[0].forward(x, y, stream=stream)
            stage = (ctypes.c_float * 5)()
            calls = ctypes.c_int()
            _capi.call("gpeed_ctx_profile_read", ctx.handle, stage, ctypes.byref(calls))
        finally:
            _capi.call("gpeed_ctx_profile", ctx.handle, 0)
        ctx.check(stream)
        gu_flops = (K_TOP + 1) * 2 * 2 * I * H * n  # gate + up, every (token, pick) and the shared expert
        out = {"tokens": n, "ms_per_layer": ms, "tokens_per_s": n / (ms / 1000.0),
               "stage_ms": dict(zip(["router", "route+gather", "gateup", "down", "combine"], list(stage))),
               "gateup_tflops": gu_flops / (stage[2] * 1e-3) / 1e12 if stage[2] > 0 else None,
               "how": f"{reps} forwards alternating {len(layers)} resident layer copies, CUDA events"}
        del x, y
        return out
    except Exception as exc:  # a side figure: the decode line stands without it
        return {"error": str(exc)[:300]}


def run_gpu(args, rank, local_rank, world):
    import torch
    import torch.distributed as dist

    from gpeed_b200 import Context, MoeConfig, MoeLayer
    from gpeed_b200 import _capi

    torch.cuda.set_device(local_rank)
    ctx = Context(local_rank)
    cfg = MoeConfig()
    L = args.layers
    layers = [MoeLayer(ctx, cfg, layer_id=l).synth(router_for(l), None, seed=1000 + l, stream0=0) for l in range(L)]
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    # one static token per layer copy
    xs = [tokens(1, 100 + l).cuda() for l in range(L)]
    ys = [torch.empty(1, H, device="cuda") for _ in range(L)]
    with torch.cuda.stream(stream):
        for l in range(L):  # sizes scratch, configures kernels (outside capture)
            layers[l].forward(xs[l], ys[l], stream=stream)
    stream.synchronize()
    ctx.check(stream)
    # graphs of consecutive layer forwards, as a model runs its MoE layers: a
    # step is one layer forward; chains[n] runs layers 0..n-1 back to back, so
    # each layer's kernel can start while the previous one drains
    def chain(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):  # consecutive steps on consecutive layer copies
                layers[i % L].forward(xs[i % L], ys[i % L], stream=stream)
        return g

    chains = {L: chain(L)}

    def run_steps(n):
        for _ in range(n // L):
            chains[L].replay()
        if n % L:
            if n % L not in chains:
                chains[n % L] = chain(n % L)
            chains[n % L].replay()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident throughput (value) ----
    # The K timed steps are one graph (cycling over the layer copies), so no
    # gap between graph launches falls inside the timed region; it is
    # replayed once untimed first, after the W warm-up steps.
    timed = chain(args.steps)
    with torch.cuda.stream(stream):
        run_steps(args.warmup)
        timed.replay()
    stream.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            ev0.record(stream)
            timed.replay()
            ev1.record(stream)
        stream.synchronize()
        ms_total = ev0.elapsed_time(ev1)
        # keep the same work running ~1.5 s so the sampler sees the clocks under this load
        soak_t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            while time.perf_counter() - soak_t0 < 1.5:
                run_steps(25 * L)
                stream.synchronize()
    barrier()
    ctx.check(stream)
    ms_step = ms_total / args.steps
    if world > 1:
        t = torch.tensor([ms_total], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    value = world * args.steps / (ms_total / 1000.0)

    # ---- per-kernel timing of the dominant kernel (events on the launch stream) ----
    _capi.call("gpeed_ctx_profile", ctx.handle, 1)
    with torch.cuda.stream(stream):
        for i in range(max(8 * L, 64)):
            layers[i % L].forward(xs[i % L], ys[i % L], stream=stream)
    stage = (ctypes.c_float * 5)()
    calls = ctypes.c_int()
    _capi.call("gpeed_ctx_profile_read", ctx.handle, stage, ctypes.byref(calls))
    _capi.call("gpeed_ctx_profile", ctx.handle, 0)
    stage_ms = list(stage)

    # ---- end to end through the public API with host buffers ----
    x_host = tokens(args.steps, 555).pin_memory()
    y_host = torch.empty(H, dtype=torch.float32).pin_memory()
    x_dev = torch.empty(1, H, dtype=torch.bfloat16, device="cuda")
    y_dev = torch.empty(1, H, dtype=torch.float32, device="cuda")
    e2e_graphs = []
    with torch.cuda.stream(stream):
        layers[0].forward(x_dev, y_dev, stream=stream)
    stream.synchronize()
    x_slot = x_host[0:1].clone().pin_memory()
    for l in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            x_dev.copy_(x_slot, non_blocking=True)
            layers[l].forward(x_dev, y_dev, stream=stream)
            y_host.copy_(y_dev[0], non_blocking=True)
        e2e_graphs.append(g)
    for i in range(args.warmup):
        with torch.cuda.stream(stream):
            e2e_graphs[i % L].replay()
        stream.synchronize()
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        x_slot.copy_(x_host[i:i + 1])       # the step's input lands in the pinned staging buffer
        with torch.cuda.stream(stream):
            e2e_graphs[i % L].replay()
        stream.synchronize()                # the step's result is on the host
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_graph_value = world * args.steps / e2e_s
    ctx.check(stream)

    # ---- end to end through the C ABI on host buffers (gpeed_moe_forward_host:
    # the reference's calling convention, x in and y out in host memory; the
    # call stages x through pinned memory, runs the layer and returns with y
    # on the host) ----
    e2e_api = "gpeed_moe_forward_host (C ABI, host buffers in and out, synchronous per step)"
    try:
        xh = tokens(args.warmup + args.steps, 556)
        yh = torch.empty(1, H, dtype=torch.float32)
        for i in range(args.warmup):
            layers[i % L].forward_host(xh[i:i + 1], yh)
        barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            layers[i % L].forward_host(xh[args.warmup + i:args.warmup + i + 1], yh)
        e2e_host_s = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([e2e_host_s], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_host_s = float(t.item())
        e2e_value = world * args.steps / e2e_host_s
    except Exception as exc:  # the graph-replay figure above stands in
        e2e_api = f"graph replay with pinned copies (host-buffer call failed: {str(exc)[:120]})"
        e2e_value = e2e_graph_value
    ctx.check(stream)

    prefill = prefill_side_timing(ctx, layers[:2], stream) if world == 1 and not args.no_prefill else None

    hbm_peak, _, peak_src = peaks()
    fused = stage_ms[0] == 0 and stage_ms[1] == 0 and stage_ms[3] == 0 and stage_ms[4] == 0
    if fused:  # the whole layer is one persistent kernel
        kern_name = "decode_layer_kernel (router, top-k, 9 experts gate/up/down, combine; batch 1)"
        kern_bytes = LAYER_TOKEN_BYTES
    else:
        kern_name = "gemv_kernel<1,gateup> (9 experts x gate+up, batch 1)"
        kern_bytes = GATEUP_BYTES
    # The timed region launches the fused kernel once per step and nothing
    # else, so its average duration there (CUDA events on its stream) is the
    # step time; the multi-kernel path takes the gate/up kernel's own events.
    kern_ms = ms_total / args.steps if fused else stage_ms[2]
    achieved = kern_bytes / (kern_ms / 1000.0) / 1e9 if kern_ms > 0 else None
    traffic = traffic_from_profiles("decode_layer_decode1.txt" if fused else "gemv_gateup_decode1.txt")
    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu and world == 1:
            from oracle import oracle
            kind = "reference" if oracle.available("reference") else "port"
            tps, done, dt, cores = cpu_time_layer(kind, args.cpu_seconds, 64)
            cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": kind,
                   "sample": f"{done} tokens x 1 layer (config 2 shapes) in {dt:.1f} s, weights RAM-resident"}
        layer_gbs = LAYER_TOKEN_BYTES * value / world / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "iq3_xxs(int8)xint16->f32", "data": "synthetic",
            "config": {"workload": "decode1: MoE layer decode, batch 1 (BASELINE config 2)", "hidden": H,
                       "n_experts": E, "top_k": K_TOP, "inter": I, "n_shared": 1, "quant": "IQ3_XXS",
                       "layer_copies": L, "l2": f"inputs larger than L2: steps rotate over {L} layer copies "
                                              f"({L * 1.454:.1f} GB of weights)",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "per_gpu_layer_hbm_gbs": layer_gbs,
                       "per_gpu_layer_hbm_frac": layer_gbs / hbm_peak,
                       "stage_ms": ({"layer_launched_alone": stage_ms[2]} if fused else
                                    dict(zip(["router", "route", "gateup", "down", "combine"], stage_ms))),
                       "prefill4096_side_timing": prefill,
                       "e2e_api": e2e_api,
                       "e2e_graph_replay_tokens_per_s": e2e_graph_value},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": (achieved / hbm_peak) if achieved else None, "traffic": traffic,
                         "kernel": kern_name, "bytes_per_launch": kern_bytes,
                         "peak_source": peak_src},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 4},
            "gpu_launches": (1 if fused else 5) * args.steps,
            "clocks": clk.summary(),
        }
    del chains, e2e_graphs, timed
    ctx.close()
    return line


def run_gpu_ep(args, rank, local_rank, world):
    """BASELINE config 2's layer, expert-parallel over `world` GPUs (the N > 1
    default).  Rank r holds units [r*NU/N, (r+1)*NU/N) of every routed expert
    of every layer copy (--ep-split units: 1/N of each expert's 1536
    intermediate rows), or routed experts [r*E/N, (r+1)*E/N) (--ep-split
    experts), plus the shared expert, and brings its own token each step.  A step (one
    token per rank through one layer) is one persistent kernel per rank,
    gpeed_moe_decode_ep: the tokens go to every rank over NVLink peer memory,
    all N are routed, this rank's share of each pick runs and adds its sums
    into the owning rank's output, the launch ends when the other ranks' sums
    into this rank's output are done.  With --ep-nccl the exchanges are NCCL
    collectives instead (all-gather of the tokens, gpeed_moe_decode_partial,
    reduce-scatter of the partial outputs).  Layer copies rotate so each
    step's weights come from HBM, and the steps are captured back to back in
    CUDA graphs."""
    import torch
    import torch.distributed as dist

    from gpeed_b200 import Context, MoeConfig, MoeLayer
    from gpeed_b200.ep import ExpertParallelLayer, PeerDecode

    torch.cuda.set_device(local_rank)
    ctx = Context(local_rank)
    cfg = MoeConfig()
    L = args.layers
    sliced = args.ep_split == "units"
    if sliced:
        u_lo, u_cnt = MoeLayer.unit_slice(cfg, rank, world)
        layers = [MoeLayer(ctx, cfg, layer_id=l).synth(router_for(l), None, 1000 + l, 0).slice_units(u_lo, u_cnt)
                  for l in range(L)]
        lo, cnt = 0, E
    else:
        lo, cnt = ExpertParallelLayer.expert_range(cfg, rank, world)
        layers = [MoeLayer(ctx, cfg, layer_id=l).synth_range(router_for(l), None, 1000 + l, 0, lo, cnt)
                  for l in range(L)]
    peer = not args.ep_nccl
    pd = PeerDecode(ctx, cfg, layers) if peer else None
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    xs = [tokens(1, 100 + l + 7919 * rank).cuda() for l in range(L)]  # this rank's token per layer copy
    x_all = [torch.empty(world, H, dtype=torch.bfloat16, device="cuda") for _ in range(L)]
    y_part = [torch.empty(world, H, device="cuda") for _ in range(L)]
    ys = [torch.empty(1, H, device="cuda") for _ in range(L)]

    def step(l, ev=None, topk_ids=None):
        if ev:
            ev[0].record(stream)
        if peer:
            if ev:
                ev[1].record(stream)
            pd.forward(l, xs[l], ys[l], topk_ids=topk_ids, stream=stream)
            if ev:
                ev[2].record(stream)
        else:
            dist.all_gather_into_tensor(x_all[l], xs[l])
            if ev:
                ev[1].record(stream)
            layers[l].decode_partial(x_all[l], rank, y_part[l], topk_ids=topk_ids, stream=stream)
            if ev:
                ev[2].record(stream)
            dist.reduce_scatter_tensor(ys[l], y_part[l], op=dist.ReduceOp.SUM)
        if ev:
            ev[3].record(stream)

    with torch.cuda.stream(stream):
        for l in range(L):  # communicators, scratch and kernel attributes set up outside capture
            step(l)
    stream.synchronize()
    ctx.check(stream)

    def chain(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for l in range(n):
                step(l)
        return g

    chains = {L: chain(L)}
    if args.steps % L:
        chains[args.steps % L] = chain(args.steps % L)

    def run_steps(n):
        for _ in range(n // L):
            chains[L].replay()
        if n % L:
            if n % L not in chains:
                chains[n % L] = chain(n % L)
            chains[n % L].replay()

    with torch.cuda.stream(stream):
        run_steps(args.warmup)
    stream.synchronize()
    dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            ev0.record(stream)
            run_steps(args.steps)
            ev1.record(stream)
        stream.synchronize()
        ms_total = ev0.elapsed_time(ev1)
        # the same work ~1.5 s more, so the sampler sees the clocks under load:
        # the round count is agreed first (every rank runs the same collectives)
        t = torch.tensor([ms_total], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
        n_soak = max(1, min(400, int(1500.0 / max(ms_max / args.steps * 25 * L, 1e-3))))
        with torch.cuda.stream(stream):
            for _ in range(n_soak):
                run_steps(25 * L)
        stream.synchronize()
    dist.barrier()
    ctx.check(stream)
    value = world * args.steps / (ms_max / 1000.0)

    # ---- per-phase split (events between the phases, eager launches) ----
    n_prof = max(4 * L, 32)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_prof)]
    with torch.cuda.stream(stream):
        for i in range(n_prof):
            step(i % L, evs[i])
    stream.synchronize()
    ph = [sum(evs[i][k].elapsed_time(evs[i][k + 1]) for i in range(n_prof)) / n_prof for k in range(3)]
    # routed slots this rank ran per layer copy (picks of all tokens in its range): the kernel's bytes
    slots = []
    for l in range(L):  # (a step on every rank)
        ids = torch.empty(world, K_TOP, dtype=torch.int32, device="cuda")
        with torch.cuda.stream(stream):
            step(l, topk_ids=ids)
        stream.synchronize()
        g = ids.cpu().numpy()
        slots.append(int(((g >= lo) & (g < lo + cnt)).sum()))
    torch.cuda.synchronize()
    mean_slots = sum(slots) / L
    # expert bytes this rank streams: its slice of every pick, or its range's
    # picks, and its own token's shared expert
    expert_units = (mean_slots / world if sliced else mean_slots) + 1
    kern_bytes = expert_units * EXPERT_BYTES + ROUTER_BYTES + world * H * (2 + 4)
    achieved = kern_bytes / (ph[1] * 1e-3) / 1e9

    # ---- end to end through the public API with host buffers ----
    x_host = tokens(args.steps, 555 + rank).pin_memory()
    y_host = torch.empty(H, dtype=torch.float32).pin_memory()
    x_slot = x_host[0:1].clone().pin_memory()
    e2e_graphs = []
    for l in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            xs[l].copy_(x_slot, non_blocking=True)
            step(l)
            y_host.copy_(ys[l][0], non_blocking=True)
        e2e_graphs.append(g)
    for i in range(args.warmup):
        with torch.cuda.stream(stream):
            e2e_graphs[i % L].replay()
        stream.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        x_slot.copy_(x_host[i:i + 1])       # the step's input lands in the pinned staging buffer
        with torch.cuda.stream(stream):
            e2e_graphs[i % L].replay()
        stream.synchronize()                # the step's result is on the host
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = world * args.steps / float(t.item())
    ctx.check(stream)

    hbm_peak, _, peak_src = peaks()
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "iq3_xxs(int8)xint16->f32", "data": "synthetic",
            "config": {"workload": "decode1: MoE layer decode, batch 1 (BASELINE config 2)", "hidden": H,
                       "n_experts": E, "top_k": K_TOP, "inter": I, "n_shared": 1, "quant": "IQ3_XXS",
                       "layer_copies": L, "l2": f"inputs larger than L2: steps rotate over {L} layer copies",
                       "parallelism": (f"ep{world}: " + (f"1/{world} of every routed expert's units per GPU ({u_cnt} "
                                                         f"of {I // 32} units of 32 rows) + the shared expert"
                                                         if sliced else
                                                         f"{cnt} routed experts per GPU + the shared expert") +
                                       "; one token per GPU per step; " +
                                       ("one persistent kernel per GPU exchanging tokens and partial outputs over "
                                        "NVLink peer memory (no collective library)" if peer else
                                        "NCCL all-gather of tokens, one persistent kernel per GPU, NCCL "
                                        "reduce-scatter of partial outputs")),
                       "phase_ms": ({"kernel": ph[1]} if peer else
                                    {"all_gather": ph[0], "experts_kernel": ph[1], "reduce_scatter": ph[2]}),
                       "routed_slots_per_gpu_rank0": mean_slots,
                       "expert_equivalents_streamed_per_gpu": expert_units,
                       "per_gpu_kernel_hbm_gbs": achieved},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "traffic": None,
                         "kernel": "decode_layer_kernel, expert-parallel share (rank 0): routing of all tokens, "
                                   "its routed picks + own shared expert" + (", peer exchange" if peer else ""),
                         "bytes_per_launch": kern_bytes, "peak_source": peak_src},
            "cpu_baseline": None,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 4},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
        }
    del chains, e2e_graphs
    if pd is not None:
        pd.close()
    ctx.close()
    return line


def run_glm5_decode(args):
    """Batch-1 decode of one MoE layer at the reference model's own default
    MoE shape (model_config.h:25, 59-60: hidden 4096, moe_inter 2048, 288
    routed experts, top-8, one shared expert) through the same persistent
    kernel: the kernel instantiated for H = 4096 (16 compute warps, down
    chunks of 2048 rows).  Steps rotate over --layers layer copies (3.7 GB
    each with the column-slab copy of W_down), captured back to back in CUDA
    graphs as for decode1; algorithmic bytes per step: 9 experts x 3 matrices
    of IQ3_XXS + the fp32 router + x and y."""
    import torch

    from gpeed_b200 import Context, MoeConfig, MoeLayer

    Hg, Ig, Eg = 4096, 2048, 288
    cfg = MoeConfig(hidden=Hg, inter=Ig, n_experts=Eg)
    L = min(args.layers, 6)
    ctx = Context(0)
    rng = np.random.default_rng(7)
    layers = [MoeLayer(ctx, cfg, layer_id=l).synth((rng.standard_normal((Eg, Hg)) * 0.02).astype(np.float32), None,
                                                     seed=2000 + l, stream0=0) for l in range(L)]
    xs = [torch.from_numpy(rng.standard_normal((1, Hg)).astype(np.float32)).to(torch.bfloat16).cuda() for _ in range(L)]
    ys = [torch.empty(1, Hg, device="cuda") for _ in range(L)]
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for l in range(L):
            layers[l].forward(xs[l], ys[l], stream=stream)
    stream.synchronize()
    ctx.check(stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for l in range(L):
            layers[l].forward(xs[l], ys[l], stream=stream)
    reps = max(1, args.steps // L)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup // L)):
            g.replay()
    stream.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(reps):
                g.replay()
            ev1.record(stream)
        stream.synchronize()
        soak_t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            while time.perf_counter() - soak_t0 < 1.0:
                for _ in range(25):
                    g.replay()
                stream.synchronize()
    ctx.check(stream)
    steps = reps * L
    ms = ev0.elapsed_time(ev1) / steps
    expert = 3 * Ig * (Hg // 256) * 98
    step_bytes = 9 * expert + Eg * Hg * 4 + Hg * (2 + 4)
    hbm_peak, _, peak_src = peaks()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    del g
    ctx.close()
    return {"metric": METRIC, "value": 1000.0 / ms, "unit": "tokens/s", "n_gpus": 1, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "iq3_xxs(int8)xint16->f32", "data": "synthetic",
            "config": {"workload": "glm5: MoE layer decode, batch 1, at the reference model's default MoE shape",
                       "hidden": Hg, "n_experts": Eg, "top_k": 8, "inter": Ig, "n_shared": 1, "quant": "IQ3_XXS",
                       "layer_copies": L, "l2": "inputs larger than L2: steps rotate over the layer copies"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "traffic": None, "kernel": "decode_layer_kernel<4096, 2048> (batch 1)",
                         "bytes_per_launch": step_bytes, "peak_source": peak_src},
            "cpu_baseline": None, "e2e": None, "gpu_launches": steps, "clocks": clk.summary()}


PREFILL_FLOPS_PER_TOKEN = (K_TOP + 1) * 3 * 2 * I * H + 2 * E * H   # experts + router, per token


def run_prefill(args, rank, local_rank, world):
    """one MoE layer over a 4096-token batch (tensor-bound).
    A step is one forward of the whole batch through one layer; the experts run
    as grouped GEMMs on the tensor cores (fp16 operands, fp32 accumulation)."""
    import torch
    import torch.distributed as dist

    from gpeed_b200 import Context, MoeConfig, MoeLayer
    from gpeed_b200 import _capi

    n = args.tokens
    torch.cuda.set_device(local_rank)
    ctx = Context(local_rank)
    cfg = MoeConfig()
    L = max(1, min(args.layers, 2))
    layers = [MoeLayer(ctx, cfg, layer_id=l).synth(router_for(l), None, seed=1000 + l, stream0=0) for l in range(L)]
    stream = torch.cuda.Stream()
    xs = [tokens(n, 300 + l).cuda() for l in range(L)]
    ys = [torch.empty(n, H, device="cuda") for _ in range(L)]
    with torch.cuda.stream(stream):
        for l in range(L):
            layers[l].forward(xs[l], ys[l], stream=stream)
    stream.synchronize()
    ctx.check(stream)
    graphs = []
    for l in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            layers[l].forward(xs[l], ys[l], stream=stream)
        graphs.append(g)

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs[i % L].replay()
    stream.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for i in range(args.steps):
                graphs[i % L].replay()
            ev1.record(stream)
        stream.synchronize()
        ms_total = ev0.elapsed_time(ev1)
    barrier()
    ctx.check(stream)
    if world > 1:
        t = torch.tensor([ms_total], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    value = world * n * args.steps / (ms_total / 1000.0)

    # per-kernel timing (events between the forward's kernels): gate/up and down GEMMs
    _capi.call("gpeed_ctx_profile", ctx.handle, 1)
    with torch.cuda.stream(stream):
        for i in range(max(args.steps, 4)):
            layers[i % L].forward(xs[i % L], ys[i % L], stream=stream)
    stage = (ctypes.c_float * 5)()
    calls = ctypes.c_int()
    _capi.call("gpeed_ctx_profile_read", ctx.handle, stage, ctypes.byref(calls))
    _capi.call("gpeed_ctx_profile", ctx.handle, 0)
    stage_ms = list(stage)

    # end to end with host buffers: x in, y out every step
    x_host = tokens(n, 555).pin_memory()
    y_host = torch.empty(n, H, dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_steps = max(3, args.steps // 4)
    for i in range(e2e_steps):
        with torch.cuda.stream(stream):
            xs[0].copy_(x_host, non_blocking=True)
            layers[0].forward(xs[0], ys[0], stream=stream)
            y_host.copy_(ys[0], non_blocking=True)
        stream.synchronize()
    e2e_s = time.perf_counter() - t0
    ctx.check(stream)

    _, tf_peak, peak_src = peaks()
    gu_flops = n * (K_TOP + 1) * 2 * 2 * I * H
    dn_flops = n * (K_TOP + 1) * 2 * I * H
    line = None
    if rank == 0:
        gu_tf = gu_flops / (stage_ms[2] * 1e-3) / 1e12 if stage_ms[2] > 0 else None
        dn_tf = dn_flops / (stage_ms[3] * 1e-3) / 1e12 if stage_ms[3] > 0 else None
        step_tf = PREFILL_FLOPS_PER_TOKEN * n / (ms_total / args.steps * 1e-3) / 1e12
        cpu = None
        if not args.no_cpu and world == 1:
            from oracle import oracle
            kind = "reference" if oracle.available("reference") else "port"
            tps, done, dt, cores = cpu_time_layer(kind, args.cpu_seconds, 64)
            cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": kind,
                   "sample": f"{done} tokens x 1 layer (config 2 shapes, token by token) in {dt:.1f} s"}
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 x f16 -> f32 (tcgen05), IQ3_XXS weights decoded in-kernel",
            "data": "synthetic",
            "config": {"workload": f"prefill{n}: MoE layer over a {n}-token batch (BASELINE config 4)", "hidden": H,
                       "n_experts": E, "top_k": K_TOP, "inter": I, "n_shared": 1, "quant": "IQ3_XXS",
                       "layer_copies": L, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "step_tflops": step_tf,
                       "stage_ms": dict(zip(["router", "route+gather", "gateup_gemm", "down_gemm", "combine"],
                                            stage_ms))},
            "roofline": {"bound": "tensor", "achieved": gu_tf, "peak": tf_peak, "unit": "TFLOP/s",
                         "frac": (gu_tf / tf_peak) if gu_tf and tf_peak else None, "traffic": None,
                         "kernel": "tc_moe_kernel<gate/up> (grouped GEMM over the expert slot list)",
                         "flops_per_launch": gu_flops, "down_tflops": dn_tf, "peak_source": peak_src},
            "cpu_baseline": cpu,
            "e2e": {"value": n * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": n * H * 2,
                    "d2h_bytes_per_step": n * H * 4},
            "gpu_launches": 7 * args.steps,
            "clocks": clk.summary(),
        }
    del graphs
    ctx.close()
    return line


def zipf_bias(seed):
    """Selection bias that skews expert loads toward Zipf(s=1.1):
    b_e = 0.25 * (-1.1 * ln(rank_e + 1)) over a seeded random ranking."""
    rank = np.random.default_rng(seed).permutation(E)
    return (0.25 * (-1.1 * np.log(rank + 1.0))).astype(np.float32)


def run_ragged(args, rank, local_rank, world):
    """a ragged continuous-batching decode step, 64 tokens
    through one MoE layer with Zipf-skewed expert loads (quantised GEMV path).
    Steps cycle over the layer copies (each step's weights come from HBM)."""
    import torch

    from gpeed_b200 import Context, MoeConfig, MoeLayer
    from gpeed_b200 import _capi

    n = args.batch
    torch.cuda.set_device(local_rank)
    ctx = Context(local_rank)
    cfg = MoeConfig()
    L = max(1, args.layers)
    layers = [MoeLayer(ctx, cfg, layer_id=l).synth(router_for(l), zipf_bias(50 + l), seed=1000 + l, stream0=0)
              for l in range(L)]
    stream = torch.cuda.Stream()
    xs = [tokens(n, 700 + l).cuda() for l in range(L)]
    ys = [torch.empty(n, H, device="cuda") for _ in range(L)]
    ids = [torch.empty(n, K_TOP, dtype=torch.int32, device="cuda") for _ in range(L)]
    with torch.cuda.stream(stream):
        for l in range(L):
            layers[l].forward(xs[l], ys[l], topk_ids=ids[l], stream=stream)
    stream.synchronize()
    ctx.check(stream)
    # algorithmic bytes per step: router, every touched routed expert once, the shared expert
    touched = [len(np.unique(t.cpu().numpy())) for t in ids]
    step_bytes = [E * H * 4 + (k + 1) * EXPERT_BYTES + n * H * 2 + n * H * 4 for k in touched]
    graphs = []
    for l in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            layers[l].forward(xs[l], ys[l], stream=stream)
        graphs.append(g)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs[i % L].replay()
    stream.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for i in range(args.steps):
                graphs[i % L].replay()
            ev1.record(stream)
        stream.synchronize()
        ms_total = ev0.elapsed_time(ev1)
    ctx.check(stream)
    value = world * n * args.steps / (ms_total / 1000.0)
    mean_bytes = sum(step_bytes[i % L] for i in range(args.steps)) / args.steps

    _capi.call("gpeed_ctx_profile", ctx.handle, 1)
    with torch.cuda.stream(stream):
        for i in range(max(args.steps, 4)):
            layers[i % L].forward(xs[i % L], ys[i % L], stream=stream)
    stage = (ctypes.c_float * 5)()
    calls = ctypes.c_int()
    _capi.call("gpeed_ctx_profile_read", ctx.handle, stage, ctypes.byref(calls))
    _capi.call("gpeed_ctx_profile", ctx.handle, 0)
    stage_ms = list(stage)

    x_host = tokens(n, 555).pin_memory()
    y_host = torch.empty(n, H, dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_steps = max(3, args.steps // 4)
    for i in range(e2e_steps):
        with torch.cuda.stream(stream):
            xs[i % L].copy_(x_host, non_blocking=True)
            layers[i % L].forward(xs[i % L], ys[i % L], stream=stream)
            y_host.copy_(ys[i % L], non_blocking=True)
        stream.synchronize()
    e2e_s = time.perf_counter() - t0
    ctx.check(stream)

    hbm_peak, _, peak_src = peaks()
    tc = n >= _capi.TC_MIN_TOKENS_DEFAULT
    tc_dtype = "f16 x f16 -> f32 (tcgen05), IQ3_XXS weights decoded in-kernel"
    line = None
    if rank == 0:
        achieved = mean_bytes / (ms_total / args.steps * 1e-3) / 1e9
        expert_ms = stage_ms[2] + stage_ms[3]
        expert_bytes = sum((k + 1) * EXPERT_BYTES for k in touched) / L
        cpu = None
        if not args.no_cpu and world == 1:
            from oracle import oracle
            kind = "reference" if oracle.available("reference") else "port"
            tps, done, dt, cores = cpu_time_layer(kind, args.cpu_seconds, 64)
            cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": kind,
                   "sample": f"{done} tokens x 1 layer (config 2 shapes, token by token) in {dt:.1f} s"}
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": tc_dtype if tc else "iq3_xxs(int8)xint16->f32", "data": "synthetic",
            "config": {"workload": f"ragged{n}: {n}-token decode step, Zipf(1.1)-skewed expert loads (BASELINE config 3)",
                       "hidden": H, "n_experts": E, "top_k": K_TOP, "inter": I, "n_shared": 1, "quant": "IQ3_XXS",
                       "layer_copies": L, "touched_experts_per_layer": touched,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "each step's layer copy (>1 GB of experts) exceeds L2",
                       "expert_path": "tensor-core grouped GEMMs" if tc else "quantised GEMV",
                       "stage_ms": dict(zip(["router", "route+gather" if tc else "route", "gateup", "down", "combine"],
                                            stage_ms))},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak if hbm_peak else None, "traffic": None,
                         "kernel": "whole layer step (router, route, expert gate/up and down, combine): algorithmic "
                                   "bytes of the touched experts / step time",
                         "bytes_per_step": mean_bytes,
                         "expert_stage_gbs": expert_bytes / (expert_ms * 1e-3) / 1e9 if expert_ms > 0 else None,
                         "peak_source": peak_src},
            "cpu_baseline": cpu,
            "e2e": {"value": n * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": n * H * 2,
                    "d2h_bytes_per_step": n * H * 4},
            # per step: router 2 (GEMM, split sum), top-k, route, gather, gate/up, down, combine; GEMV path: 6
            "gpu_launches": (8 if tc else 6) * args.steps,
            "clocks": clk.summary(),
        }
    del graphs
    ctx.close()
    return line


def run_stack(args, rank, local_rank, world):
    """BASELINE config 5 on one GPU: a 40-layer MoE decode stack (160 experts +
    shared each, IQ3_XXS, ~58 GB), swept over decode batches of 1, 8, 32, 128
    and 256 tokens with uniform-random router logits.  A step is one batch
    through all 40 layers, the 40 forwards captured back to back in one CUDA
    graph (batch 1: the fused decode kernel; 2-7: the quantised GEMV path; 8
    and up: the tensor-core grouped GEMMs).  Each layer reads its own static
    input (the timing does not depend on the values, and chaining unnormalised
    MoE outputs through 40 layers would overflow)."""
    import torch

    from gpeed_b200 import Context, MoeConfig, MoeLayer

    torch.cuda.set_device(local_rank)
    ctx = Context(local_rank)
    cfg = MoeConfig()
    NL = 40
    layers = [MoeLayer(ctx, cfg, layer_id=l).synth(router_for(2000 + l), None, seed=5000 + l, stream0=0)
              for l in range(NL)]
    stream = torch.cuda.Stream()
    sweep = []
    with ClockSampler(local_rank) as clk:
        for B in (1, 8, 32, 128, 256):
            xs = [tokens(B, 9000 + 7 * l + B).cuda() for l in range(NL)]
            ys = [torch.empty(B, H, device="cuda") for _ in range(NL)]
            with torch.cuda.stream(stream):
                for l in range(NL):
                    layers[l].forward(xs[l], ys[l], stream=stream)
            stream.synchronize()
            ctx.check(stream)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for l in range(NL):
                    layers[l].forward(xs[l], ys[l], stream=stream)
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    g.replay()
            stream.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                ev0.record(stream)
                for _ in range(args.steps):
                    g.replay()
                ev1.record(stream)
            stream.synchronize()
            ctx.check(stream)
            ms = ev0.elapsed_time(ev1) / args.steps
            sweep.append({"batch": B, "ms_per_stack": ms, "ms_per_layer": ms / NL, "tokens_per_s": B / (ms * 1e-3)})
            del g
    hbm_peak, _, peak_src = peaks()
    line = None
    if rank == 0:
        b1 = sweep[0]
        achieved = LAYER_TOKEN_BYTES / (b1["ms_per_layer"] * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": world * sweep[-1]["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sweep[-1]["ms_per_stack"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "batch 1: iq3_xxs(int8)xint16->f32; 8+: f16 x f16 -> f32 (tcgen05)", "data": "synthetic",
            "config": {"workload": "stack40: 40 MoE layers, decode batch sweep 1/8/32/128/256 (BASELINE config 5, "
                                   "one GPU; value = batch 256 through the stack)",
                       "hidden": H, "n_experts": E, "top_k": K_TOP, "inter": I, "n_shared": 1, "quant": "IQ3_XXS",
                       "layers": NL, "expert_bytes_per_layer": E * EXPERT_BYTES + EXPERT_BYTES,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU (all 40 layers resident)",
                       "sweep": sweep},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak if hbm_peak else None, "traffic": None,
                         "kernel": "batch 1: decode_layer_kernel per layer inside the 40-layer graph",
                         "bytes_per_launch": LAYER_TOKEN_BYTES, "peak_source": peak_src},
            "cpu_baseline": None,
            "e2e": None,
            "gpu_launches": NL * args.steps,
            "clocks": clk.summary(),
        }
    ctx.close()
    return line


def run_prefill_ep(args, rank, local_rank, world):
    """BASELINE config 4, expert-parallel over the GPUs of one box: each rank
    holds E/world routed experts (a contiguous range) plus the shared expert and
    its own 4096-token batch; every step routes the batch, sends each (token,
    expert) row to its expert's rank and the results back with NCCL all-to-all,
    runs the received rows and the shared expert through the tensor-core GEMMs
    and combines.  Weak scaling: tokens per GPU are fixed as N grows."""
    import torch
    import torch.distributed as dist

    from gpeed_b200 import Context, MoeConfig
    from gpeed_b200.ep import CudaExecutor, ExpertParallelLayer

    n = args.tokens
    torch.cuda.set_device(local_rank)
    ctx = Context(local_rank)
    cfg = MoeConfig()
    L = max(1, min(args.layers, 2))
    lo, cnt = ExpertParallelLayer.expert_range(cfg, rank, world)
    layers = []
    for l in range(L):
        ex = CudaExecutor(ctx, cfg, 500 + l, lo, cnt)
        ex.synth(router_for(l), None, 1000 + l, 0)
        layers.append(ExpertParallelLayer(cfg, ex))
    xs = [tokens(n, 300 + 17 * rank + l).cuda() for l in range(L)]

    for i in range(args.warmup):
        layers[i % L].forward(xs[i % L])
    torch.cuda.synchronize()
    ctx.check()
    dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        ev0.record()
        for i in range(args.steps):
            layers[i % L].forward(xs[i % L])
        ev1.record()
        torch.cuda.synchronize()
        ms_total = ev0.elapsed_time(ev1)
    dist.barrier()
    ctx.check()
    t = torch.tensor([ms_total], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    value = world * n * args.steps / (ms_total / 1000.0)

    # end to end: this rank's batch from pinned host memory, y back to the host, every step
    x_host = tokens(n, 555 + rank).pin_memory()
    y_host = torch.empty(n, H, dtype=torch.float32).pin_memory()
    e2e_steps = max(3, args.steps // 4)
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        xs[0].copy_(x_host, non_blocking=True)
        y = layers[0].forward(xs[0])
        y_host.copy_(y, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = torch.tensor([time.perf_counter() - t0], device="cuda")
    dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    ctx.check()

    _, tf_peak, peak_src = peaks()
    line = None
    if rank == 0:
        gpu_tf = PREFILL_FLOPS_PER_TOKEN * n / (ms_total / args.steps * 1e-3) / 1e12  # per GPU, whole step
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 x f16 -> f32 (tcgen05), IQ3_XXS weights decoded in-kernel",
            "data": "synthetic",
            "config": {"workload": f"prefill{n}-ep: MoE layer over {n} tokens per GPU, experts split over the GPUs "
                                   "(BASELINE config 4)", "hidden": H, "n_experts": E, "top_k": K_TOP, "inter": I,
                       "n_shared": 1, "quant": "IQ3_XXS", "layer_copies": L, "experts_per_gpu": cnt,
                       "parallelism": f"ep{world}: NCCL all-to-all dispatch and combine, shared expert replicated"},
            "roofline": {"bound": "tensor", "achieved": gpu_tf, "peak": tf_peak, "unit": "TFLOP/s",
                         "frac": gpu_tf / tf_peak if tf_peak else None, "traffic": None,
                         "kernel": "whole expert-parallel step per GPU (routing, two all-to-alls, grouped GEMMs, "
                                   "combine)", "flops_per_token": PREFILL_FLOPS_PER_TOKEN, "peak_source": peak_src},
            "cpu_baseline": None,
            "e2e": {"value": world * n * e2e_steps / float(e2e_s.item()), "unit": "tokens/s",
                    "h2d_bytes_per_step": n * H * 2, "d2h_bytes_per_step": n * H * 4},
            # per step: route 4 (router, split sum, top-k, route), pack 3, experts 2 x 6, combine 1
            "gpu_launches": 20 * args.steps,
            "clocks": clk.summary(),
        }
    ctx.close()
    return line


CODEC_TYPES = {8: ("Q8_0", 34, 32, (0,)), 10: ("Q2_K", 84, 256, (80, 82)), 11: ("Q3_K", 110, 256, (108,)),
               14: ("Q6_K", 210, 256, (208,)), 18: ("IQ3_XXS", 98, 256, (0,)), 21: ("IQ3_S", 110, 256, (0,)),
               22: ("IQ2_S", 82, 256, (0,)), 23: ("IQ4_XS", 136, 256, (0,)), 1: ("F16", 2, 1, ()),
               30: ("BF16", 2, 1, ())}


def run_codecs(args):
    """gpeed_dequantize over 2^26 values per codec (fp32 output 256 MiB, past L2):
    achieved (read + write) GB/s per codec against the measured HBM copy peak."""
    import ctypes
    import numpy as np
    import torch
    from gpeed_b200 import _capi
    hbm_peak, _, peak_src = peaks()
    n = 1 << 26
    rng = np.random.default_rng(0)
    per = {}
    tot_bytes = tot_ms = 0.0
    launches = 0
    with ClockSampler(0) as clk:
        for t, (name, bb, vals, dofs) in CODEC_TYPES.items():
            nb = n // vals
            raw = np.frombuffer(rng.bytes(bb * nb), np.uint8).reshape(nb, bb).copy()
            for o in dofs:
                raw[:, o:o + 2] = np.frombuffer((1e-4 + 1.9e-3 * rng.random(nb)).astype(np.float16).tobytes(),
                                                np.uint8).reshape(nb, 2)
            if vals == 1:  # finite values for the element-wise types
                raw = np.frombuffer((rng.standard_normal(n)).astype(np.float16 if t == 1 else np.float32)
                                    .tobytes(), np.uint8).copy()
                if t == 30:
                    raw = raw.view(np.uint32) >> 16
                    raw = raw.astype(np.uint16).view(np.uint8)
            src = torch.from_numpy(raw).cuda()
            dst = torch.empty(n, dtype=torch.float32, device="cuda")
            call = lambda: _capi.call("gpeed_dequantize", t, ctypes.c_void_p(src.data_ptr()),
                                      ctypes.c_void_p(dst.data_ptr()), ctypes.c_uint64(n), None)
            for _ in range(args.warmup):
                call()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                call()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            byt = raw.size + 4 * n
            per[name] = {"ms": ms, "gb_s": byt / ms / 1e6, "frac": byt / ms / 1e6 / hbm_peak,
                         "bytes_read_per_value": raw.size / n}
            tot_bytes += byt * args.steps
            tot_ms += ms * args.steps
            launches += args.steps
            del src, dst
    gbs = tot_bytes / tot_ms / 1e6
    return {"metric": "GGUF dequantisation throughput (read + write bytes)", "value": gbs, "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot_ms / launches,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "codecs: gpeed_dequantize, 2^26 values per codec (output 256 MiB, past L2)",
                       "codecs": per},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "traffic": None, "peak_source": peak_src},
            "gpu_launches": launches, "clocks": clk.summary()}


def run_dense(args):
    """Dense SwiGLU MLP of the leading layers (H 5120, intermediate 12288, IQ3_XXS)
    through gpeed_dense_mlp_forward: batch 1 (GEMV, HBM-bound) and --tokens
    (tensor cores)."""
    import ctypes
    import torch
    from gpeed_b200 import Context, WeightStore, _capi
    hbm_peak, tf_peak, peak_src = peaks()
    Hd, Id = H, 12288
    ctx = Context(0)
    ws = WeightStore(ctx)
    L = 4  # weight copies rotated so the batch-1 reads come from HBM (4 x 3 x 22.6 MB)
    for c in range(L):
        for m, (nm, rows, inn) in enumerate([("gate", Id, Hd), ("up", Id, Hd), ("down", Hd, Id)]):
            raw = torch.empty(rows * inn // 256 * 98, dtype=torch.uint8, device="cuda")
            _capi.call("gpeed_synth_iq3xxs", ctypes.c_void_p(raw.data_ptr()), ctypes.c_uint64(5),
                       ctypes.c_uint64(10 * c + m), ctypes.c_uint64(0), ctypes.c_uint64(rows * inn // 256), None)
            ws.add(f"{c}.{nm}", raw, rows, inn)
    wbytes = 3 * Hd * Id // 256 * 98
    res = {}
    with ClockSampler(0) as clk:
        for n in (1, args.tokens):
            X = torch.randn(n, Hd, device="cuda").to(torch.bfloat16)
            Y = torch.empty(n, Hd, dtype=torch.float32, device="cuda")
            step = lambda c: ws.dense_mlp(f"{c}.gate", f"{c}.up", f"{c}.down", X, Y)
            for i in range(args.warmup):
                step(i % L)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(args.steps):
                step(i % L)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            res[n] = {"ms": ms, "tokens_s": n / ms * 1e3, "weight_gb_s": wbytes / ms / 1e6,
                      "hbm_frac": wbytes / ms / 1e6 / hbm_peak,
                      "tflops": 2 * 3 * Hd * Id * n / ms / 1e9, "tensor_frac": 2 * 3 * Hd * Id * n / ms / 1e9 / tf_peak}
    ctx.check()
    ctx.close()
    return {"metric": "dense SwiGLU MLP tokens/s (IQ3_XXS, H 5120, intermediate 12288)", "value": res[1]["tokens_s"],
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": res[1]["ms"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint16 / fp16",
            "data": "synthetic", "config": {"workload": f"dense: batch 1 and {args.tokens} tokens, {L} weight copies rotated",
                                            "batches": res},
            "roofline": {"bound": "hbm", "achieved": res[1]["weight_gb_s"], "peak": hbm_peak, "unit": "GB/s",
                         "frac": res[1]["hbm_frac"], "traffic": None, "peak_source": peak_src},
            "gpu_launches": None, "clocks": clk.summary()}


def run_mhc(args):
    """mHC mixing + RMSNorm before the MoE layer and the stream update after it
    (N = 4 streams of H = 5120): batch 1 and --tokens.  Each measurement replays
    a CUDA graph of R calls over R different stream buffers (and, at batch 1,
    R different fn matrices, as successive layers would read), so launch
    overhead and L2 residency do not flatter the numbers."""
    import torch
    from gpeed_b200 import Context
    from gpeed_b200.moe import mhc_post, mhc_pre
    hbm_peak, _, peak_src = peaks()
    Nh, W = 4, 24
    ctx = Context(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    base, scale, nw = torch.randn(W, device="cuda"), torch.ones(3, device="cuda"), torch.ones(H, device="cuda")
    res = {}
    launches = 0
    with ClockSampler(0) as clk:
        for n in (1, args.tokens):
            R = 64 if n == 1 else 2
            S = [torch.randn(n, Nh, H, device="cuda", generator=g) for _ in range(R)]
            F = [torch.randn(W, Nh * H, device="cuda", generator=g) * 0.02 for _ in range(R if n == 1 else 1)]
            mlp = torch.randn(n, H, device="cuda", generator=g)
            outs = []
            for i in range(max(args.warmup, 3)):
                outs = [mhc_pre(ctx, S[r], F[r % len(F)], base, scale, nw) for r in range(R)]
                for r in range(R):
                    mhc_post(ctx, S[r], mlp, outs[r][1], outs[r][2], out=S[r])
            torch.cuda.synchronize()
            gp_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gp_):
                outs = [mhc_pre(ctx, S[r], F[r % len(F)], base, scale, nw) for r in range(R)]
            gq = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gq):
                for r in range(R):
                    mhc_post(ctx, S[r], mlp, outs[r][1], outs[r][2], out=S[r])
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            reps = max(1, args.steps // R)
            gp_.replay()
            gq.replay()
            torch.cuda.synchronize()
            ev[0].record()
            for _ in range(reps):
                gp_.replay()
            ev[1].record()
            for _ in range(reps):
                gq.replay()
            ev[2].record()
            torch.cuda.synchronize()
            t_pre = ev[0].elapsed_time(ev[1]) / (reps * R)
            t_post = ev[1].elapsed_time(ev[2]) / (reps * R)
            launches += reps * R * 3
            pre_bytes = 2 * n * Nh * H * 4 + W * Nh * H * 4 + n * H * 2   # streams twice, fn once, bf16 x
            post_bytes = 2 * n * Nh * H * 4 + n * H * 4
            res[n] = {"pre_us": t_pre * 1e3, "post_us": t_post * 1e3, "pre_gb_s": pre_bytes / t_pre / 1e6,
                      "pre_frac": pre_bytes / t_pre / 1e6 / hbm_peak, "post_gb_s": post_bytes / t_post / 1e6,
                      "post_frac": post_bytes / t_post / 1e6 / hbm_peak}
            del gp_, gq
    ctx.check()
    ctx.close()
    big = res[args.tokens]
    return {"metric": "mHC mixing + RMSNorm around the MoE layer, tokens/s (pre + post)",
            "value": args.tokens / ((big["pre_us"] + big["post_us"]) * 1e-6), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": (big["pre_us"] + big["post_us"]) / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"mhc: N=4 streams of {H}, batch 1 and {args.tokens}", "batches": res},
            "roofline": {"bound": "hbm", "achieved": big["pre_gb_s"], "peak": hbm_peak, "unit": "GB/s",
                         "frac": big["pre_frac"], "traffic": None, "peak_source": peak_src,
                         "kernel": "mhc_dot_kernel + mhc_finish_kernel"},
            "gpu_launches": launches, "clocks": clk.summary()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="gpeed", choices=["gpeed", "reference"])
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true",
                    help="decode1 at N=1: skip the one-shot config-4 timing reported beside the line")
    ap.add_argument("--workload", default="decode1",
                    choices=["decode1", "ragged64", "prefill", "stack40", "codecs", "dense", "mhc", "glm5"],
                    help="decode1: BASELINE config 2 (default); ragged64: config 3; prefill: config 4")
    ap.add_argument("--tokens", type=int, default=4096, help="batch of the prefill workload")
    ap.add_argument("--batch", type=int, default=64, help="tokens per step of the ragged64 workload")
    ap.add_argument("--ep-nccl", action="store_true",
                    help="expert-parallel decode (--gpus N > 1) with NCCL collectives instead of the peer-memory exchange")
    ap.add_argument("--ep-split", default="units", choices=["units", "experts"],
                    help="expert-parallel decode: each GPU holds 1/N of every expert (units, default) or E/N experts")
    ap.add_argument("--ep", action="store_true",
                    help="prefill with the experts split over the GPUs (NCCL all-to-all); needs --gpus >= 2")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, local_rank, world = env_rank()
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, world)
        return 0
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if args.workload == "prefill" and args.ep and world > 1:
        line = run_prefill_ep(args, rank, local_rank, world)
    elif args.workload == "prefill":
        line = run_prefill(args, rank, local_rank, world)
    elif args.workload == "ragged64":
        line = run_ragged(args, rank, local_rank, world)
    elif args.workload == "stack40":
        line = run_stack(args, rank, local_rank, world)
    elif args.workload in ("codecs", "dense", "mhc", "glm5"):
        fn = {"codecs": run_codecs, "dense": run_dense, "mhc": run_mhc, "glm5": run_glm5_decode}[args.workload]
        line = fn(args) if rank == 0 else None
    elif world > 1:
        line = run_gpu_ep(args, rank, local_rank, world)
    else:
        line = run_gpu(args, rank, local_rank, world)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
