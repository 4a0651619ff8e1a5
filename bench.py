"""Benchmark of the B200 routed-MoE layer (decode) -> one JSON line.

Metric: routed-MoE layer tokens/s + % HBM roofline (decode).
Workload at N=1: configuration C1 -- a DeepSeek-V4-Flash-shaped layer
(hidden 4096, 256 experts, top-6, inter 2048, 2-bit affine g64, routed scaling
2.5, clamped SwiGLU limit 10) decoding one token per step, all experts
resident in HBM arena slots.  A step is one pass of the layer (router ->
dispatch -> gate/up+SwiGLU -> down+combine) over one batch.

* ``value``: tokens/s over exactly K steps replayed from a CUDA graph, inputs
  already in HBM; each step uses its own input and one of ``--layers``
  distinct layers in rotation, so the expert bytes touched between two uses of
  a layer exceed the 126 MB L2 several times over (the inputs are larger than
  L2 in aggregate; no explicit flush).
* ``e2e``: the same metric through the public module API
  (``V4ArenaMoE.__call__``) with the activations in pinned host memory: every
  step copies its input host->device and reads the output back.
* ``roofline``: the gate/up kernel (the dominant one): algorithmic expert bytes
  per launch / its mean duration from CUDA events recorded on its stream
  (``lmoe_moe_layer_staged``), against the measured HBM copy bandwidth.
* ``cpu_baseline``: the CPU oracle (numpy restatement of the reference MLX
  path, which cannot run here) timed on this host on a bounded sample.

Multi-GPU (``--gpus N`` under torchrun): every rank runs the same decode
workload on its own GPU with all experts resident (data-parallel replicas,
weak scaling; the layer has no exchange step in this mode).
``--impl reference`` times the reference's CPU path stand-in (the oracle)
on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "routed-MoE layer tokens/s + % HBM roofline (decode)"
UNIT = "tokens/s"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0  # burst figure of the profiling recipe


def parse():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default="c1")
    p.add_argument("--tokens", type=int, default=None)
    p.add_argument("--experts", type=int, default=None,
                   help="override the expert count (small cases for profiler captures)")
    p.add_argument("--layers", type=int, default=0, help="distinct layers cycled (0 = auto)")
    p.add_argument("--e2e-steps", type=int, default=1000)
    p.add_argument("--kernel-steps", type=int, default=200)
    p.add_argument("--cpu-sample", type=int, default=24, help="decode steps timed for the CPU baseline")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--path", choices=["auto", "decode", "prefill"], default="auto",
                   help="expert-product path of the main workload (lmoe_moe_layer_path)")
    p.add_argument("--prefill-steps", type=int, default=20,
                   help="timed C3 prefill steps reported in the line's 'prefill' object (0 = skip; N=1 only)")
    p.add_argument("--ep", action="store_true",
                   help="expert-parallel layer (experts sharded over the ranks, NCCL all-to-all dispatch/combine)")
    p.add_argument("--layout", choices=["tiled", "rowmajor"], default="tiled",
                   help="expert weights in HBM: pre-tiled (one bulk copy per 16-row tile) or the row-major arrays")
    return p.parse_args()


# ------------------------------------------------------------------ helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peak():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak():
    """Burst cuBLAS bf16 TFLOP/s: the prefill kernels are timed over a region
    of tens of milliseconds, not a seconds-long loop under the power cap."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured burst"
    return FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """NVML sampling of SM clock and throttle reasons during the timed region."""

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        names = {
            "hw_slowdown": getattr(nv, "nvmlClocksThrottleReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksThrottleReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksThrottleReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(nv, "nvmlClocksThrottleReasonSwPowerCap", 0x4),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for k, bit in names.items():
                    if r & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(0.0005)

    def __enter__(self):
        if self.nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thr is not None:
            self._thr.join()

    def summary(self):
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def cpu_baseline_sample(cfg, layer_cpu, xs_cpu, n_tokens: int):
    """Time the numpy oracle (stand-in for the reference MLX CPU path)."""
    import numpy as np

    from oracle import moe_oracle as O
    from oracle.bridge import layer_np, t2np

    L = layer_np(layer_cpu)
    threads = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info

        info = threadpool_info()
        if info:
            threads = max(int(i.get("num_threads", 1)) for i in info)
    except Exception:
        pass
    t0 = time.perf_counter()
    for i in range(n_tokens):
        O.moe_layer(t2np(xs_cpu[i]), L, acc=np.float32)
    dt = time.perf_counter() - t0
    T = xs_cpu[0].shape[0]
    return {"value": T * n_tokens / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n_tokens} decode steps of {cfg.name} (T={T}) through the numpy oracle, float32 "
                      f"accumulation, {dt:.1f}s"}


def workload_config(cfg, T, world, n_layers, layout):
    """The ``config`` object of the JSON line (identical for both arms)."""
    return {
        "workload": f"{cfg.name} decode: hidden {cfg.hidden}, {cfg.n_experts} experts top-{cfg.top_k}, inter "
                    f"{cfg.inter}, {cfg.bits_gate}/{cfg.bits_up}/{cfg.bits_down}-bit affine g{cfg.group_size}, "
                    f"routed scaling {cfg.routed_scaling}, T={T} tokens/step, all experts HBM-resident",
        "global_batch": T * world, "parallelism": f"replicas{world}" if world > 1 else "single",
        "layers_cycled": n_layers,
        "l2": f"{n_layers} distinct layers cycled; >{4 * 126} MB of expert bytes touched between reuses",
        "weights": f"gate/up/down {cfg.bits_gate}/{cfg.bits_up}/{cfg.bits_down}-bit affine g{cfg.group_size} "
                   "(uint32 codes, bf16 scales/biases)",
        "layout": layout,
    }


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from locali_b200 import synth

    cfg = synth.config(args.config) if args.tokens is None else synth.config(args.config, tokens=args.tokens)
    layer = synth.make_layer(cfg, seed=0, device="cpu")
    n = args.steps + args.warmup
    xs = [synth.make_tokens(cfg, cfg.tokens, seed=10 + i, device="cpu") for i in range(n)]
    import numpy as np

    from oracle import moe_oracle as O
    from oracle.bridge import layer_np, t2np

    L = layer_np(layer)
    # each step is one decode step of the workload; the run is bounded to
    # about a minute of CPU work (at most one warm-up step, timed steps until
    # --steps or the time budget is reached)
    for i in range(min(args.warmup, 1)):
        O.moe_layer(t2np(xs[i]), L, acc=np.float32)
    budget_s = 60.0
    done = 0
    t0 = time.perf_counter()
    for i in range(args.warmup, n):
        O.moe_layer(t2np(xs[i]), L, acc=np.float32)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    value = cfg.tokens * done / dt
    threads = os.cpu_count() or 1
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * dt / done, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
        "config": workload_config(cfg, cfg.tokens, world, args.layers or 16, args.layout),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{done} timed decode steps of {cfg.name} ({dt:.1f}s; at most {args.steps} "
                                   "or about 60s) through the numpy oracle (the reference MLX CPU path is not "
                                   "importable here)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(args):
    world, rank, local = dist_env()
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())

    from locali_b200 import _lib, ops, synth

    over = {}
    if args.tokens is not None:
        over["tokens"] = args.tokens
    if args.experts is not None:
        over["n_experts"] = args.experts
    cfg = synth.config(args.config, **over)
    T = cfg.tokens
    n_layers = args.layers or 16
    layers = [synth.make_layer(cfg, seed=1000 * rank + i, device=dev) for i in range(n_layers)]
    if args.layout == "tiled":
        for l in layers:
            l.experts.pack_tiles()
    kerns = [ops.MoEKernel(l.router, l.experts, l.expert_slot, cfg.swiglu_limit, path=args.path) for l in layers]
    K, W = args.steps, args.warmup
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    xs = torch.randn((K + W, T, cfg.hidden), generator=g, device=dev).to(torch.bfloat16)
    outs = torch.empty_like(xs)

    # warm-up (also sizes every workspace before graph capture)
    for i in range(W):
        kerns[i % n_layers](xs[i], out=outs[i])
    torch.cuda.synchronize()

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for s in range(K):
            kerns[(W + s) % n_layers](xs[W + s], out=outs[W + s])
    graph.replay()  # untimed: loads the graph
    torch.cuda.synchronize()

    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        start.record()
        graph.replay()
        end.record()
        while not end.query():  # sleep-poll: the sampler thread runs meanwhile
            time.sleep(0.0005)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = world * T * K / (ms / 1e3)

    # ---- per-kernel timing pass (events on the launching stream)
    nk = args.kernel_steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(nk)]
    for e4 in ev:
        for e in e4:
            e.record()
    idx_buf = torch.empty((nk, T, cfg.top_k), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    chunk = 25
    for c0 in range(0, nk, chunk):
        torch.cuda._sleep(int(4e6))  # lets the host queue the chunk before it runs
        for s in range(c0, min(nk, c0 + chunk)):
            i = W + (s % K)
            ev[s][0].record()
            kerns[i % n_layers].staged(xs[i], outs[i], ev[s][1], ev[s][2], idx=idx_buf[s])
            ev[s][3].record()
    torch.cuda.synchronize()
    t_router = [ev[s][0].elapsed_time(ev[s][1]) for s in range(nk)]
    t_gu = [ev[s][1].elapsed_time(ev[s][2]) for s in range(nk)]
    t_down = [ev[s][2].elapsed_time(ev[s][3]) for s in range(nk)]
    distinct = [len(torch.unique(idx_buf[s]).tolist()) for s in range(nk)]
    gu_bytes = sum(d * cfg.gateup_bytes() for d in distinct) / nk
    gu_ms = sum(t_gu) / nk
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    traffic = None
    prof = ROOT / "profiles" / f"gateup_{cfg.name}_traffic.json"
    if prof.exists():
        try:
            traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    layer_bytes = (sum(d * cfg.expert_bytes() for d in distinct) / nk + cfg.router_bytes()
                   + 2 * T * cfg.hidden * 2)
    layer_ms = ms / K
    # the gate/up kernel the layer ran (AUTO picks by the routes per step)
    path = args.path
    if path == "auto":
        path = "prefill" if _lib.auto_takes_prefill(T, cfg.top_k, cfg.n_experts) else "decode"
    gu_kernel = ("gemv_kernel<bf16, gate/up>" if path == "decode"
                 else f"pf_gemm_kernel<bf16, {cfg.bits_gate}, {cfg.group_size}, gate/up> (tcgen05)")

    # ---- e2e through the public module API with host buffers
    e2e = None
    if args.e2e_steps > 0:
        e2e = run_e2e(args, cfg, layers, n_layers, dev)
    prefill = None
    if world == 1 and args.prefill_steps > 0:
        prefill = run_prefill(args, dev)

    if rank != 0:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        layer_cpu = synth.layer_to(layers[0], "cpu")
        n_cpu = min(args.cpu_sample, xs.shape[0])
        xs_cpu = [xs[i].cpu() for i in range(n_cpu)]
        del layers
        cpu = cpu_baseline_sample(cfg, layer_cpu, xs_cpu, n_cpu)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": workload_config(cfg, T, world, n_layers, args.layout),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "kernel": gu_kernel, "algorithmic_bytes_per_launch": gu_bytes},
        "layer_roofline": {"bytes_per_step": layer_bytes, "achieved_gbs": layer_bytes / (layer_ms / 1e3) / 1e9,
                           "frac": layer_bytes / (layer_ms / 1e3) / 1e9 / peak},
        "kernels_us": {"router_dispatch": 1e3 * sum(t_router) / nk, "gateup_swiglu": 1e3 * gu_ms,
                       "down_combine": 1e3 * sum(t_down) / nk},
        "gpu_launches": 3 * K,
        "clocks": clocks.summary(),
        "e2e": e2e,
        "cpu_baseline": cpu,
        "prefill": prefill,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_prefill(args, dev):
    """C3: the prefill grouped GEMM on the config-1 layer (4096 tokens, uniform
    routing, 2-bit g64).  Tokens/s of the whole layer step (inputs in HBM,
    CUDA events), and the tensor roofline of the gate/up kernel (gate + up
    FLOPs of the routes / its mean duration)."""
    from locali_b200 import ops, synth

    cfg = synth.config("c3")
    T = cfg.tokens
    layer = synth.make_layer(cfg, seed=5, device=dev)
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, path="prefill")
    K, W = args.prefill_steps, 3
    g = torch.Generator(device=dev).manual_seed(99)
    xs = torch.randn((2, T, cfg.hidden), generator=g, device=dev).to(torch.bfloat16)  # 2 x 32 MB, cycled
    out = torch.empty_like(xs[0])
    for i in range(W):
        kern(xs[i % 2], out=out)
    torch.cuda.synchronize()
    kern.ws.check()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(K):
        kern(xs[i % 2], out=out)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / K
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    for i in range(K):
        ev[i][0].record()
        kern.staged(xs[i % 2], out, ev[i][1], ev[i][2])
        ev[i][3].record()
    torch.cuda.synchronize()
    gu_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / K
    dn_ms = sum(e[2].elapsed_time(e[3]) for e in ev) / K
    rt_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / K
    R = T * cfg.top_k
    gu_flops = R * 2 * 2 * cfg.hidden * cfg.inter
    all_flops = R * 3 * 2 * cfg.hidden * cfg.inter
    peak, kind = measured_tensor_peak()
    achieved = gu_flops / (gu_ms / 1e3) / 1e12
    return {
        "workload": f"c3 prefill: {T} tokens, hidden {cfg.hidden}, {cfg.n_experts} experts top-{cfg.top_k} "
                    f"(uniform routing), inter {cfg.inter}, 2-bit affine g{cfg.group_size}",
        "value": T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": K, "warmup": W,
        "layer_tflops": all_flops / (ms / 1e3) / 1e12,
        "kernels_us": {"router_dispatch": 1e3 * rt_ms, "gateup_swiglu": 1e3 * gu_ms, "down_combine": 1e3 * dn_ms},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": f"{kind} (MEASURED_PEAKS.json bf16_tflops)",
                     "kernel": "pf_gemm_kernel<bf16, 2, 64, gate/up> (tcgen05)",
                     "algorithmic_flops_per_launch": gu_flops},
    }


def run_e2e(args, cfg, layers, n_layers, dev):
    """Public-API path: V4ArenaMoE over an HBM-resident store, host buffers."""
    from locali_b200.dsv4_arena import V4ArenaMoE, V4ArenaStore
    from locali_b200.router import V4Gate

    store = V4ArenaStore.from_layers([l.experts for l in layers], top_k=cfg.top_k, device=dev)
    mods = [V4ArenaMoE(store, i, V4Gate(layers[i].router), cfg.top_k, swiglu_limit=cfg.swiglu_limit,
                       fused_decode=True) for i in range(n_layers)]
    T = cfg.tokens
    n = args.e2e_steps
    # untimed warm-up: every layer module once (its first call builds the
    # kernel descriptor and zeroes its workspace), then steady state
    w = max(3, n_layers)
    g = torch.Generator().manual_seed(5)
    host_x = torch.randn((n + w, T, cfg.hidden), generator=g).to(torch.bfloat16).pin_memory()
    # pinned host tensors in and out: the module stages the rows on the
    # device with a kernel and the combine writes the result into pinned host
    # memory (both transfers inside every step)
    outs = []
    for i in range(w):
        outs.append(mods[i % n_layers](host_x[i]))
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(w, n + w):
        outs.append(mods[i % n_layers](host_x[i]))
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    bytes_step = T * cfg.hidden * 2
    return {"value": world * T * n / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": bytes_step,
            "d2h_bytes_per_step": bytes_step, "api": "V4ArenaMoE.__call__ on pinned host tensors (rows staged by a kernel, result written "
            "into pinned host memory by the combine; fused router+experts, device slot table)"}


def run_ep(args):
    """Expert-parallel mode: rank r owns experts [r*E/N, (r+1)*E/N) of every
    layer, routes its own T tokens, and exchanges token rows and partial
    outputs with NCCL all-to-all.  Timed with CUDA events around K steps (the
    variable all-to-all splits need host-side counts, so no graph), max over
    ranks."""
    import datetime

    import torch.distributed as dist

    from locali_b200 import ep, synth

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    over = {}
    if args.tokens is not None:
        over["tokens"] = args.tokens
    if args.experts is not None:
        over["n_experts"] = args.experts
    cfg = synth.config(args.config, **over)
    T = cfg.tokens
    n_layers = args.layers or 16
    mods = []
    for i in range(n_layers):
        layer = synth.make_layer(cfg, seed=1000 + i, device=dev)  # same weights on every rank
        shard = ep.shard_experts(layer.experts, rank, world, cfg.n_experts)
        if args.layout == "tiled":
            shard.pack_tiles()
        st = ep.EPRank(layer.router, shard, rank, world, cfg.n_experts, cfg.swiglu_limit)
        mods.append(ep.ExpertParallelMoE(st) if world > 1 else st)
        del layer
    torch.cuda.empty_cache()
    K, W = args.steps, args.warmup
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    xs = torch.randn((K + W, T, cfg.hidden), generator=g, device=dev).to(torch.bfloat16)

    def step(i):
        m = mods[i % n_layers]
        if world > 1:
            return m(xs[i])
        return ep.loopback_forward([m], [xs[i]])[0]

    for i in range(W):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        start.record()
        for s in range(K):
            step(W + s)
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * T * K / (ms / 1e3)
    # algorithmic bytes: every selected expert's weights once per step
    # (all ranks together), plus the router weights on every rank
    layer_bytes = 6 * cfg.expert_bytes() if T == 1 else None
    peak, peak_kind = measured_peak()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": dict(workload_config(cfg, T, world, n_layers, args.layout), parallelism=f"ep{world}"),
        "roofline": {"bound": "hbm", "achieved": None, "peak": peak, "unit": "GB/s", "frac": None, "traffic": None,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "note": "expert-parallel mode: per-kernel rooflines are in the single-GPU line"},
        "gpu_launches": None, "clocks": clocks.summary(), "e2e": None, "cpu_baseline": None,
    }
    if layer_bytes:
        line["layer_bytes_per_step_all_ranks"] = layer_bytes
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.ep:
        run_ep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
