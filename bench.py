"""Benchmark of the B200 routed-MoE layer -> one JSON line.

Metric: routed-MoE layer tokens/s + % HBM roofline (decode)
at 1/2/4/8 B200.

N = 1 (``python bench.py``): configuration C1 -- a DeepSeek-V4-Flash-shaped
layer (hidden 4096, 256 experts, top-6, inter 2048, 2-bit affine g64, routed
scaling 2.5, clamped SwiGLU limit 10) decoding one token per step, all
experts resident in HBM arena slots.  A step is one pass of the layer
(router -> dispatch -> gate/up+SwiGLU -> down+combine) over one batch.

* ``value``: tokens/s over exactly K steps replayed from a CUDA graph, inputs
  already in HBM; each step uses its own input and one of ``--layers``
  distinct layers in rotation, so the expert bytes touched between two uses of
  a layer exceed the 126 MB L2 several times over (no explicit flush).
* ``e2e``: the same metric through the public module API
  (``V4ArenaMoE.__call__``) with the activations in pinned host memory.
* ``roofline``: the gate/up kernel (the dominant one): algorithmic expert bytes
  per launch / its mean duration from CUDA events recorded on its stream
  (``lmoe_moe_layer_staged``), against the measured HBM copy bandwidth.
* ``decode_sweep``: C2 (gate/up 2-bit, down 4-bit, Zipf routing) at
  T = 1/4/16/64 with the HBM fraction of each batch's distinct expert bytes.
* ``prefill`` / ``prefill_zipf``: C3, 4096 tokens, uniform and Zipf routing,
  with the tensor roofline of the gate/up grouped GEMM.
* ``ep_c4``: the expert-parallel C4 stack on this one GPU (the N = 1 point of
  the multi-GPU curve).
* ``cpu_baseline``: the CPU oracle (numpy restatement of the reference MLX
  path, which cannot run here) timed on this host on a bounded sample.

N > 1 (under torchrun, one rank per GPU): configuration C4 -- a stack of 43
C2-shaped layers (mixed 2/4-bit, Zipf routing) in expert-parallel mode:
rank r owns experts [r*256/N, (r+1)*256/N) of every layer, routes its own
256 tokens, and the rows and partial outputs cross NVLink in two NCCL
all-to-alls per layer; the residual stream is added between layers.  A step
is one layer of the stack for every rank's 256 tokens; ``value`` is the
whole job's layer tokens/s (weak scaling: fixed tokens per rank), the max
over ranks of the device time.  ``replicas`` keeps the C1 decode of every
rank on its own full copy of the experts.  ``--replicas`` makes that the
main line again.

``--impl reference`` times the reference's CPU path stand-in (the oracle)
on rank 0 only, on the same workload.
"""

from __future__ import annotations

import argparse
import datetime
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
EP_LAYERS = 43


def parse():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default=None, help="c1 (N = 1 default) or c4 (N > 1 default)")
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
                   help="timed C3 prefill steps of the 'prefill' objects (0 = skip; N = 1 only)")
    p.add_argument("--sweep-steps", type=int, default=500, help="timed steps per batch of the C2 sweep (0 = skip)")
    p.add_argument("--ep", action="store_true", help="expert-parallel stack as the main line at any N")
    p.add_argument("--ep-steps", type=int, default=0, help="timed steps of the N = 1 ep_c4 object (0 = --steps)")
    p.add_argument("--no-ep-c4", action="store_true", help="skip the N = 1 ep_c4 object")
    p.add_argument("--replicas", action="store_true", help="N > 1: C1 replicas as the main line")
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


def max_over_ranks(v: float, dev, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        torch.distributed.barrier()


def timed_replay(graph, dev, world: int):
    """One replay of ``graph`` bracketed by a barrier and synchronisation on
    both sides, timed with CUDA events on the replaying stream; max over
    ranks.  Clocks are sampled during the replay."""
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        start.record()
        graph.replay()
        end.record()
        while not end.query():  # sleep-poll: the sampler thread runs meanwhile
            time.sleep(0.0005)
        torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(end), dev, world), clocks.summary()


def free_gpu():
    import gc

    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def cpu_threads() -> int:
    threads = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info

        info = threadpool_info()
        if info:
            threads = max(int(i.get("num_threads", 1)) for i in info)
    except Exception:
        pass
    return threads


def cpu_baseline_sample(cfg, layer_cpu, xs_cpu, n_steps: int):
    """Time the numpy oracle (stand-in for the reference MLX CPU path)."""
    import numpy as np

    from oracle import moe_oracle as O
    from oracle.bridge import layer_np, t2np

    L = layer_np(layer_cpu)
    t0 = time.perf_counter()
    for i in range(n_steps):
        O.moe_layer(t2np(xs_cpu[i]), L, acc=np.float32)
    dt = time.perf_counter() - t0
    T = xs_cpu[0].shape[0]
    return {"value": T * n_steps / dt, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
            "sample": f"{n_steps} decode steps of {cfg.name} (T={T}) through the numpy oracle, float32 "
                      f"accumulation, {dt:.1f}s"}


def workload_config(cfg, T, world, n_layers, layout):
    """The ``config`` object of a C1/C2 decode line (identical for both arms)."""
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


def ep_workload_config(cfg, T, world, n_layers):
    """The ``config`` object of the expert-parallel C4 line (identical for both arms)."""
    return {
        "workload": f"c4 expert-parallel stack: {n_layers} layers of hidden {cfg.hidden}, {cfg.n_experts} experts "
                    f"top-{cfg.top_k}, inter {cfg.inter}, {cfg.bits_gate}/{cfg.bits_up}/{cfg.bits_down}-bit affine "
                    f"g{cfg.group_size}, Zipf routing, routed scaling {cfg.routed_scaling}, T={T} tokens per rank "
                    f"per layer step, residual add between layers (the combine adds the residual and writes the "
                    f"weightless LayerNorm of the stream as the next layer's MoE input), {cfg.n_experts // world} "
                    f"experts per GPU",
        "global_batch": T * world, "parallelism": f"ep{world}", "layers_cycled": n_layers,
        "l2": f"{n_layers} distinct layers ({n_layers * cfg.n_experts // world * cfg.expert_bytes() / 1e9:.1f} GB "
              "of expert bytes per GPU) cycled",
        "weights": f"gate/up/down {cfg.bits_gate}/{cfg.bits_up}/{cfg.bits_down}-bit affine g{cfg.group_size} "
                   "(uint32 codes, bf16 scales/biases), row-major arena arrays",
        "exchange": "NCCL all_to_all_single of token rows (bf16 + route trailer) and fp32 partial rows, "
                    "equal splits of T rows per rank pair, CUDA-graph captured, no host wait",
    }


def _cfg(name, args):
    from locali_b200 import synth

    over = {}
    if args.tokens is not None:
        over["tokens"] = args.tokens
    if args.experts is not None:
        over["n_experts"] = args.experts
    return synth.config(name, **over)


def _default_config(args, world):
    if args.config:
        return args.config
    return "c4" if (args.ep or (world > 1 and not args.replicas)) else "c1"


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import numpy as np

    from locali_b200 import synth
    from oracle import moe_oracle as O
    from oracle.bridge import layer_np, t2np

    name = _default_config(args, world)
    cfg = _cfg(name, args)
    ep_mode = name == "c4"
    # a bounded sample of the workload: the C4 layer step holds 256 tokens
    # per rank, far too many for the scalar oracle, so each reference step is
    # 4 of those tokens through one layer of the stack
    T = min(cfg.tokens, 4) if ep_mode else cfg.tokens
    layer = synth.make_layer(cfg, seed=0, device="cpu")
    n = args.steps + args.warmup
    L = layer_np(layer)
    for i in range(min(args.warmup, 1)):
        O.moe_layer(t2np(synth.make_tokens(cfg, T, seed=10 + i, device="cpu")), L, acc=np.float32)
    budget_s = 60.0
    done = 0
    t0 = time.perf_counter()
    for i in range(args.warmup, n):
        O.moe_layer(t2np(synth.make_tokens(cfg, T, seed=10 + i, device="cpu")), L, acc=np.float32)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    value = T * done / dt
    threads = cpu_threads()
    conf = ep_workload_config(cfg, cfg.tokens, world, args.layers or EP_LAYERS) if ep_mode else \
        workload_config(cfg, cfg.tokens, world, args.layers or 16, args.layout)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * dt / done, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
        "config": conf,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{done} timed steps of {T} tokens of one {cfg.name} layer ({dt:.1f}s; at most "
                                   f"{args.steps} or about 60s) through the numpy oracle on one process (the "
                                   "reference MLX CPU path is not importable here; the reference has no "
                                   "multi-device mode)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ decode (C1 / C2)
def decode_layers(cfg, n_layers, layout, path, dev, seed_base):
    from locali_b200 import ops, synth

    layers = [synth.make_layer(cfg, seed=seed_base + i, device=dev) for i in range(n_layers)]
    if layout == "tiled":
        for l in layers:
            l.experts.pack_tiles()
    kerns = [ops.MoEKernel(l.router, l.experts, l.expert_slot, cfg.swiglu_limit, path=path) for l in layers]
    return layers, kerns


def measure_decode(cfg, kerns, K, W, dev, world, rank, kernel_steps, path):
    """K decode steps replayed from one CUDA graph (each step its own input,
    layers in rotation), then a per-kernel pass with events on the launching
    stream.  Returns the numbers of a decode line."""
    from locali_b200 import _lib

    T = cfg.tokens
    n_layers = len(kerns)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    xs = torch.randn((K + W, T, cfg.hidden), generator=g, device=dev).to(torch.bfloat16)
    outs = torch.empty_like(xs)
    # warm-up (also sizes every workspace before graph capture)
    for i in range(max(W, n_layers)):
        kerns[i % n_layers](xs[i % (K + W)], out=outs[i % (K + W)])
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for s in range(K):
            kerns[(W + s) % n_layers](xs[W + s], out=outs[W + s])
    graph.replay()  # untimed: loads the graph
    torch.cuda.synchronize()
    ms, clocks = timed_replay(graph, dev, world)
    del graph
    value = world * T * K / (ms / 1e3)

    # ---- per-kernel timing pass (events on the launching stream, at the
    # kernel boundaries of the same launches the graph replays)
    nk = kernel_steps
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
            kerns[i % n_layers].timed(xs[i], outs[i], ev[s][1], ev[s][2], idx=idx_buf[s])
            ev[s][3].record()
    torch.cuda.synchronize()
    for k in kerns:
        k.ws.check()
    t_router = [ev[s][0].elapsed_time(ev[s][1]) for s in range(nk)]
    t_gu = [ev[s][1].elapsed_time(ev[s][2]) for s in range(nk)]
    t_down = [ev[s][2].elapsed_time(ev[s][3]) for s in range(nk)]
    distinct = [len(torch.unique(idx_buf[s]).tolist()) for s in range(nk)]
    gu_ms = sum(t_gu) / nk
    # one token over the pre-tiled copy: gate/up and down run in one kernel
    # (the event after "gate/up" follows it), so its bytes are all three
    # projections'
    fused = T == 1 and path != "prefill" and kerns[0].experts.gate.tiles is not None
    gu_bytes = sum(d * (cfg.expert_bytes() if fused else cfg.gateup_bytes()) for d in distinct) / nk
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    layer_bytes = (sum(d * cfg.expert_bytes() for d in distinct) / nk + cfg.router_bytes()
                   + 2 * T * cfg.hidden * 2)
    layer_ms = ms / K
    if path == "auto":
        path = "prefill" if _lib.auto_takes_prefill(T, cfg.top_k, cfg.n_experts) else "decode"
    if fused:
        gu_kernel = (f"vec_layer_kernel<bf16, {cfg.bits_gate}, {cfg.bits_down}, {cfg.group_size}> "
                     "(single-token gate/up + down + combine, integer mma.sync)")
    elif path == "decode":
        gu_kernel = "stream_kernel<bf16, gate/up> (decode GEMV)"
    else:
        gu_kernel = f"pf_gemm_kernel<bf16, {cfg.bits_gate}, {cfg.group_size}, gate/up> (tcgen05)"
    # kernels of one step: router (+ logits on tensor cores and top-k for
    # T > 64), gate/up, down+combine (prefill: panel, dispatch, 2 GEMMs, combine)
    per_step = 2 if fused else (3 if path == "decode" and T <= 64 else (5 if path == "decode" else 7))
    return {
        "value": value, "ms": ms, "ms_per_step": layer_ms, "clocks": clocks, "path": path,
        "distinct_experts_mean": sum(distinct) / nk,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)", "kernel": gu_kernel,
                     "algorithmic_bytes_per_launch": gu_bytes},
        "layer_roofline": {"bytes_per_step": layer_bytes, "achieved_gbs": layer_bytes / (layer_ms / 1e3) / 1e9,
                           "frac": layer_bytes / (layer_ms / 1e3) / 1e9 / peak},
        "kernels_us": ({"router_dispatch": 1e3 * sum(t_router) / nk, "experts_fused": 1e3 * gu_ms,
                        "after_experts": 1e3 * sum(t_down) / nk} if fused else
                       {"router_dispatch": 1e3 * sum(t_router) / nk, "gateup_swiglu": 1e3 * gu_ms,
                        "down_combine": 1e3 * sum(t_down) / nk}),
        "gpu_launches": per_step * K,
    }


def run_decode_sweep(args, dev):
    """C2 at T = 1, 4, 16, 64 (AUTO path), 16 layers in rotation."""
    out = {}
    K = args.sweep_steps
    from locali_b200 import synth

    for T in (1, 4, 16, 64):
        cfg = synth.config("c2", tokens=T)
        layers, kerns = decode_layers(cfg, 16, "tiled", "auto", dev, seed_base=3000)
        r = measure_decode(cfg, kerns, K, 3, dev, 1, 0, min(100, K), "auto")
        out[f"T{T}"] = {"tokens_per_s": r["value"], "ms_per_step": r["ms_per_step"], "path": r["path"],
                        "distinct_experts": r["distinct_experts_mean"],
                        "layer_bytes_per_step": r["layer_roofline"]["bytes_per_step"],
                        "layer_frac": r["layer_roofline"]["frac"], "gateup_frac": r["roofline"]["frac"],
                        "kernels_us": r["kernels_us"]}
        del layers, kerns
        free_gpu()
    out["note"] = ("C2: gate/up 2-bit, down 4-bit g64, Zipf routing (selection-bias tilt); frac = distinct "
                   "expert bytes + router bytes per step / step time / measured HBM copy bandwidth")
    return out


# ------------------------------------------------------------------ prefill (C3)
def run_prefill(args, dev, zipf=False):
    """C3: the prefill grouped GEMM on the config-1 layer (4096 tokens, 2-bit
    g64, uniform or Zipf routing).  Tokens/s of the whole layer step (inputs
    in HBM, CUDA events), and the tensor roofline of the gate/up kernel (gate
    + up FLOPs of the routes / its mean duration)."""
    from locali_b200 import ops, synth

    cfg = synth.config("c3", zipf=zipf)
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
    idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device=dev)
    for i in range(K):
        ev[i][0].record()
        kern.staged(xs[i % 2], out, ev[i][1], ev[i][2], idx=idx)
        ev[i][3].record()
    torch.cuda.synchronize()
    gu_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / K
    dn_ms = sum(e[2].elapsed_time(e[3]) for e in ev) / K
    rt_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / K
    counts = torch.bincount(idx.reshape(-1).long(), minlength=cfg.n_experts)
    R = T * cfg.top_k
    gu_flops = R * 2 * 2 * cfg.hidden * cfg.inter
    all_flops = R * 3 * 2 * cfg.hidden * cfg.inter
    peak, kind = measured_tensor_peak()
    achieved = gu_flops / (gu_ms / 1e3) / 1e12
    return {
        "workload": f"c3 prefill: {T} tokens, hidden {cfg.hidden}, {cfg.n_experts} experts top-{cfg.top_k} "
                    f"({'Zipf' if zipf else 'uniform'} routing), inter {cfg.inter}, 2-bit affine g{cfg.group_size}",
        "value": T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": K, "warmup": W,
        "tokens_per_expert": {"max": int(counts.max()), "min": int(counts.min()),
                              "mean": float(counts.float().mean())},
        "layer_tflops": all_flops / (ms / 1e3) / 1e12,
        "kernels_us": {"router_dispatch": 1e3 * rt_ms, "gateup_swiglu": 1e3 * gu_ms, "down_combine": 1e3 * dn_ms},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": f"{kind} (MEASURED_PEAKS.json bf16_tflops)",
                     "kernel": "pf_gemm_kernel<bf16, 2, 64, gate/up> (tcgen05)",
                     "algorithmic_flops_per_launch": gu_flops},
    }


# ------------------------------------------------------------------ e2e (public API, host buffers)
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
    world = int(os.environ.get("WORLD_SIZE", "1"))
    ms = max_over_ranks(start.elapsed_time(end), dev, world)
    bytes_step = T * cfg.hidden * 2
    return {"value": world * T * n / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": bytes_step,
            "d2h_bytes_per_step": bytes_step, "api": "V4ArenaMoE.__call__ on pinned host tensors (rows staged by a "
            "kernel, result written into pinned host memory by the combine; fused router+experts, device slot "
            "table)"}


# ------------------------------------------------------------------ expert parallel (C4)
def ep_launches_per_step(T, k, world, path):
    """Kernels of this repository one EP layer step launches (NCCL's not counted)."""
    route = 1 if T <= 64 else 2              # router (+ top-k)
    R = world * T * k
    disp = 1 if R <= 512 else 4              # receive-side dispatch
    experts = 1 + disp + 3 + 1               # unpack, dispatch, panel + gate/up + down, partial
    return route + 1 + experts + 1           # + source dispatch, + combine


def measure_ep(cfg, n_layers, K, W, dev, world, rank, path="auto", phase_steps=None, e2e_steps=0):
    """The expert-parallel stack: K layer steps (layer s % n_layers, the
    residual stream carried between layers, a fresh batch entering layer 0)
    replayed from one CUDA graph with its NCCL calls; then an eager pass with
    events around each phase of a step; then (e2e_steps > 0) layer steps
    through the module API with the rows copied in from pinned host memory
    and the result read back every step."""
    from locali_b200 import ep, synth

    T = cfg.tokens
    E = cfg.n_experts
    mods = []
    for i in range(n_layers):
        layer = synth.make_layer(cfg, seed=1000 + i, device=dev)  # the same layer on every rank
        shard = ep.shard_experts(layer.experts, rank, world, E)
        router = layer.router
        del layer
        mods.append(ep.ExpertParallelMoE(ep.EPRank(router, shard, rank, world, E, cfg.swiglu_limit, path=path)))
    free_gpu()
    n_batches = 4
    g = torch.Generator(device=dev).manual_seed(177 + rank)
    xs = torch.randn((n_batches, T, cfg.hidden), generator=g, device=dev).to(torch.bfloat16)
    xf = xs.float()
    xc = xf - xf.mean(-1, keepdim=True)
    xns = (xc * torch.rsqrt(xc.square().mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    del xc
    del xf
    # the residual stream and its weightless LayerNorm (each layer's MoE input,
    # written by the previous layer's combine)
    x = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=dev)
    xn = torch.empty_like(x)

    def steps(s0, n):
        for s in range(s0, s0 + n):
            li = s % n_layers
            if li == 0:
                x.copy_(xs[(s // n_layers) % n_batches])
                xn.copy_(xns[(s // n_layers) % n_batches])
            mods[li](xn, residual=x, out=x, normed=xn)

    steps(0, max(W, n_layers))  # warm-up: every layer once (sizes workspaces, NCCL communicator)
    torch.cuda.synchronize()
    barrier(world)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        steps(0, n_layers)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    barrier(world)
    with torch.cuda.graph(graph):
        steps(0, K)
    graph.replay()  # untimed: loads the graph
    torch.cuda.synchronize()
    ms, clocks = timed_replay(graph, dev, world)
    value = world * T * K / (ms / 1e3)
    del graph
    torch.cuda.synchronize()
    for m in mods:
        m.r.check()

    # ---- eager phase pass: events around each phase of a layer step
    nph = phase_steps or 2 * n_layers
    names = ["route_dispatch", "exchange_rows", "experts", "exchange_partials", "combine"]
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(nph)]
    idxs = []
    barrier(world)
    torch.cuda.synchronize()
    for s_ in range(nph):
        li = s_ % n_layers
        m = mods[li]
        r, b = m.r, m._bufs[T]
        if li == 0:
            x.copy_(xs[(s_ // n_layers) % n_batches])
            xn.copy_(xns[(s_ // n_layers) % n_batches])
        ev[s_][0].record()
        idx, w = r.route(xn)
        r.dispatch(idx, w, xn, b["send"], b["slot_of"])
        ev[s_][1].record()
        m._exchange(b["recv"], b["send"])
        ev[s_][2].record()
        r.experts_partial(b["recv"].view(-1, r.row_bytes), b["part"])
        ev[s_][3].record()
        m._exchange(b["back"], b["part"])
        ev[s_][4].record()
        r.combine(b["back"], b["slot_of"], x, x, xn)
        ev[s_][5].record()
        idxs.append(idx)
    torch.cuda.synchronize()
    phase = {n: max_over_ranks(sum(ev[s_][j].elapsed_time(ev[s_][j + 1]) for s_ in range(nph)) / nph * 1e3,
                               dev, world) for j, n in enumerate(names)}
    step_us = sum(phase.values())
    # expert bytes each rank streams per layer step: its distinct experts hit
    # by any rank's routes
    allidx = torch.stack(idxs)  # [nph, T, k]
    if world > 1:
        gathered = torch.empty((world,) + tuple(allidx.shape), dtype=allidx.dtype, device=dev)
        torch.distributed.all_gather_into_tensor(gathered, allidx.contiguous())
    else:
        gathered = allidx.unsqueeze(0)
    lo, hi = ep.owned_range(E, rank, world)
    local_distinct = []
    for s_ in range(nph):
        e = gathered[:, s_].reshape(-1)
        local_distinct.append(int(torch.unique(e[(e >= lo) & (e < hi)]).numel()))
    d_mean = sum(local_distinct) / nph
    bytes_rank = d_mean * cfg.expert_bytes()

    e2e = None
    if e2e_steps > 0:
        gh = torch.Generator().manual_seed(277 + rank)
        xh = torch.randn((n_batches, T, cfg.hidden), generator=gh).to(torch.bfloat16).pin_memory()
        oh = torch.empty((n_batches, T, cfg.hidden), dtype=torch.bfloat16).pin_memory()
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for s_ in range(e2e_steps):
            # the step's MoE input rows from the host; the updated residual
            # stream back to the host
            xn.copy_(xh[s_ % n_batches], non_blocking=True)
            mods[s_ % n_layers](xn, residual=x, out=x, normed=xn)
            oh[s_ % n_batches].copy_(x, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        ems = max_over_ranks(e0.elapsed_time(e1), dev, world)
        e2e = {"value": world * T * e2e_steps / (ems / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": T * cfg.hidden * 2, "d2h_bytes_per_step": T * cfg.hidden * 2,
               "api": "ExpertParallelMoE.__call__ (eager, no graph) per layer step; the rows copied in from pinned "
                      "host memory and the result read back into pinned host memory every step"}
    peak, peak_kind = measured_peak()
    exp_gbs = bytes_rank / (phase["experts"] / 1e6) / 1e9
    row_b = mods[0].r.row_bytes
    path_taken = path
    if path == "auto":
        from locali_b200 import _lib

        routes = T * cfg.top_k
        path_taken = "prefill" if (routes >= _lib.PREFILL_MIN_ROUTES and
                                   4 * routes >= _lib.PREFILL_ROUTES_PER_4_EXPERTS * (E // world)) else "decode"
    res = {
        "value": value, "ms": ms, "ms_per_step": ms / K, "clocks": clocks,
        "per_gpu_value": value / world,
        "stack_tokens_per_s": value / n_layers,
        "phases_us": phase,
        "exchange_share": (phase["exchange_rows"] + phase["exchange_partials"]) / step_us,
        "limiting_phase": max(phase, key=phase.get),
        "expert_path": path_taken,
        "expert_roofline": {"bound": "hbm", "achieved": exp_gbs, "peak": peak, "unit": "GB/s",
                            "frac": exp_gbs / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                            "kernel": f"expert phase of a layer step on one GPU ({path_taken} path)",
                            "algorithmic_bytes_per_step": bytes_rank,
                            "distinct_local_experts": d_mean},
        "exchange_bytes_per_step": {"rows": world * T * row_b, "partials": world * T * cfg.hidden * 4,
                                    "note": "send buffer sizes per GPU (fixed capacity of T rows per rank pair)"},
        "gpu_launches": ep_launches_per_step(T, cfg.top_k, world, path_taken) * K,
        "e2e": e2e,
    }
    del mods
    free_gpu()
    return res


def init_dist(world, local):
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    else:
        torch.cuda.set_device(0)
    return torch.device("cuda", torch.cuda.current_device())


# ------------------------------------------------------------------ our arm
def run_ours(args):
    world, rank, local = dist_env()
    dev = init_dist(world, local)
    name = _default_config(args, world)
    if name == "c4":
        line = run_ep_main(args, world, rank, dev)
    else:
        line = run_decode_main(args, world, rank, dev, name)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_decode_main(args, world, rank, dev, name):
    """C1 (or another decode config) as the main line; at N = 1 with the
    sweep, prefill and ep_c4 objects."""
    cfg = _cfg(name, args)
    T = cfg.tokens
    n_layers = args.layers or 16
    layers, kerns = decode_layers(cfg, n_layers, args.layout, args.path, dev, seed_base=1000 * rank)
    K, W = args.steps, args.warmup
    r = measure_decode(cfg, kerns, K, W, dev, world, rank, args.kernel_steps, args.path)
    traffic = None
    # ncu DRAM bytes of the roofline kernel (one launch), when a capture of
    # it for this config is committed
    kname = "vec_layer" if r["roofline"]["kernel"].startswith("vec_layer") else "gateup"
    prof = ROOT / "profiles" / f"{kname}_{cfg.name}_traffic.json"
    if prof.exists():
        try:
            traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    r["roofline"]["traffic"] = traffic
    e2e = run_e2e(args, cfg, layers, n_layers, dev) if args.e2e_steps > 0 else None
    layer_cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from locali_b200 import synth

        layer_cpu = synth.layer_to(layers[0], "cpu")
    del layers, kerns
    free_gpu()
    line = {
        "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": workload_config(cfg, T, world, n_layers, args.layout),
        "roofline": r["roofline"], "layer_roofline": r["layer_roofline"], "kernels_us": r["kernels_us"],
        "gpu_launches": r["gpu_launches"], "clocks": r["clocks"], "e2e": e2e,
    }
    if world == 1:
        if args.sweep_steps > 0:
            line["decode_sweep"] = run_decode_sweep(args, dev)
        if args.prefill_steps > 0:
            line["prefill"] = run_prefill(args, dev)
            free_gpu()
            line["prefill_zipf"] = run_prefill(args, dev, zipf=True)
            free_gpu()
        if not args.no_ep_c4:
            c4 = _cfg("c4", args)
            ep = measure_ep(c4, args.layers or EP_LAYERS, args.ep_steps or K, max(W, 3), dev, 1, 0)
            line["ep_c4"] = {"config": ep_workload_config(c4, c4.tokens, 1, args.layers or EP_LAYERS),
                             **{k: v for k, v in ep.items() if k not in ("clocks", "ms")}}
    if layer_cpu is not None:
        n_cpu = args.cpu_sample
        g = torch.Generator().manual_seed(77)
        xs_cpu = [torch.randn((T, cfg.hidden), generator=g).to(torch.bfloat16) for _ in range(n_cpu)]
        line["cpu_baseline"] = cpu_baseline_sample(cfg, layer_cpu, xs_cpu, n_cpu)
    else:
        line["cpu_baseline"] = None
    return line


def run_ep_main(args, world, rank, dev):
    """The expert-parallel C4 stack as the main line (N > 1 default), with
    the C1 replicas of every rank as an extra field."""
    K, W = args.steps, args.warmup
    replicas = None
    if world > 1 and not args.ep:
        c1 = _cfg("c1", args)
        layers, kerns = decode_layers(c1, 16, args.layout, "auto", dev, seed_base=1000 * rank)
        r = measure_decode(c1, kerns, K, W, dev, world, rank, 50, "auto")
        replicas = {"config": workload_config(c1, c1.tokens, world, 16, args.layout), "value": r["value"],
                    "per_gpu_value": r["value"] / world, "ms_per_step": r["ms_per_step"],
                    "roofline": r["roofline"], "kernels_us": r["kernels_us"]}
        del layers, kerns
        free_gpu()
    cfg = _cfg(args.config or "c4", args)
    n_layers = args.layers or EP_LAYERS
    ep = measure_ep(cfg, n_layers, K, W, dev, world, rank, args.path,
                    e2e_steps=min(args.e2e_steps, 2 * n_layers) if args.e2e_steps > 0 else 0)
    return {
        "metric": METRIC, "value": ep["value"], "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ep["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": ep_workload_config(cfg, cfg.tokens, world, n_layers),
        "per_gpu_value": ep["per_gpu_value"], "stack_tokens_per_s": ep["stack_tokens_per_s"],
        "roofline": ep["expert_roofline"],
        "phases_us": ep["phases_us"], "exchange_share": ep["exchange_share"],
        "limiting_phase": ep["limiting_phase"], "exchange_bytes_per_step": ep["exchange_bytes_per_step"],
        "gpu_launches": ep["gpu_launches"], "clocks": ep["clocks"],
        "e2e": ep["e2e"], "cpu_baseline": None, "replicas": replicas,
        "note": "value: layer tokens/s of all ranks together; the reference arm is one CPU process, so compare "
                "per_gpu_value with it",
    }


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
