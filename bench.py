#!/usr/bin/env python
"""Benchmark of the GGUF quantized-linear hot path on B200.

Headline workload (config 2 of the benchmark plan): the Q4_K decode GEMV over
the seven projections of one Llama-7B-shaped decoder layer (q, k, v, o
4096x4096; gate, up 11008x4096; down 4096x11008), fp32 activations at batch 1.
One "step" = one grouped dequant-GEMV launch over the whole layer set.  The metric is HBM GB/s of algorithmic bytes
(packed weights + fp32 x + fp32 y) per second.

Timing rules applied:
* W warm-up steps, then exactly K timed steps between barrier +
  cuda.synchronize on both sides, CUDA events on the launching stream; the
  max over ranks is reported (one rank at N=1).
* Inputs larger than L2: R distinct copies of the layer set (R * 113.8 MB >=
  4x the 126 MB L2) are used round-robin, one per step, so no step finds its
  weights in L2.
* SM clock and clock-event reasons are sampled through NVML during the run.

Usage:
  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--mix q4_k|q4_k_m]
  python bench.py --impl reference ...   # the reference's CPU path (oracle port) on host cores
Multi-GPU (N > 1, under torchrun): the layer set is sharded tensor-parallel,
column-parallel q/k/v/gate/up and row-parallel o/down (super-block aligned
K ranges).  The gather of the column outputs and the sum of the row partials
run over NVLink inside the kernels (the GEMV stores every output into every
rank's exchange buffer; a finish kernel waits for all ranks and reduces); the
same step with an NCCL all-gather + all-reduce is timed beside it
("tp_nccl").

The same JSON line carries the second half of the metric under "prefill":
config 3, the mixed Q4_K/Q6_K prefill dequant-GEMM (gate and up 11008x4096
Q4_K, down 4096x11008 Q6_K, M = 2048 bf16 tokens, fp32 accumulation), one step
= one grouped tcgen05 GEMM launch over the three projections (tensor-parallel
at N > 1: gate/up column shards, down row shard + NCCL all-reduce), reported
in TFLOP/s with its roofline against the measured dense-bf16 peak.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
METRIC = "Q4_K dequant-GEMV HBM GB/s (% of 8 TB/s); prefill dequant-GEMM TFLOP/s"


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--mix", choices=["q4_k", "q4_k_m"], default="q4_k")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-sweep", dest="sweep", action="store_false",
                    help="skip timing batch 4 and 16 (reported under 'batches')")
    ap.add_argument("--prefill-steps", type=int, default=200, help="timed steps of the prefill GEMM leg")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill GEMM leg")
    ap.add_argument("--moe-steps", type=int, default=50, help="timed steps of the MoE (config 5) leg")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE expert-parallel leg")
    ap.add_argument("--model-steps", type=int, default=20, help="timed steps of the 32-layer decode leg")
    ap.add_argument("--no-model", action="store_true", help="skip the 32-layer decode (config 4) leg")
    ap.add_argument("--decode-steps", type=int, default=20, help="timed steps of the GGUF decode-step leg")
    ap.add_argument("--decode-layers", type=int, default=32, help=argparse.SUPPRESS)
    ap.add_argument("--no-decode", action="store_true", help="skip the 32-layer GGUF decode-step (f4) leg")
    ap.add_argument("--q8-steps", type=int, default=2000, help="timed steps of the Q8_0 (config 1) leg")
    ap.add_argument("--no-q8", action="store_true", help="skip the Q8_0 GEMV (config 1) leg")
    return ap.parse_args(argv)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return dict(FALLBACK_PEAKS)


def profiled_traffic(key: str):
    """Per-launch DRAM bytes of `key` from profiles/traffic.txt (ncu capture summaries)."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == key and not line.startswith("#"):
            try:
                return int(parts[1])
            except ValueError:
                return None
    return None


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ---------------------------------------------------------------------------
# CPU leg: the reference's own algorithm (oracle port of gguf._dequantize +
# GenericGemmKernel.matmul_f32) on the host cores
# ---------------------------------------------------------------------------
def host_cpu_info():
    """Logical and physical core counts and the BLAS thread pools numpy uses."""
    info = {"logical_cores": os.cpu_count()}
    try:
        import psutil

        info["physical_cores"] = psutil.cpu_count(logical=False)
    except Exception:  # pragma: no cover - psutil is in the image
        info["physical_cores"] = None
    try:
        from threadpoolctl import threadpool_info

        info["blas"] = [{"api": p.get("internal_api"), "threads": p.get("num_threads")} for p in threadpool_info()
                        if p.get("user_api") == "blas"]
    except Exception:  # pragma: no cover
        info["blas"] = []
    return info


def blas_threads(info):
    return max([b["threads"] or 0 for b in info.get("blas", [])] or [0]) or None


def workload_config(mix, batch, world):
    """The config keys that name the workload; both arms report them."""
    return {"workload": f"config2_{mix}_layer_decode_gemv", "batch": batch,
            "weights": "q,k,v,o 4096x4096; gate,up 11008x4096; down 4096x11008"
                       + (" (Q6_K v and down)" if mix == "q4_k_m" else ""),
            "step": "the 7 projections of one decoder layer, one pass each",
            "parallelism": f"tp{world}"}


def cpu_layer_steps(specs, packed, batch, seed, warmup, steps, threads=None, budget_s=None):
    """The reference's decode path on the host for whole layer-set steps: the
    fp32 cache from gguf._dequantize (first touch, timed once), then per step
    the 7 projections' matmul_f32 (executor._linear, executor.py:47-79).
    Returns per-step seconds and the first-touch dequant time."""
    from oracle import gguf_oracle as O

    import contextlib

    ctx = contextlib.nullcontext()
    if threads:
        from threadpoolctl import threadpool_limits

        ctx = threadpool_limits(limits=threads, user_api="blas")
    with ctx:
        rng = np.random.default_rng(seed + 7)
        t0 = time.perf_counter()
        weights = [O.dequantize_matrix(s.qtype, p, s.n_rows, s.k) for s, p in zip(specs, packed)]
        t_dequant = time.perf_counter() - t0
        xs = [rng.standard_normal((batch, s.k)).astype(np.float32) for s in specs]

        def step():
            for x, w in zip(xs, weights):
                O.matmul_f32(x, w)

        for _ in range(max(0, warmup)):
            step()
        per = []
        t_end = None if budget_s is None else time.perf_counter() + budget_s
        while len(per) < max(1, steps) and (t_end is None or time.perf_counter() < t_end or not per):
            t = time.perf_counter()
            step()
            per.append(time.perf_counter() - t)
        return per, t_dequant


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from dracort_b200.workloads import algorithmic_bytes, encode_specs, layer_specs

    specs = layer_specs(args.mix)
    packed = encode_specs(specs, args.seed)
    info = host_cpu_info()
    # a step is one pass over the layer set (the same step as the GPU arm's);
    # the run is bounded to a few minutes of host time
    per, t_dequant = cpu_layer_steps(specs, packed, args.batch, args.seed, args.warmup, args.steps)
    alg = algorithmic_bytes(specs, args.batch)
    total_t = float(sum(per))
    value = alg * len(per) / total_t / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": len(per),
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * total_t / len(per), 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights, GGUF-encoded; N(0,1) activations)",
        "config": workload_config(args.mix, args.batch, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": blas_threads(info) or os.cpu_count(),
                         "kind": "port", **info,
                         "sample": f"{len(per)} layer-set steps after {args.warmup} warm-up steps: the 7 "
                                   f"projections' matmul_f32 on the fp32 dequant cache (reference steady "
                                   f"state, numpy/OpenBLAS default threads); first-touch dequant of the layer "
                                   f"set {t_dequant:.2f} s"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_prefill:
        from dracort_b200.workloads import encode_specs as enc, prefill_specs

        pspecs = prefill_specs("mixed")
        pres = cpu_prefill_leg(pspecs, enc(pspecs, args.seed + 100), args.seed)
        line["prefill"] = {
            "metric": "prefill dequant-GEMM TFLOP/s", "value": round(pres["tflops"], 5), "unit": "TFLOP/s",
            "config": {"workload": "config3_mixed_q4k_q6k_prefill_gemm", "tokens_sampled": pres["tokens"]},
            "cpu_baseline": {"value": round(pres["tflops"], 5), "unit": "TFLOP/s",
                             "cores": blas_threads(info) or os.cpu_count(), "kind": "port",
                             "sample": f"{pres['tokens']} tokens through gate, up, down on the fp32 dequant cache"},
        }
    print(json.dumps(line), flush=True)
    return 0


def cpu_prefill_leg(specs, packed, seed, tokens=64):
    """Reference prefill path on the host: fp32 dequant cache @ a token sample."""
    from oracle import gguf_oracle as O

    rng = np.random.default_rng(seed + 11)
    t0 = time.perf_counter()
    weights = [O.dequantize_matrix(s.qtype, p, s.n_rows, s.k) for s, p in zip(specs, packed)]
    t_dequant = time.perf_counter() - t0
    xs = [rng.standard_normal((tokens, s.k)).astype(np.float32) for s in specs]
    for x, w in zip(xs, weights):
        O.matmul_f32(x, w)
    best = []
    for x, w in zip(xs, weights):
        ts = []
        for _ in range(3):
            t = time.perf_counter()
            O.matmul_f32(x, w)
            ts.append(time.perf_counter() - t)
        best.append(float(np.median(ts)))
    flops = sum(2 * tokens * s.n_rows * s.k for s in specs)
    return {"tflops": flops / sum(best) / 1e12, "tokens": tokens, "dequant_s": t_dequant,
            "step_s": sum(best)}


_DEQ_LAYER = {}


def dequant_layer(specs, layer_packed):
    """The reference's first-access transform of one layer's projections (the
    fp32 cache, oracle port of gguf._dequantize) and its time in seconds; the
    last layer is kept, so the config-4 and decode-step CPU legs share it."""
    from oracle import gguf_oracle as O

    key = id(layer_packed)
    if key not in _DEQ_LAYER:
        t0 = time.perf_counter()
        weights = [O.dequantize_matrix(s.qtype, p, s.n_rows, s.k) for s, p in zip(specs, layer_packed)]
        _DEQ_LAYER.clear()
        _DEQ_LAYER[key] = (layer_packed, weights, time.perf_counter() - t0)
    return _DEQ_LAYER[key][1], _DEQ_LAYER[key][2]


def cpu_model_leg(specs, layer_packed, seed, n_layers, batches=(1, 32)):
    """Config 4 on the host (the reference's path): one layer's seven projections
    dequantized to the fp32 cache, then x @ W.T per projection (median of 3),
    times the number of layers."""
    from oracle import gguf_oracle as O

    rng = np.random.default_rng(seed + 13)
    weights, t_dequant = dequant_layer(specs, layer_packed)
    out = {"dequant_layer_s": round(t_dequant, 3)}
    for b in batches:
        xs = [rng.standard_normal((b, s.k)).astype(np.float32) for s in specs]
        layer_s = 0.0
        for x, w in zip(xs, weights):
            O.matmul_f32(x, w)
            ts = []
            for _ in range(3):
                t = time.perf_counter()
                O.matmul_f32(x, w)
                ts.append(time.perf_counter() - t)
            layer_s += float(np.median(ts))
        out[str(b)] = {"ms_per_step": round(layer_s * n_layers * 1e3, 3),
                       "tokens_per_s": round(b / (layer_s * n_layers), 2)}
    return out


def cpu_decode_leg(specs, layer_packed, seed, n_layers, pos0, vocab=32000, batches=(1, 32)):
    """The decode step on the host, the reference's path: CPUExecutionBackend's
    per-layer body over the fp32 weight cache and an fp32 key/value cache
    (the oracle's restatement, layer_decode_step / layer_decode_batch, pinned
    to OracleLlama), one layer of the model over pos0 cached positions per
    sequence (median of 3) times n_layers, plus the final norm and a Q6_K
    output head of `vocab` rows sampled from the layer's v rows."""
    from oracle import llama_decode as D

    rng = np.random.default_rng(seed + 17)
    names = ["q", "k", "v", "o", "gate", "up", "down"]
    weights, t_dequant = dequant_layer(specs, layer_packed)
    w = dict(zip(names, weights))
    # the head's rows are v rows (as in the GPU leg's model): its fp32 cache is
    # the dequantized v rows gathered
    w_out = w["v"][rng.integers(0, specs[2].n_rows, vocab)]
    hidden_size = specs[0].k
    heads = kvh = 32
    hd = hidden_size // heads
    w["attn_norm"] = (1 + 0.1 * rng.standard_normal(hidden_size)).astype(np.float32)
    w["ffn_norm"] = (1 + 0.1 * rng.standard_normal(hidden_size)).astype(np.float32)
    norm_out = (1 + 0.1 * rng.standard_normal(hidden_size)).astype(np.float32)
    cos, sin = D.build_rope_cache(hd, pos0 + 1, 10000.0)
    out = {"dequant_s": round(t_dequant, 3)}
    for b in batches:
        # one sequence's rows drawn, every sequence its own copy (distinct memory)
        k0 = rng.standard_normal((pos0 + 1, kvh, hd)).astype(np.float32)
        v0 = rng.standard_normal((pos0 + 1, kvh, hd)).astype(np.float32)
        caches = [(k0.copy(), v0.copy()) for _ in range(b)]
        x = rng.standard_normal((b, hidden_size)).astype(np.float32)

        def layer():
            if b == 1:
                return D.layer_decode_step(x, w, caches[0][0], caches[0][1], pos0, cos, sin, 1e-5, heads, kvh)
            return D.layer_decode_batch(x, w, caches, [pos0] * b, cos, sin, 1e-5, heads, kvh)

        def head():
            return D.head_step(x, norm_out, w_out, 1e-5)

        times = {}
        for nm, fn in (("layer", layer), ("head", head)):
            fn()
            ts = []
            for _ in range(3):
                t = time.perf_counter()
                fn()
                ts.append(time.perf_counter() - t)
            times[nm] = float(np.median(ts))
        step_s = times["layer"] * n_layers + times["head"]
        out[str(b)] = {"ms_per_step": round(step_s * 1e3, 2), "tokens_per_s": round(b / step_s, 2),
                       "layer_ms": round(times["layer"] * 1e3, 3), "head_ms": round(times["head"] * 1e3, 3)}
        del caches
    return out


def cpu_moe_leg(expert, hidden, ffn, tokens_per_expert, n_experts, seed):
    """Config 5 on the host (the reference's ExpertGroup path on fp32
    dequantized weights, torch CPU): one expert's gate/up/down MLP on its share
    of the routed tokens, median of 3, times the number of experts."""
    import torch
    import torch.nn.functional as F

    from oracle import gguf_oracle as O

    qt, g, u, d = expert
    t0 = time.perf_counter()
    wg = torch.from_numpy(O.dequantize_matrix(qt, g, ffn, hidden))
    wu = torch.from_numpy(O.dequantize_matrix(qt, u, ffn, hidden))
    wd = torch.from_numpy(O.dequantize_matrix(qt, d, hidden, ffn))
    t_dequant = time.perf_counter() - t0
    x = torch.from_numpy(np.random.default_rng(seed + 17).standard_normal((tokens_per_expert, hidden))
                         .astype(np.float32))
    ts = []
    for _ in range(4):
        t = time.perf_counter()
        (F.silu(x @ wg.T) * (x @ wu.T)) @ wd.T
        ts.append(time.perf_counter() - t)
    expert_s = float(np.median(ts[1:]))
    return {"step_s": expert_s * n_experts, "expert_s": expert_s, "dequant_expert_s": t_dequant,
            "threads": torch.get_num_threads()}


def pipelined_e2e(dev, x_dev, y_dev, make_run, n_copies, timed, K, warmup):
    """End-to-end steps through the public API with host buffers, the way a
    serving loop overlaps them: two device input/output buffer pairs, step i's
    inputs uploaded from pinned memory on one copy stream while step i-1
    computes, its outputs downloaded on another.  Every step still moves its
    own inputs in and its outputs out inside the timed region (the first
    upload starts after the timing event, the timing ends after the last
    download).  make_run(x, y) -> [callable per weight copy] launching one
    step's GEMV on the current stream with inputs x and outputs y.
    Returns (ms over K steps, h2d bytes per step, d2h bytes per step)."""
    import torch

    xs = [x_dev, torch.empty_like(x_dev)]
    ys = [y_dev, torch.empty_like(y_dev)]
    runs = [make_run(xs[j], ys[j]) for j in range(2)]
    g = torch.Generator().manual_seed(977)
    xh = [torch.randn(x_dev.shape, generator=g).pin_memory() for _ in range(2)]
    yh = [torch.empty(y_dev.shape).pin_memory() for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_up = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_down = [torch.cuda.Event() for _ in range(2)]

    def steps(n):
        start = torch.cuda.Event()
        start.record(comp)
        up.wait_event(start)
        down.wait_event(start)
        for i in range(n):
            j = i & 1
            up.wait_event(ev_comp[j])  # step i-2's GEMV has read buffer j
            with torch.cuda.stream(up):
                xs[j].copy_(xh[j], non_blocking=True)
                ev_up[j].record(up)
            comp.wait_event(ev_up[j])
            comp.wait_event(ev_down[j])  # step i-2's outputs have left buffer j
            runs[j][i % n_copies]()
            ev_comp[j].record(comp)
            down.wait_event(ev_comp[j])
            with torch.cuda.stream(down):
                yh[j].copy_(ys[j], non_blocking=True)
                ev_down[j].record(down)
        comp.wait_event(ev_down[0])
        comp.wait_event(ev_down[1])

    steps(max(3, warmup))
    torch.cuda.synchronize()
    ms, _, _ = timed(lambda: steps(K))
    return ms, xh[0].numel() * 4, yh[0].numel() * 4


def q8_0_leg(args, dev, peaks, timed, want_e2e, want_cpu):
    """Config 1: the Q8_0 GEMV, W 4096x4096 (fp16 d = max|w|/127, int8 rint(w/d)
    per 32-element block, as the reference test encoder), x fp32 [1, 4096],
    y fp32, one GEMV launch per step; distinct weight copies rotated so no
    step finds its weight in L2.  N = 1 only (the weight is one GPU's work)."""
    import torch

    from dracort_b200 import gguf_ops as G
    from dracort_b200.telemetry import ClockSampler
    from dracort_b200.workloads import algorithmic_bytes, encode_specs, q8_0_spec

    specs = q8_0_spec()
    s = specs[0]
    packed = encode_specs(specs, args.seed + 300)[0]
    t0 = G.repack(s.qtype, torch.from_numpy(packed.reshape(-1)).to(dev), s.n_rows, s.k)
    n_copies = max(2, math.ceil(4 * L2_BYTES / t0.numel()))
    copies = [t0] + [t0.clone() for _ in range(n_copies - 1)]
    g = torch.Generator().manual_seed(args.seed + 301)
    x = torch.randn((1, s.k), generator=g).to(dev)
    y = torch.empty((1, s.n_rows), device=dev)
    plans = [G.GemvPlan([G.GemvProblem(s.qtype, c, x, y, s.n_rows, s.k)]) for c in copies]
    for i in range(max(3, args.warmup)):
        plans[i % n_copies].run()
    torch.cuda.synchronize()
    if plans[0].status():
        raise RuntimeError(f"Q8_0 GEMV reported device status {plans[0].status()}")
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
        for pl in plans:
            pl.run()
    graph.replay()
    torch.cuda.synchronize()
    reps = max(1, args.q8_steps // n_copies)
    K = reps * n_copies
    sampler = ClockSampler(dev.index or 0).start()

    def steps():
        for _ in range(reps):
            graph.replay()

    ms, tw0, tw1 = timed(steps)
    clocks = sampler.summary(tw0, tw1)
    sampler.stop()
    ms_step = ms / K
    alg = algorithmic_bytes(specs, 1)
    gbs = alg / (ms_step * 1e-3) / 1e9
    out = {
        "metric": "Q8_0 dequant-GEMV HBM GB/s (config 1)", "value": round(gbs, 2), "unit": "GB/s",
        "ms_per_step": round(ms_step, 6), "steps": K, "higher_is_better": True, "dtype": "f32",
        "config": {"workload": "config1_q8_0_gemv", "batch": 1, "weights": "4096x4096 Q8_0",
                   "l2": f"{n_copies} weight copies rotated ({n_copies * t0.numel() / 1e6:.0f} MB > 4x126 MB L2)",
                   "graph": True},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "traffic": profiled_traffic("gemv_q8_0_config1"),
                     "peak_source": f"{peaks['source']} MEASURED_PEAKS.json hbm_gbs",
                     "kernel": f"gemv_kernel, one launch per step; algorithmic bytes {alg} per step"},
        "gpu_launches": plans[0].launches * K,
        "clocks": clocks,
    }
    if want_e2e:
        def make_run(xd, yd):
            pls = plans if xd is x else [G.GemvPlan([G.GemvProblem(s.qtype, c, xd, yd, s.n_rows, s.k)]) for c in copies]
            return [pl.run for pl in pls]

        ms_e, h2d, d2h = pipelined_e2e(dev, x, y, make_run, n_copies, timed, K, args.warmup)
        out["e2e"] = {"value": round(alg / (ms_e / K * 1e-3) / 1e9, 3), "unit": "GB/s",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "ms_per_step": round(ms_e / K, 6),
                      "path": "pinned host x -> H2D copy stream -> GemvPlan.run (C ABI) -> D2H copy stream -> "
                              "pinned host y; two buffer pairs, step i's copies overlap its neighbours' GEMVs"}
    if want_cpu:
        per, t_dq = cpu_layer_steps(specs, [packed], 1, args.seed, 3, 200)
        cpu_gbs = alg * len(per) / sum(per) / 1e9
        info = host_cpu_info()
        out["cpu_baseline"] = {
            "value": round(cpu_gbs, 3), "unit": "GB/s", "cores": blas_threads(info) or os.cpu_count(),
            "kind": "port", **info,
            "sample": (f"{len(per)} matmul_f32 steps on the fp32 cache after 3 warm-up steps (oracle port of "
                       f"gguf._dequantize + GenericGemmKernel.matmul_f32, numpy/OpenBLAS default threads), "
                       f"{np.median(per) * 1e3:.3f} ms median; first-touch dequant {t_dq * 1e3:.0f} ms")}
    del graph, plans, copies
    torch.cuda.empty_cache()
    return out


def prefill_leg(args, dev, peaks, rank, world, pg, timed, want_e2e, want_cpu):
    """Config 3 prefill dequant-GEMM (TP-sharded at N > 1); returns the 'prefill' object."""
    import torch

    from dracort_b200 import gguf_ops as G
    from dracort_b200.parallel.prefill import TPPrefillLayer
    from dracort_b200.telemetry import ClockSampler
    from dracort_b200.workloads import PREFILL_TOKENS, encode_specs, prefill_specs

    specs = prefill_specs("mixed")
    packed = encode_specs(specs, args.seed + 100)
    m = PREFILL_TOKENS
    layer = TPPrefillLayer(specs, packed, rank, world, m, dev, seed=args.seed, group=pg, copies=2)
    K = max(1, args.prefill_steps)
    for i in range(max(3, args.warmup)):
        layer.step(i)
    torch.cuda.synchronize()
    if layer.check_status() != 0:
        raise RuntimeError(f"prefill GEMM reported status {layer.check_status()}")
    sampler = ClockSampler(dev.index or 0).start()

    def steps():
        for i in range(K):
            layer.step(i)

    ms, tw0, tw1 = timed(steps)
    clocks = sampler.summary(tw0, tw1)
    sampler.stop()
    ms_step = ms / K
    value = layer.flops_total / (ms_step * 1e-3) / 1e12

    # the GEMM launch alone (no collective), on the launching stream, for the roofline
    gemm_ms = ms_step
    if world > 1:
        def gemm_only():
            for i in range(K):
                G.gemm_grouped(layer.problems[i % layer.n_copies], layer.status)

        gemm_ms, _, _ = timed(gemm_only)
        gemm_ms /= K
    achieved = layer.flops_local / (gemm_ms * 1e-3) / 1e12
    # the timed loop is ~0.1 s, at the boost clock (its own clock record
    # shows it): the burst cuBLAS figure is the denominator
    peak = peaks["bf16_tflops"]
    out = {
        "metric": "prefill dequant-GEMM TFLOP/s",
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "ms_per_step": round(ms_step, 5),
        "steps": K,
        "higher_is_better": True,
        "scaling": "strong",
        "dtype": "bf16",
        "config": {"workload": "config3_mixed_q4k_q6k_prefill_gemm", "tokens": m,
                   "weights": "gate,up 11008x4096 Q4_K; down 4096x11008 Q6_K",
                   "accumulate": "fp32 (TMEM)", "output": "bf16",
                   "parallelism": f"tp{world}" + (" (gate/up column, down row + NCCL all-reduce)" if world > 1 else ""),
                   "l2": f"step working set {layer.local_weight_bytes / 1e6:.0f} MB packed weights x 2 copies "
                         f"rotated + {sum(x.numel() * 2 for x in layer.x_local) / 1e6:.0f} MB bf16 inputs + "
                         f"{sum(y.numel() * 2 for y in layer.y_local) / 1e6:.0f} MB bf16 outputs > 126 MB L2"},
        "roofline": {
            "bound": "tensor",
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "frac_of_sustained": round(achieved / peaks.get("bf16_tflops_sustained", peak), 4),
            "traffic": profiled_traffic("gemm_config3_prefill") if world == 1 else None,
            "peak_source": f"{peaks['source']} MEASURED_PEAKS.json bf16_tflops (burst: a {K}-launch loop of "
                           f"about 0.1 s runs at the boost clock); frac_of_sustained uses bf16_tflops_sustained",
            "kernel": f"gemm_kernel, one launch per step, {layer.flops_local} algorithmic FLOP per launch per GPU",
        },
        "gpu_launches": layer.launches_per_step * K,
        "clocks": clocks,
    }
    if want_e2e and world == 1:
        pairs = []  # (device input, pinned host copy); gate and up share one input
        for x in layer.x_local:
            if all(x is not a for a, _ in pairs):
                pairs.append((x, x.cpu().pin_memory()))
        yh = [torch.empty(y.shape, dtype=y.dtype).pin_memory() for y in layer.y_local]
        h2d = sum(a.numel() * 2 for a, _ in pairs)
        d2h = sum(y.numel() * 2 for y in layer.y_local)

        def e2e_steps():
            for i in range(K):
                for a, b in pairs:
                    a.copy_(b, non_blocking=True)
                layer.step(i)
                for a, b in zip(yh, layer.y_local):
                    a.copy_(b, non_blocking=True)

        ms_e, _, _ = timed(e2e_steps)
        out["e2e"] = {"value": round(layer.flops_total / (ms_e / K * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e / K, 5),
                      "path": "pinned host bf16 x -> cuda -> gemm_grouped (C ABI) -> pinned host bf16 y, eager"}
    if want_cpu and rank == 0 and world == 1:
        res = cpu_prefill_leg(specs, packed, args.seed)
        out["cpu_baseline"] = {
            "value": round(res["tflops"], 5), "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
            "sample": (f"reference prefill path (oracle port of gguf._dequantize + GenericGemmKernel.matmul_f32, "
                       f"fp32) on {res['tokens']} of the {m} tokens through gate, up and down on the warm fp32 "
                       f"cache: {res['step_s'] * 1e3:.1f} ms; first-touch dequant of the three weights "
                       f"{res['dequant_s']:.1f} s; numpy/OpenBLAS default threads")}
    layer.close()
    return out


def model_leg(args, dev, peaks, rank, world, pg, timed):
    """Config 4: decode step of a 32-layer Llama-7B-shaped Q4_K_M model (the 7
    quantized projections of every layer, back to back), batch 1 and 32,
    tensor-parallel at N > 1."""
    import torch

    from dracort_b200 import gguf_ops as G
    from dracort_b200.parallel.decode import TPDecodeLayer
    from dracort_b200.telemetry import ClockSampler
    from dracort_b200.workloads import algorithmic_bytes, model_layers

    specs, layers = model_layers(args.seed + 700)
    n_layers = len(layers)
    out = {"metric": f"{n_layers}-layer Q4_K_M decode step (config 4): linear-layer HBM GB/s and tokens/s",
           "unit": "GB/s", "scaling": "strong", "dtype": "f32",
           "config": {"workload": "config4_llama7b_q4_k_m_decode_step", "layers": n_layers,
                      "weights": "per layer q,k,o,gate,up Q4_K; v,down Q6_K (Llama-7B shapes)",
                      "parallelism": f"tp{world}" + (" (in-kernel NVLink exchange + finish kernel per layer)"
                                                     if world > 1 else ""),
                      "step": "the 7 projections of every layer (one grouped GEMV call per layer: the GEMV "
                              "kernel, after an activation conversion kernel from batch 2, and a partial-sum "
                              "kernel on the tensor-memory path)"},
           "batches": {}}
    for batch in (1, 32):
        if world == 1:
            tiled = [[G.repack(s.qtype, torch.from_numpy(p.reshape(-1)).to(dev), s.n_rows, s.k)
                      for s, p in zip(specs, lay)] for lay in layers]
            xs = [torch.randn((batch, s.k), device=dev) for s in specs]
            ys = [torch.empty((batch, s.n_rows), device=dev) for s in specs]
            plans = [G.GemvPlan([G.GemvProblem(s.qtype, t[i], xs[i], ys[i], s.n_rows, s.k)
                                 for i, s in enumerate(specs)]) for t in tiled]

            def step():
                for pl in plans:
                    pl.run()
            launches = sum(pl.launches for pl in plans)
            graph = torch.cuda.CUDAGraph()
            for _ in range(3):
                step()
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
                step()
            run = graph.replay
        else:
            tp = [TPDecodeLayer(specs, lay, rank, world, batch, dev, seed=args.seed, group=pg, copies=1, fused=True)
                  for lay in layers]

            def step():
                for layer in tp:
                    layer.step(0)
            launches = n_layers * tp[0].launches_per_step
            for _ in range(3):
                step()
            torch.cuda.synchronize()
            bad = [layer.status() for layer in tp if layer.status()]
            if bad:
                raise RuntimeError(f"tensor-parallel decode step reported device status {bad[0]}")
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
                step()
            run = graph.replay
        for _ in range(max(3, args.warmup)):
            run()
        torch.cuda.synchronize()
        K = max(1, args.model_steps)
        sampler = ClockSampler(dev.index or 0).start()

        def steps():
            for _ in range(K):
                run()

        ms, tw0, tw1 = timed(steps)
        clocks = sampler.summary(tw0, tw1)
        sampler.stop()
        ms_step = ms / K
        gbs = n_layers * algorithmic_bytes(specs, batch) / (ms_step * 1e-3) / 1e9
        out["batches"][str(batch)] = {
            "ms_per_step": round(ms_step, 4), "tokens_per_s": round(batch / (ms_step * 1e-3), 1),
            "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / (peaks["hbm_gbs"] * world), 4),
            "gpu_launches": launches * K, "clocks": clocks}
        del graph
        if world == 1:
            del plans, tiled
        else:
            for layer in tp:
                layer.close()
            del tp
        torch.cuda.empty_cache()
    out["value"] = out["batches"]["1"]["gbs"]
    if rank == 0 and world == 1 and not args.no_cpu:
        res = cpu_model_leg(specs, layers[0], args.seed, n_layers)
        out["cpu_baseline"] = {
            "value": res["1"]["tokens_per_s"], "unit": "tokens/s (batch 1)", "cores": os.cpu_count(), "kind": "port",
            "batches": {b: res[b] for b in ("1", "32")},
            "sample": (f"reference path (oracle port of gguf._dequantize + GenericGemmKernel.matmul_f32): one "
                       f"layer's 7 projections on the warm fp32 cache, median of 3 per projection, x {n_layers} "
                       f"layers; first-touch dequant of one layer {res['dequant_layer_s']:.1f} s; numpy/OpenBLAS "
                       f"default threads")}
    return out


def decode_backend(seed, dev, n_layers=32, pos0=1024, max_num_seqs=32):
    """A GPUExecutionBackend over a synthetic Llama-7B Q4_K_M GGUF file of
    n_layers layers (q,k,o,gate,up Q4_K; v,down Q6_K; Q6_K output head over
    32000 tokens; F16 embedding), with room for pos0 + 64 positions per
    sequence.  The file is written to a temporary directory and removed once
    loaded."""
    import shutil
    import tempfile

    from dracort_b200.format.gguf_file import write_gguf
    from dracort_b200.gguf_executor import GPUExecutionBackend
    from dracort_b200.workloads import model_layers

    vocab, hidden, ffn, heads = 32000, 4096, 11008, 32
    specs, layers = model_layers(seed + 700, n_layers=n_layers)
    rng = np.random.default_rng(seed + 701)

    def raw(a):
        return np.ascontiguousarray(a).reshape(-1).view(np.uint8)

    names = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]
    tensors = [("token_embd.weight", 1, (vocab, hidden),
                raw((rng.standard_normal((vocab, hidden)) * 0.5).astype(np.float16)))]
    for li, lay in enumerate(layers):
        norm = raw((1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32))
        tensors.append((f"blk.{li}.attn_norm.weight", 0, (hidden,), norm))
        tensors.append((f"blk.{li}.ffn_norm.weight", 0, (hidden,), norm))
        for nm, sp, pk in zip(names, specs, lay):
            tensors.append((f"blk.{li}.{nm}.weight", sp.qtype, (sp.n_rows, sp.k), raw(pk)))
    v_spec, v_rows = specs[2], layers[0][2]  # Q6_K rows of width 4096
    head_rows = v_rows[rng.integers(0, v_spec.n_rows, vocab)]
    tensors += [("output_norm.weight", 0, (hidden,), raw((1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32))),
                ("output.weight", v_spec.qtype, (vocab, hidden), raw(head_rows))]
    meta = {"general.architecture": "llama", "general.name": "bench-llama7b-q4_k_m",
            "llama.embedding_length": hidden, "llama.block_count": n_layers, "llama.feed_forward_length": ffn,
            "llama.attention.head_count": heads, "llama.attention.head_count_kv": heads,
            "llama.context_length": 4096, "llama.rope.freq_base": 10000.0,
            "llama.attention.layer_norm_rms_epsilon": 1e-5, "llama.vocab_size": vocab}
    tmp = tempfile.mkdtemp(prefix="draco_decode_")
    try:
        path = os.path.join(tmp, "llama7b_q4_k_m.gguf")
        write_gguf(path, tensors, meta)
        del tensors, layers
        return GPUExecutionBackend(path, device=dev, max_num_seqs=max_num_seqs, max_seq_len=pos0 + 64,
                                   q6k_order="d_first")
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def decode_leg(args, dev, peaks, timed):
    """The f4 row: one full decode step of a 32-layer Llama-7B Q4_K_M GGUF model
    through GPUExecutionBackend (the drop-in for the reference's
    CPUExecutionBackend): embedding, per layer RMSNorm-fused q/k/v GEMV, RoPE +
    key/value append, cached attention over 1025 positions, o_proj with the
    residual add, RMSNorm-fused gate/up, SwiGLU-fused down with the residual
    add, then the final norm and a Q6_K output head over 32000 tokens.
    Batch 1 (forward_step) and batch 32 (forward_batch_decode), device-timed
    (logits left on the device) and end to end (host token ids in, host
    logits out, through the public methods)."""
    import torch

    from dracort_b200 import gguf_ops as G
    from dracort_b200.telemetry import ClockSampler

    n_layers = getattr(args, "decode_layers", 32)
    pos0, vocab = 1024, 32000
    rng = np.random.default_rng(args.seed + 702)
    be = decode_backend(args.seed, dev, n_layers, pos0)
    for t in be.k_cache + be.v_cache:  # 1024 cached positions of every sequence
        t.normal_()
    seqs = [be.new_sequence() for _ in range(32)]
    for s in seqs:
        be._len[s] = pos0
    hd = be.config.head_dim
    w_bytes = sum(G.tiled_nbytes(w.qtype, w.n_rows, w.k) for L in be.layers for key, w in L.items()
                  if hasattr(w, "qtype")) + G.tiled_nbytes(be.lm_head.qtype, be.lm_head.n_rows, be.lm_head.k)
    kv_bytes = 2 * n_layers * be.config.num_key_value_heads * (pos0 + 1) * hd * 4  # per sequence, read
    K = max(1, args.decode_steps)
    out = {"metric": "32-layer Q4_K_M decode step through GPUExecutionBackend: tokens/s",
           "unit": "tokens/s", "dtype": "f32",
           "config": {"workload": "llama7b_q4_k_m_gguf_decode", "layers": n_layers, "vocab": vocab,
                      "cached_positions": pos0, "kv_cache": "fp32 [slot, kv_heads, capacity, head_dim]",
                      "weights": "per layer q,k,o,gate,up Q4_K; v,down Q6_K; output Q6_K; embedding F16",
                      "graph": bool(be.use_graphs)},
           "launches_per_layer": be.launches_per_layer, "batches": {}}
    for batch in (1, 32):
        ss = seqs[:batch]
        toks = [int(t) for t in rng.integers(0, vocab, batch)]
        bufs = be._buffers(batch)
        per_layer = sum(g.launches for g in bufs["layers"][0]) + 1  # GEMV steps + the decode attention
        head_launches = bufs["head"].launches
        slots = [be._slot[s] for s in ss]

        def device_steps(k=K):
            for _ in range(k):
                be._forward(slots, toks, [pos0] * batch)

        def e2e_steps(k=K):
            for _ in range(k):
                for s in ss:
                    be.truncate_sequence(s, pos0)
                if batch == 1:
                    be.forward_step(ss[0], np.array(toks), pos0)
                else:
                    be.forward_batch_decode(ss, toks, [pos0] * batch)

        device_steps(max(3, args.warmup))
        e2e_steps(3)
        torch.cuda.synchronize()
        sampler = ClockSampler(dev.index or 0).start()
        ms, tw0, tw1 = timed(device_steps)
        clocks = sampler.summary(tw0, tw1)
        sampler.stop()
        ms_e2e, _, _ = timed(e2e_steps)
        step = ms / K
        alg = w_bytes + batch * kv_bytes
        gbs = alg / (step * 1e-3) / 1e9
        out["batches"][str(batch)] = {
            "ms_per_step": round(step, 4), "tokens_per_s": round(batch / (step * 1e-3), 1),
            "e2e": {"value": round(batch / (ms_e2e / K * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(ms_e2e / K, 4), "h2d_bytes_per_step": 3 * 8 * batch,
                    "d2h_bytes_per_step": batch * vocab * 4},
            "algorithmic_bytes": alg, "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4),
            "gpu_launches": (per_layer * n_layers + head_launches) * K, "clocks": clocks}
    out["value"] = out["batches"]["1"]["tokens_per_s"]
    del be
    torch.cuda.empty_cache()
    if not args.no_cpu:
        from dracort_b200.workloads import model_layers

        specs, layers = model_layers(args.seed + 700, n_layers=n_layers)  # the GPU leg's model (cached)
        res = cpu_decode_leg(specs, layers[0], args.seed, n_layers, pos0, vocab=vocab)
        out["cpu_baseline"] = {
            "value": res["1"]["tokens_per_s"], "unit": "tokens/s (batch 1)", "cores": os.cpu_count(),
            "kind": "port", "batches": {b: res[b] for b in ("1", "32")},
            "sample": (f"reference path (oracle port of CPUExecutionBackend's layer body: RMSNorm, matmul_f32 on "
                       f"the fp32 weight cache, RoPE, float64-score attention over {pos0} cached fp32 positions, "
                       f"SwiGLU, residuals; pinned to OracleLlama): one layer timed (median of 3) x {n_layers} "
                       f"layers + the final norm and head; batch 32 as forward_batch_decode (attention per "
                       f"sequence); first-touch dequant of one layer {res['dequant_s']:.1f} s; numpy/OpenBLAS "
                       f"default threads")}
    return out


def moe_leg(args, dev, peaks, rank, world, pg, timed):
    """Config 5: Mixtral-shaped MoE FFN, expert-parallel over the ranks."""
    import torch

    from dracort_b200.parallel.moe import EPMoELayer
    from dracort_b200.telemetry import ClockSampler
    from dracort_b200.workloads import MOE_FFN, MOE_HIDDEN, MOE_TOKENS, MOE_TOP_K, moe_experts

    experts = moe_experts(args.seed + 500)
    n_exp = len(experts)
    if n_exp % world or MOE_TOKENS % world:
        return {"unavailable": f"{n_exp} experts / {MOE_TOKENS} tokens do not split over {world} ranks"}
    g = torch.Generator().manual_seed(args.seed + 501)
    x_all = torch.randn((MOE_TOKENS, MOE_HIDDEN), generator=g).to(torch.bfloat16)
    logits_all = torch.randn((MOE_TOKENS, n_exp), generator=g)
    tl = MOE_TOKENS // world
    x = x_all[rank * tl:(rank + 1) * tl].to(dev)
    logits = logits_all[rank * tl:(rank + 1) * tl].to(dev)
    layer = EPMoELayer(experts, MOE_HIDDEN, MOE_FFN, MOE_TOP_K, rank, world, dev, group=pg)
    for _ in range(max(3, args.warmup)):
        layer.forward(x, logits)
    torch.cuda.synchronize()
    if layer.check_status() != 0:
        raise RuntimeError(f"MoE GEMM reported status {layer.check_status()}")
    K = max(1, args.moe_steps)
    # the layer never waits for the host (device-side routing and counts), so
    # at one rank the whole step is replayed from a CUDA graph
    graph = None
    if world == 1:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
            layer.forward(x, logits)
        graph.replay()
        torch.cuda.synchronize()
    sampler = ClockSampler(dev.index or 0).start()

    def steps():
        for _ in range(K):
            if graph is not None:
                graph.replay()
            else:
                layer.forward(x, logits)

    ms, tw0, tw1 = timed(steps)
    clocks = sampler.summary(tw0, tw1)
    sampler.stop()
    ms_step = ms / K
    flops = 2 * 3 * MOE_HIDDEN * MOE_FFN * MOE_TOKENS * MOE_TOP_K  # routed expert FLOP, whole job
    wbytes = sum(p.size for e in experts for p in e[1:])          # every expert's packed weights, read once
    gbs = wbytes / (ms_step * 1e-3) / 1e9
    return {
        "metric": "MoE FFN layer (config 5) TFLOP/s of routed expert work",
        "value": round(flops / (ms_step * 1e-3) / 1e12, 3),
        "unit": "TFLOP/s",
        "ms_per_step": round(ms_step, 5),
        "tokens_per_s": round(MOE_TOKENS / (ms_step * 1e-3), 1),
        "steps": K,
        "scaling": "strong",
        "dtype": "bf16",
        "config": {"workload": "config5_mixtral_moe_ffn", "experts": n_exp, "top_k": MOE_TOP_K,
                   "hidden": MOE_HIDDEN, "ffn": MOE_FFN, "tokens": MOE_TOKENS, "qtype": "Q4_K",
                   "parallelism": f"ep{world}" + (" (NCCL all-to-all dispatch + combine)" if world > 1 else ""),
                   "step": "route -> dispatch -> grouped gate/up GEMM -> SwiGLU -> grouped down GEMM -> combine",
                   "host_sync": "none (device-side routing counts; equal-split all-to-alls)",
                   "graph": graph is not None},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"] * world, "unit": "GB/s",
                     "frac": round(gbs / (peaks["hbm_gbs"] * world), 4),
                     "note": f"{wbytes} B of packed expert weights per step (each expert read once) over the "
                             f"whole step time incl. routing and collectives"},
        "gpu_launches": 3 * K * max(1, -(-2 * (n_exp // world) // 16)),
        "clocks": clocks,
        **({"cpu_baseline": _moe_cpu_baseline(experts, n_exp)} if rank == 0 and world == 1 and not args.no_cpu
           else {}),
    }


def _moe_cpu_baseline(experts, n_exp):
    from dracort_b200.workloads import MOE_FFN, MOE_HIDDEN, MOE_TOKENS, MOE_TOP_K

    per_expert = MOE_TOKENS * MOE_TOP_K // n_exp
    res = cpu_moe_leg(experts[0], MOE_HIDDEN, MOE_FFN, per_expert, n_exp, 0)
    flops = 2 * 3 * MOE_HIDDEN * MOE_FFN * MOE_TOKENS * MOE_TOP_K
    return {"value": round(flops / res["step_s"] / 1e12, 5), "unit": "TFLOP/s", "cores": os.cpu_count(),
            "kind": "port", "ms_per_step": round(res["step_s"] * 1e3, 2),
            "sample": (f"reference ExpertGroup math (down(silu(gate(x)) * up(x))) on the oracle's fp32 dequantized "
                       f"weights, torch CPU ({res['threads']} threads): one expert on {per_expert} tokens (the "
                       f"mean routed share), median of 3, x {n_exp} experts; first-touch dequant of one expert "
                       f"{res['dequant_expert_s']:.1f} s")}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist.group.WORLD

    from dracort_b200 import gguf_ops as G
    from dracort_b200.telemetry import ClockSampler
    from dracort_b200.workloads import algorithmic_bytes, encode_specs, layer_specs

    peaks = measured_peaks()
    specs_full = layer_specs(args.mix)
    packed_full = encode_specs(specs_full, args.seed)  # same seed on every rank
    batch = args.batch

    if world > 1:
        from dracort_b200.parallel.decode import TPDecodeLayer

        layer = TPDecodeLayer(specs_full, packed_full, rank, world, batch, dev, seed=args.seed, group=pg,
                              fused=True)
        step_fn = layer.step
        n_copies = layer.n_copies
        gpu_launches_per_step = layer.launches_per_step
        local_bytes = layer.local_weight_bytes
    else:
        layer = None

    sampler = ClockSampler(local).start()
    result = {}

    if world == 1:
        raw = [torch.from_numpy(p.reshape(-1)).to(dev) for p in packed_full]
        tiled0 = [G.repack(s.qtype, r, s.n_rows, s.k) for s, r in zip(specs_full, raw)]
        del raw
        set_bytes = sum(t.numel() for t in tiled0)
        n_copies = max(2, math.ceil(4 * L2_BYTES / set_bytes))
        copies = [tiled0] + [[t.clone() for t in tiled0] for _ in range(n_copies - 1)]
        rng = torch.Generator(device="cpu").manual_seed(args.seed + 1)
        # every projection's x [batch, k] and y [batch, n] is a block of one
        # buffer, so the end-to-end leg moves each with one copy
        xbuf = torch.randn(batch * sum(s.k for s in specs_full), generator=rng).to(dev)
        ybuf = torch.empty(batch * sum(s.n_rows for s in specs_full), device=dev)
        xs, ys, ox, oy = [], [], 0, 0
        for s in specs_full:
            xs.append(xbuf[ox:ox + batch * s.k].view(batch, s.k))
            ys.append(ybuf[oy:oy + batch * s.n_rows].view(batch, s.n_rows))
            ox += batch * s.k
            oy += batch * s.n_rows
        plans = [G.GemvPlan([G.GemvProblem(s.qtype, c[i], xs[i], ys[i], s.n_rows, s.k)
                             for i, s in enumerate(specs_full)]) for c in copies]
        local_bytes = set_bytes
        gpu_launches_per_step = plans[0].launches  # the grouped GEMV (batch 1: one kernel)

        def step_fn(i):
            plans[i % n_copies].run()

    # -- warm-up (eager), then CUDA-graph capture of one rotation ---------------
    for i in range(max(3, args.warmup)):
        step_fn(i)
    torch.cuda.synchronize()
    if layer is not None and layer.status():
        raise RuntimeError(f"tensor-parallel step reported device status {layer.status()}")
    stream = torch.cuda.Stream(device=dev)
    graphs = {}

    def graph_for(nsteps):
        if nsteps not in graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(nsteps):
                    step_fn(i)
            graphs[nsteps] = g
        return graphs[nsteps]

    use_graph = world == 1 or (layer is not None and layer.graph_safe)
    if use_graph:
        gfull = graph_for(n_copies)
        for _ in range(2):
            gfull.replay()
        torch.cuda.synchronize()

    K = args.steps

    def timed(fn_steps):
        if pg is not None:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        t_wall0 = time.perf_counter()
        s_ev = torch.cuda.Event(enable_timing=True)
        e_ev = torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream()
        s_ev.record(cur)
        fn_steps()
        e_ev.record(cur)
        torch.cuda.synchronize()
        if pg is not None:
            torch.distributed.barrier()
        t_wall1 = time.perf_counter()
        ms = s_ev.elapsed_time(e_ev)
        if pg is not None:
            t = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms, t_wall0, t_wall1

    def graph_steps():
        full, rem = divmod(K, n_copies)
        for _ in range(full):
            gfull.replay()
        if rem:
            graph_for(rem).replay()

    def eager_steps():
        for i in range(K):
            step_fn(i)

    if use_graph:
        graph_for(K % n_copies) if K % n_copies else None
        torch.cuda.synchronize()
    ms, tw0, tw1 = timed(graph_steps if use_graph else eager_steps)
    ms_step = ms / K
    alg = algorithmic_bytes(specs_full, batch)
    value = alg / (ms_step * 1e-3) / 1e9  # whole-job GB/s (all ranks' shards together)
    clocks = sampler.summary(tw0, tw1)

    # -- batch sweep (config 2 lists batch 1, 4 and 16) -------------------------
    batches = {}
    if args.sweep and world == 1:
        for b2 in (4, 16):
            xs2 = [torch.randn((b2, s.k), device=dev) for s in specs_full]
            ys2 = [torch.empty((b2, s.n_rows), device=dev) for s in specs_full]
            plans2 = [G.GemvPlan([G.GemvProblem(s.qtype, c[i], xs2[i], ys2[i], s.n_rows, s.k)
                                  for i, s in enumerate(specs_full)]) for c in copies]
            for i in range(10):
                plans2[i % n_copies].run()
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=stream):
                for i in range(n_copies):
                    plans2[i].run()
            reps = max(1, K // n_copies)
            torch.cuda.synchronize()
            s_ev = torch.cuda.Event(enable_timing=True)
            e_ev = torch.cuda.Event(enable_timing=True)
            s_ev.record()
            for _ in range(reps):
                g2.replay()
            e_ev.record()
            torch.cuda.synchronize()
            ms2 = s_ev.elapsed_time(e_ev) / (reps * n_copies)
            batches[str(b2)] = {"gbs": round(algorithmic_bytes(specs_full, b2) / (ms2 * 1e-3) / 1e9, 1),
                                "us_per_step": round(ms2 * 1e3, 3)}
            del g2, plans2

    # -- end to end through the public API, host buffers -----------------------
    e2e = None
    if not args.no_e2e and world == 1:
        def make_run(xd, yd):
            if xd is xbuf:
                return [pl.run for pl in plans]
            xv, yv, ox, oy = [], [], 0, 0
            for s in specs_full:
                xv.append(xd[ox:ox + batch * s.k].view(batch, s.k))
                yv.append(yd[oy:oy + batch * s.n_rows].view(batch, s.n_rows))
                ox += batch * s.k
                oy += batch * s.n_rows
            return [G.GemvPlan([G.GemvProblem(s.qtype, c[i], xv[i], yv[i], s.n_rows, s.k)
                                for i, s in enumerate(specs_full)]).run for c in copies]

        ms_e2e, h2d, d2h = pipelined_e2e(dev, xbuf, ybuf, make_run, n_copies, timed, K, args.warmup)
        e2e = {"value": round(alg / (ms_e2e / K * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": round(ms_e2e / K, 5),
               "path": "pinned host x (one buffer) -> H2D copy stream -> GemvPlan.run (C ABI) -> D2H copy "
                       "stream -> pinned host y (one buffer); two buffer pairs, step i's copies overlap its "
                       "neighbours' GEMVs"}
    elif world > 1 and not args.no_e2e and layer is not None:
        e2e = layer.e2e(K, timed)
        e2e.update({"value": round(alg / (e2e["ms_per_step"] * 1e-3) / 1e9, 3), "unit": "GB/s",
                    "path": "pinned host x -> cuda -> tensor-parallel GEMV (C ABI) with NVLink exchange + "
                            "finish kernel -> pinned host, eager"})

    # -- the same tensor-parallel step with NCCL collectives, for comparison ---
    tp_nccl = None
    if world > 1:
        layer.close()
        nl = TPDecodeLayer(specs_full, packed_full, rank, world, batch, dev, seed=args.seed, group=pg)
        for i in range(max(3, args.warmup)):
            nl.step(i)
        torch.cuda.synchronize()
        kn = min(K, 500)

        def nccl_steps():
            for i in range(kn):
                nl.step(i)

        ms_n, _, _ = timed(nccl_steps)
        tp_nccl = {"ms_per_step": round(ms_n / kn, 5), "gbs": round(alg / (ms_n / kn * 1e-3) / 1e9, 1),
                   "steps": kn, "path": "same shards; GemvPlan.run + NCCL all-gather + all-reduce, eager"}
        nl.close()
        del nl

    sampler.stop()

    # -- prefill dequant-GEMM (config 3), the second half of the metric --------
    # each leg runs inside an NVTX range named after it, so that a profiler
    # can select one leg's launches (ncu --nvtx --nvtx-include "<leg>/")
    nvtx = torch.cuda.nvtx

    def leg(name, fn):
        """One leg inside an NVTX range.  At one rank a leg that fails reports
        its error in the line instead of ending the run (the headline value is
        already measured); with several ranks an error propagates, so that no
        rank skips collectives the others enter."""
        nvtx.range_push(name)
        try:
            if world > 1:
                return fn()
            try:
                return fn()
            except Exception as e:  # noqa: BLE001 - reported in the JSON line
                import traceback

                traceback.print_exc()
                err = {"error": f"{type(e).__name__}: {e}"[:500]}
                del e
                try:
                    torch.cuda.synchronize()
                    torch.cuda.empty_cache()
                except Exception:  # noqa: BLE001 - a sticky device error: later legs report theirs
                    pass
                return err
        finally:
            nvtx.range_pop()

    prefill = None
    if not args.no_prefill:
        prefill = leg("prefill", lambda: prefill_leg(args, dev, peaks, rank, world, pg, timed, not args.no_e2e,
                                                     not args.no_cpu))
    q8 = None
    if not args.no_q8 and world == 1:
        q8 = leg("q8_0", lambda: q8_0_leg(args, dev, peaks, timed, not args.no_e2e, rank == 0 and not args.no_cpu))
    moe = None
    if not args.no_moe:
        moe = leg("moe", lambda: moe_leg(args, dev, peaks, rank, world, pg, timed))
    model = None
    if not args.no_model:
        model = leg("model", lambda: model_leg(args, dev, peaks, rank, world, pg, timed))
    decode = None
    if not args.no_decode and world == 1:
        decode = leg("decode", lambda: decode_leg(args, dev, peaks, timed))

    # -- CPU baseline (rank 0, N=1) --------------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        info = host_cpu_info()
        per, t_dq = cpu_layer_steps(specs_full, packed_full, batch, args.seed, 3, 100000, budget_s=8.0)
        warm = alg * len(per) / sum(per) / 1e9
        phys = info.get("physical_cores")
        per_p, _ = (cpu_layer_steps(specs_full, packed_full, batch, args.seed, 3, 100000, threads=phys, budget_s=4.0)
                    if phys else (None, None))
        cpu = {"value": round(warm, 3), "unit": "GB/s", "cores": blas_threads(info) or os.cpu_count(),
               "kind": "port", **info,
               "value_physical_threads": round(alg * len(per_p) / sum(per_p) / 1e9, 3) if per_p else None,
               "value_cold": round(alg / (t_dq + float(np.median(per))) / 1e9, 4),
               "sample": (f"reference path (oracle port of gguf._dequantize + GenericGemmKernel.matmul_f32) over "
                          f"the same layer set at batch {batch}: {len(per)} layer-set steps on the fp32 cache "
                          f"after 3 warm-up steps, {float(np.median(per)) * 1e3:.2f} ms median (warm, BLAS default "
                          f"threads); value_physical_threads with BLAS limited to the physical cores; cold first "
                          f"touch incl. dequant {t_dq:.2f} s per layer set")}

    if rank == 0:
        achieved = value
        traffic = profiled_traffic(f"gemv_{args.mix}_layer_b{batch}") if world == 1 else None
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 6),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights, GGUF-encoded; N(0,1) fp32 activations)",
            "config": {
                **workload_config(args.mix, batch, world),
                "l2": f"inputs larger than L2: {n_copies} layer-set copies rotated "
                      f"({n_copies * local_bytes / 1e6:.0f} MB per GPU > 4x126 MB L2)",
                "exchange": ("in-kernel NVLink exchange: peer stores + finish kernel" if world > 1 else None),
                "graph": bool(use_graph),
            },
            "roofline": {
                "bound": "hbm",
                "achieved": round(achieved, 2),
                "peak": peaks["hbm_gbs"] * world,
                "unit": "GB/s",
                "frac": round(achieved / (peaks["hbm_gbs"] * world), 4),
                "traffic": traffic,
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs x {world} GPUs)",
                "kernel": ("gemv_kernel, one launch per step" if world == 1 else
                           "gemv_kernel (tensor-parallel, stores to every rank) + tp_finish_kernel per step")
                          + f"; algorithmic bytes {alg} per step / device time per step",
            },
            "gpu_launches": gpu_launches_per_step * K,
            "clocks": clocks,
        }
        if batches:
            line["batches"] = batches
        if e2e is not None:
            line["e2e"] = e2e
        if tp_nccl is not None:
            line["tp_nccl"] = tp_nccl
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if q8 is not None:
            line["q8_0"] = q8
        if prefill is not None:
            line["prefill"] = prefill
        if moe is not None:
            line["moe"] = moe
        if model is not None:
            line["model"] = model
        if decode is not None:
            line["decode"] = decode
        print(json.dumps(line), flush=True)

    if layer is not None:
        layer.close()
    graphs.clear()
    if pg is not None:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
