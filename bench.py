#!/usr/bin/env python3
"""MoE-block benchmark: Qwen3-30B-A3B-shaped 4-bit MoE layer decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl ours|reference]

A step is one MoE-block forward (router + cache bias -> top-k -> dispatch ->
4-bit SwiGLU experts -> combine) of one layer over a decode batch of T tokens
(default 64; the workload also sweeps T = 1 and 8). Layers rotate over
--layers distinct weight sets (48 x 340 MB = 16.3 GB, far above the 126 MB
L2), each with its own seeded input batch, so no step reads weights another
recent step left in L2. Inputs are synthetic and seeded: experts fp16
N(0, 0.02) quantised to MLX affine 4-bit (group 64), router bf16 N(0, 0.02),
activations bf16 N(0, 1), routing bias +0.5 on a seeded 25% expert subset.

Prints one JSON line (rank 0). `value` = tokens/s with inputs resident in HBM
(CUDA graphs of the C-ABI call, CUDA events); `e2e` = tokens/s through the
public C-ABI call with pinned host buffers, host->device inputs and
device->host output inside the timed region; `roofline` = the dominant
kernel's algorithmic bytes per launch / its CUDA-event duration against the
measured HBM copy bandwidth; `cpu_baseline` = the C restatement of the block
timed on this host's cores.

--impl reference times the reference's algorithm on the host cores (the C
restatement in oracle/; the reference's own MLX path cannot run on Linux x86
here) on the same workload and prints the same line with "impl": "reference".
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
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "MoE-layer decode tokens/s (Qwen3-30B-A3B-shaped 4-bit layer)"
UNIT = "tokens/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--kernel-path", default="auto",
                    choices=["auto", "decode", "tensor", "tensor-small"],
                    help="expert-FFN kernels of the decode line (es_moe_cfg.kernel_path)")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--sweep", default="1,8", help="extra decode batch sizes to time (\"\" for none)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--placement", default="bounded", choices=["hrw", "bounded"],
                    help="--gpus N > 1: expert placement over gpu0..gpuN-1: the reference's "
                         "rendezvous hashing (hrw) or its capacity-bounded variant (bounded)")
    ap.add_argument("--ep-mode", default="p2p", choices=["p2p", "nccl"],
                    help="--gpus N > 1: expert-parallel exchange: NVLink peer-to-peer windows "
                         "(default) or NCCL all_gather + all_to_all")
    ap.add_argument("--model", default="qwen3-30b-a3b",
                    choices=["qwen3-30b-a3b", "qwen3-235b-a22b", "olmoe-1b-7b"],
                    help="--gpus N > 1: layer shape of the expert-parallel workload")
    ap.add_argument("--ep-graphs", action="store_true",
                    help="--gpus N > 1: replay each layer's step (kernels + NCCL collectives) "
                         "as a CUDA graph instead of launching eagerly")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill"],
                    help="decode: the headline line (it also carries a short prefill "
                         "measurement); prefill: only the Qwen3-Next layer prefill")
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--prefill-steps", type=int, default=50)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-decoder", action="store_true",
                    help="skip the 48-layer decoder measurement in the decode line")
    return ap.parse_args()


# --------------------------------------------------------------------------- #
# helpers
# --------------------------------------------------------------------------- #

def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 100 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def stop(self):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if self.proc is None:
            return out
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return out
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        out.update(sm_mhz=statistics.median(sm) if sm else None,
                   sm_max_mhz=max(mx) if mx else None, reasons=reasons, samples=len(rows),
                   power_w_max=max(float(r[3]) for r in rows
                                   if r[3].replace(".", "").isdigit()) if rows else None)
        return out


def block_bytes(cfg, T, U):
    """Algorithmic HBM bytes of one MoE-block step: the packed bytes of the
    distinct experts selected, logits, x, out and the bias vector."""
    return (U * cfg.bytes_per_expert + T * cfg.num_experts * 2 + T * cfg.hidden * 2 * 2
            + cfg.num_experts * 4)


def kernel_bytes(cfg, T, U, path="decode"):
    """Algorithmic bytes per launch of each kernel of the block. `path` is
    the expert-FFN kernels that ran: the decode kernels keep per-pair rows
    in fp32 and x as bf16 fragments plus 64-column sums; the tensor-core
    kernels keep fp16 rows and x as scaled fp16 with one scale per token."""
    D, I, E, k = cfg.hidden, cfg.inter, cfg.num_experts, cfg.top_k
    P = T * k
    if path == "fused":
        # one kernel: the instrumentation puts the whole block in "front"
        return {"front": block_bytes(cfg, T, U), "gap": 0, "gateup": 0, "down": 0,
                "combine": 0}
    yb = 4 if path == "decode" else 2
    xprep = T * D * 2 + (T * (D // 64) * 4 if path == "decode" else T * 4)
    return {
        # router + dispatch + operand prep: logits, bias, x in, prepared x out,
        # routing lists out
        "front": T * E * 2 + E * 4 + T * D * 2 + xprep + 3 * T * k * 8 + E * 16,
        "gap": 0,
        # packed gate+up tiles of the distinct experts, prepared x in, fp16 h out
        "gateup": U * 2 * D * I * 9 // 16 + T * D * 2 + P * I * 2,
        # packed down tiles, fp16 h in, per-pair rows out
        "down": U * D * I * 9 // 16 + P * I * 2 + P * D * yb,
        # per-pair rows in, bf16 out
        "combine": P * D * yb + T * D * 2 + T * k * 8,
    }


# intervals between the six events es_moe_forward_timed records: the fused
# front-end kernel, the (empty) gap before the FFN, gate/up, down, combine
KERNELS = ["front", "gap", "gateup", "down", "combine"]


# --------------------------------------------------------------------------- #
# CPU baseline (oracle C restatement)
# --------------------------------------------------------------------------- #

def cpu_baseline(cfg, T, seconds, layer_np=None, seed=0):
    from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
    from oracle import c_oracle
    c_oracle.build()
    if layer_np is None:
        lay = synthetic_layer(cfg, seed=1000)
        layer_np = {k: v.numpy() for k, v in lay.items()}
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=seed)
    xf = x.float().numpy()
    lf = logits.float().numpy()
    bias = cache_bias_vector(cfg.num_experts, 0.5, 0)[0].numpy()
    cores = os.cpu_count() or 1
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        idx, w = c_oracle.route(lf, bias, cfg.top_k, cfg.norm_topk_prob)
        c_oracle.expert_ffn(xf, layer_np, idx, w, nthreads=cores)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": T / med, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{len(times)} calls of one {cfg.name} layer at T={T} "
                      f"(router + experts + combine), median {med * 1e3:.1f} ms/call"}


def cpu_baselines_other(seconds):
    """The C restatement on the host cores for the other configurations'
    layers (BASELINE: OLMoE T = 1 and 32, Qwen3-Next prefill T = 4096 with
    the shared expert, Qwen3-235B T = 256 with bias +0.5), each timed for
    about `seconds` (at least one call); CPU-generated seeded weights."""
    from expert_sniper_b200 import PRESETS
    from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
    from oracle import c_oracle
    c_oracle.build()
    cores = os.cpu_count() or 1
    out = []
    cases = [("olmoe-1b-7b", 1, 0.0), ("olmoe-1b-7b", 32, 0.0),
             ("qwen3-next-80b-a3b", 4096, 0.0), ("qwen3-235b-a22b", 256, 0.5)]
    layers = {}
    for name, T, b in cases:
        cfg = PRESETS[name]
        if name not in layers:
            layers.clear()
            import torch
            dev = "cuda" if torch.cuda.is_available() else "cpu"
            layers[name] = {k: v.cpu().numpy()
                            for k, v in synthetic_layer(cfg, seed=7, device=dev).items()}
        lay = layers[name]
        x, _, logits, sg = synthetic_inputs(cfg, T, seed=8)
        bias = cache_bias_vector(cfg.num_experts, b, 0)[0].numpy() if b > 0 else None
        xf, lf = x.float().numpy(), logits.float().numpy()
        sgn = None if sg is None else sg.float().numpy()
        times = []
        t_end = time.perf_counter() + seconds
        while not times or time.perf_counter() < t_end:
            t0 = time.perf_counter()
            idx, w = c_oracle.route(lf, bias, cfg.top_k, cfg.norm_topk_prob)
            c_oracle.expert_ffn(xf, lay, idx, w, sgn, nthreads=cores)
            times.append(time.perf_counter() - t0)
        med = statistics.median(times)
        out.append({"model": name, "tokens": T, "bias": b, "ms_per_call": med * 1e3,
                    "tokens_per_s": T / med, "calls": len(times), "cores": cores,
                    "kind": "port"})
    return out


# --------------------------------------------------------------------------- #
# prefill: Qwen3-Next-80B-A3B layer, T = 4096 (tensor-core path)
# --------------------------------------------------------------------------- #

PREFILL_METRIC = "MoE-layer prefill tokens/s (Qwen3-Next-80B-A3B-shaped 4-bit layer, shared expert)"


def measure_prefill(T, steps, warmup, layers=2):
    """One step = one MoE-block forward of a Qwen3-Next-shaped layer (E = 512,
    k = 10, I = 512, shared expert I = 512 with sigmoid gate) over T prompt
    tokens. Two layers alternate (2 x 908 MB, far above L2), each graph-
    captured; CUDA events on the launching stream."""
    import torch
    from expert_sniper_b200 import MoEBlock, PRESETS
    from expert_sniper_b200.block import ffn_kernels
    from expert_sniper_b200.quant import synthetic_inputs, synthetic_layer

    cfg = PRESETS["qwen3-next-80b-a3b"]
    dev = torch.device("cuda:0")
    ws = MoEBlock.new_workspace(cfg, T, dev)
    blocks, xs, lgs, outs, U = [], [], [], [], []
    for l in range(layers):
        lay = synthetic_layer(cfg, seed=2000 + l, device=dev)
        x, _, lg, sg = synthetic_inputs(cfg, T, seed=3000 + l, device=dev)
        blk = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=T, workspace=ws)
        del lay
        idx, _ = blk.route(lg, None)
        U.append(int(torch.unique(idx).numel()))
        blocks.append(blk)
        xs.append(x)
        lgs.append(lg)
        outs.append(torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=dev))
    torch.cuda.empty_cache()
    stream = torch.cuda.Stream(dev)
    events = []
    for l in range(layers):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        for e in evs:
            e.record(stream)
        events.append(evs)
    graphs, tgraphs = [], []
    with torch.cuda.stream(stream):
        for l in range(layers):
            blocks[l].forward(xs[l], lgs[l], None, out=outs[l])
        torch.cuda.synchronize()
        for l in range(layers):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                blocks[l].forward(xs[l], lgs[l], None, out=outs[l])
            graphs.append(g)
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=stream):
                blocks[l].forward_timed(xs[l], lgs[l], None, events[l], outs[l])
            tgraphs.append(g2)
        for s_ in range(max(3, warmup)):
            graphs[s_ % layers].replay()
        torch.cuda.synchronize()
        clocks = ClockSampler(0).start()
        time.sleep(0.3)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for s_ in range(steps):
            graphs[s_ % layers].replay()
        e1.record(stream)
        e1.synchronize()
        clk = clocks.stop()
        ms = e0.elapsed_time(e1) / steps
        kt = {k: [] for k in KERNELS}
        for rep in range(4):
            for l in range(layers):
                tgraphs[l].replay()
                torch.cuda.synchronize()
                for i, name in enumerate(KERNELS):
                    kt[name].append(events[l][i].elapsed_time(events[l][i + 1]))
    err = blocks[0].read_device_error()
    del graphs, tgraphs
    kmean = {k: statistics.mean(v) for k, v in kt.items()}
    D, I, k = cfg.hidden, cfg.inter, cfg.top_k
    flops = 2 * T * (k * 3 * D * I + 3 * D * cfg.shared_inter)
    ffn_flops = {"gateup": 2 * T * (k + 1) * 2 * D * I, "down": 2 * T * (k + 1) * D * I}
    mean_u = statistics.mean(U)
    step_bytes = ((mean_u + 1) * cfg.bytes_per_expert + T * cfg.num_experts * 2
                  + T * D * 2 * 2)
    peaks = {}
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peaks = json.load(f)
    tpeak = float(peaks.get("bf16_tflops", 1590.0))
    tkind = "measured" if "bf16_tflops" in peaks else "fallback"
    hbm, hkind = measured_peaks()
    dom = max(["gateup", "down"], key=lambda n: kmean[n])
    return {
        "metric": PREFILL_METRIC, "value": T / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms,
        "steps": steps, "tokens": T, "kernel_path": ffn_kernels(cfg, T),
        "config": {"workload": f"{cfg.name} MoE layer prefill, {T} tokens, no routing bias, "
                               f"{layers} alternating layers of {cfg.packed_bytes / 1e6:.0f} MB",
                   "model": cfg.name, "hidden": D, "experts": cfg.num_experts, "top_k": k,
                   "inter": I, "shared_inter": cfg.shared_inter},
        "tflops": flops / (ms * 1e-3) / 1e12,
        "roofline": {"bound": "tensor", "kernel": dom,
                     "achieved": ffn_flops[dom] / (kmean[dom] * 1e-3) / 1e12, "peak": tpeak,
                     "peak_kind": tkind, "unit": "TFLOP/s",
                     "frac": ffn_flops[dom] / (kmean[dom] * 1e-3) / 1e12 / tpeak,
                     "flops_per_launch": ffn_flops[dom], "launch_ms": kmean[dom]},
        "block_roofline": {"tensor_frac": flops / (ms * 1e-3) / 1e12 / tpeak,
                           "hbm_frac": step_bytes / (ms * 1e-3) / 1e9 / hbm,
                           "flops_per_step": flops, "bytes_per_step": step_bytes,
                           "mean_distinct_experts": mean_u},
        "kernel_ms": kmean, "clocks": clk, "device_error": err,
    }


# --------------------------------------------------------------------------- #
# our arm, one GPU
# --------------------------------------------------------------------------- #

def run_ours_single(args):
    import torch
    from expert_sniper_b200 import MoEBlock, PRESETS, prepare_packed
    from expert_sniper_b200.block import ffn_kernels
    from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer

    cfg = PRESETS[args.model].with_(kernel_path=args.kernel_path)
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    T, L = args.tokens, args.layers
    sweep = [int(s) for s in args.sweep.split(",") if s.strip() and int(s) != T]
    t_setup = time.time()
    packed = []
    cpu_layer = None
    for l in range(L):
        lay = synthetic_layer(cfg, seed=1000 + l, device=dev)
        packed.append(prepare_packed(cfg, lay))
        if l == 0 and not args.no_cpu_baseline:
            cpu_layer = {k: v.cpu().numpy() for k, v in lay.items()}
        del lay
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    setup_s = time.time() - t_setup
    bias = cache_bias_vector(cfg.num_experts, 0.5, 0)[0].to(dev)
    Tmax = max([T] + sweep)
    ws = MoEBlock.new_workspace(cfg, Tmax, dev)  # layers run in sequence: one workspace
    blocks = [MoEBlock(cfg, packed=p, max_tokens=Tmax, workspace=ws) for p in packed]
    stream = torch.cuda.Stream(dev)
    peak, peak_kind = measured_peaks()

    def make_case(Tc, seed_base):
        xs, lgs, outs, U = [], [], [], []
        for l in range(L):
            x, _, lg, _ = synthetic_inputs(cfg, Tc, seed=seed_base + l, device=dev)
            xs.append(x)
            lgs.append(lg)
            outs.append(torch.empty((Tc, cfg.hidden), dtype=torch.bfloat16, device=dev))
            idx, _ = blocks[l].route(lg, bias)
            U.append(int(torch.unique(idx).numel()))
        return xs, lgs, outs, U

    def capture(xs, lgs, outs, events=None):
        graphs = []
        with torch.cuda.stream(stream):
            for l in range(L):
                blocks[l].forward(xs[l], lgs[l], bias, out=outs[l])
            torch.cuda.synchronize()
            for l in range(L):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    if events is None:
                        blocks[l].forward(xs[l], lgs[l], bias, out=outs[l])
                    else:
                        blocks[l].forward_timed(xs[l], lgs[l], bias, events[l], outs[l])
                graphs.append(g)
        torch.cuda.synchronize()
        return graphs

    def time_graphs(graphs, K, W):
        with torch.cuda.stream(stream):
            for s in range(W):
                graphs[s % L].replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            for s in range(W, W + K):
                graphs[s % L].replay()
            e1.record(stream)
            e1.synchronize()
        return e0.elapsed_time(e1) / K

    def step_distribution(graphs, n):
        """ms of single graph replays, each bracketed by CUDA events on the
        launching stream (includes the event records' own gap)."""
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
        with torch.cuda.stream(stream):
            torch.cuda.synchronize()
            evs[0].record(stream)
            for s in range(n):
                graphs[s % L].replay()
                evs[s + 1].record(stream)
            evs[-1].synchronize()
        v = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(n))
        q = lambda f: v[min(n - 1, int(f * n))]
        return {"n": n, "p10": q(0.1), "median": q(0.5), "p90": q(0.9)}

    def profile_kernels(xs, lgs, outs, K):
        events = []
        for l in range(L):
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            for e in evs:
                e.record(stream)  # creates the underlying cudaEvent_t
            events.append(evs)
        torch.cuda.synchronize()
        graphs = capture(xs, lgs, outs, events)
        tot = {k: [] for k in KERNELS}
        done = 0
        with torch.cuda.stream(stream):
            while done < K:
                n = min(L, K - done)
                for l in range(n):
                    graphs[l].replay()
                torch.cuda.synchronize()
                for l in range(n):
                    evs = events[l]
                    for i, name in enumerate(KERNELS):
                        tot[name].append((l, evs[i].elapsed_time(evs[i + 1])))
                done += n
        del graphs
        return tot

    results = {}
    for Tc in [T] + sweep:
        xs, lgs, outs, U = make_case(Tc, seed_base=10_000 * Tc)
        graphs = capture(xs, lgs, outs)
        K = args.steps if Tc == T else min(args.steps, 4000)
        W = max(3, args.warmup)
        clocks = ClockSampler(0).start() if Tc == T else None
        if clocks:
            time.sleep(0.3)
        ms = time_graphs(graphs, K, W)
        clk = clocks.stop() if clocks else None
        dist_ms = step_distribution(graphs, min(K, 1000))
        del graphs
        mean_bytes = sum(block_bytes(cfg, Tc, U[s % L]) for s in range(W, W + K)) / K
        prof = profile_kernels(xs, lgs, outs, min(K, 4 * L))
        kmean = {k: statistics.mean(v for _, v in prof[k]) for k in KERNELS}
        path_c = ffn_kernels(cfg, Tc)
        kb = {k: statistics.mean(kernel_bytes(cfg, Tc, U[l], path_c)[k] for l, _ in prof[k])
              for k in KERNELS}
        if path_c == "fused":
            # one kernel: its time is the first interval of the instrumentation
            # (the others are empty event pairs)
            kmean, kb = {"fused": kmean["front"]}, {"fused": kb["front"]}
        results[Tc] = dict(ms=ms, bytes=mean_bytes, U=statistics.mean(U), U_layers=U, kmean=kmean,
                           kb=kb, clocks=clk, xs=xs, lgs=lgs, outs=outs, path=path_c,
                           dist=dist_ms)

    # e2e through the public API with host buffers: every step copies its x
    # and logits from pinned host memory and reads its output back. The
    # copies run on a second stream, double-buffered, so step s + 1's inputs
    # travel while step s's kernels run (a serving loop's overlap); events
    # order each buffer's reuse.
    r = results[T]
    xs_h = [x.cpu().pin_memory() for x in r["xs"]]
    lg_h = [g.cpu().pin_memory() for g in r["lgs"]]
    out_h = [torch.empty((T, cfg.hidden), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(r["xs"][0]) for _ in range(2)]
    ld = [torch.empty_like(r["lgs"][0]) for _ in range(2)]
    od = [torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    copy = torch.cuda.Stream(dev)
    K_e2e = min(args.steps, 2000)
    ev = lambda: torch.cuda.Event()   # noqa: E731 (ordering only)
    in_ready, fwd_done, out_done = {}, {}, {}

    def h2d(s):
        b = s % 2
        if s - 2 in fwd_done:
            copy.wait_event(fwd_done[s - 2])    # step s - 2 has read this buffer
        with torch.cuda.stream(copy):
            xd[b].copy_(xs_h[s % L], non_blocking=True)
            ld[b].copy_(lg_h[s % L], non_blocking=True)
            in_ready[s] = ev()
            in_ready[s].record(copy)

    def run(s):
        b = s % 2
        stream.wait_event(in_ready.pop(s))
        if s - 2 in out_done:
            stream.wait_event(out_done.pop(s - 2))   # step s - 2's output was read
        with torch.cuda.stream(stream):
            blocks[s % L].forward(xd[b], ld[b], bias, out=od[b])
            fwd_done[s] = ev()
            fwd_done[s].record(stream)
        copy.wait_event(fwd_done[s])
        with torch.cuda.stream(copy):
            out_h[b].copy_(od[b], non_blocking=True)
            out_done[s] = ev()
            out_done[s].record(copy)
        fwd_done.pop(s - 2, None)

    def steps(n):
        h2d(0)
        for s in range(n):
            if s + 1 < n:
                h2d(s + 1)
            run(s)

    steps(max(3, args.warmup))
    torch.cuda.synchronize()
    in_ready.clear(); fwd_done.clear(); out_done.clear()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy.wait_stream(stream)
    steps(K_e2e)
    stream.wait_stream(copy)
    e1.record(stream)
    e1.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K_e2e

    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, T, args.cpu_seconds, cpu_layer)

    dom = max([k for k in r["kmean"] if k != "gap"], key=lambda k: r["kmean"][k])
    achieved = r["kb"][dom] / (r["kmean"][dom] * 1e-3) / 1e9
    # DRAM traffic of the dominant kernel from one ncu capture (profiles/),
    # scaled from the captured launch's algorithmic bytes to this run's mean
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            rec = json.load(f).get(f"{cfg.name}:T{T}:{r['path']}:{dom}")
        if rec:
            traffic = rec["dram_bytes"] * r["kb"][dom] / rec["algorithmic_bytes"]
    metric = METRIC if args.model == "qwen3-30b-a3b" else \
        f"MoE-layer decode tokens/s ({args.model}-shaped 4-bit layer)"
    line = {
        "metric": metric, "value": T / (r["ms"] * 1e-3), "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": r["ms"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4xbf16->f32",
        "data": "synthetic (seeded; random-init 4-bit MLX-affine experts)",
        "config": {"workload": f"{cfg.name} MoE layer decode, batch {T} tokens, routing bias +0.5 "
                               f"on 25% cached experts, {L} rotating layers",
                   "model": cfg.name, "hidden": cfg.hidden, "experts": cfg.num_experts,
                   "top_k": cfg.top_k, "inter": cfg.inter, "tokens": T, "layers_rotated": L,
                   "l2": f"working set {L} layers x {cfg.packed_bytes / 1e6:.0f} MB > L2",
                   "parallelism": "single GPU"},
        "gbs": r["bytes"] / (r["ms"] * 1e-3) / 1e9,
        "block_roofline": {"bound": "hbm", "achieved": r["bytes"] / (r["ms"] * 1e-3) / 1e9,
                           "peak": peak, "unit": "GB/s",
                           "frac": r["bytes"] / (r["ms"] * 1e-3) / 1e9 / peak,
                           "bytes_per_step": r["bytes"], "mean_distinct_experts": r["U"],
                           "distinct_experts_per_layer": r["U_layers"]},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "traffic_note": "ncu dram read+write of one launch "
                     "(profiles/traffic.json), scaled by algorithmic bytes to this run's mean",
                     "algorithmic_bytes_per_launch": r["kb"][dom], "launch_ms": r["kmean"][dom]},
        "kernel_ms": r["kmean"],
        "step_ms_distribution": r["dist"],
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": T * cfg.hidden * 2 + T * cfg.num_experts * 2,
                "d2h_bytes_per_step": T * cfg.hidden * 2, "ms_per_step": e2e_ms,
                "copies": "pinned host buffers, double-buffered on a second stream: step s+1's "
                          "inputs and step s-1's output move while step s's kernels run"},
        # per step: fused tiny-batch kernel 1; decode kernels front, gate/up,
        # down, combine; tensor-core kernels front, (scatter above 8192
        # slots), gate/up, down, combine
        "gpu_launches": {"fused": 1, "decode": 4}.get(r["path"], 5 if T * cfg.top_k > 8192 else 4)
        * args.steps,
        "kernel_path": r["path"],
        "clocks": r["clocks"],
        "cpu_baseline": cpu,
        "sweep": [{"tokens": Tc, "ms_per_step": results[Tc]["ms"],
                   "value": Tc / (results[Tc]["ms"] * 1e-3),
                   "gbs": results[Tc]["bytes"] / (results[Tc]["ms"] * 1e-3) / 1e9,
                   "frac": results[Tc]["bytes"] / (results[Tc]["ms"] * 1e-3) / 1e9 / peak,
                   "kernel_ms": results[Tc]["kmean"], "kernel_path": results[Tc]["path"],
                   "step_ms_distribution": results[Tc]["dist"]}
                  for Tc in sweep],
        "setup_s": setup_s,
    }
    if not args.no_prefill:
        line["prefill"] = measure_prefill(args.prefill_tokens, min(args.prefill_steps, 50),
                                          3)
    if not args.no_decoder:
        # the Qwen3-30B-shaped 48-layer decoder around the block (attention,
        # norms, rotary, KV cache with a 2048-token context; one CUDA graph
        # per step): whole-model decode tokens/s at batch 1 and 16
        from expert_sniper_b200.decoder import measure as measure_decoder
        del blocks, packed
        torch.cuda.empty_cache()
        dec = measure_decoder((1, 16), 2048, 40, 48)
        for res in dec["results"].values():
            res["roofline"] = {"bound": "hbm", "achieved": res["gbs"], "peak": peak,
                               "peak_kind": peak_kind, "unit": "GB/s",
                               "frac": res["gbs"] / peak, "bytes_per_step": res["bytes_per_step"]}
        line["decoder"] = dec
    if not args.no_cpu_baseline:
        line["cpu_baselines"] = cpu_baselines_other(args.cpu_seconds / 3)
    print(json.dumps(line), flush=True)


def run_ours_ep(args):
    """N GPUs, one process each, experts sharded by rendezvous hashing over
    gpu0..gpu{N-1} (or its capacity-bounded variant). Every rank keeps
    --tokens home tokens (weak scaling: N x T tokens per step). The default
    exchange (--ep-mode p2p) is this library's NVLink peer-to-peer path:
    rows go straight into their owners' exchange windows and partials
    straight back (es_ep_dispatch / receive / return / combine_p2p), with no
    collective library on the data path and no host synchronisation; each
    layer's whole step is one CUDA graph. --ep-mode nccl runs the earlier
    all_gather + all_to_all exchange. Timed with CUDA events, max over ranks;
    NCCL is used only for barriers and the max outside the timed region."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    from expert_sniper_b200 import MoEBlock, PRESETS, ep
    from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    # --workload prefill: the Qwen3-Next layer over --prefill-tokens prompt
    # tokens split across the GPUs (strong scaling), no routing bias, two
    # alternating layers, as the one-GPU prefill line
    prefill = args.workload == "prefill"
    cfg = PRESETS["qwen3-next-80b-a3b" if prefill else args.model]
    if prefill:
        if args.prefill_tokens % world:
            raise SystemExit("--prefill-tokens must divide by the number of GPUs")
        T, L = args.prefill_tokens // world, 2
    else:
        T, L = args.tokens, max(2, args.layers)
    pl = ep.make_placement(cfg.num_experts, world, args.placement)
    lcfg = cfg.with_(num_experts=max(1, max(pl.counts)))
    bias = None if prefill else cache_bias_vector(cfg.num_experts, 0.5, 0)[0].to(dev)
    p2p = args.ep_mode == "p2p"
    wins = ep.EpWindows(world, rank, T, cfg.hidden, cfg.top_k, dev) if p2p else None
    ws = MoEBlock.new_workspace(lcfg, world * T, dev)
    backends, xs, lgs, touched = [], [], [], []
    t_setup = time.time()
    for l in range(L):
        lay = synthetic_layer(cfg, seed=1000 + l, device=dev)
        x, _, lg, sg = synthetic_inputs(cfg, T, seed=100_000 * rank + l, device=dev)
        if sg is not None:   # one shared-gate vector per layer on every rank
            sg = synthetic_inputs(cfg, 1, seed=1000 + l, device=dev)[3]
        if p2p:
            backends.append(ep.P2PEPBackend(cfg, pl, rank, wins, layer=lay, shared_gate_w=sg,
                                            local_workspace=ws))
        else:
            backends.append(ep.CudaEPBackend(cfg, pl, rank, layer=lay, max_tokens=T, device=dev,
                                             workspace=ws))
        del lay
        xs.append(x)
        lgs.append(lg)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    setup_s = time.time() - t_setup
    # experts this rank reads per layer: owned and chosen by any rank's token
    for l in range(L):
        b = backends[l]
        if p2p:
            b.route(lgs[l], bias)
            idx = b.idx[:T]
        else:
            idx, _ = b.route(lgs[l], bias)
        sel = torch.zeros(cfg.num_experts, dtype=torch.int32, device=dev)
        sel[idx.long().flatten()] = 1
        dist.all_reduce(sel, op=dist.ReduceOp.MAX)
        owned = pl.owned[rank]
        touched.append(int(sel[torch.tensor(owned, dtype=torch.long, device=dev)].sum())
                       if owned else 0)

    def step(s):
        b = backends[s % L]
        if p2p:
            return b.step(xs[s % L], lgs[s % L], bias)
        return ep.ep_forward(b, xs[s % L], lgs[s % L], bias)

    W = max(3, args.warmup)
    K = min(args.steps, args.prefill_steps) if prefill else args.steps
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for s in range(max(W, L)):   # warm every layer before capture
            step(s)
    torch.cuda.synchronize()
    dist.barrier()
    graphs = []
    use_graphs = p2p or args.ep_graphs
    if use_graphs:
        with torch.cuda.stream(stream):
            for l in range(L):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    step(l)
                graphs.append(g)
        torch.cuda.synchronize()
        dist.barrier()
    note = ("p2p exchange over NVLink peer memory (CUDA IPC windows), one CUDA graph per "
            "layer step" if p2p else
            ("NCCL all_gather + all_to_all, " + ("CUDA graphs" if graphs else "eager launches")))

    def timed(s):
        if graphs:
            graphs[s % L].replay()
        else:
            step(s)

    with torch.cuda.stream(stream):
        for s in range(W):
            timed(s)
    torch.cuda.synchronize()
    dist.barrier()
    clocks = ClockSampler(local_rank).start() if rank == 0 else None
    if clocks:
        time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    dist.barrier()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for s in range(W, W + K):
            timed(s)
        e1.record(stream)
    e1.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / K], device=dev)
    clk = clocks.stop() if clocks else None
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    err = wins.read_error() if p2p else 0
    # per-phase device times of one eager step on every rank (max over ranks)
    phases = None
    if p2p:
        names = ["route", "dispatch", "receive", "expert_ffn", "return", "combine"]
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        acc = torch.zeros(len(names), device=dev)
        n_rep = min(L, 8)
        torch.cuda.synchronize()
        dist.barrier()
        with torch.cuda.stream(stream):
            for s in range(n_rep):
                b = backends[s % L]
                evs[0].record(stream)
                b.route(lgs[s % L], bias)
                evs[1].record(stream)
                b.dispatch(xs[s % L], T)
                evs[2].record(stream)
                b.receive()
                evs[3].record(stream)
                b.ffn()
                evs[4].record(stream)
                b.ret()
                evs[5].record(stream)
                b.combine(b.shared(xs[s % L], T), T)
                evs[6].record(stream)
                evs[6].synchronize()
                acc += torch.tensor([evs[i].elapsed_time(evs[i + 1]) for i in range(len(names))],
                                    device=dev)
        dist.all_reduce(acc, op=dist.ReduceOp.MAX)
        phases = {n: float(v) / n_rep for n, v in zip(names, acc.tolist())}
    # e2e: host buffers in, host buffer out, through the same public path;
    # as on one GPU, the copies run on a second stream, double-buffered, so
    # step s + 1's inputs travel while step s runs
    xs_h = [x.cpu().pin_memory() for x in xs]
    lg_h = [g.cpu().pin_memory() for g in lgs]
    out_h = [torch.empty((T, cfg.hidden), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(xs[0]) for _ in range(2)]
    ld = [torch.empty_like(lgs[0]) for _ in range(2)]
    copy = torch.cuda.Stream(dev)
    K2 = min(K, 500)
    in_ready, fwd_done, out_done = {}, {}, {}

    def h2d(s):
        bb = s % 2
        if s - 2 in fwd_done:
            copy.wait_event(fwd_done[s - 2])
        with torch.cuda.stream(copy):
            xd[bb].copy_(xs_h[s % L], non_blocking=True)
            ld[bb].copy_(lg_h[s % L], non_blocking=True)
            in_ready[s] = torch.cuda.Event()
            in_ready[s].record(copy)

    def run(s):
        bb = s % 2
        stream.wait_event(in_ready.pop(s))
        if s - L in out_done:   # the layer's output buffer was read back
            stream.wait_event(out_done.pop(s - L))
        with torch.cuda.stream(stream):
            b = backends[s % L]
            o = b.step(xd[bb], ld[bb], bias) if p2p else ep.ep_forward(b, xd[bb], ld[bb], bias)
            fwd_done[s] = torch.cuda.Event()
            fwd_done[s].record(stream)
        copy.wait_event(fwd_done[s])
        with torch.cuda.stream(copy):
            out_h[bb].copy_(o, non_blocking=True)
            out_done[s] = torch.cuda.Event()
            out_done[s].record(copy)
        fwd_done.pop(s - 2, None)

    torch.cuda.synchronize()
    dist.barrier()
    e0.record(stream)
    copy.wait_stream(stream)
    h2d(0)
    for s in range(K2):
        if s + 1 < K2:
            h2d(s + 1)
        run(s)
    stream.wait_stream(copy)
    e1.record(stream)
    e1.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / K2], device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    per_gpu_bytes = torch.tensor([statistics.mean(touched) * cfg.bytes_per_expert], device=dev)
    dist.all_reduce(per_gpu_bytes, op=dist.ReduceOp.MAX)
    errs = torch.tensor([float(err)], device=dev)
    dist.all_reduce(errs, op=dist.ReduceOp.MAX)
    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = float(per_gpu_bytes.item()) / (ms * 1e-3) / 1e9
        if prefill:
            metric = PREFILL_METRIC[:-1] + ", expert-parallel)"
            workload = (f"{cfg.name} MoE layer prefill, {world * T} tokens split over {world} "
                        f"GPUs ({T} each), experts sharded ({args.placement}), no routing bias, "
                        f"{L} alternating layers")
        else:
            metric = (METRIC if args.model == "qwen3-30b-a3b" else
                      f"MoE-layer decode tokens/s ({args.model}-shaped 4-bit layer, "
                      "expert-parallel)")
            workload = (f"{cfg.name} MoE layer decode, {T} home tokens per GPU, experts sharded "
                        f"over {world} GPUs ({args.placement}), routing bias +0.5, {L} rotating "
                        "layers")
        line = {
            "metric": metric,
            "value": world * T / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if prefill else "weak", "vs_baseline": None,
            "dtype": "u4xbf16->f32",
            "data": "synthetic (seeded; random-init 4-bit MLX-affine experts)",
            "config": {"workload": workload,
                       "model": cfg.name, "tokens_per_gpu": T, "global_batch": world * T,
                       "parallelism": f"ep{world}", "placement": args.placement,
                       "exchange": args.ep_mode, "experts_per_gpu": pl.counts,
                       "l2": f"working set {L} layers x {cfg.packed_bytes / world / 1e6:.0f} MB "
                             "per GPU > L2"},
            "roofline": {"bound": "hbm", "kernel": "whole step (max over GPUs of expert bytes)",
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": achieved / peak, "traffic": None},
            "e2e": {"value": world * T / (float(e2e_ms.item()) * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": T * (cfg.hidden + cfg.num_experts) * 2,
                    "d2h_bytes_per_step": T * cfg.hidden * 2,
                    "copies": "pinned host buffers on every rank, double-buffered on a second "
                              "stream: step s+1's inputs and step s-1's output move while step "
                              "s runs"},
            # p2p: route, dispatch, receive, front, gate/up, down, combine (FFN:
            # front + 2 GEMMs + combine, or front + scatter + 2 + combine on the
            # tensor-core kernels), return, combine_p2p
            "gpu_launches": (10 if p2p else 7) * K,
            "phase_ms": phases,
            "tflops": (2 * world * T * (cfg.top_k * 3 * cfg.hidden * cfg.inter
                                         + 3 * cfg.hidden * cfg.shared_inter)
                       / (ms * 1e-3) / 1e12) if prefill else None,
            "device_error": int(errs.item()),
            "clocks": clk,
            "cpu_baseline": None,
            "setup_s": setup_s,
            "note": note,
        }
        if prefill:
            tpeak, tkind = 1590.0, "fallback"
            pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
            if os.path.exists(pp):
                with open(pp) as f:
                    tpeak, tkind = float(json.load(f).get("bf16_tflops", 1590.0)), "measured"
            line["roofline"] = {"bound": "tensor", "kernel": "whole step (all GPUs)",
                                "achieved": line["tflops"] / world, "peak": tpeak,
                                "peak_kind": tkind, "unit": "TFLOP/s per GPU",
                                "frac": line["tflops"] / world / tpeak, "traffic": None}
        print(json.dumps(line), flush=True)
    del graphs
    torch.cuda.synchronize()
    dist.barrier()
    del backends
    if wins is not None:
        wins.close()
    dist.barrier()
    dist.destroy_process_group()


def run_reference(args):
    """The reference's algorithm on the host cores: oracle C restatement."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from expert_sniper_b200 import PRESETS
    cfg = PRESETS[args.model]
    T = args.tokens
    per_step = max(1.0, min(10.0, 60.0 / max(1, args.steps + args.warmup)))
    base = cpu_baseline(cfg, T, per_step * (args.steps + args.warmup))
    ms = T / base["value"] * 1e3
    line = {
        "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
        "data": "synthetic (seeded)",
        "config": {"workload": f"{cfg.name} MoE layer decode, batch {T} tokens, routing bias +0.5",
                   "model": cfg.name, "tokens": T},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "C restatement of generate.py:122-136 + engine.py:15-42 on the host cores "
                "(MLX, the reference's own backend, is not installable on Linux x86)",
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gpus > 1 or world > 1:
        run_ours_ep(args)
        return
    if args.workload == "prefill":
        run_prefill_only(args)
        return
    run_ours_single(args)


def run_prefill_only(args):
    """--workload prefill: the prefill measurement as its own JSON line."""
    import torch
    torch.cuda.set_device(0)
    r = measure_prefill(args.prefill_tokens, args.prefill_steps, args.warmup)
    line = {"metric": r["metric"], "value": r["value"], "unit": UNIT, "n_gpus": 1,
            "steps": args.prefill_steps, "warmup": max(3, args.warmup),
            "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u4->f16 x f16 -> f32",
            "data": "synthetic (seeded; random-init 4-bit MLX-affine experts)",
            "config": r["config"], "roofline": r["roofline"],
            "block_roofline": r["block_roofline"], "tflops": r["tflops"],
            "kernel_ms": r["kernel_ms"], "clocks": r["clocks"],
            "gpu_launches": 5 * args.prefill_steps, "kernel_path": r["kernel_path"]}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
