"""bench.py on the CPU: the algorithmic bytes per kernel for each
expert-FFN kernel family (the roofline numerators), the traffic records it
scales, the peak it divides by, and the reference arm's line."""
from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys

from expert_sniper_b200 import PRESETS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_kernel_bytes_by_kernel_family():
    b = _bench()
    cfg = PRESETS["qwen3-30b-a3b"]
    D, I, k = cfg.hidden, cfg.inter, cfg.top_k
    T, U = 64, 120
    P = T * k
    dec = b.kernel_bytes(cfg, T, U, "decode")
    ts = b.kernel_bytes(cfg, T, U, "tensor-small")
    # weights read once per distinct expert, activations in, fp16 h out
    assert dec["gateup"] == ts["gateup"] == U * 2 * D * I * 9 // 16 + T * D * 2 + P * I * 2
    # per-pair rows: fp32 on the decode kernels, fp16 on the tensor-core ones
    assert dec["down"] - ts["down"] == P * D * 2
    assert dec["combine"] - ts["combine"] == P * D * 2
    # prepared activations: 64-column sums (decode) vs one scale per token
    assert dec["front"] - ts["front"] == T * (D // 64) * 4 - T * 4
    assert b.kernel_bytes(cfg, T, U, "tensor") == ts
    assert b.kernel_bytes(cfg, T, U) == dec


def test_block_bytes_counts_distinct_experts():
    b = _bench()
    cfg = PRESETS["qwen3-30b-a3b"]
    one = b.block_bytes(cfg, 64, 1)
    assert b.block_bytes(cfg, 64, 2) - one == cfg.bytes_per_expert


def test_traffic_records_name_their_kernel_family():
    with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
        rec = json.load(f)
    fams = {"decode", "tensor", "tensor-small", "fused"}
    for key, v in rec.items():
        model, t, fam, kernel = key.split(":")
        assert model in PRESETS and t.startswith("T") and fam in fams and kernel
        # DRAM traffic within a few percent of the algorithmic bytes: no
        # re-reads (the fused kernel's split-K partials, a few MB per call,
        # partly spill from L2: up to 10 % more)
        limit = 1.10 if fam == "fused" else 1.05
        assert 1.0 <= v["dram_bytes"] / v["algorithmic_bytes"] < limit


def test_measured_peak():
    b = _bench()
    hbm, kind = b.measured_peaks()
    assert kind in ("measured", "fallback") and hbm > 1000


def _run_bench(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                          capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)


def test_reference_arm_prints_one_line_on_rank_zero_only():
    """`bench.py --impl reference` (the reference's algorithm on the host
    cores) under a multi-process launch: rank 0 prints one JSON line with
    impl "reference", the workload's metric and a zero-copy e2e; any other
    rank exits 0 without work or output."""
    other = _run_bench({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"},
                       "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0")
    assert other.returncode == 0 and other.stdout.strip() == ""
    zero = _run_bench({"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0"},
                      "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0")
    assert zero.returncode == 0, zero.stderr[-2000:]
    lines = [l for l in zero.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["metric"] == _bench().METRIC
