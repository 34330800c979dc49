"""The CUDA block against outputs of the reference's own MoE-block code.

tests/golden/reference_block.{npz,json}: the reference's make_forward layer
loop (src/mlx_expert_sniper/generate.py:92-187) and run_expert_ffn
(src/mlx_expert_sniper/engine.py:15-42) executed unmodified on the MLX
stand-in, on seeded inputs that are regenerated here on the CPU and moved
to the GPU. Two checks per case, through the C ABI:
  * the whole block (es_moe_forward, our router on the same logits and cache
    bias): top-k sets equal to the reference's except at near-ties of its
    own selection keys; outputs of the tokens whose sets agree within the
    bar of the case;
  * the expert FFN alone (es_moe_expert_ffn) on the reference's own indices
    and scores.
Bars, max |ours - reference| / RMS(reference): 1e-2 with fp16 scales (the
configurations' format), 5e-2 with bf16 scales, where the reference keeps
its intermediates in bf16 (its own distance from exact arithmetic is up to
~4e-2; tests/test_cpu_reference_exec.py).
"""
from __future__ import annotations

import functools
import json
import os

import numpy as np
import pytest
import torch

from expert_sniper_b200 import MoEBlock
from expert_sniper_b200.block import ffn_kernels
from oracle import moe_oracle as mo
from tests import _refexec as rx

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
BAR = {"f16": 1e-2, "bf16": 5e-2}
# With unbiased bf16 logits the reference's routing weights stay bf16 (MLX's
# softmax keeps its input dtype) while this build and the oracle keep them
# in fp32: that rounding alone puts whole blocks up to ~1.1e-2 x RMS apart
# (measured: olmoe_T16_f16). Block comparisons of such cases get this bar;
# the expert FFN fed the reference's own scores keeps the plain one.
BF16_SCORES_BLOCK_BAR = 2e-2


def block_bar(m):
    bar = BAR[m["scales"]]
    return max(bar, BF16_SCORES_BLOCK_BAR) if m["scores_dtype"] == "bfloat16" else bar


@functools.lru_cache(maxsize=None)
def _golden():
    with open(os.path.join(GOLDEN, "reference_block.json")) as f:
        meta = json.load(f)
    return {c["name"]: c for c in meta["cases"]}, dict(np.load(os.path.join(GOLDEN,
                                                                            "reference_block.npz")))


@functools.lru_cache(maxsize=1)
def _case(name):
    case = next(c for c in rx.CASES if c["name"] == name)
    cfg, lay, x, logits, sg, cb, cached = rx.case_inputs(case)
    return case, cfg, rx.fp16_layer(lay), x, logits, sg, cb


@pytest.mark.parametrize("name", [c["name"] for c in rx.CASES])
def test_block_against_reference_vectors(cuda, name):
    meta, arrays = _golden()
    m = meta[name]
    case, cfg, lay, x, logits, sg, cb = _case(name)
    dev = cuda
    lay_d = {k: v.to(dev) for k, v in lay.items()}
    T = case["T"]
    blk = MoEBlock(cfg, weights=lay_d, shared_gate_w=None if sg is None else sg.to(dev),
                   max_tokens=T)
    xd, ld = x.to(dev), logits.to(dev)
    cbd = None if cb is None else cb.to(dev)
    out, idx, w = blk.forward(xd, ld, cbd, out_dtype=torch.float32, return_routing=True)
    ref_inds = arrays[f"{name}/inds"]
    ref_scores = arrays[f"{name}/scores"]
    rows = arrays[f"{name}/rows"]
    ref = arrays[f"{name}/out"]
    ffn = blk.expert_ffn(xd, torch.from_numpy(ref_inds).to(dev),
                         torch.from_numpy(ref_scores).to(dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    bar = BAR[m["scales"]]

    # routing: sets equal to the reference's except at its near-ties
    ours = idx.cpu().numpy()
    lg = logits.float().numpy()
    ok, _, _, bad = mo.topk_parity(ours, lg, None if cb is None else cb.numpy(), cfg.top_k)
    assert ok, f"{name}: top-k beyond near-ties at tokens {bad}"
    # tokens whose sets differ are reference near-ties (checked above); with
    # bf16 selection keys and 512 experts most tokens of a batch can be
    same = np.array([set(ours[t]) == set(ref_inds[t]) for t in range(T)])
    keep = same[rows]
    err_blk = 0.0
    if keep.any():
        err_blk = float(np.abs(out.cpu().numpy()[rows][keep] - ref[keep]).max()) / rms
    assert err_blk <= block_bar(m), f"{name} [{ffn_kernels(cfg, T)}]: block {err_blk:.3e} x RMS"

    err_ffn = float(np.abs(ffn.cpu().numpy()[rows] - ref).max()) / rms
    assert err_ffn <= bar, f"{name} [{ffn_kernels(cfg, T)}]: expert FFN {err_ffn:.3e} x RMS"
    print(f"{name} [{ffn_kernels(cfg, T)}]: block {err_blk:.2e}, ffn {err_ffn:.2e} x RMS "
          f"(oracle {m['oracle_block_rel']:.2e}), sets equal on {int(same.sum())}/{T} tokens")
