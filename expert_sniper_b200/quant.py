"""MLX-affine 4-bit weight format: quantise, pack, and synthetic experts.

Format (the reference's expert tensors, src/mlx_expert_sniper/download.py:73-77,
engine.py:12-13): per row, 64-column groups; code q in [0, 15] of column k is
stored in bits 4*(k % 8) of uint32 word k // 8; w = scale * q + bias with fp16
scale and bias per (row, group).

The quantiser here is this library's own min/max affine rule (scale =
(max - min) / 15, bias = min, q = round((w - bias) / scale)); the kernels and
the oracle both consume the packed tensors it produces, so parity does not
depend on which affine rule made them. It runs on CPU or GPU tensors.
"""
from __future__ import annotations

import torch

from .config import MoEConfig

GROUP = 64
PROJS = ("gate_proj", "up_proj", "down_proj")
KINDS = ("weight", "scales", "biases")


def quantize_affine(w: torch.Tensor):
    """w [..., N, K] (any float dtype) -> (q int32 [..., N, K/8] holding uint32
    bits, scales fp16 [..., N, K/64], biases fp16 [..., N, K/64])."""
    *lead, n, k = w.shape
    if k % GROUP:
        raise ValueError("K must be a multiple of 64")
    wg = w.float().reshape(*lead, n, k // GROUP, GROUP)
    wmin = wg.amin(dim=-1)
    wmax = wg.amax(dim=-1)
    scale = ((wmax - wmin) / 15.0).half()
    bias = wmin.half()
    s = scale.float().unsqueeze(-1)
    b = bias.float().unsqueeze(-1)
    safe = torch.where(s > 0, s, torch.ones_like(s))
    q = torch.round((wg - b) / safe).clamp_(0, 15)
    q = torch.where(s > 0, q, torch.zeros_like(q)).to(torch.int64)
    q = q.reshape(*lead, n, k // 8, 8)
    shifts = (torch.arange(8, device=w.device, dtype=torch.int64) * 4)
    words = (q << shifts).sum(dim=-1)                       # < 2**32
    words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    return words, scale, bias


def unpack_codes(words: torch.Tensor) -> torch.Tensor:
    """int32 [..., N, K/8] -> uint8 codes [..., N, K]."""
    w = words.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, device=words.device, dtype=torch.int64) * 4
    codes = (w.unsqueeze(-1) >> shifts) & 0xF
    return codes.reshape(*words.shape[:-1], words.shape[-1] * 8).to(torch.uint8)


def dequantize_affine(words, scales, biases) -> torch.Tensor:
    """Packed tensors -> fp32 [..., N, K] (w = scale * q + bias)."""
    codes = unpack_codes(words).float()
    *lead, n, k = codes.shape
    cg = codes.reshape(*lead, n, k // GROUP, GROUP)
    out = cg * scales.float().unsqueeze(-1) + biases.float().unsqueeze(-1)
    return out.reshape(*lead, n, k)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def synthetic_layer(cfg: MoEConfig, seed: int, device="cpu", std: float = 0.02,
                    experts_per_chunk: int = 16) -> dict:
    """Seeded synthetic expert weights of one layer in the reference's tensor
    naming: {"switch_mlp.<proj>.<kind>": [E, ...]} plus, with a shared expert,
    {"shared_expert.<proj>.<kind>": [...]}. Weights are fp16 N(0, std)
    quantised with `quantize_affine`, generated in chunks of experts so a GPU
    holds only one chunk of fp16 weights at a time."""
    device = torch.device(device)
    g = _gen(seed, device)
    D, I, E = cfg.hidden, cfg.inter, cfg.num_experts
    shapes = {"gate_proj": (I, D), "up_proj": (I, D), "down_proj": (D, I)}
    out = {}
    for proj in PROJS:
        n, k = shapes[proj]
        out[f"switch_mlp.{proj}.weight"] = torch.empty((E, n, k // 8), dtype=torch.int32, device=device)
        out[f"switch_mlp.{proj}.scales"] = torch.empty((E, n, k // GROUP), dtype=torch.float16, device=device)
        out[f"switch_mlp.{proj}.biases"] = torch.empty((E, n, k // GROUP), dtype=torch.float16, device=device)
    for e0 in range(0, E, experts_per_chunk):
        e1 = min(E, e0 + experts_per_chunk)
        for proj in PROJS:
            n, k = shapes[proj]
            w = (torch.randn((e1 - e0, n, k), generator=g, device=device,
                             dtype=torch.float32) * std).half()
            q, s, b = quantize_affine(w)
            out[f"switch_mlp.{proj}.weight"][e0:e1] = q
            out[f"switch_mlp.{proj}.scales"][e0:e1] = s
            out[f"switch_mlp.{proj}.biases"][e0:e1] = b
    if cfg.has_shared:
        for proj in PROJS:
            n, k = shapes[proj]
            w = (torch.randn((n, k), generator=g, device=device, dtype=torch.float32) * std).half()
            q, s, b = quantize_affine(w)
            out[f"shared_expert.{proj}.weight"] = q
            out[f"shared_expert.{proj}.scales"] = s
            out[f"shared_expert.{proj}.biases"] = b
    return out


def synthetic_inputs(cfg: MoEConfig, T: int, seed: int, device="cpu",
                     router_std: float = 0.02, with_shared_gate: bool = True):
    """Seeded x [T, D] bf16 N(0, 1), router weight [E, D] bf16 N(0, router_std),
    logits = x @ Wr^T rounded to bf16 (an MLX bf16 Linear), and, with a shared
    expert, the shared gate weight [D] bf16 N(0, router_std)."""
    device = torch.device(device)
    g = _gen(seed, device)
    x = torch.randn((T, cfg.hidden), generator=g, device=device).to(torch.bfloat16)
    wr = (torch.randn((cfg.num_experts, cfg.hidden), generator=g, device=device)
          * router_std).to(torch.bfloat16)
    logits = (x.float() @ wr.float().t()).to(torch.bfloat16)
    sg = None
    if cfg.has_shared and with_shared_gate:
        sg = (torch.randn((cfg.hidden,), generator=g, device=device) * router_std).to(torch.bfloat16)
    return x, wr, logits, sg


def cache_bias_vector(num_experts: int, bias: float, seed: int, frac: float = 0.25):
    """The reference's cache-aware routing mask (generate.py:124-129): `bias`
    on a seeded subset of round(frac*E) "cached" experts, 0 elsewhere, fp32.
    The subset is numpy.random.default_rng(seed).choice(E, n, replace=False)."""
    import numpy as np
    n = int(round(frac * num_experts))
    ids = np.random.default_rng(seed).choice(num_experts, n, replace=False)
    mask = np.zeros(num_experts, dtype=np.float32)
    mask[ids] = bias
    return torch.from_numpy(mask), sorted(int(i) for i in ids)
