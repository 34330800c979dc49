"""GPU parity of the MoE block against the CPU oracle, through the C ABI.

Each case generates seeded MLX-format experts on the GPU, runs the CUDA block,
and compares against oracle/ (numpy + C restatements of the reference's
generate.py:122-136 router and engine.py:15-42 run_expert_ffn):
  * top-k index sets equal except at reference-dtype near-ties;
  * routing weights within 1e-5 of the oracle's fp32 softmax;
  * fp32 outputs within 1e-2 x RMS of the oracle (expected ~1e-5);
  * bf16 outputs within that plus half a bf16 ulp;
  * bitwise-identical results on repeated calls.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig, PRESETS, run_expert_ffn
from expert_sniper_b200 import _native
from expert_sniper_b200.block import uses_tensor_path
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
from oracle import c_oracle as co
from oracle import moe_oracle as mo
from tests._helpers import (assert_bf16_close, assert_close_rms, layer_to_numpy,
                            oracle_weights_for)

pytestmark = pytest.mark.gpu

SMALL = MoEConfig(256, 16, 4, 256, True, name="small")
SMALL_SHARED = MoEConfig(512, 32, 6, 512, True, shared_inter=512, name="small-shared")
SMALL_NORENORM = MoEConfig(768, 24, 3, 768, False, name="small-norenorm")

_LAYERS = {}


def _layer(cfg, seed, device):
    key = (cfg, seed)
    if key not in _LAYERS:
        if len(_LAYERS) > 2:
            _LAYERS.clear()
            torch.cuda.empty_cache()
        lay = synthetic_layer(cfg, seed=seed, device=device)
        _LAYERS[key] = (lay, layer_to_numpy(lay))
    return _LAYERS[key]


def _check_forward(cfg, T, bias, seed, device, check_bf16=True):
    lay, lay_np = _layer(cfg, 100 + seed, device)
    x, _, logits, sg = synthetic_inputs(cfg, T, seed=seed, device=device)
    cb = cache_bias_vector(cfg.num_experts, 0.5, seed)[0].to(device) if bias else None
    blk = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=T)
    out32, idx, w = blk.forward(x, logits, cb, out_dtype=torch.float32, return_routing=True)
    out16 = blk.forward(x, logits, cb)
    out32b = blk.forward(x, logits, cb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    # determinism
    assert torch.equal(out32, out32b)

    lg = logits.float().cpu().numpy()
    cbn = None if cb is None else cb.cpu().numpy()
    idx_n = idx.cpu().numpy()
    ok, n_exact, n_tie, bad = mo.topk_parity(idx_n, lg, cbn, cfg.top_k)
    assert ok, f"top-k mismatch beyond near-ties at tokens {bad[:10]}"
    # descending probability order within the k
    w_n = w.cpu().numpy()
    assert (np.diff(w_n, axis=1) <= 1e-7).all()
    w_ref = oracle_weights_for(idx_n, lg, cbn, cfg.norm_topk_prob)
    assert np.abs(w_n - w_ref).max() <= 1e-5

    xf = x.float().cpu().numpy()
    sgn = None if sg is None else sg.float().cpu().numpy()
    ref = co.expert_ffn(xf, lay_np, idx_n, w_ref, sgn)
    err, rms = assert_close_rms(out32.cpu().numpy(), ref, what=f"{cfg.name} T={T} f32")
    if check_bf16:
        assert_bf16_close(out16.float().cpu().numpy(), ref, what=f"{cfg.name} T={T} bf16")
    return err / rms, n_exact, n_tie


# The parity bar is 1e-2 x RMS; the decode kernels land near 1e-3 (h is
# carried in fp16 into the down projection), which these tighter checks pin.
# Batches that select the tensor-core path (fp16 weights, h and y) are held
# to the level pinned in test_gpu_tensor.py.
KERNEL_REL = 3e-3
TENSOR_REL = 6e-3


def _rel_bound(cfg, T):
    return TENSOR_REL if uses_tensor_path(cfg, T) else KERNEL_REL


@pytest.mark.parametrize("T", [1, 5, 33, 100])
@pytest.mark.parametrize("bias", [False, True])
def test_small_forward(cuda, T, bias):
    rel, _, _ = _check_forward(SMALL, T, bias, seed=T, device=cuda)
    assert rel < _rel_bound(SMALL, T)


@pytest.mark.parametrize("T", [1, 17, 70])
def test_small_shared_expert(cuda, T):
    rel, _, _ = _check_forward(SMALL_SHARED, T, True, seed=3 + T, device=cuda)
    assert rel < _rel_bound(SMALL_SHARED, T)


@pytest.mark.parametrize("T", [2, 40])
def test_small_no_renorm(cuda, T):
    _check_forward(SMALL_NORENORM, T, False, seed=T, device=cuda)


# the reference's configurations, full shapes
@pytest.mark.parametrize("T", [1, 32])
def test_olmoe_layer(cuda, T):
    _check_forward(PRESETS["olmoe-1b-7b"], T, False, seed=0, device=cuda)


@pytest.mark.parametrize("T", [1, 8, 64])
def test_qwen3_30b_layer(cuda, T):
    _check_forward(PRESETS["qwen3-30b-a3b"], T, True, seed=T, device=cuda)


@pytest.mark.parametrize("T", [4, 48])
def test_qwen3_next_layer_shared(cuda, T):
    _check_forward(PRESETS["qwen3-next-80b-a3b"], T, False, seed=T, device=cuda)


def test_qwen3_235b_layer(cuda):
    _check_forward(PRESETS["qwen3-235b-a22b"], 16, True, seed=5, device=cuda)


@pytest.mark.parametrize("E,k,renorm", [(16, 4, True), (512, 10, True), (64, 8, False),
                                         (1000, 16, True)])
def test_route_only_matches_oracle(cuda, E, k, renorm):
    """es_moe_route on bf16 and fp32 logits, with and without a cache bias."""
    cfg = MoEConfig(256, E, k, 256, renorm)
    lay = synthetic_layer(cfg, seed=1, device=cuda)
    blk = MoEBlock(cfg, weights=lay, max_tokens=1)
    T = 37
    g = torch.Generator(device=cuda).manual_seed(E)
    for dt in (torch.bfloat16, torch.float32):
        for bias in (None, cache_bias_vector(E, 0.5, 9)[0].to(cuda)):
            logits = torch.randn((T, E), generator=g, device=cuda).to(dt)
            idx, w = blk.route(logits, bias)
            lg = logits.float().cpu().numpy()
            bn = None if bias is None else bias.cpu().numpy()
            ok, _, _, bad = mo.topk_parity(idx.cpu().numpy(), lg, bn, k)
            assert ok, bad
            ridx, rw, _ = mo.route(lg, bn, k, renorm)
            same = (idx.cpu().numpy() == ridx).all(axis=1)
            assert same.mean() > 0.5
            assert np.abs(w.cpu().numpy()[same] - rw[same]).max() <= 1e-5


def test_expert_ffn_masked_and_duplicates(cuda):
    cfg = SMALL
    lay, lay_np = _layer(cfg, 7, cuda)
    T = 9
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=11, device=cuda)
    g = np.random.default_rng(3)
    idx = np.stack([g.choice(cfg.num_experts, cfg.top_k, replace=False) for _ in range(T)]).astype(np.int32)
    idx[0, :] = -1                    # a token that owns nothing here
    idx[1, 1] = -1
    idx[2, 2] = idx[2, 0]             # duplicate expert in one token
    w = g.random((T, cfg.top_k)).astype(np.float32)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    out = blk.expert_ffn(x, torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                         out_dtype=torch.float32)
    ref = mo.expert_ffn(x.float().cpu().numpy(), lay_np, idx, w)
    assert_close_rms(out.cpu().numpy(), ref, what="masked")
    assert torch.count_nonzero(out[0]) == 0
    assert blk.read_device_error() == 0


def test_out_of_range_id_is_flagged_and_skipped(cuda):
    cfg = SMALL
    lay, lay_np = _layer(cfg, 7, cuda)
    T = 4
    x, _, _, _ = synthetic_inputs(cfg, T, seed=12, device=cuda)
    idx = np.array([[0, 1, 2, 3]] * T, np.int32)
    idx[1, 3] = cfg.num_experts + 5   # bounds-checked by the kernel
    w = np.full((T, cfg.top_k), 0.25, np.float32)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    out = blk.expert_ffn(x, torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                         out_dtype=torch.float32)
    assert blk.read_device_error() & _native.DEVERR_BAD_EXPERT_ID
    assert blk.read_device_error() == 0  # cleared by the first read
    masked = idx.copy()
    masked[1, 3] = -1
    ref = mo.expert_ffn(x.float().cpu().numpy(), lay_np, masked, w)
    assert_close_rms(out.cpu().numpy(), ref, what="oob")


def test_nan_logit_is_flagged(cuda):
    cfg = SMALL
    lay, _ = _layer(cfg, 7, cuda)
    x, _, logits, _ = synthetic_inputs(cfg, 3, seed=13, device=cuda)
    logits = logits.clone()
    logits[1, 5] = float("nan")
    blk = MoEBlock(cfg, weights=lay, max_tokens=3)
    _, idx, _ = blk.forward(x, logits, return_routing=True)
    assert blk.read_device_error() & _native.DEVERR_NONFINITE_LOGIT
    assert 5 not in idx[1].tolist()


def test_fp16_range_of_h_is_flagged(cuda):
    """Activations large enough that silu(g)*u leaves the fp16 range: the
    kernel saturates h and sets ES_DEVERR_RANGE instead of producing inf."""
    cfg = SMALL
    lay, _ = _layer(cfg, 7, cuda)
    x, _, logits, _ = synthetic_inputs(cfg, 2, seed=16, device=cuda)
    big = (x.float() * 2000.0).to(torch.bfloat16)
    blk = MoEBlock(cfg, weights=lay, max_tokens=2)
    out = blk.forward(big, logits, out_dtype=torch.float32)
    assert blk.read_device_error() & 0x10
    assert torch.isfinite(out).all()


def test_empty_batch(cuda):
    cfg = SMALL
    lay, _ = _layer(cfg, 7, cuda)
    blk = MoEBlock(cfg, weights=lay, max_tokens=4)
    x = torch.empty((0, cfg.hidden), dtype=torch.bfloat16, device=cuda)
    lg = torch.empty((0, cfg.num_experts), dtype=torch.bfloat16, device=cuda)
    out = blk.forward(x, lg)
    assert out.shape == (0, cfg.hidden)


def test_batched_leading_dims(cuda):
    """[1, T, D] inputs as make_forward passes them."""
    cfg = SMALL
    lay, lay_np = _layer(cfg, 7, cuda)
    x, _, logits, _ = synthetic_inputs(cfg, 6, seed=14, device=cuda)
    blk = MoEBlock(cfg, weights=lay, max_tokens=6)
    out = blk.forward(x[None], logits[None], out_dtype=torch.float32)
    assert out.shape == (1, 6, cfg.hidden)
    flat = blk.forward(x, logits, out_dtype=torch.float32)
    assert torch.equal(out[0], flat)


def test_run_expert_ffn_dropin(cuda):
    """The reference's per-call signature: dict of active experts."""
    cfg = SMALL
    lay, lay_np = _layer(cfg, 7, cuda)
    T = 5
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=15, device=cuda)
    idx, w, _ = mo.route(logits.float().cpu().numpy(), None, cfg.top_k, True)
    active = sorted(set(int(e) for e in idx.ravel()))
    expert_data = {e: {name: t[e] for name, t in lay.items()} for e in active}
    out = run_expert_ffn(x[None], expert_data, torch.from_numpy(idx)[None].to(cuda),
                         torch.from_numpy(w)[None].to(cuda))
    assert out.shape == (1, T, cfg.hidden) and out.dtype == torch.bfloat16
    ref = mo.expert_ffn(x.float().cpu().numpy(), lay_np, idx, w)
    assert_bf16_close(out[0].float().cpu().numpy(), ref, what="run_expert_ffn")


def test_full_size_properties_235b(cuda):
    """Qwen3-235B-shaped layer at decode batch 256: size-independent
    properties instead of a full oracle pass. (1) scaling the routing
    weights by 2 doubles the output bit-exactly; (2) the sum of the
    per-owner partials of an 8-way expert partition equals the full block
    to fp32 rounding (the expert-parallel invariant of reader.py:278-286)."""
    from expert_sniper_b200 import hrw
    cfg = PRESETS["qwen3-235b-a22b"]
    lay, _ = _layer(cfg, 21, cuda)
    T = 256
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=21, device=cuda)
    cb = cache_bias_vector(cfg.num_experts, 0.5, 21)[0].to(cuda)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    full, idx, w = blk.forward(x, logits, cb, out_dtype=torch.float32, return_routing=True)
    twice = blk.expert_ffn(x, idx, 2 * w, out_dtype=torch.float32)
    assert torch.equal(twice, 2 * full)
    roster = hrw.gpu_roster(8)
    table = torch.tensor(hrw.owner_table(hrw.plan(roster, cfg.num_experts), roster,
                                         cfg.num_experts), device=cuda)
    total = torch.zeros_like(full)
    for r in range(8):
        mine = torch.where(table[idx.long()] == r, idx, torch.full_like(idx, -1))
        total += blk.expert_ffn(x, mine, w, out_dtype=torch.float32)
    rms = full.pow(2).mean().sqrt()
    assert (total - full).abs().max() <= 1e-5 * rms
