"""Tensor-core (tcgen05) path of the MoE block against the CPU oracle.

The path dequantises weights to fp16 (w = scale * q + bias rounded once),
carries activations as fp16 rows with a per-token power-of-two scale, h and
the per-pair rows y as fp16, and accumulates in fp32 in tensor memory. Each
fp16 rounding is at most 2^-11 relative, so outputs stay far inside the
parity bar (1e-2 x RMS); TENSOR_REL pins the level the path reaches
(about 4e-3 at worst over ~1e5 outputs: four fp16 roundings -- gate/up
weights, h, down weights, y -- against the decode path's one).
Cases cover several token tiles per expert, masked and duplicate slots,
rows of very different magnitude, repeated calls (bitwise), agreement with
the decode path, and the Qwen3-Next prefill and Qwen3-30B shapes at full
size (sampled tokens against the oracle). Each runs on both variants of
the GEMMs: "tensor" (128-token tiles, dequantised weights in shared memory)
and "tensor-small" (32-token tiles, dequantised weights in tensor memory).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig, PRESETS
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
from oracle import c_oracle as co
from oracle import moe_oracle as mo
from tests._helpers import assert_close_rms, layer_to_numpy, oracle_weights_for

pytestmark = pytest.mark.gpu

TENSOR_REL = 6e-3

SMALL = MoEConfig(512, 32, 6, 512, True, shared_inter=512, name="tc-small")
PLAIN = MoEConfig(256, 16, 4, 256, True, name="tc-plain")

_LAYERS = {}


def _layer(cfg, seed, device):
    key = (cfg.hidden, cfg.num_experts, cfg.inter, cfg.shared_inter, seed)
    if key not in _LAYERS:
        if len(_LAYERS) > 1:
            _LAYERS.clear()
            torch.cuda.empty_cache()
        lay = synthetic_layer(cfg, seed=seed, device=device)
        _LAYERS[key] = (lay, layer_to_numpy(lay))
    return _LAYERS[key]


def _sample_check(out, x, idx, w_ref, lay_np, sg, rows, what):
    xs = x.float().cpu().numpy()[rows]
    sgn = None if sg is None else sg.float().cpu().numpy()
    ref = co.expert_ffn(xs, lay_np, idx[rows], w_ref[rows], sgn)
    err, rms = assert_close_rms(out[rows], ref, what=what)
    return err / rms


PATHS = ["tensor", "tensor-small"]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("T", [16, 64, 200])
@pytest.mark.parametrize("bias", [False, True])
def test_tensor_path_small(cuda, T, bias, path):
    cfg = SMALL.with_(kernel_path=path)
    lay, lay_np = _layer(cfg, 31, cuda)
    x, _, logits, sg = synthetic_inputs(cfg, T, seed=40 + T, device=cuda)
    cb = cache_bias_vector(cfg.num_experts, 0.5, T)[0].to(cuda) if bias else None
    blk = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=T)
    out, idx, w = blk.forward(x, logits, cb, out_dtype=torch.float32, return_routing=True)
    again = blk.forward(x, logits, cb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    assert torch.equal(out, again), "repeated calls must agree bitwise"
    lg = logits.float().cpu().numpy()
    cbn = None if cb is None else cb.cpu().numpy()
    idx_n = idx.cpu().numpy()
    ok, _, _, bad = mo.topk_parity(idx_n, lg, cbn, cfg.top_k)
    assert ok, bad
    w_ref = oracle_weights_for(idx_n, lg, cbn, cfg.norm_topk_prob)
    rel = _sample_check(out.cpu().numpy(), x, idx_n, w_ref, lay_np, sg, np.arange(T), "tensor")
    assert rel < TENSOR_REL
    # the decode kernels on the same inputs
    dec = MoEBlock(cfg.with_(kernel_path="decode"), packed=blk.packed, shared_gate_w=sg,
                   max_tokens=T).forward(x, logits, cb, out_dtype=torch.float32)
    assert_close_rms(out.cpu().numpy(), dec.cpu().numpy(), rel=TENSOR_REL, what="vs decode")


@pytest.mark.parametrize("path", PATHS)
def test_tensor_path_many_tiles_masked_duplicates(cuda, path):
    """Experts 0..3 in every token (T = 300: three 128-token tiles each, or
    ten 32-token tiles), masked slots (-1), a duplicated expert in one token,
    a token with nothing routed."""
    cfg = PLAIN.with_(kernel_path=path)
    lay, lay_np = _layer(cfg, 32, cuda)
    T = 300
    x, _, _, _ = synthetic_inputs(cfg, T, seed=5, device=cuda)
    g = np.random.default_rng(8)
    idx = np.stack([np.concatenate([[0, 1], g.choice(np.arange(2, cfg.num_experts), 2,
                                                      replace=False)]) for _ in range(T)])
    idx[:, 2] = np.where(np.arange(T) % 2 == 0, 2, idx[:, 2])
    idx[:, 3] = np.where(np.arange(T) % 3 == 0, 3, idx[:, 3])
    idx = idx.astype(np.int32)
    idx[7, 3] = -1
    idx[9, :] = -1
    idx[11, 2] = idx[11, 0]
    w = g.random((T, cfg.top_k)).astype(np.float32)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    out = blk.expert_ffn(x, torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                         out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    ref = mo.expert_ffn(x.float().cpu().numpy(), lay_np, idx, w)
    err, rms = assert_close_rms(out.cpu().numpy(), ref, what="tiles")
    assert err / rms < TENSOR_REL
    assert torch.count_nonzero(out[9]) == 0


@pytest.mark.parametrize("path", PATHS)
def test_tensor_path_row_scales(cuda, path):
    """Rows scaled by 1e2 and 1e-1 against each row's own RMS: the
    activations' per-token power-of-two scale keeps every row's relative
    accuracy. (h and y are plain fp16 on both paths: much larger rows
    saturate h and are flagged, much smaller ones lose h to fp16 underflow;
    normalised hidden states stay far from both.)"""
    cfg = PLAIN.with_(kernel_path=path)
    lay, lay_np = _layer(cfg, 32, cuda)
    T = 96
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=6, device=cuda)
    f = torch.ones(T, 1, device=cuda)
    f[::3] = 1e2
    f[1::3] = 1e-1
    xs = (x.float() * f).to(torch.bfloat16)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    out, idx, w = blk.forward(xs, logits, out_dtype=torch.float32, return_routing=True)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    ref = co.expert_ffn(xs.float().cpu().numpy(), lay_np, idx.cpu().numpy(),
                        oracle_weights_for(idx.cpu().numpy(), logits.float().cpu().numpy(), None,
                                           True))
    o = out.cpu().numpy()
    for t in range(T):  # relative to each row's own RMS
        rms = float(np.sqrt(np.mean(ref[t].astype(np.float64) ** 2)))
        assert np.abs(o[t] - ref[t]).max() <= TENSOR_REL * rms, t


@pytest.mark.parametrize("name,T,bias,path", [("qwen3-next-80b-a3b", 4096, False, "auto"),
                                              ("qwen3-30b-a3b", 512, True, "auto"),
                                              ("qwen3-30b-a3b", 256, True, "auto"),
                                              ("qwen3-30b-a3b", 64, True, "tensor-small"),
                                              ("qwen3-30b-a3b", 1, True, "tensor-small"),
                                              ("qwen3-next-80b-a3b", 8, False, "tensor-small")])
def test_tensor_path_full_shapes(cuda, name, T, bias, path):
    """Full-size layers: prefill batch sizes (the automatic choice picks the
    tensor path there) and decode sizes on the small-tile variant; up to 64
    sampled tokens against the oracle, all tokens against the decode
    kernels."""
    cfg = PRESETS[name].with_(kernel_path=path)
    lay, lay_np = _layer(cfg, 50, cuda)
    x, _, logits, sg = synthetic_inputs(cfg, T, seed=51, device=cuda)
    cb = cache_bias_vector(cfg.num_experts, 0.5, 3)[0].to(cuda) if bias else None
    blk = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=T)
    out, idx, w = blk.forward(x, logits, cb, out_dtype=torch.float32, return_routing=True)
    again = blk.forward(x, logits, cb, out_dtype=torch.float32)
    for _ in range(8):  # back-to-back calls: every bounded wait completes
        blk.forward(x, logits, cb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    words = blk.workspace[:16].view(torch.int32).cpu().tolist()
    assert words[:4] == [0, 0, 0, 0], f"device error / timed-out wait site: {words[:4]}"
    assert torch.equal(out, again)
    lg = logits.float().cpu().numpy()
    cbn = None if cb is None else cb.cpu().numpy()
    idx_n = idx.cpu().numpy()
    ok, _, _, bad = mo.topk_parity(idx_n, lg, cbn, cfg.top_k)
    assert ok, bad
    w_ref = oracle_weights_for(idx_n, lg, cbn, cfg.norm_topk_prob)
    rows = np.random.default_rng(T).choice(T, min(T, 64), replace=False)
    rel = _sample_check(out.cpu().numpy(), x, idx_n, w_ref, lay_np, sg, rows, name)
    assert rel < TENSOR_REL
    dec = MoEBlock(cfg.with_(kernel_path="decode"), packed=blk.packed, shared_gate_w=sg,
                   max_tokens=T).forward(x, logits, cb, out_dtype=torch.float32)
    assert_close_rms(out.cpu().numpy(), dec.cpu().numpy(), rel=TENSOR_REL, what="vs decode")


def test_fp16_activations(cuda):
    """x given in fp16 (es_moe_cfg.x_dtype, the Expert Network wire dtype):
    read without rounding, against the oracle on the same fp16 values."""
    cfg = SMALL.with_(x_dtype="f16")
    lay, lay_np = _layer(cfg, 31, cuda)
    T = 40
    x, _, logits, sg = synthetic_inputs(cfg, T, seed=77, device=cuda)
    x16 = (x.float() * 3.0).half()
    blk = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=T)
    out, idx, w = blk.forward(x16, logits, None, out_dtype=torch.float32, return_routing=True)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    idx_n = idx.cpu().numpy()
    w_ref = oracle_weights_for(idx_n, logits.float().cpu().numpy(), None, cfg.norm_topk_prob)
    ref = co.expert_ffn(x16.float().cpu().numpy(), lay_np, idx_n, w_ref, sg.float().cpu().numpy())
    err, rms = assert_close_rms(out.cpu().numpy(), ref, what="fp16 x")
    assert err / rms < TENSOR_REL
    with pytest.raises(ValueError):
        blk.forward(x, logits)  # bf16 given to an fp16-x block
