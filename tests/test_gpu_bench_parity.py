"""Parity at the benchmarked workloads, at their timed sizes, with the
benchmark's own seeds (bench.py), against the C oracle.

  * Qwen3-Next-80B-A3B layer prefill, T = 4096, shared expert, no bias: the
    128-token tensor-core kernels. Routing is checked for every token; the
    outputs on a seeded subset of 256 rows (rows are independent tokens), in
    fp32 and in the benchmark's bf16; ten back-to-back calls bitwise equal
    with a clear error block.
  * Qwen3-235B-A22B layer, decode batch T = 256, bias +0.5 on the seeded 25%
    hot set: all rows.
  * Qwen3-30B-A3B layer, decode batches 64, 8 and 1 with bias +0.5: all rows.
  * The 48-layer Qwen3-30B-shaped decoder, one step at batch 1 with the
    2048-token context, against an fp32 restatement of the step.
Reference functions: generate.py:122-136 (router), engine.py:15-42
(run_expert_ffn), generate.py:173-178 (shared expert), generate.py:108-194
(the decoder's layer loop).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from expert_sniper_b200 import MoEBlock, PRESETS
from expert_sniper_b200.block import ffn_kernels
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
from oracle import c_oracle as co
from oracle import moe_oracle as mo
from tests._helpers import (assert_bf16_close, assert_close_rms, layer_to_numpy,
                            oracle_weights_for)

pytestmark = pytest.mark.gpu

TENSOR_REL = 6e-3   # tensor-core kernels: fp16 weights, h and y
DECODE_REL = 3e-3   # decode kernels: fp16 h


def _check(cfg, lay, x, logits, sg, cb, rows, rel, repeats=1):
    blk = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=x.shape[0])
    out32, idx, w = blk.forward(x, logits, cb, out_dtype=torch.float32, return_routing=True)
    out16 = blk.forward(x, logits, cb)
    for _ in range(repeats):
        again = blk.forward(x, logits, cb, out_dtype=torch.float32)
        assert torch.equal(again, out32)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    lg = logits.float().cpu().numpy()
    cbn = None if cb is None else cb.cpu().numpy()
    idx_n = idx.cpu().numpy()
    ok, _, _, bad = mo.topk_parity(idx_n, lg, cbn, cfg.top_k)
    assert ok, f"top-k beyond near-ties at tokens {bad[:10]}"
    w_ref = oracle_weights_for(idx_n, lg, cbn, cfg.norm_topk_prob)
    assert np.abs(w.cpu().numpy() - w_ref).max() <= 1e-5
    lay_np = layer_to_numpy(lay)
    sgn = None if sg is None else sg.float().cpu().numpy()
    xf = x.float().cpu().numpy()[rows]
    ref = co.expert_ffn(xf, lay_np, idx_n[rows], w_ref[rows], sgn)
    err, rms = assert_close_rms(out32.cpu().numpy()[rows], ref, rel=rel)
    assert_bf16_close(out16.float().cpu().numpy()[rows], ref)
    return err / rms


def test_prefill_qwen3_next_T4096(cuda):
    cfg = PRESETS["qwen3-next-80b-a3b"]
    T = 4096
    assert ffn_kernels(cfg, T) == "tensor"
    lay = synthetic_layer(cfg, seed=2000, device=cuda)
    x, _, logits, sg = synthetic_inputs(cfg, T, seed=3000, device=cuda)
    rows = np.sort(np.random.default_rng(0).choice(T, 256, replace=False))
    _check(cfg, lay, x, logits, sg, None, rows, TENSOR_REL, repeats=10)


def test_decode_qwen3_235b_T256_bias(cuda):
    cfg = PRESETS["qwen3-235b-a22b"]
    T = 256
    lay = synthetic_layer(cfg, seed=5000, device=cuda)
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=6000, device=cuda)
    cb = cache_bias_vector(cfg.num_experts, 0.5, 0)[0].to(cuda)
    rel = TENSOR_REL if ffn_kernels(cfg, T) != "decode" else DECODE_REL
    _check(cfg, lay, x, logits, None, cb, np.arange(T), rel)


@pytest.mark.parametrize("T", [64, 8, 1])
def test_decode_qwen3_30b_bench_batches(cuda, T):
    cfg = PRESETS["qwen3-30b-a3b"]
    lay = synthetic_layer(cfg, seed=1000, device=cuda)
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=10_000 * T, device=cuda)
    cb = cache_bias_vector(cfg.num_experts, 0.5, 0)[0].to(cuda)
    rel = TENSOR_REL if ffn_kernels(cfg, T) != "decode" else DECODE_REL
    _check(cfg, lay, x, logits, None, cb, np.arange(T), rel)


def _attention_ref(dec, l, h, caches, pos):
    """fp32 restatement of the attention half of layer l (Qwen3 attention:
    q/k/v projections, per-head RMS norm, rotary, grouped-query attention
    over the cached context plus the new token, output projection, residual
    add) from the residual h [B, D]."""
    c = dec.dcfg
    L = dec.layers[l]
    B, H, KV, hd = dec.batch, c.heads, c.kv_heads, c.head_dim
    f = lambda t: t.float()

    def norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + c.eps) * f(w)

    inv = c.rope_theta ** (-torch.arange(0, hd, 2, dtype=torch.float64, device=dec.device) / hd)
    ang = (pos * inv).float()
    cos, sin = ang.cos(), ang.sin()

    def rope(x):
        x1, x2 = x[..., :hd // 2], x[..., hd // 2:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)

    x = norm(h, L["in_norm"])
    wq, wk, wv = f(L["qkv"]).split([H * hd, KV * hd, KV * hd])
    q = rope(norm((x @ wq.t()).view(B, H, hd), L["q_norm"]))
    k = rope(norm((x @ wk.t()).view(B, KV, hd), L["k_norm"]))
    v = (x @ wv.t()).view(B, KV, hd)
    kc = torch.cat([f(caches[l][0][:, :, :pos]), k[:, :, None]], 2)
    vc = torch.cat([f(caches[l][1][:, :, :pos]), v[:, :, None]], 2)
    rep = H // KV
    att = torch.softmax(torch.einsum("bhd,bhsd->bhs", q, kc.repeat_interleave(rep, 1))
                        / math.sqrt(hd), -1)
    o = torch.einsum("bhs,bhsd->bhd", att, vc.repeat_interleave(rep, 1)).reshape(B, H * hd)
    return h + o @ f(L["o"]).t()


def _moe_ref(dec, l, n, logits, expert_seed=1000):
    """fp32 MoE block of layer l on the decoder's own normed input n and
    router logits (top-k on those logits, ties to the lower id, softmax
    renormalised over the k): engine.py:15-42 with generate.py:131-136."""
    from expert_sniper_b200.quant import dequantize_affine
    moe = dec.dcfg.moe
    probs = torch.softmax(logits, -1)
    order = torch.sort(-logits, dim=-1, stable=True).indices[:, :moe.top_k]
    w = torch.gather(probs, -1, order)
    w = w / w.sum(-1, keepdim=True)
    lay = synthetic_layer(moe, seed=expert_seed + l, device=dec.device)
    y = torch.zeros_like(n)
    for b in range(n.shape[0]):
        for j in range(moe.top_k):
            e = int(order[b, j])
            W = {p: dequantize_affine(lay[f"switch_mlp.{p}.weight"][e],
                                      lay[f"switch_mlp.{p}.scales"][e],
                                      lay[f"switch_mlp.{p}.biases"][e]).float()
                 for p in ("gate_proj", "up_proj", "down_proj")}
            g_ = W["gate_proj"] @ n[b]
            u_ = W["up_proj"] @ n[b]
            y[b] += w[b, j] * (W["down_proj"] @ (torch.nn.functional.silu(g_) * u_))
    return y


def test_decoder_qwen3_30b_48_layers_batch1(cuda):
    """The benchmarked decoder (48 layers, 2048-token context) for one step
    at batch 1, every layer at full size against fp32 restatements, each
    part from the decoder's own inputs so that bf16 rounding and routing
    choices of earlier parts do not compound:
      * the residual after each layer, read by running the decoder
        truncated to 0, 1, ..., 48 layers;
      * each MoE block's input n, router logits and output, recorded by
        wrapping the layer's block;
      * attention half: the restatement from the residual before the layer
        against (residual after the layer - the block's output), within
        5e-2 x RMS of the attention's contribution plus two bf16 roundings
        of the residual;
      * router: logits against n @ W_router^T within a bf16 rounding;
      * MoE block: output against the fp32 block on the decoder's n and
        logits within 1e-2 x RMS plus half a bf16 ulp;
      * final norm and lm_head from the last residual; the graph-replayed
        step equals the eager one bitwise."""
    from expert_sniper_b200.decoder import Decoder, DecoderConfig
    dcfg = DecoderConfig(layers=48)
    ctx = 2048
    dec = Decoder(dcfg, 1, ctx, max_steps=4, seed=0)
    caches = [(L["k_cache"][:, :, :ctx].clone(), L["v_cache"][:, :, :ctx].clone())
              for L in dec.layers]
    toks = torch.tensor([12345], device=cuda)
    layers = dec.layers
    rec = {}
    for l, L in enumerate(layers):
        blk = L["moe"]
        orig = blk.forward

        def wrapped(n, logits, bias=None, *a, _l=l, _orig=orig, **kw):
            out = _orig(n, logits, bias, *a, **kw)
            rec[_l] = (n.float().clone(), logits.float().clone(), out.float().clone())
            return out
        blk.forward = wrapped
    hs = []
    for l in range(len(layers) + 1):
        dec.layers = layers[:l]
        dec.pos.fill_(ctx)
        dec.step(toks)
        torch.cuda.synchronize()
        hs.append(dec.h.float().clone())
    dec.layers = layers
    dec.pos.fill_(ctx)
    eager = dec.step(toks).float().clone()
    torch.cuda.synchronize()
    for L in layers:
        del L["moe"].forward          # back to the class method for capture
    dec.pos.fill_(ctx)
    dec.capture()
    graph = dec.step(toks).float().clone()
    torch.cuda.synchronize()
    assert torch.equal(graph, eager)

    bf16_ulp = lambda v: 2.0 ** (torch.floor(torch.log2(v.abs().clamp_min(2.0 ** -126))) - 7)
    for l in range(len(layers)):
        n, logits, delta = rec[l]
        h1 = _attention_ref(dec, l, hs[l], caches, ctx)
        h1_dec = hs[l + 1] - delta
        attn = h1 - hs[l]
        tol = 5e-2 * float(attn.pow(2).mean().sqrt()) + 2 * bf16_ulp(hs[l + 1])
        assert ((h1_dec - h1).abs() <= tol).all(), \
            f"layer {l} attention: {float((h1_dec - h1).abs().max()):.3e}"
        lg_ref = n @ layers[l]["router"].float().t()
        assert ((logits - lg_ref).abs() <= bf16_ulp(lg_ref) + 1e-3).all(), f"layer {l} router"
        y = _moe_ref(dec, l, n, logits)
        rms = float(y.pow(2).mean().sqrt())
        assert ((delta - y).abs() <= 1e-2 * rms + 0.5 * bf16_ulp(y)).all(), \
            f"layer {l} MoE: {float((delta - y).abs().max()) / rms:.3e} x RMS"
    c = dec.dcfg
    hN = hs[-1]
    nN = hN * torch.rsqrt(hN.pow(2).mean(-1, keepdim=True) + c.eps) * dec.final_norm.float()
    ref_logits = nN @ dec.lm_head.float().t()
    rms = float(ref_logits.pow(2).mean().sqrt())
    ulp = 2.0 ** -7 * float(ref_logits.abs().max())
    assert float((eager - ref_logits).abs().max()) <= 1e-2 * rms + ulp
