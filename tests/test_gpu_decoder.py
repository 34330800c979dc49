"""The decoder around the MoE block (generate.py:98-194 restated) against an
independent fp32 restatement: embedding, RMS norms, Qwen3 attention (q/k
head norms, rotary theta, grouped-query attention over the cached context
plus the new token), MoE through the oracle's dequantised experts, final norm
and lm_head. The decoder runs bf16 activations, so logits are compared at
5e-2 x RMS (a wrong rotary, mask, norm or residual shows as O(1)); the graph
replay must equal the eager step bitwise."""
from __future__ import annotations

import math

import pytest
import torch

from expert_sniper_b200.config import MoEConfig
from expert_sniper_b200.decoder import Decoder, DecoderConfig
from expert_sniper_b200.quant import dequantize_affine, synthetic_layer

pytestmark = pytest.mark.gpu

SMALL = DecoderConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, vocab=512,
                      moe=MoEConfig(256, 16, 4, 256, True, name="dec-moe"), name="dec-small")
LOGIT_REL = 5e-2


def _ref_step(dec: Decoder, caches, tokens, pos, expert_seed=1000):
    c = dec.dcfg
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

    h = f(dec.embed[tokens])
    for l, L in enumerate(dec.layers):
        x = norm(h, L["in_norm"])
        wq, wk, wv = f(L["qkv"]).split([H * hd, KV * hd, KV * hd])
        q = rope(norm((x @ wq.t()).view(B, H, hd), L["q_norm"]))
        k = rope(norm((x @ wk.t()).view(B, KV, hd), L["k_norm"]))
        v = (x @ wv.t()).view(B, KV, hd)
        kc = torch.cat([f(caches[l][0][:, :, :pos]), k[:, :, None]], 2)
        vc = torch.cat([f(caches[l][1][:, :, :pos]), v[:, :, None]], 2)
        rep = H // KV
        kc = kc.repeat_interleave(rep, 1)
        vc = vc.repeat_interleave(rep, 1)
        att = torch.softmax(torch.einsum("bhd,bhsd->bhs", q, kc) / math.sqrt(hd), -1)
        o = torch.einsum("bhs,bhsd->bhd", att, vc).reshape(B, H * hd)
        h = h + o @ f(L["o"]).t()
        n = norm(h, L["post_norm"])
        probs = torch.softmax(n @ f(L["router"]).t(), -1)
        w, idx = probs.topk(c.moe.top_k, -1)
        w = w / w.sum(-1, keepdim=True)
        lay = synthetic_layer(c.moe, seed=expert_seed + l, device=dec.device)
        W = {p: dequantize_affine(lay[f"switch_mlp.{p}.weight"], lay[f"switch_mlp.{p}.scales"],
                                  lay[f"switch_mlp.{p}.biases"]).float()
             for p in ("gate_proj", "up_proj", "down_proj")}
        y = torch.zeros_like(h)
        for b in range(B):
            for j in range(c.moe.top_k):
                e = int(idx[b, j])
                g_ = W["gate_proj"][e] @ n[b]
                u_ = W["up_proj"][e] @ n[b]
                y[b] += w[b, j] * (W["down_proj"][e] @ (torch.nn.functional.silu(g_) * u_))
        h = h + y
    return norm(h, dec.final_norm) @ f(dec.lm_head).t()


@pytest.mark.parametrize("fused", [True, False])
def test_decoder_step_matches_fp32_restatement(cuda, fused):
    B, ctx = 3, 20
    dec = Decoder(SMALL, B, ctx, max_steps=4, seed=3, fused=fused)
    caches = [(L["k_cache"].clone(), L["v_cache"].clone()) for L in dec.layers]
    toks = torch.tensor([5, 77, 300], device=cuda)
    eager = dec.step(toks).float().clone()
    ref = _ref_step(dec, caches, toks, ctx)
    rms = float(ref.pow(2).mean().sqrt())
    err = float((eager - ref).abs().max())
    assert err <= LOGIT_REL * rms, (err, rms)
    assert int(dec.pos) == ctx + 1


def test_graph_replay_equals_eager(cuda):
    B, ctx = 2, 16
    a = Decoder(SMALL, B, ctx, max_steps=6, seed=4)
    b = Decoder(SMALL, B, ctx, max_steps=6, seed=4).capture()
    toks = torch.tensor([1, 2], device=cuda)
    for _ in range(3):
        la = a.step(toks).clone()
        lb = b.step(toks).clone()
        torch.cuda.synchronize()
        assert torch.equal(la, lb)
        toks = la.argmax(-1)
    assert int(a.pos) == int(b.pos) == ctx + 3


def test_fused_step_matches_unfused(cuda):
    """The fused kernels (add + RMS norm, q/k norm + rotary + cache write,
    one q|k|v projection, and at batch <= 4 weight-streaming GEMVs for the
    projections) round at the same points as the torch ops they replace;
    the GEMVs sum in another fp32 order than cuBLAS, which can move a bf16
    rounding by one step. Logits agree within 1e-2 x RMS plus one bf16 ulp
    of the largest logit; the written cache rows within 2e-2 x RMS."""
    B, ctx = 3, 20
    a = Decoder(SMALL, B, ctx, max_steps=4, seed=5, fused=True)
    b = Decoder(SMALL, B, ctx, max_steps=4, seed=5, fused=False)
    toks = torch.tensor([9, 100, 511], device=cuda)
    for _ in range(2):
        la = a.step(toks).float().clone()
        lb = b.step(toks).float().clone()
        rms = float(lb.pow(2).mean().sqrt())
        ulp = 2.0 ** -7 * float(lb.abs().max())
        assert float((la - lb).abs().max()) <= 1e-2 * rms + ulp
        toks = lb.argmax(-1)
    for La, Lb in zip(a.layers, b.layers):
        for name in ("k_cache", "v_cache"):
            x, y = La[name][:, :, ctx:ctx + 2].float(), Lb[name][:, :, ctx:ctx + 2].float()
            assert float((x - y).abs().max()) <= 2e-2 * float(y.pow(2).mean().sqrt())
            assert torch.equal(La[name][:, :, :ctx], Lb[name][:, :, :ctx])
