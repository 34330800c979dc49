"""A Qwen3-MoE-shaped decoder around the MoE block: the caller side of the
hot path.

Restates the per-layer loop of the reference's `make_forward`
(src/mlx_expert_sniper/generate.py:98-194) for batched decode on one GPU:

  h = embed(tokens)
  for each layer:
      h = h + attention(rms_norm(h))                      (generate.py:112-118)
      n = rms_norm(h)                                      (:120)
      h = h + MoE block(n, gate(n) [+ cache bias])         (:121-178)
  logits = lm_head(rms_norm(h))                            (:192-193)

Attention is the Qwen3 one: q/k/v projections, RMS norm per head on q and
k, rotary embedding (theta 1e6), grouped-query attention over a KV cache,
output projection. The MoE block is MoEBlock (router, dispatch, 4-bit
experts, combine; the kernels of this package). A whole decode step, all
layers, is one CUDA graph: the position lives on the device (KV write index,
rotary angle and attention mask are computed from it), so the same graph
replays step after step.

Two forms of the code around the block, same arithmetic (fp32 math on bf16
tensors, bf16 rounding at the same points):
  fused=True   one q|k|v projection; the residual add + RMS norm and
               the q/k norm + rotary + cache write are single kernels of
               libes_moe.so (es_dec_add_rmsnorm, es_dec_qk_norm_rope_kv);
               at batch <= 4 the q|k|v, output and router projections are
               weight-streaming GEMVs (es_dec_gemv), cuBLAS above;
  fused=False  the same steps as separate torch ops (the restatement the
               fused kernels are checked against).
Attention itself is torch's scaled_dot_product_attention in both.

Weights are random (seeded): attention and embeddings bf16 N(0, 0.02),
experts quantised MLX-affine 4-bit, norms 1; the KV cache holds a seeded
N(0, 1) bf16 context. The model is a shape and timing stand-in, not a
trained network.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import ctypes

import torch
import torch.nn.functional as F

from . import _native
from .block import MoEBlock, prepare_packed
from .config import MoEConfig, PRESETS
from .quant import synthetic_layer


@dataclass
class DecoderConfig:
    layers: int = 48
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6
    moe: MoEConfig = field(default_factory=lambda: PRESETS["qwen3-30b-a3b"])
    name: str = "qwen3-30b-a3b-decoder"


QWEN3_30B_DECODER = DecoderConfig()


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def rope_tables(head_dim: int, max_pos: int, theta: float, device):
    inv = theta ** (-torch.arange(0, head_dim, 2, device=device, dtype=torch.float64) / head_dim)
    ang = torch.arange(max_pos, device=device, dtype=torch.float64)[:, None] * inv[None]
    return ang.cos().float(), ang.sin().float()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., head_dim]; rotate the two halves (the non-interleaved form)."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h].float(), x[..., h:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).to(x.dtype)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def add_rmsnorm_(h: torch.Tensor, delta, w: torch.Tensor, out: torch.Tensor,
                 eps: float) -> torch.Tensor:
    """h += delta (bf16, in place; skipped when delta is None), then
    out = rms_norm(h, w): one es_dec_add_rmsnorm launch."""
    rows, cols = h.shape
    for t in (h, w, out) + ((delta,) if delta is not None else ()):
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()):
            raise ValueError("add_rmsnorm_ takes contiguous bf16 CUDA tensors")
    if out.shape != h.shape or w.numel() != cols or (delta is not None and delta.shape != h.shape):
        raise ValueError("add_rmsnorm_: shape mismatch")
    _native.check("es_dec_add_rmsnorm", _native.lib().es_dec_add_rmsnorm(
        h.data_ptr(), 0 if delta is None else delta.data_ptr(), w.data_ptr(), out.data_ptr(),
        rows, cols, ctypes.c_float(eps), _stream(h)))
    return out


GEMV_MAX_BATCH = 4


def gemv(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out = x @ w.T for x [B, K] (B <= 4), w [N, K], out [B, N], all bf16:
    one es_dec_gemv launch (weight-streaming, fp32 accumulation)."""
    B, K = x.shape
    N = w.shape[0]
    for t in (x, w, out):
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()):
            raise ValueError("gemv takes contiguous bf16 CUDA tensors")
    if w.shape[1] != K or out.shape != (B, N) or B > GEMV_MAX_BATCH:
        raise ValueError("gemv: shape mismatch or batch above 4")
    _native.check("es_dec_gemv", _native.lib().es_dec_gemv(
        w.data_ptr(), x.data_ptr(), out.data_ptr(), B, N, K, _stream(x)))
    return out


def qk_norm_rope_kv(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor,
                    cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor, q_out: torch.Tensor,
                    k_cache: torch.Tensor, v_cache: torch.Tensor, eps: float) -> torch.Tensor:
    """qkv [B, (H + 2 KV) * hd] -> q_out [B, H, hd] (normed, rotated); the
    normed, rotated k and the v of every sequence written into the caches
    [B, KV, max_ctx, hd] at position pos (a device int64 scalar tensor)."""
    B, H, hd = q_out.shape
    KV, max_ctx = k_cache.shape[1], k_cache.shape[2]
    if qkv.shape != (B, (H + 2 * KV) * hd) or v_cache.shape != k_cache.shape:
        raise ValueError("qk_norm_rope_kv: shape mismatch")
    if cos.shape != (max_ctx, hd // 2) or sin.shape != cos.shape or pos.dtype != torch.int64:
        raise ValueError("qk_norm_rope_kv: rotary tables must be [max_ctx, hd/2] f32")
    for t in (qkv, q_norm, k_norm, q_out, k_cache, v_cache, cos, sin, pos):
        if not (t.is_cuda and t.is_contiguous()):
            raise ValueError("qk_norm_rope_kv takes contiguous CUDA tensors")
    _native.check("es_dec_qk_norm_rope_kv", _native.lib().es_dec_qk_norm_rope_kv(
        qkv.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(), cos.data_ptr(), sin.data_ptr(),
        pos.data_ptr(), q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), B, H, KV, hd,
        max_ctx, ctypes.c_float(eps), _stream(qkv)))
    return q_out


class Decoder:
    """Batched decode: `batch` sequences, each with a `context`-token KV cache,
    one new token per sequence per step."""

    def __init__(self, dcfg: DecoderConfig, batch: int, context: int, max_steps: int = 64,
                 seed: int = 0, device="cuda", expert_seed: int = 1000, fused: bool = True):
        self.dcfg = dcfg
        self.fused = fused
        self.device = torch.device(device)
        self.batch = batch
        self.max_ctx = context + max_steps
        D, H, KV, hd, V = dcfg.hidden, dcfg.heads, dcfg.kv_heads, dcfg.head_dim, dcfg.vocab
        g = torch.Generator(device=self.device).manual_seed(seed)

        def rnd(*shape, std=0.02):
            return (torch.randn(shape, generator=g, device=self.device) * std).to(torch.bfloat16)

        self.embed = rnd(V, D)
        self.lm_head = rnd(V, D)
        self.final_norm = torch.ones(D, dtype=torch.bfloat16, device=self.device)
        self.layers = []
        mcfg = dcfg.moe
        self.ws = MoEBlock.new_workspace(mcfg, batch, self.device)
        for l in range(dcfg.layers):
            lay = synthetic_layer(mcfg, seed=expert_seed + l, device=self.device)
            sg = rnd(D) if mcfg.has_shared else None
            blk = MoEBlock(mcfg, packed=prepare_packed(mcfg, lay), shared_gate_w=sg,
                           max_tokens=batch, workspace=self.ws)
            del lay
            self.layers.append({
                "in_norm": torch.ones(D, dtype=torch.bfloat16, device=self.device),
                "post_norm": torch.ones(D, dtype=torch.bfloat16, device=self.device),
                # q, k and v projections stacked as one [(H + 2 KV) hd, D] matrix
                "qkv": torch.cat([rnd(H * hd, D), rnd(KV * hd, D), rnd(KV * hd, D)]),
                "o": rnd(D, H * hd),
                "q_norm": torch.ones(hd, dtype=torch.bfloat16, device=self.device),
                "k_norm": torch.ones(hd, dtype=torch.bfloat16, device=self.device),
                "router": rnd(mcfg.num_experts, D),
                "moe": blk,
                "k_cache": torch.zeros(batch, KV, self.max_ctx, hd, dtype=torch.bfloat16,
                                       device=self.device),
                "v_cache": torch.zeros(batch, KV, self.max_ctx, hd, dtype=torch.bfloat16,
                                       device=self.device),
            })
        # seeded N(0, 1) context in the caches
        for L in self.layers:
            L["k_cache"][:, :, :context] = torch.randn(
                (batch, KV, context, hd), generator=g, device=self.device).to(torch.bfloat16)
            L["v_cache"][:, :, :context] = torch.randn(
                (batch, KV, context, hd), generator=g, device=self.device).to(torch.bfloat16)
        self.cos, self.sin = rope_tables(hd, self.max_ctx, dcfg.rope_theta, self.device)
        self.pos = torch.full((1,), context, dtype=torch.long, device=self.device)
        self.ar = torch.arange(self.max_ctx, device=self.device)
        self.tokens = torch.zeros(batch, dtype=torch.long, device=self.device)
        self.logits = torch.empty(batch, V, dtype=torch.bfloat16, device=self.device)
        self.h = torch.empty(batch, D, dtype=torch.bfloat16, device=self.device)
        self.n = torch.empty(batch, D, dtype=torch.bfloat16, device=self.device)
        self.q = torch.empty(batch, H, hd, dtype=torch.bfloat16, device=self.device)
        # projection outputs of the fused step (weight-streaming GEMVs at batch <= 4)
        self.qkv_out = torch.empty(batch, (H + 2 * KV) * hd, dtype=torch.bfloat16,
                                   device=self.device)
        self.attn_out = torch.empty(batch, D, dtype=torch.bfloat16, device=self.device)
        self.router_out = torch.empty(batch, mcfg.num_experts, dtype=torch.bfloat16,
                                      device=self.device)
        self.cache_bias = [None] * dcfg.layers   # per-layer [E] routing bias, optional
        self.graph = None

    # -- one step, eager ----------------------------------------------------
    def _sdpa(self, L: dict, q: torch.Tensor, mask) -> torch.Tensor:
        B, H, hd = q.shape
        o = F.scaled_dot_product_attention(q.unsqueeze(2), L["k_cache"], L["v_cache"],
                                           attn_mask=mask, scale=1.0 / math.sqrt(hd),
                                           enable_gqa=True)
        return o.reshape(B, H * hd) @ L["o"].t()

    def _attention(self, L: dict, x: torch.Tensor, cos, sin, mask) -> torch.Tensor:
        c = self.dcfg
        B, H, KV, hd = self.batch, c.heads, c.kv_heads, c.head_dim
        w = L["qkv"]
        q = (x @ w[:H * hd].t()).view(B, H, hd)
        k = (x @ w[H * hd:(H + KV) * hd].t()).view(B, KV, hd)
        v = (x @ w[(H + KV) * hd:].t()).view(B, KV, hd)
        q = apply_rope(rms_norm(q, L["q_norm"], c.eps), cos, sin)
        k = apply_rope(rms_norm(k, L["k_norm"], c.eps), cos, sin)
        L["k_cache"].index_copy_(2, self.pos, k.unsqueeze(2))
        L["v_cache"].index_copy_(2, self.pos, v.unsqueeze(2))
        return self._sdpa(L, q, mask)

    def _mask(self):
        # positions <= pos are visible
        mask = torch.where(self.ar <= self.pos, 0.0, float("-inf")).to(torch.bfloat16)
        return mask.view(1, 1, 1, -1)

    def _step(self):
        if self.fused:
            return self._step_fused()
        c = self.dcfg
        h = self.embed.index_select(0, self.tokens)
        cos = self.cos.index_select(0, self.pos)   # [1, hd/2]
        sin = self.sin.index_select(0, self.pos)
        mask = self._mask()
        for i, L in enumerate(self.layers):
            h = h + self._attention(L, rms_norm(h, L["in_norm"], c.eps), cos, sin, mask)
            n = rms_norm(h, L["post_norm"], c.eps)
            logits = n @ L["router"].t()
            h = h + L["moe"].forward(n, logits, self.cache_bias[i])
        self.logits.copy_(rms_norm(h, self.final_norm, c.eps) @ self.lm_head.t())
        self.pos.add_(1)

    def _proj(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        # batch <= 4: weight-streaming GEMV; larger batches: cuBLAS
        if self.batch <= GEMV_MAX_BATCH:
            return gemv(x, w, out)
        return torch.matmul(x, w.t(), out=out)

    def _step_fused(self):
        c = self.dcfg
        h, n = self.h, self.n
        B, H, hd = self.batch, c.heads, c.head_dim
        torch.index_select(self.embed, 0, self.tokens, out=h)
        mask = self._mask()
        delta = None
        for i, L in enumerate(self.layers):
            add_rmsnorm_(h, delta, L["in_norm"], n, c.eps)
            qkv_proj = self._proj(n, L["qkv"], self.qkv_out)
            qk_norm_rope_kv(qkv_proj, L["q_norm"], L["k_norm"], self.cos, self.sin, self.pos,
                            self.q, L["k_cache"], L["v_cache"], c.eps)
            o = F.scaled_dot_product_attention(self.q.unsqueeze(2), L["k_cache"], L["v_cache"],
                                               attn_mask=mask, scale=1.0 / math.sqrt(hd),
                                               enable_gqa=True).reshape(B, H * hd)
            add_rmsnorm_(h, self._proj(o, L["o"], self.attn_out), L["post_norm"], n, c.eps)
            logits = self._proj(n, L["router"], self.router_out)
            delta = L["moe"].forward(n, logits, self.cache_bias[i])
        add_rmsnorm_(h, delta, self.final_norm, n, c.eps)
        torch.matmul(n, self.lm_head.t(), out=self.logits)
        self.pos.add_(1)

    # -- graph ----------------------------------------------------------------
    def capture(self):
        """Capture one decode step (all layers) as a CUDA graph; the position
        advances on the device at the end of every replay."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        p0 = self.pos.clone()
        with torch.cuda.stream(s):
            self._step()   # warm up (cuBLAS / SDPA workspaces) outside capture
            torch.cuda.synchronize()
            self.pos.copy_(p0)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self._step()
        torch.cuda.synchronize()
        self.pos.copy_(p0)
        self._stream = s
        return self

    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        """Feed one token per sequence; returns the next-token logits [B, V]."""
        self.tokens.copy_(tokens)
        if self.graph is None:
            self._step()
        else:
            with torch.cuda.stream(self._stream):
                self.graph.replay()
            torch.cuda.current_stream(self.device).wait_stream(self._stream)
        return self.logits


def distinct_experts(dec: "Decoder", tokens: torch.Tensor) -> list:
    """Distinct experts each layer's MoE block selects in one eager step
    (the step's position is restored afterwards)."""
    counts = []
    wrapped = []
    for L in dec.layers:
        blk = L["moe"]
        orig = blk.forward

        def rec(n, logits, bias=None, *a, _blk=blk, _orig=orig, **kw):
            idx, _ = _blk.route(logits, bias)
            counts.append(int(torch.unique(idx).numel()))
            return _orig(n, logits, bias, *a, **kw)
        blk.forward = rec
        wrapped.append(blk)
    p0 = dec.pos.clone()
    graph, dec.graph = dec.graph, None
    try:
        dec.step(tokens)
        torch.cuda.synchronize()
    finally:
        dec.graph = graph
        dec.pos.copy_(p0)
        for blk in wrapped:
            del blk.forward
    return counts


def step_bytes(dec: "Decoder", distinct: list) -> int:
    """Algorithmic HBM bytes of one decode step: every layer's attention,
    router and selected experts' weights, the KV cache read up to the
    position (plus the new row written), embedding rows, final norm and
    lm_head. `distinct` = distinct experts per layer."""
    c = dec.dcfg
    D, H, KV, hd, V = c.hidden, c.heads, c.kv_heads, c.head_dim, c.vocab
    B = dec.batch
    ctx = int(dec.pos.item())
    per_layer = ((H + 2 * KV) * hd * D + D * H * hd + c.moe.num_experts * D) * 2
    kv = B * KV * (ctx + 1) * hd * 2 * 2
    total = len(dec.layers) * (per_layer + kv)
    total += sum(distinct) * c.moe.bytes_per_expert
    total += V * D * 2 + B * D * 2
    return int(total)


def measure(batches=(1, 16), context: int = 2048, steps: int = 40, layers: int = 48,
            fused: bool = True) -> dict:
    """Decode tokens/s of the Qwen3-30B-shaped decoder: graph replays with
    greedy next tokens, timed with CUDA events after 3 warm-up steps."""
    dcfg = DecoderConfig(layers=layers)
    res = {}
    for B in batches:
        t0 = time.time()
        dec = Decoder(dcfg, B, context, max_steps=steps + 8, fused=fused).capture()
        build_s = time.time() - t0
        g = torch.Generator(device="cuda").manual_seed(B)
        toks = torch.randint(0, dcfg.vocab, (B,), generator=g, device="cuda")
        for _ in range(3):
            toks = dec.step(toks).argmax(-1)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            toks = dec.step(toks).argmax(-1)
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1) / steps
        U = distinct_experts(dec, toks)
        nbytes = step_bytes(dec, U)
        res[str(B)] = {"ms_per_step": ms, "tokens_per_s": B / (ms * 1e-3), "build_s": build_s,
                       "bytes_per_step": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9,
                       "mean_distinct_experts": sum(U) / len(U)}
        del dec
        torch.cuda.empty_cache()
    return {"decoder": dcfg.name, "layers": layers, "context": context, "steps": steps,
            "fused": fused, "results": res}


def _bench(argv=None):
    """Decode tokens/s of the 48-layer Qwen3-30B-shaped decoder (graph
    replays, CUDA events) at batch 1 and 16 with a 2048-token context."""
    import argparse
    import json
    ap = argparse.ArgumentParser(description="decoder decode throughput")
    ap.add_argument("--batches", default="1,16")
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--unfused", action="store_true",
                    help="torch ops around the block instead of the fused helper kernels")
    args = ap.parse_args(argv)
    print(json.dumps(measure([int(b) for b in args.batches.split(",")], args.context,
                             args.steps, args.layers, fused=not args.unfused)))


if __name__ == "__main__":
    _bench()
