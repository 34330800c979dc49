"""torch.ops.expert_sniper.moe_forward / moe_forward_out (ops.py) against the
C ABI's es_moe_forward called directly: bitwise equal, eagerly and inside a
captured CUDA graph. The operator stands where the reference calls
run_expert_ffn from make_forward (engine.py:15, generate.py:170)."""
from __future__ import annotations

import ctypes

import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig, PRESETS, _native
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer

pytestmark = pytest.mark.gpu


def _direct(blk, x, logits, bias, out_dtype):
    T = x.shape[0]
    out = torch.empty((T, blk.cfg.hidden), dtype=out_dtype, device=x.device)
    idx = torch.empty((T, blk.cfg.top_k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, blk.cfg.top_k), dtype=torch.float32, device=x.device)
    code = {torch.bfloat16: 0, torch.float32: 2}
    _native.check("es_moe_forward", _native.lib().es_moe_forward(
        ctypes.byref(blk.ccfg), x.data_ptr(), logits.data_ptr(), code[logits.dtype],
        0 if bias is None else bias.data_ptr(),
        0 if blk.shared_gate_w is None else blk.shared_gate_w.data_ptr(),
        blk.packed.data_ptr(), out.data_ptr(), code[out_dtype], idx.data_ptr(), w.data_ptr(), T,
        blk.workspace.data_ptr(), blk.workspace.numel(),
        torch.cuda.current_stream().cuda_stream))
    return out, idx, w


@pytest.mark.parametrize("name,T", [("qwen3-30b-a3b", 8), ("qwen3-30b-a3b", 64),
                                    ("small-shared", 100)])
def test_op_matches_c_abi_bitwise(cuda, name, T):
    cfg = (PRESETS[name] if name in PRESETS
           else MoEConfig(512, 32, 6, 512, True, shared_inter=512, name=name))
    lay = synthetic_layer(cfg, seed=7, device=cuda)
    x, _, logits, sg = synthetic_inputs(cfg, T, seed=8, device=cuda)
    bias = cache_bias_vector(cfg.num_experts, 0.5, 1)[0].to(cuda)
    blk = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=T)
    ref = _direct(blk, x, logits, bias, torch.float32)
    got = torch.ops.expert_sniper.moe_forward(
        x, logits, bias, blk.packed, blk.shared_gate_w, None, cfg.num_experts, cfg.top_k,
        cfg.inter, cfg.norm_topk_prob, cfg.shared_inter, 0, 2)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    # MoEBlock.forward goes through moe_forward_out
    o, i, w = blk.forward(x, logits, bias, out_dtype=torch.float32, return_routing=True)
    assert torch.equal(o, ref[0]) and torch.equal(i, ref[1]) and torch.equal(w, ref[2])
    assert blk.read_device_error() == 0


def test_op_in_cuda_graph(cuda):
    cfg = PRESETS["qwen3-30b-a3b"]
    T = 16
    lay = synthetic_layer(cfg, seed=9, device=cuda)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=10, device=cuda)
    x2, _, logits2, _ = synthetic_inputs(cfg, T, seed=11, device=cuda)
    bias = cache_bias_vector(cfg.num_experts, 0.5, 2)[0].to(cuda)
    xs, ls = x.clone(), logits.clone()
    out = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=cuda)
    idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device=cuda)
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device=cuda)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        args = (xs, ls, bias, blk.packed, None, blk.workspace, out, idx, w, cfg.num_experts,
                cfg.top_k, cfg.inter, cfg.norm_topk_prob, 0, 0)
        torch.ops.expert_sniper.moe_forward_out(*args)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            torch.ops.expert_sniper.moe_forward_out(*args)
    torch.cuda.synchronize()
    for xi, li in ((x, logits), (x2, logits2), (x, logits)):
        xs.copy_(xi)
        ls.copy_(li)
        g.replay()
        torch.cuda.synchronize()
        ref = _direct(blk, xi, li, bias, torch.bfloat16)
        assert torch.equal(out, ref[0]) and torch.equal(idx, ref[1]) and torch.equal(w, ref[2])
    del g


def test_run_expert_ffn_pool_reuses_packed_experts(cuda):
    """The run_expert_ffn drop-in repacks an expert once: a second call with
    the same tensors adds no slot, and ids outside the dict map to the first
    active expert (the reference's id_to_local.get(v, 0))."""
    import numpy as np
    from expert_sniper_b200 import run_expert_ffn
    from expert_sniper_b200.block import expert_pool
    from oracle import moe_oracle as mo
    from tests._helpers import assert_bf16_close, layer_to_numpy
    cfg = MoEConfig(256, 16, 4, 256, True, name="pool")
    lay = synthetic_layer(cfg, seed=12, device=cuda)
    lay_np = layer_to_numpy(lay)
    T = 6
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=13, device=cuda)
    idx, w, _ = mo.route(logits.float().cpu().numpy(), None, cfg.top_k, True)
    active = sorted(set(int(e) for e in idx.ravel()))
    expert_data = {e: {n: t[e] for n, t in lay.items()} for e in active}
    pool = expert_pool(cfg.hidden, cfg.inter, cuda)
    pool.clear()
    a = run_expert_ffn(x, expert_data, torch.from_numpy(idx).to(cuda),
                       torch.from_numpy(w).to(cuda))
    n = len(pool.slots)
    assert n == len(active)
    b = run_expert_ffn(x, expert_data, torch.from_numpy(idx).to(cuda),
                       torch.from_numpy(w).to(cuda))
    assert len(pool.slots) == n and torch.equal(a, b)
    assert_bf16_close(a.float().cpu().numpy(), mo.expert_ffn(x.float().cpu().numpy(), lay_np,
                                                             idx, w), what="pool")
    odd = idx.copy()
    odd[0, 0] = 99                     # not in expert_data: the first active expert
    c = run_expert_ffn(x, expert_data, torch.from_numpy(odd).to(cuda),
                       torch.from_numpy(w).to(cuda))
    sub = idx.copy()
    sub[0, 0] = active[0]
    ref = mo.expert_ffn(x.float().cpu().numpy(), lay_np, sub, w)
    assert_bf16_close(c.float().cpu().numpy(), ref, what="unknown id")
