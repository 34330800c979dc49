"""The fused tiny-batch kernel (es_small.cu, kernel_path "fused", the
automatic choice for T <= 16) against the CPU oracle, through the C ABI:
routing as in test_gpu_block.py, outputs within 3e-3 x RMS (the decode
kernels' arithmetic: exact 4-bit weights, fp16 h), bitwise-repeatable calls,
given routing with masked / duplicate / out-of-range ids, the shared expert,
every reference shape, and replay inside a CUDA graph."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig, PRESETS, _native
from expert_sniper_b200.block import ffn_kernels
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
from oracle import c_oracle as co
from oracle import moe_oracle as mo
from tests._helpers import (assert_bf16_close, assert_close_rms, layer_to_numpy,
                            oracle_weights_for)

pytestmark = pytest.mark.gpu

FUSED_REL = 3e-3
SMALL = MoEConfig(256, 16, 4, 256, True, name="small")
SHARED = MoEConfig(512, 32, 6, 512, True, shared_inter=512, name="small-shared")


def _check(cfg, T, bias, seed, dev):
    lay = synthetic_layer(cfg, seed=100 + seed, device=dev)
    x, _, logits, sg = synthetic_inputs(cfg, T, seed=seed, device=dev)
    cb = cache_bias_vector(cfg.num_experts, 0.5, seed)[0].to(dev) if bias else None
    blk = MoEBlock(cfg.with_(kernel_path="fused"), weights=lay, shared_gate_w=sg, max_tokens=T)
    assert ffn_kernels(blk.cfg, T) == "fused"
    out32, idx, w = blk.forward(x, logits, cb, out_dtype=torch.float32, return_routing=True)
    again = blk.forward(x, logits, cb, out_dtype=torch.float32)
    out16 = blk.forward(x, logits, cb)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    assert torch.equal(out32, again)
    lg = logits.float().cpu().numpy()
    cbn = None if cb is None else cb.cpu().numpy()
    idx_n = idx.cpu().numpy()
    ok, _, _, bad = mo.topk_parity(idx_n, lg, cbn, cfg.top_k)
    assert ok, bad
    w_ref = oracle_weights_for(idx_n, lg, cbn, cfg.norm_topk_prob)
    assert np.abs(w.cpu().numpy() - w_ref).max() <= 1e-5
    ref = co.expert_ffn(x.float().cpu().numpy(), layer_to_numpy(lay), idx_n, w_ref,
                        None if sg is None else sg.float().cpu().numpy())
    err, rms = assert_close_rms(out32.cpu().numpy(), ref, rel=FUSED_REL, what=f"{cfg.name} T={T}")
    assert_bf16_close(out16.float().cpu().numpy(), ref)
    return blk, x, logits, cb


@pytest.mark.parametrize("T", [1, 2, 3, 4, 5, 6, 7, 8, 9, 12, 16])
@pytest.mark.parametrize("bias", [False, True])
def test_fused_small(cuda, T, bias):
    _check(SMALL, T, bias, seed=T, dev=cuda)


@pytest.mark.parametrize("T", [1, 4, 8, 9, 16])
def test_fused_shared_expert(cuda, T):
    _check(SHARED, T, True, seed=10 + T, dev=cuda)


@pytest.mark.parametrize("name,T", [("olmoe-1b-7b", 2), ("qwen3-30b-a3b", 1),
                                    ("qwen3-30b-a3b", 4), ("qwen3-next-80b-a3b", 3),
                                    ("qwen3-235b-a22b", 4), ("qwen3-30b-a3b", 8),
                                    ("qwen3-next-80b-a3b", 6), ("qwen3-235b-a22b", 8),
                                    ("qwen3-30b-a3b", 16), ("olmoe-1b-7b", 13),
                                    ("qwen3-next-80b-a3b", 16), ("qwen3-235b-a22b", 16)])
def test_fused_reference_shapes(cuda, name, T):
    _check(PRESETS[name], T, name == "qwen3-30b-a3b", seed=20 + T, dev=cuda)


def test_fused_given_routing_masked_duplicate_out_of_range(cuda):
    cfg = SMALL.with_(kernel_path="fused")
    lay = synthetic_layer(cfg, seed=7, device=cuda)
    T = 4
    x, _, _, _ = synthetic_inputs(cfg, T, seed=11, device=cuda)
    g = np.random.default_rng(3)
    idx = np.stack([g.choice(cfg.num_experts, cfg.top_k, replace=False) for _ in range(T)]).astype(np.int32)
    idx[0, :] = -1                     # a token with nothing routed
    idx[1, 1] = -1
    idx[2, 2] = idx[2, 0]              # duplicate expert in one token
    idx[3, 3] = cfg.num_experts + 3    # out of range: flagged, skipped
    w = g.random((T, cfg.top_k)).astype(np.float32)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    out = blk.expert_ffn(x, torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                         out_dtype=torch.float32)
    assert blk.read_device_error() & _native.DEVERR_BAD_EXPERT_ID
    masked = idx.copy()
    masked[3, 3] = -1
    ref = mo.expert_ffn(x.float().cpu().numpy(), layer_to_numpy(lay), masked, w)
    assert_close_rms(out.cpu().numpy(), ref, rel=FUSED_REL, what="given routing")
    assert torch.count_nonzero(out[0]) == 0


@pytest.mark.parametrize("T", [2, 13])
def test_fused_f32_logits_match_decode_kernels(cuda, T):
    """fp32 router logits (the dtype biased MLX logits promote to) through
    the fused kernel: the same top-k and weights as the decode kernels, and
    outputs within the parity tolerance of them."""
    cfg = PRESETS["qwen3-30b-a3b"]
    lay = synthetic_layer(cfg, seed=61, device=cuda)
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=62, device=cuda)
    lg32 = logits.float() + 0.01 * torch.randn(logits.shape, device=cuda)
    cb = cache_bias_vector(cfg.num_experts, 0.5, 7)[0].to(cuda)
    fused = MoEBlock(cfg.with_(kernel_path="fused"), weights=lay, max_tokens=T)
    dec = MoEBlock(cfg.with_(kernel_path="decode"), packed=fused.packed, max_tokens=T)
    o1, i1, w1 = fused.forward(x, lg32, cb, out_dtype=torch.float32, return_routing=True)
    o2, i2, w2 = dec.forward(x, lg32, cb, out_dtype=torch.float32, return_routing=True)
    torch.cuda.synchronize()
    assert fused.read_device_error() == 0 and dec.read_device_error() == 0
    assert torch.equal(i1, i2) and torch.equal(w1, w2)
    assert_close_rms(o1.cpu().numpy(), o2.cpu().numpy(), rel=FUSED_REL, what=f"f32 logits T={T}")


def test_fused_reports_capacity_for_repeated_experts(cuda):
    """Given routing that repeats one expert 17 times across 8 tokens (a
    token listing it in several slots) cuts more expert entries than the
    partials hold at this shape: the call sets ES_DEVERR_CAPACITY and writes
    zeros instead of running past the workspace, and the next call on the
    same workspace is exact again."""
    cfg = MoEConfig(512, 16, 4, 512, True, name="dup", kernel_path="fused")
    lay = synthetic_layer(cfg, seed=71, device=cuda)
    T = 8
    x, _, _, _ = synthetic_inputs(cfg, T, seed=72, device=cuda)
    idx = np.zeros((T, cfg.top_k), dtype=np.int32)
    others = iter(range(1, 16))
    for t in range(4, T):
        for j in range(cfg.top_k):
            if not (t == 4 and j == 0):
                idx[t, j] = next(others)
    w = np.random.default_rng(5).random((T, cfg.top_k)).astype(np.float32)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    out = blk.expert_ffn(x, torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                         out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert blk.read_device_error(clear=True) & _native.DEVERR_CAPACITY
    assert torch.count_nonzero(out) == 0
    ok_idx = np.stack([np.random.default_rng(t).choice(16, 4, replace=False)
                       for t in range(T)]).astype(np.int32)
    out2 = blk.expert_ffn(x, torch.from_numpy(ok_idx).to(cuda), torch.from_numpy(w).to(cuda),
                          out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert blk.read_device_error() == 0
    ref = mo.expert_ffn(x.float().cpu().numpy(), layer_to_numpy(lay), ok_idx, w)
    assert_close_rms(out2.cpu().numpy(), ref, rel=FUSED_REL, what="after a capacity error")


@pytest.mark.parametrize("T", [8, 11, 16])
def test_fused_all_tokens_one_expert(cuda, T):
    """Every token routed to expert 0 (8 tokens fill the 8 columns of one
    expert entry; 11 and 16 take two entries) next to scattered slots,
    duplicates and masked ones."""
    cfg = SMALL.with_(kernel_path="fused")
    lay = synthetic_layer(cfg, seed=8, device=cuda)
    x, _, _, _ = synthetic_inputs(cfg, T, seed=12, device=cuda)
    g = np.random.default_rng(4)
    idx = np.stack([g.choice(np.arange(1, cfg.num_experts), cfg.top_k, replace=False)
                    for _ in range(T)]).astype(np.int32)
    idx[:, 0] = 0
    idx[5, 2] = idx[5, 1]
    idx[6, 3] = -1
    w = g.random((T, cfg.top_k)).astype(np.float32)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    assert ffn_kernels(blk.cfg, T) == "fused"
    out = blk.expert_ffn(x, torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                         out_dtype=torch.float32)
    assert blk.read_device_error() == 0
    ref = mo.expert_ffn(x.float().cpu().numpy(), layer_to_numpy(lay), idx, w)
    assert_close_rms(out.cpu().numpy(), ref, rel=FUSED_REL, what="8 tokens on one expert")


def test_one_workspace_across_batch_sizes(cuda):
    """Calls of different T on one workspace: a 64-token call (decode
    kernels) leaves every region the small-batch kernels count in at zero,
    so fused and split-K decode calls after it match fresh blocks bitwise."""
    cfg = PRESETS["qwen3-30b-a3b"]
    lay = synthetic_layer(cfg, seed=31, device=cuda)
    packed = MoEBlock(cfg, weights=lay, max_tokens=1).packed
    ws = MoEBlock.new_workspace(cfg, 64, cuda)
    for T, path in [(64, "auto"), (1, "auto"), (8, "fused"), (64, "auto"), (3, "decode"),
                    (16, "auto"), (4, "auto"), (12, "decode"), (2, "fused")]:
        x, _, logits, _ = synthetic_inputs(cfg, T, seed=50 + T, device=cuda)
        big = MoEBlock(cfg.with_(kernel_path=path), packed=packed, max_tokens=64, workspace=ws)
        got = big.forward(x, logits, None, out_dtype=torch.float32)
        fresh = MoEBlock(cfg.with_(kernel_path=path), packed=packed, max_tokens=T)
        want = fresh.forward(x, logits, None, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert big.read_device_error() == 0 and fresh.read_device_error() == 0, (T, path)
        assert torch.equal(got, want), (T, path)


def test_fused_in_cuda_graph(cuda):
    blk, x, logits, cb = _check(PRESETS["qwen3-30b-a3b"], 1, True, seed=40, dev=cuda)
    xs, ls = x.clone(), logits.clone()
    out = torch.empty((1, blk.cfg.hidden), dtype=torch.float32, device=cuda)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        blk.forward(xs, ls, cb, out=out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            blk.forward(xs, ls, cb, out=out)
    torch.cuda.synchronize()
    for seed in (41, 42, 41):
        x2, _, l2, _ = synthetic_inputs(blk.cfg, 1, seed=seed, device=cuda)
        xs.copy_(x2)
        ls.copy_(l2)
        g.replay()
        torch.cuda.synchronize()
        want = blk.forward(x2, l2, cb, out_dtype=torch.float32)
        assert torch.equal(out, want)
    assert blk.read_device_error() == 0
    del g
