"""The decoder's helper kernels (es_dec_add_rmsnorm, es_dec_qk_norm_rope_kv,
es_dec_gemv) against the torch ops they replace: bf16 results
within one bf16 ulp (the fp32 sums are reduced in another order, which can
move a rounding by one step), the residual update and the v copy bit-exact,
cache rows other than the written position untouched."""
from __future__ import annotations

import pytest
import torch

from expert_sniper_b200.decoder import (add_rmsnorm_, apply_rope, gemv, qk_norm_rope_kv, rms_norm,
                                        rope_tables)

pytestmark = pytest.mark.gpu

ULP = 2.0 ** -7   # bf16: 8 significant bits


def _within_ulp(got, want):
    g, w = got.float(), want.float()
    return bool(((g - w).abs() <= w.abs() * ULP + 1e-30).all())


@pytest.mark.parametrize("rows,cols", [(1, 2048), (5, 256), (64, 2048), (3, 1000), (2, 4096),
                                       (16, 2048), (4, 8192), (2, 9000), (1, 24)])
@pytest.mark.parametrize("with_delta", [True, False])
def test_add_rmsnorm(cuda, rows, cols, with_delta):
    g = torch.Generator(device=cuda).manual_seed(rows * cols)
    h = torch.randn(rows, cols, generator=g, device=cuda).to(torch.bfloat16)
    d = torch.randn(rows, cols, generator=g, device=cuda).to(torch.bfloat16) if with_delta else None
    w = (1 + 0.1 * torch.randn(cols, generator=g, device=cuda)).to(torch.bfloat16)
    h_ref = h + d if with_delta else h.clone()
    out_ref = rms_norm(h_ref, w, 1e-6)
    out = torch.empty_like(h)
    add_rmsnorm_(h, d, w, out, 1e-6)
    assert torch.equal(h, h_ref)
    assert _within_ulp(out, out_ref)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("pos", [0, 7, 11])
def test_qk_norm_rope_kv(cuda, hd, pos):
    B, H, KV, max_ctx = 3, 8, 2, 12
    g = torch.Generator(device=cuda).manual_seed(hd + pos)
    qkv = torch.randn(B, (H + 2 * KV) * hd, generator=g, device=cuda).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(hd, generator=g, device=cuda)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(hd, generator=g, device=cuda)).to(torch.bfloat16)
    cos, sin = rope_tables(hd, max_ctx, 1e6, cuda)
    kc = torch.full((B, KV, max_ctx, hd), 7.0, dtype=torch.bfloat16, device=cuda)
    vc = torch.full_like(kc, -7.0)
    q = torch.empty(B, H, hd, dtype=torch.bfloat16, device=cuda)
    p = torch.tensor(pos, dtype=torch.int64, device=cuda)
    qk_norm_rope_kv(qkv, qn, kn, cos, sin, p, q, kc, vc, 1e-6)

    q_in, k_in, v_in = qkv.view(B, H + 2 * KV, hd).split([H, KV, KV], 1)
    q_ref = apply_rope(rms_norm(q_in, qn, 1e-6), cos[pos], sin[pos])
    k_ref = apply_rope(rms_norm(k_in, kn, 1e-6), cos[pos], sin[pos])
    assert _within_ulp(q, q_ref)
    assert _within_ulp(kc[:, :, pos], k_ref)
    assert torch.equal(vc[:, :, pos], v_in)
    others = [i for i in range(max_ctx) if i != pos]
    assert bool((kc[:, :, others] == 7.0).all()) and bool((vc[:, :, others] == -7.0).all())


def test_position_outside_cache_writes_nothing(cuda):
    B, H, KV, hd, max_ctx = 2, 4, 2, 64, 8
    qkv = torch.randn(B, (H + 2 * KV) * hd, device=cuda).to(torch.bfloat16)
    ones = torch.ones(hd, dtype=torch.bfloat16, device=cuda)
    cos, sin = rope_tables(hd, max_ctx, 1e6, cuda)
    kc = torch.zeros(B, KV, max_ctx, hd, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    q = torch.full((B, H, hd), 3.0, dtype=torch.bfloat16, device=cuda)
    p = torch.tensor(max_ctx, dtype=torch.int64, device=cuda)
    qk_norm_rope_kv(qkv, ones, ones, cos, sin, p, q, kc, vc, 1e-6)
    torch.cuda.synchronize()
    assert not kc.any() and not vc.any() and bool((q == 3.0).all())


@pytest.mark.parametrize("B", [1, 2, 3, 4])
@pytest.mark.parametrize("N,K", [(5120, 2048), (2048, 4096), (128, 2048), (37, 264)])
def test_gemv(cuda, B, N, K):
    """x @ W^T against an fp32 product of the same bf16 values: the kernel
    accumulates in fp32 and rounds once to bf16, so the error is within one
    bf16 ulp of each output plus summation-order noise."""
    g = torch.Generator(device=cuda).manual_seed(B * N + K)
    w = (torch.randn(N, K, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(B, K, generator=g, device=cuda).to(torch.bfloat16)
    out = torch.empty(B, N, dtype=torch.bfloat16, device=cuda)
    gemv(x, w, out)
    ref = x.float() @ w.float().t()
    rms = float(ref.pow(2).mean().sqrt())
    assert bool(((out.float() - ref).abs() <= ref.abs() * ULP + 1e-3 * rms).all())
