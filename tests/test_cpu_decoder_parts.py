"""The decoder's building blocks on the CPU: RMS norm, the rotary tables
and the half-split rotation against their defining formulas (the decoder
itself runs on the GPU; tests/test_gpu_decoder.py compares whole steps)."""
from __future__ import annotations

import numpy as np
import torch

from expert_sniper_b200.decoder import apply_rope, rms_norm, rope_tables


def test_rms_norm_formula():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 64, generator=g)
    w = torch.randn(64, generator=g)
    got = rms_norm(x, w, 1e-6)
    want = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6) * w
    assert torch.allclose(got, want, rtol=1e-5, atol=1e-6)


def test_rope_rotation_is_complex_multiplication():
    hd, pos, theta = 16, 37, 1e6
    cos, sin = rope_tables(hd, 64, theta, "cpu")
    x = torch.randn(2, 4, hd, dtype=torch.float64).float()
    got = apply_rope(x, cos[pos], sin[pos]).double().numpy()
    h = hd // 2
    z = x[..., :h].double().numpy() + 1j * x[..., h:].double().numpy()
    ang = np.array([pos * theta ** (-2 * i / hd) for i in range(h)])
    r = z * np.exp(1j * ang)
    want = np.concatenate([r.real, r.imag], -1)
    assert np.allclose(got, want, atol=1e-5)


def test_rope_preserves_norm_and_position_zero_is_identity():
    cos, sin = rope_tables(8, 4, 1e4, "cpu")
    x = torch.randn(5, 8)
    assert torch.allclose(apply_rope(x, cos[0], sin[0]), x)
    y = apply_rope(x, cos[3], sin[3])
    assert torch.allclose(y.norm(dim=-1), x.norm(dim=-1), rtol=1e-5)
