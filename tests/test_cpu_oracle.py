"""The oracle itself: format, router semantics, parity classifier, FFN."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from expert_sniper_b200 import quant
from expert_sniper_b200.config import MoEConfig
from oracle import c_oracle as co
from oracle import moe_oracle as mo
from tests._helpers import layer_to_numpy


def test_pack_unpack_roundtrip():
    g = torch.Generator().manual_seed(0)
    w = (torch.randn((5, 3, 128), generator=g) * 0.02).half()
    q, s, b = quant.quantize_affine(w)
    assert q.shape == (5, 3, 16) and s.shape == (5, 3, 2) and s.dtype == torch.float16
    codes = quant.unpack_codes(q)
    assert int(codes.max()) <= 15
    # numpy unpack agrees with torch unpack, bit for bit
    assert np.array_equal(mo.unpack_codes(q.numpy()), codes.numpy())
    deq = mo.dequant(q.numpy(), s.numpy(), b.numpy())
    assert np.array_equal(deq, quant.dequantize_affine(q, s, b).numpy())
    # an affine 4-bit quantiser is within half a step of the input
    step = s.float().numpy().repeat(64, axis=-1)
    assert (np.abs(deq - w.float().numpy()) <= 0.5 * step + 1e-3).all()


def test_code_layout_is_low_nibble_first():
    # word 0x76543210: column k holds k
    words = np.array([[0x76543210]], dtype=np.uint32)
    assert mo.unpack_codes(words).tolist() == [[0, 1, 2, 3, 4, 5, 6, 7]]


def test_bf16_rounding_helpers():
    a = np.array([1.0, 1.00390625, 1.005859375, -3.0, 0.0], np.float32)
    r = mo.round_bf16(a)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even
    assert r[2] == np.float32(1.0078125)
    assert (np.abs(r - a) <= mo.bf16_half_ulp(a)).all()


def test_route_semantics():
    rng = np.random.default_rng(0)
    lg = rng.standard_normal((20, 64)).astype(np.float32)
    idx, w, probs = mo.route(lg, None, 8, renorm=False)
    assert np.allclose(probs.sum(-1), 1.0, atol=1e-6)
    assert (np.diff(w, axis=1) <= 0).all()                    # descending
    assert np.allclose(np.sort(lg, -1)[:, ::-1][:, :8], np.take_along_axis(lg, idx, -1))
    _, wr, _ = mo.route(lg, None, 8, renorm=True)
    assert np.allclose(wr.sum(-1), 1.0, atol=1e-6)
    # the bias moves selection AND weights (softmax of the biased logits)
    bias = np.zeros(64, np.float32)
    bias[[1, 2, 3]] = 5.0
    ib, wb, _ = mo.route(lg, bias, 8, renorm=True)
    assert all({1, 2, 3} <= set(r) for r in ib.tolist())
    # ties go to the lower id
    tie = np.zeros((1, 8), np.float32)
    it, _, _ = mo.route(tie, None, 3, False)
    assert it.tolist() == [[0, 1, 2]]


def test_c_oracle_matches_numpy_oracle():
    cfg = MoEConfig(256, 16, 4, 256, True, shared_inter=256)
    lay = layer_to_numpy(quant.synthetic_layer(cfg, seed=1))
    x, _, logits, sg = quant.synthetic_inputs(cfg, 9, seed=2)
    xf, lf = x.float().numpy(), logits.float().numpy()
    for bias in (None, quant.cache_bias_vector(16, 0.5, 3)[0].numpy()):
        i1, w1, _ = mo.route(lf, bias, 4, True)
        i2, w2 = co.route(lf, bias, 4, True)
        assert np.array_equal(i1, i2) and np.abs(w1 - w2).max() < 1e-6
    o1 = mo.expert_ffn(xf, lay, i1, w1, sg.float().numpy())
    o2 = co.expert_ffn(xf, lay, i1, w1, sg.float().numpy())
    rms = np.sqrt((o1 ** 2).mean())
    assert np.abs(o1 - o2).max() < 1e-4 * rms


def test_expert_ffn_matches_dense_per_token_loop():
    """engine.py:15-42 restated literally: per token, per slot, three dense
    products with dequantised weights."""
    cfg = MoEConfig(256, 8, 2, 256, False)
    lay = layer_to_numpy(quant.synthetic_layer(cfg, seed=4))
    x, _, logits, _ = quant.synthetic_inputs(cfg, 3, seed=5)
    xf = x.float().numpy()
    idx, w, _ = mo.route(logits.float().numpy(), None, 2, False)
    out = mo.expert_ffn(xf, lay, idx, w)

    def deq(proj, e):
        return mo.dequant(lay[f"switch_mlp.{proj}.weight"][e], lay[f"switch_mlp.{proj}.scales"][e],
                          lay[f"switch_mlp.{proj}.biases"][e])
    want = np.zeros_like(out)
    for t in range(3):
        for j in range(2):
            e = idx[t, j]
            g = deq("gate_proj", e) @ xf[t]
            u = deq("up_proj", e) @ xf[t]
            h = g / (1 + np.exp(-g)) * u
            want[t] += w[t, j] * (deq("down_proj", e) @ h)
    assert np.abs(out - want).max() < 1e-5 * np.sqrt((want ** 2).mean()) + 1e-9


def test_partial_and_node_order_combine():
    """compute_partial masking + reader.py fixed-order fp32 sum == full."""
    cfg = MoEConfig(256, 8, 3, 256, True)
    lay = layer_to_numpy(quant.synthetic_layer(cfg, seed=6))
    x, _, logits, _ = quant.synthetic_inputs(cfg, 4, seed=7)
    xf = x.float().numpy()
    idx, w, _ = mo.route(logits.float().numpy(), None, 3, True)
    full = mo.expert_ffn(xf, lay, idx, w)
    parts = [mo.partial(xf, lay, idx, w, p) for p in ([0, 1, 2], [3, 4], [5, 6, 7])]
    tot = mo.combine_nodes(parts)
    assert np.abs(tot - full).max() < 1e-5 * np.sqrt((full ** 2).mean())


def test_topk_parity_classifier():
    """Planted mistakes are caught; a tie flip in the reference dtype is not."""
    lg = np.array([[3.0, 2.0, 1.0, 0.0, -1.0]], np.float32)
    ok, n_exact, _, _ = mo.topk_parity(np.array([[0, 1]]), lg, None, 2)
    assert ok and n_exact == 1
    ok, _, _, bad = mo.topk_parity(np.array([[0, 2]]), lg, None, 2)   # wrong expert
    assert not ok and bad == [0]
    ok, _, _, bad = mo.topk_parity(np.array([[0, 0]]), lg, None, 2)   # duplicate
    assert not ok
    ok, _, _, bad = mo.topk_parity(np.array([[0, 9]]), lg, None, 2)   # out of range
    assert not ok
    # near-tie: logits 1e-6 apart at the boundary -> either choice accepted
    lt = np.array([[3.0, 2.0, 2.0 - 1e-6, 0.0]], np.float32)
    ok, _, n_tie, _ = mo.topk_parity(np.array([[0, 2]]), lt, None, 2)
    assert ok and n_tie == 1
    # bf16-probability tie (unbiased reference keys are bf16): logits 1e-3
    # apart round to the same bf16 probability
    lb = np.array([[0.0, 0.001, -5.0, -5.0]], np.float32)
    keys = mo.reference_selection_keys(lb, None)
    assert keys[0, 0] == keys[0, 1]
    ok, _, n_tie, _ = mo.topk_parity(np.array([[1]]), lb, None, 1)
    assert ok and n_tie == 1
    # with a bias the keys are fp32, so the same gap is NOT a tie
    ok, _, _, _ = mo.topk_parity(np.array([[0]]), lb, np.zeros(4, np.float32), 1)
    assert not ok


@pytest.mark.parametrize("frac", [0.25])
def test_cache_bias_vector_matches_reference_rule(frac):
    m, ids = quant.cache_bias_vector(128, 0.5, 42, frac)
    assert len(ids) == 32 and float(m.sum()) == pytest.approx(16.0)
    want = sorted(np.random.default_rng(42).choice(128, 32, replace=False).tolist())
    assert ids == want
