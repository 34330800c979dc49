"""The device-resident routing-bias table reproduces the reference's
per-layer host mask (generate.py:124-129): `bias` at the cached expert ids,
0 elsewhere, None when bias <= 0 (CPU tensors here; the CUDA path is the
same code with a side-stream copy)."""
from __future__ import annotations

import numpy as np
import pytest

from expert_sniper_b200.bias_table import CacheBiasTable


def _ref_mask(E, ids, bias):
    m = np.zeros(E, np.float32)
    if ids:
        m[list(ids)] = bias
    return m


def test_rows_match_reference_mask():
    pytest.importorskip("torch")
    t = CacheBiasTable(3, 16, 0.5, device="cpu")
    t.set_cached(0, [1, 5, 9])
    t.set_cached(2, [])
    t.set_cached(1, {15, 0})
    assert np.array_equal(t.row(0).numpy(), _ref_mask(16, [1, 5, 9], 0.5))
    assert np.array_equal(t.row(1).numpy(), _ref_mask(16, [0, 15], 0.5))
    assert not t.row(2).numpy().any()
    t.set_cached(0, [2])  # the cached set changes: the row is replaced
    assert np.array_equal(t.row(0).numpy(), _ref_mask(16, [2], 0.5))


def test_no_bias_means_no_mask():
    t = CacheBiasTable(2, 8, 0.0, device="cpu")
    t.set_cached(0, [1])
    assert t.row(0) is None


def test_out_of_range_rejected():
    t = CacheBiasTable(1, 8, 0.5, device="cpu")
    with pytest.raises(ValueError):
        t.set_cached(0, [8])
