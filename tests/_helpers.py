"""Shared helpers for the parity tests (test side only)."""
from __future__ import annotations

import numpy as np

from oracle import moe_oracle as mo

# Output tolerance of the parity bar: max |ours - oracle| <= REL_TOL * RMS(oracle)
# on fp32 outputs (the kernels accumulate in fp32). A bf16 output may move by a
# further half bf16 ulp of the value from its own final rounding.
REL_TOL = 1e-2


def layer_to_numpy(layer: dict) -> dict:
    out = {}
    for k, v in layer.items():
        a = v.detach().cpu().numpy()
        out[k] = a
    return out


def assert_close_rms(ours: np.ndarray, ref: np.ndarray, rel: float = REL_TOL, what: str = ""):
    ours = np.asarray(ours, np.float32)
    ref = np.asarray(ref, np.float32)
    assert ours.shape == ref.shape, (ours.shape, ref.shape)
    assert np.isfinite(ours).all(), f"{what}: non-finite output"
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    err = float(np.max(np.abs(ours - ref))) if ref.size else 0.0
    assert err <= rel * rms, f"{what}: max|diff|={err:.3e} > {rel} * rms {rms:.3e}"
    return err, rms


def assert_bf16_close(ours_bf16_as_f32: np.ndarray, ref: np.ndarray, rel: float = REL_TOL,
                      what: str = ""):
    ours = np.asarray(ours_bf16_as_f32, np.float32)
    ref = np.asarray(ref, np.float32)
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    tol = rel * rms + mo.bf16_half_ulp(ref)
    diff = np.abs(ours - ref)
    assert (diff <= tol).all(), f"{what}: max excess {float(np.max(diff - tol)):.3e}"


def oracle_weights_for(idx: np.ndarray, logits: np.ndarray, cache_bias, renorm: bool) -> np.ndarray:
    """Oracle routing weights of the experts WE selected (so a legitimate tie
    flip does not pollute the output comparison)."""
    z = logits.astype(np.float32)
    if cache_bias is not None:
        z = z + np.asarray(cache_bias, np.float32)[None]
    probs = mo.softmax_f32(z)
    w = np.take_along_axis(probs, idx.astype(np.int64), axis=-1)
    if renorm:
        w = w / w.sum(-1, keepdims=True)
    return w.astype(np.float32)
