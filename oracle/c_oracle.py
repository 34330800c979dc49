"""ctypes wrapper of oracle/liboracle.so (the C restatement in moe_oracle.c).

TEST INFRASTRUCTURE ONLY (see moe_oracle.py). Same inputs and outputs as
moe_oracle.route / moe_oracle.expert_ffn, with numpy arrays.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
_lib = None


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "moe_oracle.c")
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-B", "-C", HERE, "liboracle.so"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        _lib = ctypes.CDLL(LIB)
        _lib.oracle_route.restype = ctypes.c_int
        _lib.oracle_expert_ffn.restype = ctypes.c_int
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def route(logits: np.ndarray, cache_bias, k: int, renorm: bool):
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = lg.shape
    b = None if cache_bias is None else np.ascontiguousarray(cache_bias, dtype=np.float32)
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    rc = lib().oracle_route(_p(lg), _p(b), T, E, k, int(renorm), _p(idx), _p(w))
    if rc:
        raise RuntimeError(f"oracle_route failed ({rc})")
    return idx, w


def _mlx(layer, prefix, proj):
    out = []
    for kind, dt in (("weight", np.uint32), ("scales", np.uint16), ("biases", np.uint16)):
        a = np.asarray(layer[f"{prefix}.{proj}.{kind}"])
        out.append(np.ascontiguousarray(a).view(dt))
    return out


def expert_ffn(x: np.ndarray, layer: dict, idx: np.ndarray, w: np.ndarray,
               shared_gate_w=None, nthreads: int = 0) -> np.ndarray:
    """x [T, D] fp32, layer: numpy arrays named like the reference's tensors
    (scales/biases as float16 or uint16 bits). Returns fp32 [T, D]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, D = x.shape
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    k = idx.shape[1]
    gw = _mlx(layer, "switch_mlp", "gate_proj")
    uw = _mlx(layer, "switch_mlp", "up_proj")
    dw = _mlx(layer, "switch_mlp", "down_proj")
    E, I = gw[0].shape[0], gw[0].shape[1]
    sh = [None] * 9
    if "shared_expert.gate_proj.weight" in layer:
        sh = (_mlx(layer, "shared_expert", "gate_proj") + _mlx(layer, "shared_expert", "up_proj")
              + _mlx(layer, "shared_expert", "down_proj"))
    sgw = None if shared_gate_w is None else np.ascontiguousarray(shared_gate_w, dtype=np.float32)
    out = np.empty((T, D), np.float32)
    args = [_p(a) for a in gw + uw + dw] + [_p(a) for a in sh]
    rc = lib().oracle_expert_ffn(_p(x), T, D, I, E, k, *args, _p(sgw), _p(idx), _p(w), _p(out),
                                 int(nthreads))
    if rc:
        raise RuntimeError(f"oracle_expert_ffn failed ({rc})")
    return out
