"""ctypes binding of libes_moe.so (include/es_moe.h).

There is no fallback: if the library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import re

from .config import CMoECfg

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libes_moe.so")
HEADER = os.path.join(os.path.dirname(PKG_DIR), "include", "es_moe.h")

ES_OK = 0
ES_DTYPE_BF16, ES_DTYPE_F16, ES_DTYPE_F32 = 0, 1, 2
DEVERR_BAD_EXPERT_ID = 0x1
DEVERR_NONFINITE_LOGIT = 0x2
DEVERR_CAPACITY = 0x4
DEVERR_TIMEOUT = 0x8
DEVERR_RANGE = 0x10


class EsError(RuntimeError):
    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: {msg} (status {status})")
        self.status = status


class CMlxProj(ctypes.Structure):
    _fields_ = [("weight", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("biases", ctypes.c_void_p)]


class CMlxLayer(ctypes.Structure):
    _fields_ = [("gate", CMlxProj), ("up", CMlxProj), ("down", CMlxProj),
                ("shared_gate_proj", CMlxProj), ("shared_up_proj", CMlxProj),
                ("shared_down_proj", CMlxProj)]


class CEpPlan(ctypes.Structure):
    """Mirror of `es_ep_plan` in include/es_moe.h."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("cap", ctypes.c_int32),
                ("hidden", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("num_experts", ctypes.c_int32), ("owner", ctypes.c_void_p),
                ("local_id", ctypes.c_void_p), ("peers", ctypes.c_void_p),
                ("window", ctypes.c_void_p), ("err", ctypes.c_void_p)]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t
_CFG = ctypes.POINTER(CMoECfg)

_SIGNATURES = {
    "es_status_str": (ctypes.c_char_p, [ctypes.c_int]),
    "es_version": (_I32, []),
    "es_moe_packed_bytes": (ctypes.c_int, [_CFG, ctypes.POINTER(_SZ)]),
    "es_moe_prepare": (ctypes.c_int, [_CFG, ctypes.POINTER(CMlxLayer), _P, _SZ, _P]),
    "es_moe_prepare_blocks": (ctypes.c_int, [_CFG, _P, _SZ, ctypes.POINTER(ctypes.c_int64),
                                             ctypes.POINTER(CMlxLayer), _P, _SZ, _P]),
    "es_moe_workspace_bytes": (ctypes.c_int, [_CFG, _I32, ctypes.POINTER(_SZ)]),
    "es_moe_route": (ctypes.c_int, [_CFG, _P, _I32, _P, _I32, _P, _P, _P]),
    "es_moe_expert_ffn": (ctypes.c_int, [_CFG, _P, _P, _P, _P, _P, _P, _I32, _I32, _P, _SZ, _P]),
    "es_moe_forward": (ctypes.c_int, [_CFG, _P, _P, _I32, _P, _P, _P, _P, _I32, _P, _P, _I32,
                                      _P, _SZ, _P]),
    "es_moe_forward_timed": (ctypes.c_int, [_CFG, _P, _P, _I32, _P, _P, _P, _P, _I32, _P, _P,
                                            _I32, _P, _SZ, _P, _P, _I32]),
    "es_ep_mask": (ctypes.c_int, [_P, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P, _P, _P]),
    "es_ep_combine": (ctypes.c_int, [_P, _P, _I32, _I32, _I32, _P, _I32, _P]),
    "es_ep_window_bytes": (ctypes.c_int, [_I32, _I32, _I32, _I32, ctypes.POINTER(_SZ)]),
    "es_ep_window_alloc": (ctypes.c_int, [_SZ, ctypes.POINTER(_P), _P]),
    "es_ep_window_open": (ctypes.c_int, [_P, ctypes.POINTER(_P)]),
    "es_ep_window_close": (ctypes.c_int, [_P]),
    "es_ep_window_free": (ctypes.c_int, [_P]),
    "es_ep_dispatch": (ctypes.c_int, [ctypes.POINTER(CEpPlan), _P, _P, _P, _I32, _P]),
    "es_ep_receive": (ctypes.c_int, [ctypes.POINTER(CEpPlan), _P, _P, _P]),
    "es_ep_rows_offset": (ctypes.c_int, [ctypes.POINTER(CEpPlan), ctypes.POINTER(_SZ)]),
    "es_ep_return": (ctypes.c_int, [ctypes.POINTER(CEpPlan), _P, _P]),
    "es_ep_combine_p2p": (ctypes.c_int, [ctypes.POINTER(CEpPlan), _P, _P, _I32, _P, _I32, _P]),
    "es_moe_forward_noalloc": (ctypes.c_int, [_CFG, _P, _P, _I32, _P, _P, _P, _P, _I32, _P, _P,
                                              _I32, _P]),
    "es_moe_read_error": (ctypes.c_int, [_P, _I32, ctypes.POINTER(ctypes.c_uint32), _P]),
    "es_moe_noalloc_read_error": (ctypes.c_int, [_I32, ctypes.POINTER(ctypes.c_uint32), _P]),
    "es_moe_kernel_family": (ctypes.c_int, [_CFG, _I32, ctypes.POINTER(ctypes.c_int32)]),
    "es_dec_add_rmsnorm": (ctypes.c_int, [_P, _P, _P, _P, _I32, _I32, ctypes.c_float, _P]),
    "es_dec_qk_norm_rope_kv": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32,
                                              _I32, _I32, _I32, ctypes.c_float, _P]),
    "es_dec_gemv": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I32, _P]),
}

_lib = None


def header_functions() -> list:
    """Names of the functions include/es_moe.h declares."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    pat = r"^\s*(?:ES_API\s+)?(?:const\s+)?\w+\s*\*?\s*(es_\w+)\s*\("
    return sorted(set(re.findall(pat, text, flags=re.M)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m expert_sniper_b200.build` "
                "(the MoE block has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(fn: str, status: int) -> None:
    if status != ES_OK:
        msg = lib().es_status_str(status).decode()
        raise EsError(fn, status, msg)


def packed_bytes(ccfg: CMoECfg) -> int:
    out = _SZ(0)
    check("es_moe_packed_bytes", lib().es_moe_packed_bytes(ctypes.byref(ccfg), ctypes.byref(out)))
    return out.value


def workspace_bytes(ccfg: CMoECfg, max_tokens: int) -> int:
    out = _SZ(0)
    check("es_moe_workspace_bytes",
          lib().es_moe_workspace_bytes(ctypes.byref(ccfg), int(max_tokens), ctypes.byref(out)))
    return out.value
