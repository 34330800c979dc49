"""PyTorch custom operators over the C ABI (torch.library).

    torch.ops.expert_sniper.moe_forward(x, logits, cache_bias, packed,
        shared_gate_w, workspace, num_experts, top_k, inter, norm_topk_prob,
        shared_inter, kernel_path, out_dtype) -> (out, topk_idx, topk_w)
    torch.ops.expert_sniper.moe_forward_out(..., out, topk_idx, topk_w)

The MoE part of one make_forward layer (src/mlx_expert_sniper/generate.py:
122-181: router with cache bias, top-k, run_expert_ffn of engine.py:15-42,
shared expert of generate.py:173-178) as operators of PyTorch's dispatcher,
so the block traces (a fake kernel gives output shapes without running
anything), composes with other ops and is captured by torch.cuda.graph like
any CUDA op. Both run es_moe_forward on the current CUDA stream.

`workspace` is the caller's zero-initialised uint8 buffer of
es_moe_workspace_bytes(max_tokens) bytes (MoEBlock owns one); None makes the
operator use one that it keeps per device and stream, grown on demand. The
operators raise on CPU tensors: there is no CPU implementation.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _native
from .config import CMoECfg

_OUT_DTYPES = {0: torch.bfloat16, 2: torch.float32}   # es_dtype codes
_X_DTYPES = {torch.bfloat16: 0, torch.float16: 1}
_LOGIT_DTYPES = {torch.bfloat16: _native.ES_DTYPE_BF16, torch.float32: _native.ES_DTYPE_F32}
_OUT_CODES = {torch.bfloat16: _native.ES_DTYPE_BF16, torch.float32: _native.ES_DTYPE_F32}

_workspaces = {}   # (device index, stream) -> zero-initialised uint8 tensor


def _ccfg(x, num_experts, top_k, inter, norm_topk_prob, shared_inter, kernel_path) -> CMoECfg:
    if x.dtype not in _X_DTYPES:
        raise ValueError("x must be bf16 or fp16")
    return CMoECfg(x.shape[-1], num_experts, top_k, inter, 64, 4, int(norm_topk_prob),
                   shared_inter, kernel_path, _X_DTYPES[x.dtype])


def _shared_workspace(ccfg: CMoECfg, T: int, device: torch.device) -> torch.Tensor:
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream)
    need = _native.workspace_bytes(ccfg, T)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def _run(x, logits, cache_bias, packed, shared_gate_w, workspace, ccfg, out, idx, w):
    for name, t in (("x", x), ("logits", logits), ("packed", packed)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (the MoE block has no CPU path)")
    T = x.shape[0]
    if logits.dtype not in _LOGIT_DTYPES:
        raise ValueError("logits must be bf16 or fp32")
    if tuple(logits.shape) != (T, ccfg.num_experts):
        raise ValueError(f"logits must be [{T}, {ccfg.num_experts}]")
    if not (x.is_contiguous() and logits.is_contiguous() and packed.is_contiguous()):
        raise ValueError("x, logits and packed must be contiguous")
    ws = workspace if workspace is not None else _shared_workspace(ccfg, T, x.device)
    if cache_bias is not None and (cache_bias.dtype != torch.float32
                                   or not cache_bias.is_contiguous()):
        raise ValueError("cache_bias must be a contiguous fp32 [E] tensor")
    if shared_gate_w is not None and shared_gate_w.dtype != torch.bfloat16:
        raise ValueError("shared_gate_w must be bf16")
    ptr = lambda t: 0 if t is None else t.data_ptr()
    _native.check("es_moe_forward", _native.lib().es_moe_forward(
        ctypes.byref(ccfg), x.data_ptr(), logits.data_ptr(), _LOGIT_DTYPES[logits.dtype],
        ptr(cache_bias), ptr(shared_gate_w), packed.data_ptr(), out.data_ptr(),
        _OUT_CODES[out.dtype], ptr(idx), ptr(w), T, ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream(x.device).cuda_stream))


@torch.library.custom_op("expert_sniper::moe_forward", mutates_args=("workspace",))
def moe_forward(x: torch.Tensor, logits: torch.Tensor, cache_bias: Optional[torch.Tensor],
                packed: torch.Tensor, shared_gate_w: Optional[torch.Tensor],
                workspace: Optional[torch.Tensor], num_experts: int, top_k: int, inter: int,
                norm_topk_prob: bool, shared_inter: int = 0, kernel_path: int = 0,
                out_dtype: int = 0) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """x [T, D] bf16 (or fp16), logits [T, E] bf16 or fp32, cache_bias [E] fp32
    or None -> (out [T, D] in out_dtype (0 bf16, 2 fp32), topk_idx [T, k]
    int32 in descending probability order, topk_w [T, k] fp32)."""
    ccfg = _ccfg(x, num_experts, top_k, inter, norm_topk_prob, shared_inter, kernel_path)
    T = x.shape[0]
    out = torch.empty((T, x.shape[1]), dtype=_OUT_DTYPES[out_dtype], device=x.device)
    idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    if T:
        _run(x, logits, cache_bias, packed, shared_gate_w, workspace, ccfg, out, idx, w)
    return out, idx, w


@moe_forward.register_fake
def _(x, logits, cache_bias, packed, shared_gate_w, workspace, num_experts, top_k, inter,
      norm_topk_prob, shared_inter=0, kernel_path=0, out_dtype=0):
    T = x.shape[0]
    return (x.new_empty((T, x.shape[1]), dtype=_OUT_DTYPES[out_dtype]),
            x.new_empty((T, top_k), dtype=torch.int32),
            x.new_empty((T, top_k), dtype=torch.float32))


@torch.library.custom_op("expert_sniper::moe_forward_out",
                         mutates_args=("workspace", "out", "topk_idx", "topk_w"))
def moe_forward_out(x: torch.Tensor, logits: torch.Tensor, cache_bias: Optional[torch.Tensor],
                    packed: torch.Tensor, shared_gate_w: Optional[torch.Tensor],
                    workspace: Optional[torch.Tensor], out: torch.Tensor,
                    topk_idx: Optional[torch.Tensor], topk_w: Optional[torch.Tensor],
                    num_experts: int, top_k: int, inter: int, norm_topk_prob: bool,
                    shared_inter: int = 0, kernel_path: int = 0) -> None:
    """moe_forward into caller-owned outputs: out [T, D] bf16 or fp32,
    topk_idx / topk_w [T, k] or None (then kept in the workspace)."""
    ccfg = _ccfg(x, num_experts, top_k, inter, norm_topk_prob, shared_inter, kernel_path)
    if out.shape != x.shape or out.dtype not in _OUT_CODES or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 or fp32 tensor shaped like x")
    if (topk_idx is None) != (topk_w is None):
        raise ValueError("pass both topk_idx and topk_w, or neither")
    if x.shape[0]:
        _run(x, logits, cache_bias, packed, shared_gate_w, workspace, ccfg, out, topk_idx, topk_w)


@moe_forward_out.register_fake
def _(x, logits, cache_bias, packed, shared_gate_w, workspace, out, topk_idx, topk_w,
      num_experts, top_k, inter, norm_topk_prob, shared_inter=0, kernel_path=0):
    return None
