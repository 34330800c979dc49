"""es_moe_forward_noalloc: the forward for callers that cannot allocate.

Hosts that own all device memory (a fixed-arena inference runtime, a plugin
whose host forbids outside allocations) cannot hand the library a workspace;
this entry point uses scratch built into the library instead. The test calls
it through the C ABI twice in a row (different inputs, the shared scratch
keeping the first call's contents) and compares each result with the
workspace-based es_moe_forward, within the parity tolerance. The file sorts
last so a stop-at-first-failure run has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig, PRESETS, _native
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
from tests._helpers import REL_TOL, assert_close_rms

pytestmark = pytest.mark.gpu


def _noalloc(blk, x, logits, bias):
    T = x.shape[0]
    out = torch.empty((T, blk.cfg.hidden), dtype=torch.float32, device=x.device)
    st = _native.lib().es_moe_forward_noalloc(
        ctypes.byref(blk.ccfg), x.data_ptr(), logits.data_ptr(), _native.ES_DTYPE_BF16,
        bias.data_ptr() if bias is not None else None,
        blk.shared_gate_w.data_ptr() if blk.shared_gate_w is not None else None,
        blk.packed.data_ptr(), out.data_ptr(), _native.ES_DTYPE_F32, None, None, T,
        torch.cuda.current_stream().cuda_stream)
    _native.check("es_moe_forward_noalloc", st)
    return out


@pytest.mark.parametrize("cfg,T", [(MoEConfig(512, 32, 4, 512, True, shared_inter=512), 7),
                                   (PRESETS["qwen3-30b-a3b"], 64)])
def test_noalloc_matches_workspace_forward_twice(cuda, cfg, T):
    lay = synthetic_layer(cfg, seed=31, device=cuda)
    blk = MoEBlock(cfg, weights=lay,
                   shared_gate_w=synthetic_inputs(cfg, 1, seed=0, device=cuda)[3], max_tokens=T)
    bias = cache_bias_vector(cfg.num_experts, 0.5, 4)[0].to(cuda)
    for call in range(2):
        x, _, logits, _ = synthetic_inputs(cfg, T, seed=40 + call, device=cuda)
        got = _noalloc(blk, x, logits, bias)
        want = blk.forward(x, logits, bias, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert_close_rms(got.cpu().numpy(), want.cpu().numpy(), rel=REL_TOL,
                         what=f"call {call}")


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    cfg = PRESETS["qwen3-235b-a22b"]
    blk_cfg = cfg.to_c()
    need = _native.workspace_bytes(blk_cfg, 4096)
    assert need > 64 << 20
    dummy = torch.zeros(16, dtype=torch.uint8, device=cuda)
    st = _native.lib().es_moe_forward_noalloc(
        ctypes.byref(blk_cfg), dummy.data_ptr(), dummy.data_ptr(), 0, None, None,
        dummy.data_ptr(), dummy.data_ptr(), 0, None, None, 4096,
        torch.cuda.current_stream().cuda_stream)
    assert st == 3  # ES_ERR_WORKSPACE, before any launch


@pytest.mark.parametrize("T", [3, 40])
def test_noalloc_reports_device_errors(cuda, T):
    """A NaN router logit sets ES_DEVERR_NONFINITE_LOGIT in the scratch's
    error word: es_moe_noalloc_read_error returns it (fused kernel at T = 3,
    decode kernels at T = 40), clears it on request, and the next clean call
    starts from zero."""
    cfg = MoEConfig(512, 32, 4, 512, True)
    lay = synthetic_layer(cfg, seed=33, device=cuda)
    blk = MoEBlock(cfg, weights=lay, max_tokens=T)
    x, _, logits, _ = synthetic_inputs(cfg, T, seed=50, device=cuda)
    bad = logits.clone()
    bad[0, 3] = float("nan")
    lib = _native.lib()
    stream = torch.cuda.current_stream().cuda_stream
    flags = ctypes.c_uint32(0)

    def read(clear):
        _native.check("es_moe_noalloc_read_error",
                      lib.es_moe_noalloc_read_error(clear, ctypes.byref(flags), stream))
        return flags.value

    _noalloc(blk, x, bad, None)
    assert read(1) & _native.DEVERR_NONFINITE_LOGIT
    assert read(0) == 0
    _noalloc(blk, x, logits, None)
    assert read(0) == 0
