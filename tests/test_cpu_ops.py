"""The registered operators trace without a GPU (fake kernels) and refuse
CPU tensors: there is no CPU implementation of the block."""
from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import expert_sniper_b200  # noqa: F401  (registers torch.ops.expert_sniper.*)


def test_fake_shapes():
    with FakeTensorMode():
        x = torch.empty(5, 256, dtype=torch.bfloat16, device="cuda")
        lg = torch.empty(5, 16, dtype=torch.bfloat16, device="cuda")
        pk = torch.empty(1024, dtype=torch.uint8, device="cuda")
        out, idx, w = torch.ops.expert_sniper.moe_forward(x, lg, None, pk, None, None, 16, 4,
                                                          256, True, 0, 0, 0)
        assert tuple(out.shape) == (5, 256) and out.dtype == torch.bfloat16
        assert tuple(idx.shape) == (5, 4) and idx.dtype == torch.int32
        assert tuple(w.shape) == (5, 4) and w.dtype == torch.float32


def test_cpu_tensors_are_refused():
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    lg = torch.zeros(2, 16, dtype=torch.bfloat16)
    pk = torch.zeros(1024, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA"):
        torch.ops.expert_sniper.moe_forward(x, lg, None, pk, None, None, 16, 4, 256, True,
                                            0, 0, 0)
