"""MoE block shapes.

`MoEConfig` carries the keys the reference reads from a streaming model's
config.json (src/mlx_expert_sniper/download.py:477-523: num_experts,
num_experts_per_tok, moe_intermediate_size, norm_topk_prob,
shared_expert_intermediate_size, quantization{bits, group_size}) and the
module constants BITS=4 / GROUP_SIZE=64 (src/mlx_expert_sniper/engine.py:12-13).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace


KERNEL_PATHS = {"auto": 0, "decode": 1, "tensor": 2, "tensor-small": 3, "fused": 4}
X_DTYPES = {"bf16": 0, "f16": 1}  # es_dtype codes


@dataclass(frozen=True)
class MoEConfig:
    hidden: int                 # D
    num_experts: int            # E (routed)
    top_k: int                  # k
    inter: int                  # I of a routed expert
    norm_topk_prob: bool        # renormalise the k selected probabilities
    shared_inter: int = 0       # 0 = no shared expert
    group_size: int = 64
    bits: int = 4
    name: str = ""
    # expert-FFN kernels: "auto", "decode" (CUDA-core GEMV) or "tensor"
    # (tcgen05 grouped GEMM); no counterpart in the reference
    kernel_path: str = "auto"
    # activation dtype: "bf16" (the model dtype) or "f16" (the Expert
    # Network's wire dtype; runs the tensor-core path)
    x_dtype: str = "bf16"

    def __post_init__(self):
        if self.group_size != 64 or self.bits != 4:
            raise ValueError("only 4-bit, group-64 MLX affine experts are supported")
        if self.hidden % 64 or self.inter % 64:
            raise ValueError("hidden and inter must be multiples of 64")
        if not 1 <= self.top_k <= 16:
            raise ValueError("top_k must be in [1, 16]")
        if self.shared_inter and self.shared_inter != self.inter:
            raise ValueError("a shared expert must have the routed experts' inter size")
        if self.kernel_path not in KERNEL_PATHS:
            raise ValueError(f"kernel_path must be one of {sorted(KERNEL_PATHS)}")
        if self.x_dtype not in X_DTYPES:
            raise ValueError(f"x_dtype must be one of {sorted(X_DTYPES)}")
        if self.x_dtype == "f16" and self.kernel_path in ("decode", "fused"):
            raise ValueError("the decode and fused kernels read bf16 activations")

    @property
    def has_shared(self) -> bool:
        return self.shared_inter > 0

    @property
    def bytes_per_expert(self) -> int:
        """Packed bytes of one expert: 3*D*I*(1/2 + 2*2/64) = 3*D*I*0.5625."""
        return 3 * self.hidden * self.inter * 9 // 16

    @property
    def experts_total(self) -> int:
        return self.num_experts + (1 if self.has_shared else 0)

    @property
    def packed_bytes(self) -> int:
        return self.bytes_per_expert * self.experts_total

    def with_(self, **kw) -> "MoEConfig":
        return replace(self, **kw)

    def to_c(self) -> "CMoECfg":
        return CMoECfg(self.hidden, self.num_experts, self.top_k, self.inter,
                       self.group_size, self.bits, int(self.norm_topk_prob),
                       self.shared_inter, KERNEL_PATHS[self.kernel_path], X_DTYPES[self.x_dtype])


class CMoECfg(ctypes.Structure):
    """Mirror of `es_moe_cfg` in include/es_moe.h."""
    _fields_ = [("hidden", ctypes.c_int32), ("num_experts", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("inter", ctypes.c_int32),
                ("group_size", ctypes.c_int32), ("bits", ctypes.c_int32),
                ("norm_topk_prob", ctypes.c_int32), ("shared_inter", ctypes.c_int32),
                ("kernel_path", ctypes.c_int32), ("x_dtype", ctypes.c_int32)]


# Shapes of the model families the reference serves (engine_olmoe.py:53-54,
# engine_30b.py:85-87, engine_next.py; Qwen3-235B-A22B is the same Qwen3-MoE
# block at hidden 4096 / inter 1536).
PRESETS = {
    "olmoe-1b-7b": MoEConfig(2048, 64, 8, 1024, False, name="olmoe-1b-7b"),
    "qwen3-30b-a3b": MoEConfig(2048, 128, 8, 768, True, name="qwen3-30b-a3b"),
    "qwen3-next-80b-a3b": MoEConfig(2048, 512, 10, 512, True, shared_inter=512,
                                    name="qwen3-next-80b-a3b"),
    "qwen3-235b-a22b": MoEConfig(4096, 128, 8, 1536, True, name="qwen3-235b-a22b"),
}
