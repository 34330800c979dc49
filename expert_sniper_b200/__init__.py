"""B200-native MoE block for Expert Sniper's 4-bit MLX-affine experts.

router (+ cache bias) -> dispatch -> 4-bit expert FFN -> combine, on
hand-written sm_100a kernels behind a C ABI (include/es_moe.h), with
expert-parallel sharding over the GPUs of one box.
"""
from .config import PRESETS, MoEConfig  # noqa: F401
from .block import MoEBlock, cache_bias_mask, prepare_packed, run_expert_ffn  # noqa: F401
from . import hrw  # noqa: F401

__all__ = ["MoEConfig", "PRESETS", "MoEBlock", "prepare_packed", "run_expert_ffn",
           "cache_bias_mask", "hrw"]
