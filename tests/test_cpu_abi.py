"""The C ABI library on the host: it loads, exports every declared entry
point, and its host-only entry points (sizes, argument checks) behave,
without touching a GPU."""
from __future__ import annotations

import ctypes
import os

import pytest

from expert_sniper_b200 import PRESETS, MoEConfig, _native
from expert_sniper_b200.config import CMoECfg


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_native.LIB_PATH):
        from expert_sniper_b200 import build
        build.build()
    return _native.lib()


def test_exports_every_header_function(lib):
    names = _native.header_functions()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), f"{n} declared in es_moe.h but not exported"
    # and nothing else is exported under the es_ prefix
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = sorted({line.split()[-1] for line in out.splitlines()
                       if line.split()[-1].startswith("es_")})
    assert exported == names


def test_signature_table_covers_header():
    assert sorted(_native._SIGNATURES) == _native.header_functions()


def test_version_and_status_strings(lib):
    assert lib.es_version() >> 16 == 1
    assert lib.es_status_str(0) == b"ok"
    assert lib.es_status_str(3) == b"workspace too small"
    assert lib.es_status_str(99) == b"unknown status"


@pytest.mark.parametrize("name", sorted(PRESETS))
def test_packed_bytes_equal_reference_block_bytes(lib, name):
    cfg = PRESETS[name]
    nb = _native.packed_bytes(cfg.to_c())
    assert nb == cfg.packed_bytes
    # the reference's per-expert block bytes: align16K of the nine tensors of
    # TENSOR_ORDER (src/mlx_expert_sniper/download.py:73-77, 197-212)
    per = {"olmoe-1b-7b": 3538944, "qwen3-30b-a3b": 2654208, "qwen3-next-80b-a3b": 1769472,
           "qwen3-235b-a22b": 10616832}[name]
    assert cfg.bytes_per_expert == per


def test_workspace_bytes_monotone(lib):
    c = PRESETS["qwen3-30b-a3b"].to_c()
    sizes = [_native.workspace_bytes(c, t) for t in (0, 1, 8, 64, 256, 4096)]
    assert sizes == sorted(sizes) and sizes[1] > 0


@pytest.mark.parametrize("bad", [
    dict(group_size=32), dict(bits=8), dict(hidden=2000), dict(hidden=8192), dict(inter=640),
    dict(num_experts=2000), dict(top_k=17), dict(top_k=0), dict(shared_inter=256),
    dict(kernel_path=5), dict(kernel_path=-1),
])
def test_unsupported_configs_rejected(lib, bad):
    base = dict(hidden=2048, num_experts=128, top_k=8, inter=768, group_size=64, bits=4,
                norm_topk_prob=1, shared_inter=0, kernel_path=0)
    base.update(bad)
    c = CMoECfg(**base)
    out = ctypes.c_size_t(0)
    st = lib.es_moe_packed_bytes(ctypes.byref(c), ctypes.byref(out))
    assert st in (1, 2)


def test_null_and_size_checks_return_status(lib):
    c = PRESETS["qwen3-30b-a3b"].to_c()
    assert lib.es_moe_packed_bytes(None, None) == 1
    assert lib.es_moe_workspace_bytes(ctypes.byref(c), -1, ctypes.byref(ctypes.c_size_t())) == 1
    # workspace too small is reported before any launch
    st = lib.es_moe_forward(ctypes.byref(c), 16, 16, 0, None, None, 256, 256, 0, None, None, 4,
                            256, 1, None)
    assert st == 3
    # T == 0 is a no-op success
    assert lib.es_moe_route(ctypes.byref(c), None, 0, None, 0, None, None, None) == 0
    # misaligned workspace
    assert lib.es_moe_expert_ffn(ctypes.byref(c), 16, 16, 16, None, 256, 256, 0, 1, 8, 1 << 30,
                                 None) == 1
    # read_error validates before touching the device
    assert lib.es_moe_read_error(None, 0, None, None) == 1
    # decoder helpers: null pointers and bad shapes are rejected before a
    # launch; zero rows / batch is a no-op success
    assert lib.es_dec_add_rmsnorm(None, None, None, None, 4, 256, 1e-6, None) == 1
    assert lib.es_dec_add_rmsnorm(16, None, 16, 16, 4, 0, 1e-6, None) == 1
    assert lib.es_dec_add_rmsnorm(16, None, 16, 16, 0, 256, 1e-6, None) == 0
    args = [16] * 9
    assert lib.es_dec_qk_norm_rope_kv(*args, 2, 4, 2, 63, 8, 1e-6, None) == 1  # odd head_dim
    assert lib.es_dec_qk_norm_rope_kv(*args, 2, 4, 2, 64, 0, 1e-6, None) == 1
    assert lib.es_dec_qk_norm_rope_kv(*([None] + args[1:]), 2, 4, 2, 64, 8, 1e-6, None) == 1
    assert lib.es_dec_qk_norm_rope_kv(*args, 0, 4, 2, 64, 8, 1e-6, None) == 0
    assert lib.es_dec_gemv(None, 16, 16, 1, 8, 8, None) == 1
    assert lib.es_dec_gemv(16, 16, 16, 5, 8, 8, None) == 1     # batch above 4
    assert lib.es_dec_gemv(16, 16, 16, 1, 8, 12, None) == 1    # k not a multiple of 8
    assert lib.es_dec_gemv(16, 24, 16, 1, 8, 8, None) == 1     # x not 16-byte aligned
    assert lib.es_dec_gemv(16, 16, 16, 0, 8, 8, None) == 0


def test_config_validation_in_python():
    with pytest.raises(ValueError):
        MoEConfig(2048, 128, 8, 768, True, shared_inter=512)
    with pytest.raises(ValueError):
        MoEConfig(2048, 4, 17, 768, True)
    with pytest.raises(ValueError):
        MoEConfig(2048, 128, 8, 768, True, kernel_path="fast")
    assert MoEConfig(2048, 128, 8, 768, True, kernel_path="tensor").to_c().kernel_path == 2
    assert MoEConfig(2048, 128, 8, 768, True, kernel_path="tensor-small").to_c().kernel_path == 3


def test_automatic_kernel_choice():
    """The automatic expert-FFN kernel rule (es_moe_cfg.kernel_path 0), by
    average pairs per routed expert p = T k / E: the fused tiny-batch kernel
    for T <= 16, decode below 4, 32-token tensor tiles up to 48, 128-token
    tiles above; tensor kernels from T = 64; fp16 activations never take the
    decode or fused kernels."""
    from expert_sniper_b200.block import ffn_kernels, uses_tensor_path
    q = PRESETS["qwen3-30b-a3b"]          # E = 128, k = 8
    assert [ffn_kernels(q, T) for T in (1, 4, 5, 8, 16, 17, 63, 64, 128, 256, 768, 769, 4096)] == [
        "fused", "fused", "fused", "fused", "fused", "decode", "decode", "tensor-small",
        "tensor-small",
        "tensor-small", "tensor-small", "tensor", "tensor"]
    assert ffn_kernels(q.with_(kernel_path="fused"), 16) == "fused"
    assert ffn_kernels(q.with_(kernel_path="fused"), 17) == "decode"
    small = MoEConfig(256, 4, 2, 256, True)  # p = T / 2: the T >= 64 floor decides
    assert ffn_kernels(small, 32) == "decode" and ffn_kernels(small, 64) == "tensor-small"
    assert ffn_kernels(small, 98) == "tensor"
    nxt = PRESETS["qwen3-next-80b-a3b"]     # E = 512, k = 10
    assert [ffn_kernels(nxt, T) for T in (64, 256, 2048, 4096)] == [
        "decode", "tensor-small", "tensor-small", "tensor"]
    f16 = q.with_(x_dtype="f16")
    assert ffn_kernels(f16, 8) == "tensor-small" and ffn_kernels(f16, 4096) == "tensor"
    for path in ("decode", "tensor", "tensor-small"):
        assert ffn_kernels(q.with_(kernel_path=path), 64) == path
    assert not uses_tensor_path(q, 63) and uses_tensor_path(q, 64)


def test_python_kernel_rule_matches_the_library():
    """block.ffn_kernels (the Python mirror used for accounting and by the
    expert-parallel wrapper) names the same kernel family as the library's
    own rule (es_moe_kernel_family), for every preset, forced path,
    activation dtype and a range of batch sizes."""
    import ctypes

    from expert_sniper_b200.block import ffn_kernels
    lib = _native.lib()
    names = {1: "decode", 2: "tensor", 3: "tensor-small", 4: "fused"}
    out = ctypes.c_int32(0)
    for cfg in list(PRESETS.values()) + [MoEConfig(256, 16, 4, 256, True),
                                         MoEConfig(3072, 64, 8, 1024, True)]:
        for path in ("auto", "decode", "tensor", "tensor-small", "fused"):
            for xd in ("bf16", "f16"):
                if xd == "f16" and path in ("decode", "fused"):
                    continue
                c = cfg.with_(kernel_path=path, x_dtype=xd)
                cc = c.to_c()
                for T in (1, 2, 5, 8, 9, 15, 16, 17, 32, 63, 64, 65, 128, 255, 1024, 4096):
                    _native.check("es_moe_kernel_family",
                                  lib.es_moe_kernel_family(ctypes.byref(cc), T, ctypes.byref(out)))
                    assert names[out.value] == ffn_kernels(c, T), (c.name, path, xd, T)
