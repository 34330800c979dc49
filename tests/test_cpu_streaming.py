"""Streaming-format layer files (src/mlx_expert_sniper/download.py:189-248,
expert_io.py:271-284 / 338-362): header, offsets, block padding, per-expert
bytes, and the reference test fixture's file (tests/conftest.py:29-54),
all on the CPU."""
from __future__ import annotations

import json

import numpy as np
import pytest

from expert_sniper_b200 import MoEConfig
from expert_sniper_b200 import streaming as sm
from expert_sniper_b200.quant import synthetic_layer

CFG = MoEConfig(256, 8, 2, 256, True, name="stream-small")


def _routed(cfg, seed):
    return {k: v for k, v in synthetic_layer(cfg, seed=seed).items() if k.startswith("switch_mlp")}


def test_write_read_round_trip(tmp_path):
    lay = _routed(CFG, 3)
    p = sm.layer_path(str(tmp_path), 4)
    nb = sm.write_layer(p, lay, layer_idx=4)
    hdr = sm.read_header(p)
    assert hdr["layer_idx"] == 4 and hdr["num_experts"] == CFG.num_experts
    block, start, offs, sdt = sm.check_layout(hdr, CFG)
    assert start == sm.PAGE_SIZE and block % sm.PAGE_SIZE == 0 and sdt == "float16"
    # cumulative offsets in TENSOR_ORDER, as the writer lays them out
    want = sm.expected_layout(CFG)
    acc = 0
    for name, o in zip(sm.TENSOR_ORDER, offs):
        assert o == acc
        acc += want[name][2]
    assert block == -(-acc // sm.PAGE_SIZE) * sm.PAGE_SIZE
    assert nb == sm.PAGE_SIZE + CFG.num_experts * block
    for e in (0, 5, CFG.num_experts - 1):
        got = sm.read_expert(p, e, hdr)
        for name in sm.TENSOR_ORDER:
            src = lay[name][e].numpy()
            assert got[name].tobytes() == src.tobytes(), (e, name)
    # padding after the last tensor is zero
    with open(p, "rb") as f:
        f.seek(sm.PAGE_SIZE + acc)
        assert f.read(block - acc) == b"\x00" * (block - acc)


def test_reference_fixture_file_parses(tmp_path):
    """The reference's own fixture layout (16 KB header, 64-byte blocks of
    two fp16 [4, 4] tensors with deterministic content)."""
    header = {"layout": {"expert_block_size": 64, "data_start": sm.PAGE_SIZE, "tensors": {
        "switch_mlp.gate_proj.weight": {"inner_offset": 0, "nbytes": 32,
                                        "shape_per_expert": [4, 4], "dtype": "float16"},
        "switch_mlp.down_proj.weight": {"inner_offset": 32, "nbytes": 32,
                                        "shape_per_expert": [4, 4], "dtype": "float16"}}}}
    p = tmp_path / "layer_01.bin"
    with open(p, "wb") as f:
        f.write(json.dumps(header).encode().ljust(sm.PAGE_SIZE, b"\x00"))
        for eid in range(16):
            f.write((np.arange(32, dtype=np.float16) + 1 * 1000 + eid).tobytes())
    got = sm.read_expert(str(p), 7)
    vals = np.arange(32, dtype=np.float16) + 1007
    assert np.array_equal(got["switch_mlp.gate_proj.weight"].ravel(), vals[:16])
    assert np.array_equal(got["switch_mlp.down_proj.weight"].ravel(), vals[16:])
    with pytest.raises(ValueError):  # not a 4-bit MoE layer of CFG
        sm.check_layout(sm.read_header(str(p)), CFG)


@pytest.mark.parametrize("bad", ["shape", "dtype", "nbytes", "missing"])
def test_layout_mismatch_rejected(tmp_path, bad):
    lay = _routed(CFG, 4)
    p = sm.layer_path(str(tmp_path), 0)
    sm.write_layer(p, lay)
    hdr = sm.read_header(p)
    t = hdr["layout"]["tensors"]
    name = "switch_mlp.up_proj.scales"
    if bad == "shape":
        t[name]["shape_per_expert"] = [1, 1]
    elif bad == "dtype":
        t[name]["dtype"] = "float32"
    elif bad == "nbytes":
        t[name]["nbytes"] += 2
    else:
        del t[name]
    with pytest.raises(ValueError):
        sm.check_layout(hdr, CFG)


def test_mlx_dtype_names_accepted(tmp_path):
    lay = _routed(CFG, 5)
    p = sm.layer_path(str(tmp_path), 0)
    sm.write_layer(p, lay)
    hdr = sm.read_header(p)
    for v in hdr["layout"]["tensors"].values():  # the writer's str(mx.dtype) spelling
        v["dtype"] = "mlx.core." + v["dtype"]
    sm.check_layout(hdr, CFG)
