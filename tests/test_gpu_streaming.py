"""Streaming-format layers loaded onto the GPU: es_moe_prepare_blocks must
produce exactly the bytes es_moe_prepare produces from the same tensors
(bit-exact), with and without a shared expert, with bf16 scales converted,
and at the full Qwen3-30B layer size."""
from __future__ import annotations

import json

import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig, PRESETS, prepare_packed
from expert_sniper_b200 import streaming as sm
from expert_sniper_b200.quant import synthetic_inputs, synthetic_layer

pytestmark = pytest.mark.gpu


def _split(lay):
    routed = {k: v for k, v in lay.items() if k.startswith("switch_mlp")}
    shared = {k: v for k, v in lay.items() if k.startswith("shared_expert")}
    return routed, shared


@pytest.mark.parametrize("cfg", [MoEConfig(512, 16, 4, 512, True, name="st-a"),
                                 MoEConfig(512, 8, 2, 512, True, shared_inter=512, name="st-b"),
                                 PRESETS["qwen3-30b-a3b"]])
def test_loaded_layer_matches_prepare(cuda, tmp_path, cfg):
    lay = synthetic_layer(cfg, seed=9, device="cpu")
    routed, shared = _split(lay)
    p = sm.layer_path(str(tmp_path), 0)
    sm.write_layer(p, routed)
    got = sm.load_layer(p, cfg, cuda, shared={k: v.to(cuda) for k, v in shared.items()} or None)
    want = prepare_packed(cfg, {k: v.to(cuda) for k, v in lay.items()})
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_bf16_scales_are_converted(cuda, tmp_path):
    cfg = MoEConfig(256, 8, 2, 256, True, name="st-bf16")
    lay = synthetic_layer(cfg, seed=10, device="cpu")
    routed, _ = _split(lay)
    as_bf16 = {k: (v.to(torch.bfloat16) if not k.endswith("weight") else v) for k, v in routed.items()}
    p = sm.layer_path(str(tmp_path), 0)
    sm.write_layer(p, {k: (v.view(torch.int16).numpy().view("<u2") if v.dtype == torch.bfloat16 else v)
                       for k, v in as_bf16.items()})
    hdr = sm.read_header(p)
    for k, v in hdr["layout"]["tensors"].items():
        if not k.endswith("weight"):
            v["dtype"] = "bfloat16"
    raw = open(p, "rb").read()
    with open(p, "wb") as f:
        f.write(json.dumps(hdr).encode().ljust(sm.PAGE_SIZE, bytes(1)))
        f.write(raw[sm.PAGE_SIZE:])
    got = sm.load_layer(p, cfg, cuda)
    ref = {k: (v.float().half() if v.dtype == torch.bfloat16 else v).to(cuda) for k, v in as_bf16.items()}
    want = prepare_packed(cfg, ref)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_forward_from_streaming_layer(cuda, tmp_path):
    """A block built from a loaded layer file computes what the block built
    from the tensors computes (identical packed bytes -> identical output)."""
    cfg = MoEConfig(512, 16, 4, 512, True, name="st-fw")
    lay = synthetic_layer(cfg, seed=11, device="cpu")
    p = sm.layer_path(str(tmp_path), 0)
    sm.write_layer(p, lay)
    x, _, lg, _ = synthetic_inputs(cfg, 9, seed=12, device=cuda)
    a = MoEBlock(cfg, packed=sm.load_layer(p, cfg, cuda), max_tokens=9).forward(x, lg, out_dtype=torch.float32)
    b = MoEBlock(cfg, weights={k: v.to(cuda) for k, v in lay.items()}, max_tokens=9).forward(
        x, lg, out_dtype=torch.float32)
    assert torch.equal(a, b)
