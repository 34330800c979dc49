"""The expert-node shim on the GPU: one node's fp16 partial against the
oracle's compute_partial restatement (node.py:142-172), the fixed-order sum
of every node's partial against the whole block (reader.py:278-292), and a
/compute_bin request served over HTTP on 127.0.0.1."""
from __future__ import annotations

import socket
import threading
import time
import urllib.request

import numpy as np
import pytest

from expert_sniper_b200 import hrw
from expert_sniper_b200 import node as nd
from expert_sniper_b200.config import MoEConfig
from expert_sniper_b200.quant import synthetic_layer
from oracle import moe_oracle as mo
from tests._helpers import assert_close_rms

pytestmark = pytest.mark.gpu

CFG = MoEConfig(512, 32, 4, 512, True, name="node-gpu")
# fp16 activations are read as fp16 (tensor-core path: fp16 weights, h and y
# rows, fp32 accumulation) and the partial is returned in fp16; the parity bar
NODE_REL = 1e-2


def _case(T, seed):
    rng = np.random.default_rng(seed)
    h = rng.standard_normal((1, T, CFG.hidden)).astype(np.float16)
    inds = np.stack([rng.choice(CFG.num_experts, CFG.top_k, replace=False) for _ in range(T)])
    w = rng.random((T, CFG.top_k)).astype(np.float32)
    return h, inds[None].astype(np.int32), w[None]


def test_node_partials_match_oracle_and_sum_to_block(cuda):
    lay = synthetic_layer(CFG, seed=4, device="cpu")
    lay_np = {k: v.numpy() for k, v in lay.items()}
    roster = hrw.gpu_roster(4)
    plan = hrw.plan(roster, CFG.num_experts)
    h, inds, w = _case(12, 5)
    ids = sorted(set(inds.ravel().tolist()))
    x32 = h.reshape(12, -1).astype(np.float32)
    total = None
    for name in roster:
        owned = sorted(plan[name])
        node = nd.NodeCompute(CFG, owned, {3: lay}, device=cuda, max_tokens=16)
        n, part = node.compute_partial(3, ids, h, inds, w)
        my = [e for e in ids if e in set(owned)]
        assert n == len(my) and part.dtype == np.float16 and part.shape == h.shape
        ref = mo.partial(x32, lay_np, inds[0], w[0], my) if my else np.zeros((12, CFG.hidden))
        assert_close_rms(part[0].astype(np.float32), ref, rel=NODE_REL, what=name)
        total = part[0].astype(np.float32) if total is None else total + part[0].astype(np.float32)
    full = mo.expert_ffn(x32, {k: v for k, v in lay_np.items() if k.startswith("switch_mlp")},
                         inds[0], w[0])
    assert_close_rms(total, full, rel=NODE_REL, what="sum of nodes")
    # a layer this node does not hold, or no owned expert requested: zeros
    n0, z = node.compute_partial(9, ids, h, inds, w)
    assert n0 == 0 and not z.any()


def test_compute_bin_over_http(cuda):
    uvicorn = pytest.importorskip("uvicorn")
    lay = synthetic_layer(CFG, seed=6, device="cpu")
    owned = sorted(hrw.plan(hrw.gpu_roster(2), CFG.num_experts)["gpu1"])
    node = nd.NodeCompute(CFG, owned, {0: lay}, device=cuda, max_tokens=8)
    h, inds, w = _case(6, 7)
    ids = sorted(set(inds.ravel().tolist()))
    req = nd.pack_request(0, ids, h, inds, w)
    direct = node.handle(req)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    server = uvicorn.Server(uvicorn.Config(nd.create_app(node), host="127.0.0.1", port=port,
                                           log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    try:
        for _ in range(200):
            if server.started:
                break
            time.sleep(0.05)
        got = urllib.request.urlopen(urllib.request.Request(
            f"http://127.0.0.1:{port}/compute_bin", data=req,
            headers={"Content-Type": "application/octet-stream"}), timeout=60).read()
        assert got == direct  # deterministic kernels: identical bytes
    finally:
        server.should_exit = True
        th.join(timeout=10)
