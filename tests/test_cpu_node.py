"""Expert-node compatibility on the CPU: the /compute_bin wire format against
bytes the reference produced (tests/golden/protocol_sizes.json, from
src/expert_network/protocol.py), the partition masking of compute_partial
(node.py:142-172) against the oracle, and the HTTP endpoint served by
uvicorn on 127.0.0.1 with an oracle-backed node."""
from __future__ import annotations

import json
import os
import socket
import threading
import time
import urllib.request

import numpy as np
import pytest

from expert_sniper_b200 import node as nd
from expert_sniper_b200.config import MoEConfig
from expert_sniper_b200.quant import synthetic_layer
from oracle import moe_oracle as mo
from tests._helpers import assert_close_rms

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "protocol_sizes.json")))


def test_request_and_response_bytes_match_reference():
    t = GOLD["tiny"]
    h = np.array(t["hidden"], np.float16)
    inds = np.array(t["inds"], np.int32)
    w = np.array(t["weights"], np.float32)
    req = nd.pack_request(t["layer"], t["expert_ids"], h, inds, w)
    assert req.hex() == t["request_hex"]
    assert nd.pack_response(2, h).hex() == t["response_hex"]
    layer, ids, h2, i2, w2 = nd.unpack_request(bytes.fromhex(t["request_hex"]))
    assert layer == t["layer"] and ids == sorted(t["expert_ids"])
    assert np.array_equal(h2, h) and np.array_equal(i2, inds) and np.array_equal(w2, w)
    n, r = nd.unpack_response(bytes.fromhex(t["response_hex"]))
    assert n == 2 and np.array_equal(r, h)


@pytest.mark.parametrize("case", GOLD["sizes"], ids=lambda c: f"D{c['D']}k{c['k']}T{c['T']}")
def test_message_sizes_match_reference(case):
    D, k, T = case["D"], case["k"], case["T"]
    h = np.zeros((1, T, D), np.float16)
    req = nd.pack_request(3, list(range(k)), h, np.zeros((1, T, k), np.int32),
                          np.zeros((1, T, k), np.float32))
    assert len(req) == case["request_bytes"]
    assert len(nd.pack_response(k, h)) == case["response_bytes"]


def test_truncated_request_rejected():
    t = GOLD["tiny"]
    raw = bytes.fromhex(t["request_hex"])
    with pytest.raises(ValueError):
        nd.unpack_request(raw[:-4])


CFG = MoEConfig(256, 16, 4, 256, True, name="node-cpu")


def _oracle_node_partial(lay, owned, layer_idx, req_ids, h, inds, w):
    """Reference semantics restated: experts requested and owned; others masked."""
    my = sorted(e for e in req_ids if e in set(owned))
    if not my:
        return 0, np.zeros(h.shape, np.float16)
    T, k = inds.shape[1], inds.shape[2]
    part = mo.partial(h.reshape(T, -1).astype(np.float32), lay, inds.reshape(T, k), w.reshape(T, k), my)
    return len(my), part.astype(np.float16).reshape(h.shape)


def test_local_routing_is_the_partition_mask():
    rng = np.random.default_rng(1)
    owned = [1, 4, 6, 9, 15]
    lut = np.full(16, -1, np.int32)
    lut[owned] = np.arange(len(owned))
    inds = rng.integers(0, 16, (1, 7, 4)).astype(np.int32)
    inds[0, 2, 1] = -1
    w = rng.random((1, 7, 4)).astype(np.float32)
    req = sorted(set(inds[inds >= 0].tolist()))
    my = [e for e in req if e in owned]
    local, lw = nd.local_routing(inds, w, my, lut)
    for t in range(7):
        for j in range(4):
            e = inds[0, t, j]
            if e in my:
                assert local[t, j] == owned.index(e) and lw[t, j] == w[0, t, j]
            else:
                assert local[t, j] == -1 and lw[t, j] == 0.0


class _OracleNode:
    """NodeCompute's interface, computed with the oracle on the CPU."""

    def __init__(self, lay, owned):
        self.lay, self.owned, self.blocks, self.device = lay, owned, {0: None}, "cpu"

    def handle(self, raw):
        layer_idx, ids, h, i, w = nd.unpack_request(raw)
        n, res = _oracle_node_partial(self.lay, self.owned, layer_idx, ids, h, i, w)
        return nd.pack_response(n, res)


def test_http_compute_bin_round_trip():
    uvicorn = pytest.importorskip("uvicorn")
    lay = {k: v.numpy() for k, v in synthetic_layer(CFG, seed=2).items()}
    owned = [0, 3, 5, 7, 8, 12]
    app = nd.create_app(_OracleNode(lay, owned))
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    try:
        for _ in range(100):
            if server.started:
                break
            time.sleep(0.05)
        rng = np.random.default_rng(3)
        T = 5
        h = rng.standard_normal((1, T, CFG.hidden)).astype(np.float16)
        inds = np.stack([rng.choice(16, 4, replace=False) for _ in range(T)])[None].astype(np.int32)
        w = rng.random((1, T, 4)).astype(np.float32)
        req = nd.pack_request(0, sorted(set(inds.ravel().tolist())), h, inds, w)
        r = urllib.request.urlopen(urllib.request.Request(
            f"http://127.0.0.1:{port}/compute_bin", data=req,
            headers={"Content-Type": "application/octet-stream"}), timeout=30)
        n, res = nd.unpack_response(r.read())
        n_ref, ref = _oracle_node_partial(lay, owned, 0, sorted(set(inds.ravel().tolist())), h, inds, w)
        assert n == n_ref and res.dtype == np.float16 and res.shape == h.shape
        assert np.array_equal(res, ref)
        health = json.loads(urllib.request.urlopen(f"http://127.0.0.1:{port}/health", timeout=10).read())
        assert health["status"] == "ok" and health["requests"] == 1
    finally:
        server.should_exit = True
        th.join(timeout=10)


def test_four_nodes_sum_to_the_block():
    """Every node answers for its HRW partition; the driver sums the fp16
    partials in fixed node order in fp32 (reader.py:278-292): the total is the
    whole block up to the fp16 rounding of each partial."""
    from expert_sniper_b200 import hrw
    lay = {k: v.numpy() for k, v in synthetic_layer(CFG, seed=8).items()}
    roster = hrw.gpu_roster(4)
    plan = hrw.plan(roster, CFG.num_experts)
    rng = np.random.default_rng(9)
    T = 7
    h = rng.standard_normal((1, T, CFG.hidden)).astype(np.float16)
    inds = np.stack([rng.choice(CFG.num_experts, CFG.top_k, replace=False)
                     for _ in range(T)])[None].astype(np.int32)
    w = rng.random((1, T, CFG.top_k)).astype(np.float32)
    ids = sorted(set(inds.ravel().tolist()))
    total = np.zeros((T, CFG.hidden), np.float32)
    counted = 0
    for name in roster:
        node = _OracleNode(lay, sorted(plan[name]))
        n, part = nd.unpack_response(node.handle(nd.pack_request(0, ids, h, inds, w)))
        counted += n
        total += part[0].astype(np.float32)
    assert counted == len(ids)
    full = mo.expert_ffn(h[0].astype(np.float32), {k: v for k, v in lay.items()
                                                   if k.startswith("switch_mlp")}, inds[0], w[0])
    assert_close_rms(total, full, rel=1e-2, what="sum of 4 nodes")
