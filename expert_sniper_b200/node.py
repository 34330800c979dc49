"""Expert-node compatibility: a B200 process that answers the Expert
Network's `/compute_bin` requests with the MoE kernels.

The Expert Network driver (src/expert_network/reader.py:237-292) posts, per
layer, the active token rows to every node and sums the fp16 partials it gets
back in fixed node order. A node (src/expert_network/node.py:142-198)
computes, over the requested experts it owns, the routed FFN with the
routing weights masked to its partition, and returns the result cast to
fp16. This module does the same on the GPU:

  wire format   pack/unpack of the request and response, byte-compatible with
                src/expert_network/protocol.py:1-65 (checked against bytes
                produced by the reference in tests/golden/protocol_sizes.json):
                request  [layer:u16][n:u16][ids:u16*n][hs_shape:u16*3]
                         [inds_shape:u16*3][wt_shape:u16*3]
                         [hidden:f16][inds:i32][weights:f32]
                response [n_computed:u16][ndim:u16][shape:u16*ndim][out:f16]
  compute       NodeCompute holds, per layer, a block with this node's experts
                only (ids remapped to local indices); slots whose expert is not
                among the requested, owned experts are masked (-1), which the
                kernels skip -- the partition mask of compute_partial. The fp16
                wire activations become bf16, the model dtype the kernels take.
  server        create_app() -> FastAPI app with POST /compute_bin and
                GET /health; run it with uvicorn like the reference's node.

A slot that names an owned expert which the request did not list is skipped
here; the reference would evaluate it with its first requested expert's
weights (its lookup table defaults to 0). Drivers list every active expert,
so the two agree on every request a driver sends.
"""
import struct
import threading
import time

import numpy as np
import torch

from .block import MoEBlock
from .config import MoEConfig
from .ep import shard_layer


# --------------------------------------------------------------------------- #
# wire format
# --------------------------------------------------------------------------- #

def pack_request(layer_idx: int, expert_ids, hidden_f16: np.ndarray, inds_i32: np.ndarray,
                 weights_f32: np.ndarray) -> bytes:
    ids = np.asarray(sorted(int(e) for e in expert_ids), dtype="<u2")
    parts = [struct.pack("<HH", layer_idx, ids.size), ids.tobytes()]
    for a in (hidden_f16, inds_i32, weights_f32):
        if a.ndim != 3:
            raise ValueError("hidden, indices and weights are rank-3 ([1, T, .])")
        parts.append(np.asarray(a.shape, dtype="<u2").tobytes())
    parts += [np.ascontiguousarray(hidden_f16, dtype="<f2").tobytes(),
              np.ascontiguousarray(inds_i32, dtype="<i4").tobytes(),
              np.ascontiguousarray(weights_f32, dtype="<f4").tobytes()]
    return b"".join(parts)


def unpack_request(raw: bytes):
    """-> (layer_idx, expert_ids, hidden f16, inds i32, weights f32)."""
    layer_idx, n = struct.unpack_from("<HH", raw, 0)
    off = 4
    ids = np.frombuffer(raw, dtype="<u2", count=n, offset=off).tolist()
    off += 2 * n
    shapes = []
    for _ in range(3):
        shapes.append(tuple(int(v) for v in np.frombuffer(raw, dtype="<u2", count=3, offset=off)))
        off += 6
    out = []
    for shape, dt, size in zip(shapes, ("<f2", "<i4", "<f4"), (2, 4, 4)):
        cnt = int(np.prod(shape))
        out.append(np.frombuffer(raw, dtype=dt, count=cnt, offset=off).reshape(shape).copy())
        off += cnt * size
    if off != len(raw):
        raise ValueError(f"request length {len(raw)} != {off} implied by its shapes")
    return layer_idx, ids, out[0], out[1], out[2]


def pack_response(n_computed: int, result_f16: np.ndarray) -> bytes:
    r = np.ascontiguousarray(result_f16, dtype="<f2")
    return (struct.pack("<HH", n_computed, r.ndim) + np.asarray(r.shape, dtype="<u2").tobytes()
            + r.tobytes())


def unpack_response(raw: bytes):
    n, ndim = struct.unpack_from("<HH", raw, 0)
    shape = tuple(int(v) for v in np.frombuffer(raw, dtype="<u2", count=ndim, offset=4))
    res = np.frombuffer(raw, dtype="<f2", offset=4 + 2 * ndim).reshape(shape)
    return n, res


# --------------------------------------------------------------------------- #
# compute
# --------------------------------------------------------------------------- #

def local_routing(inds: np.ndarray, weights: np.ndarray, my_ids, lut: np.ndarray):
    """Routing of one node's share: each slot keeps its owner-local expert id
    when its expert is among `my_ids`, else -1 (skipped: the partition mask of
    node.py:158-163); weights pass through. -> ([T, k] int32, [T, k] fp32)."""
    k = inds.shape[-1]
    flat = inds.reshape(-1, k).astype(np.int64)
    ok = (flat >= 0) & (flat < lut.size)
    safe = np.where(ok, flat, 0)
    mine = np.zeros(lut.size, dtype=bool)
    mine[list(my_ids)] = True
    sel = ok & mine[safe]
    local = np.where(sel, lut[safe], -1).astype(np.int32)
    w = np.where(sel, weights.reshape(-1, k), 0.0).astype(np.float32)
    return local, w


class NodeCompute:
    """This node's experts of each layer, resident on one GPU.

    layers: {layer_idx: MLX-format tensors of the layer's routed experts
    ({"switch_mlp.<proj>.<kind>": [E, ...]}, all E experts or already
    restricted to `owned` -- see `sharded`)}."""

    def __init__(self, cfg: MoEConfig, owned, layers: dict, device="cuda", max_tokens: int = 256,
                 sharded: bool = False):
        # the driver keeps the shared expert; activations arrive as fp16 and
        # are read as such (tensor-core path), without rounding to bf16
        self.cfg = cfg.with_(shared_inter=0, x_dtype="f16", kernel_path="auto")
        self.owned = sorted(int(e) for e in owned)
        self.owned_set = set(self.owned)
        self.device = torch.device(device)
        self.lcfg = self.cfg.with_(num_experts=max(1, len(self.owned)))
        self.lut = np.full(cfg.num_experts, -1, np.int32)
        self.lut[self.owned] = np.arange(len(self.owned), dtype=np.int32)
        self.max_tokens = max_tokens
        self.ws = MoEBlock.new_workspace(self.lcfg, max_tokens, self.device)
        self.blocks = {}
        self.lock = threading.Lock()   # calls share one workspace and stream
        for l, lay in layers.items():
            part = lay if sharded else shard_layer(
                {k: v for k, v in lay.items() if k.startswith("switch_mlp.")}, self.owned)
            part = {k: v.to(self.device) for k, v in part.items()}
            self.blocks[int(l)] = MoEBlock(self.lcfg, weights=part, max_tokens=max_tokens,
                                           workspace=self.ws)

    def compute_partial(self, layer_idx: int, req_ids, hidden: np.ndarray, inds: np.ndarray,
                        weights: np.ndarray):
        """(n_computed, fp16 partial shaped like `hidden`): node.py:142-172."""
        my_ids = sorted(e for e in req_ids if e in self.owned_set and layer_idx in self.blocks)
        if not my_ids:
            return 0, np.zeros(hidden.shape, dtype=np.float16)
        local, w = local_routing(inds, weights, my_ids, self.lut)
        T = local.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > the node's max_tokens {self.max_tokens}")
        with self.lock, torch.cuda.device(self.device):
            x = torch.from_numpy(hidden.reshape(T, -1)).to(self.device)
            idx = torch.from_numpy(local).to(self.device)
            wt = torch.from_numpy(w).to(self.device)
            out = self.blocks[layer_idx].expert_ffn(x, idx, wt, out_dtype=torch.float32)
            res = out.to(torch.float16).cpu().numpy().reshape(hidden.shape)
        return len(my_ids), res

    def handle(self, raw: bytes) -> bytes:
        layer_idx, ids, h, i, w = unpack_request(raw)
        n, res = self.compute_partial(layer_idx, ids, h, i, w)
        return pack_response(n, res)


def create_app(node: "NodeCompute"):
    """FastAPI app serving `node` (node.py:189-198's /compute_bin). (This
    module does not postpone annotations: FastAPI reads the endpoint's
    `Request` annotation at definition time.)"""
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, Response

    app = FastAPI(title="Expert node (B200)")
    stats = {"count": 0, "time": 0.0}

    @app.post("/compute_bin")
    async def compute_bin(request: Request):
        t0 = time.time()
        body = await request.body()
        out = node.handle(body)
        stats["count"] += 1
        stats["time"] += time.time() - t0
        return Response(content=out, media_type="application/octet-stream")

    @app.get("/health")
    async def health():
        return JSONResponse({"status": "ok", "experts": len(node.owned),
                             "layers": sorted(node.blocks), "requests": stats["count"],
                             "compute_s": stats["time"], "device": str(node.device)})

    return app


def _bench(argv=None):
    """Latency of one node's share of a decode layer: in-process
    compute_partial and the full HTTP round trip on 127.0.0.1."""
    import argparse
    import json
    import socket
    import urllib.request

    from . import hrw
    from .config import PRESETS
    from .quant import synthetic_layer

    ap = argparse.ArgumentParser(description="expert-node request latency")
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--nodes", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=8)
    ap.add_argument("--reps", type=int, default=50)
    args = ap.parse_args(argv)
    cfg = PRESETS[args.model]
    roster = hrw.gpu_roster(args.nodes)
    owned = sorted(hrw.plan(roster, cfg.num_experts)[roster[0]])
    lay = synthetic_layer(cfg, seed=5, device="cuda")
    node = NodeCompute(cfg, owned, {0: lay}, max_tokens=max(args.tokens, 8))
    del lay
    rng = np.random.default_rng(0)
    T, k = args.tokens, cfg.top_k
    h = rng.standard_normal((1, T, cfg.hidden)).astype(np.float16)
    inds = np.stack([rng.choice(cfg.num_experts, k, replace=False) for _ in range(T)])[None]
    inds = inds.astype(np.int32)
    w = rng.random((1, T, k)).astype(np.float32)
    ids = sorted(set(inds.ravel().tolist()))
    req = pack_request(0, ids, h, inds, w)
    for _ in range(5):
        node.handle(req)
    t0 = time.perf_counter()
    for _ in range(args.reps):
        node.handle(req)
    inproc = (time.perf_counter() - t0) / args.reps
    import uvicorn
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    server = uvicorn.Server(uvicorn.Config(create_app(node), host="127.0.0.1", port=port,
                                           log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    while not server.started:
        time.sleep(0.05)
    url = f"http://127.0.0.1:{port}/compute_bin"

    def post():
        return urllib.request.urlopen(urllib.request.Request(
            url, data=req, headers={"Content-Type": "application/octet-stream"}), timeout=60).read()
    for _ in range(5):
        post()
    t0 = time.perf_counter()
    for _ in range(args.reps):
        post()
    http = (time.perf_counter() - t0) / args.reps
    server.should_exit = True
    th.join(timeout=10)
    print(json.dumps({"model": cfg.name, "nodes": args.nodes, "owned_experts": len(owned),
                      "tokens": T, "request_bytes": len(req), "handle_ms": inproc * 1e3,
                      "http_round_trip_ms": http * 1e3}))


if __name__ == "__main__":
    _bench()
