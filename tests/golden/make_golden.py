"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a checkout where the reference project is available (it is read, not
copied):
    python tests/golden/make_golden.py --reference /path/to/expert-sniper

Fixtures
  hrw_plans.json       expert_network.hrw.plan(["gpu0".."gpuN-1"], E) and the
                       owner of every expert, for N in 1, 2, 4, 8 and E in 8,
                       64, 128, 512 (src/expert_network/hrw.py:11-30), plus a
                       roster of free-form node ids.
  protocol_sizes.json  byte sizes of expert_network.protocol.pack_request /
                       pack_response for the decode shapes, and one full
                       request/response byte string (hex) of a tiny case
                       (src/expert_network/protocol.py:1-65).
The reference's MLX arithmetic cannot be imported here (MLX is absent), so no
MLX output vectors are generated.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (read, never copied)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "src"))
    sys.dont_write_bytecode = True
    from expert_network import hrw, protocol  # the reference's own modules

    plans = []
    for n in (1, 2, 4, 8):
        roster = [f"gpu{i}" for i in range(n)]
        for e in (8, 64, 128, 512):
            plans.append({"roster": roster, "num_experts": e,
                          "plan": hrw.plan(roster, e),
                          "owners": [hrw.owner(roster, i) for i in range(e)]})
    roster = ["http://10.0.0.1:8000", "node-b", "mac-mini"]
    plans.append({"roster": roster, "num_experts": 64, "plan": hrw.plan(roster, 64),
                  "owners": [hrw.owner(roster, i) for i in range(64)],
                  "partition_node-b": hrw.partition(roster, "node-b", 64)})
    with open(os.path.join(HERE, "hrw_plans.json"), "w") as f:
        json.dump({"source": "src/expert_network/hrw.py", "plans": plans}, f, indent=0)

    sizes = []
    for D, k, T in ((2048, 8, 1), (2048, 8, 8), (2048, 10, 4), (4096, 8, 256)):
        h = np.zeros((1, T, D), np.float16)
        inds = np.zeros((1, T, k), np.int32)
        w = np.zeros((1, T, k), np.float32)
        req = protocol.pack_request(3, list(range(k)), h, inds, w)
        resp = protocol.pack_response(k, h)
        sizes.append({"D": D, "k": k, "T": T, "request_bytes": len(req),
                      "response_bytes": len(resp)})
    rng = np.random.default_rng(0)
    h = rng.standard_normal((1, 2, 8)).astype(np.float16)
    inds = np.array([[[1, 5], [2, 5]]], np.int32)
    w = np.array([[[0.75, 0.25], [0.5, 0.5]]], np.float32)
    req = protocol.pack_request(7, [5, 1, 2], h, inds, w)
    resp = protocol.pack_response(2, h)
    with open(os.path.join(HERE, "protocol_sizes.json"), "w") as f:
        json.dump({"source": "src/expert_network/protocol.py", "sizes": sizes,
                   "tiny": {"layer": 7, "expert_ids": [5, 1, 2], "hidden": h.tolist(),
                            "inds": inds.tolist(), "weights": w.tolist(),
                            "request_hex": req.hex(), "response_hex": resp.hex()}},
                  f, indent=1)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
