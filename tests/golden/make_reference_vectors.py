"""Generate tests/golden/reference_block.{npz,json}: outputs of the reference's
own MoE-block code.

    python tests/golden/make_reference_vectors.py --reference /path/to/expert-sniper

For each case of tests/_refexec.CASES the reference's make_forward layer loop
(src/mlx_expert_sniper/generate.py:92-187) and run_expert_ffn
(src/mlx_expert_sniper/engine.py:15-42) run unmodified on the MLX stand-in
(tests/mlx_standin) with seeded CPU inputs. Recorded per case: the routing
the reference handed to run_expert_ffn (indices in its argpartition order,
scores and their dtype), the block output and its dtype (rows `rows` only for
the larger batches), and the measured distance of the fp32 oracle from it:
  oracle_block_rel  oracle routing weights (fp32) on the reference's indices
  oracle_ffn_rel    the reference's own scores (its dtype's values)
both as max|oracle - reference| / RMS(reference).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests import _refexec as rx  # noqa: E402
from oracle import c_oracle as co  # noqa: E402
from oracle import moe_oracle as mo  # noqa: E402

MAX_ROWS = 16   # output rows stored per case (rows are independent tokens)


def oracle_distances(cfg, lay, x, logits, sg, cb, rec, rows):
    lay_np = {k: v.numpy() for k, v in rx.fp16_layer(lay).items()}
    lg = logits.float().numpy()
    z = lg + (cb.numpy()[None] if cb is not None else 0.0)
    p = mo.softmax_f32(z)
    inds = rec["inds"].astype(np.int32)
    w = np.take_along_axis(p, inds.astype(np.int64), -1)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdims=True)
    xf = x.float().numpy()
    sgn = None if sg is None else sg.float().numpy()
    ref = rec["out"][rows]
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    blk = co.expert_ffn(xf[rows], lay_np, inds[rows], w[rows].astype(np.float32), sgn)
    ffn = co.expert_ffn(xf[rows], lay_np, inds[rows], rec["scores"][rows], sgn)
    ok, n_exact, n_tie, _ = mo.topk_parity(inds, lg, None if cb is None else cb.numpy(),
                                           cfg.top_k)
    return {"oracle_block_rel": float(np.abs(blk - ref).max() / rms),
            "oracle_ffn_rel": float(np.abs(ffn - ref).max() / rms),
            "topk_sets_ok": bool(ok), "topk_exact_tokens": int(n_exact),
            "topk_tie_tokens": int(n_tie), "out_rms": rms}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (read, never copied)")
    args = ap.parse_args()
    root = rx.reference_root(args.reference)
    if root is None:
        raise SystemExit(f"no reference checkout at {args.reference}")
    arrays, meta = {}, {"source": "src/mlx_expert_sniper/generate.py:92-187 (make_forward) and "
                                  "src/mlx_expert_sniper/engine.py:15-42 (run_expert_ffn), "
                                  "executed unmodified on tests/mlx_standin", "cases": []}
    with rx.reference_modules(root) as mods:
        for case in rx.CASES:
            cfg, lay, x, logits, sg, cb, cached = rx.case_inputs(case)
            rec = rx.run_reference_block(mods, cfg, lay, x, logits, sg, case.get("bias", 0.0),
                                         cached)
            T = case["T"]
            rows = np.arange(T) if T <= MAX_ROWS else np.sort(
                np.random.default_rng(case["input_seed"]).choice(T, MAX_ROWS, replace=False))
            n = case["name"]
            arrays[f"{n}/inds"] = rec["inds"].astype(np.int32)
            arrays[f"{n}/scores"] = rec["scores"]
            arrays[f"{n}/rows"] = rows.astype(np.int32)
            arrays[f"{n}/out"] = rec["out"][rows]
            d = oracle_distances(cfg, lay, x, logits, sg, cb, rec, rows)
            entry = dict(case, scores_dtype=rec["scores_dtype"], out_dtype=rec["out_dtype"],
                         cached_ids=[int(e) for e in cached], **d)
            meta["cases"].append(entry)
            print(json.dumps(entry), flush=True)
    np.savez_compressed(os.path.join(HERE, "reference_block.npz"), **arrays)
    with open(os.path.join(HERE, "reference_block.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
