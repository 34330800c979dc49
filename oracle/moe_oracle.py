"""CPU restatement of Expert Sniper's MoE block, in numpy fp32.

TEST INFRASTRUCTURE ONLY. This module is the checker: the parity tests, the
smoke check and bench.py's CPU-baseline / reference arm may import it; the
product path (expert_sniper_b200) never does, and has no CPU fallback.

What it restates (file:line in the reference project):
  route        src/mlx_expert_sniper/generate.py:122-136 — additive cache bias
               (fp32 mask, only when bias > 0), softmax(precise) in fp32,
               argpartition top-k, take_along_axis, optional renormalisation.
               Same math in engine_30b.py:158-165 and
               models/qwen4_exp.py:463-472.
  expert_ffn   src/mlx_expert_sniper/engine.py:15-42 run_expert_ffn — per
               (token, slot): gate/up gather_qmm (transpose=True), silu(g)*u,
               down gather_qmm, weighted sum over the k slots; plus the shared
               expert of generate.py:173-178 (sigmoid(gate(x)) * shared(x)).
  partial      src/expert_network/node.py:142-172 compute_partial — weights
               masked to a partition; experts outside it contribute nothing.
  combine_nodes src/expert_network/reader.py:278-292 — partials summed in fp32
               in fixed node order.
  dequant      the MLX affine format (engine.py:12-13, download.py:73-77):
               w = scale * q + bias per 64-column group, q in bits 4*(k%8) of
               uint32 word k//8.

Dtype notes. The reference runs the block in the model dtype (bf16) inside
MLX; MLX is not available here, so this oracle computes in fp32 and leaves
output rounding to the caller. The one place where the reference dtype is
restated exactly is the top-k selection key (`reference_selection_keys`):
without a bias the key is the softmax output rounded to bf16 (softmax keeps
its input dtype), with a bias it is the fp32 softmax of the promoted logits.
That key decides which near-ties are legitimate top-k disagreements.
"""
from __future__ import annotations

import numpy as np

GROUP = 64


# --------------------------------------------------------------------------- #
# dtype helpers
# --------------------------------------------------------------------------- #

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (NaN kept as NaN)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def round_bf16(a: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


def bf16_half_ulp(a: np.ndarray) -> np.ndarray:
    """Half a bf16 ulp at |a| (the most a correct round-to-bf16 can move a)."""
    a = np.abs(np.asarray(a, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return np.float32(2.0) ** (e - 8)


# --------------------------------------------------------------------------- #
# format
# --------------------------------------------------------------------------- #

def unpack_codes(words: np.ndarray) -> np.ndarray:
    """uint32 (or int32 bits) [..., N, K/8] -> uint8 codes [..., N, K]."""
    w = np.asarray(words).view(np.uint32)
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    codes = (w[..., None] >> shifts) & 0xF
    return codes.reshape(*w.shape[:-1], w.shape[-1] * 8).astype(np.uint8)


def dequant(words, scales, biases) -> np.ndarray:
    """MLX affine dequantisation: fp32 [..., N, K] = scale * q + bias."""
    codes = unpack_codes(words).astype(np.float32)
    *lead, n, k = codes.shape
    cg = codes.reshape(*lead, n, k // GROUP, GROUP)
    s = np.asarray(scales, dtype=np.float16).astype(np.float32)[..., None]
    b = np.asarray(biases, dtype=np.float16).astype(np.float32)[..., None]
    return (cg * s + b).reshape(*lead, n, k)


# --------------------------------------------------------------------------- #
# router (generate.py:122-136)
# --------------------------------------------------------------------------- #

def softmax_f32(z: np.ndarray) -> np.ndarray:
    z = z.astype(np.float32)
    m = z.max(axis=-1, keepdims=True)
    e = np.exp(z - m)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def route(logits: np.ndarray, cache_bias, k: int, renorm: bool):
    """logits [T, E] (fp32 values of the bf16 logits, or fp32 logits),
    cache_bias [E] fp32 or None. Returns (idx [T, k] int32 in descending
    probability order, weights [T, k] fp32, probs [T, E] fp32).

    The bias is added only when given (the reference adds it only for
    bias > 0, generate.py:124); softmax in fp32 (`precise=True`); ties in the
    selection go to the lower expert id (argpartition's tie order is
    unspecified)."""
    z = logits.astype(np.float32)
    if cache_bias is not None:
        z = z + np.asarray(cache_bias, dtype=np.float32)[None, :]
    probs = softmax_f32(z)
    # stable descending sort on the biased fp32 logits: equal keys keep the
    # lower index first
    order = np.argsort(-z, axis=-1, kind="stable")
    idx = order[:, :k].astype(np.int32)
    w = np.take_along_axis(probs, idx, axis=-1).astype(np.float32)
    if renorm:
        w = (w / w.sum(axis=-1, keepdims=True)).astype(np.float32)
    return idx, w, probs


def reference_selection_keys(logits: np.ndarray, cache_bias) -> np.ndarray:
    """The values the reference's argpartition ranks, in its own dtype:
    bf16 logits + fp32 mask promote to fp32, so with a bias the keys are fp32
    probabilities; without one softmax returns bf16, so the keys are the fp32
    softmax rounded to bf16 (generate.py:124-133)."""
    if cache_bias is not None:
        return softmax_f32(logits.astype(np.float32) + np.asarray(cache_bias, np.float32)[None])
    return round_bf16(softmax_f32(logits.astype(np.float32)))


def topk_parity(our_idx: np.ndarray, logits: np.ndarray, cache_bias, k: int,
                logit_gap: float = 1e-5):
    """Compare our per-token top-k index SETS with the reference's.

    A token's sets may differ only at a near-tie of the reference: the k-th
    and (k+1)-th selection keys (in the reference dtype) are equal, or the
    biased logits at the boundary are within `logit_gap`. Every expert we
    picked must then rank no lower than the reference's tied k-th key.
    Returns (ok, n_exact, n_tie, bad_tokens)."""
    keys = reference_selection_keys(logits, cache_bias)
    z = logits.astype(np.float32)
    if cache_bias is not None:
        z = z + np.asarray(cache_bias, np.float32)[None]
    T, E = keys.shape
    n_exact = n_tie = 0
    bad = []
    for t in range(T):
        ref_order = np.argsort(-keys[t], kind="stable")
        ref_set = set(int(e) for e in ref_order[:k])
        ours = set(int(e) for e in our_idx[t])
        if ours == ref_set:
            n_exact += 1
            continue
        if len(ours) != k or min(ours) < 0 or max(ours) >= E:
            bad.append(t)
            continue
        kth = keys[t, ref_order[k - 1]]
        zk = z[t, ref_order[k - 1]]
        # every disagreeing expert (either side) must be tied with the k-th key
        diff = ours.symmetric_difference(ref_set)
        tied = all(keys[t, e] == kth or abs(float(z[t, e]) - float(zk)) < logit_gap
                   for e in diff)
        # and nothing we picked may rank strictly below the tie
        ranked_ok = all(keys[t, e] >= kth or abs(float(z[t, e]) - float(zk)) < logit_gap
                        for e in ours)
        if tied and ranked_ok:
            n_tie += 1
        else:
            bad.append(t)
    return (not bad), n_exact, n_tie, bad


# --------------------------------------------------------------------------- #
# expert FFN + combine (engine.py:15-42, generate.py:173-178)
# --------------------------------------------------------------------------- #

def silu(a):
    return a / (1.0 + np.exp(-a))


def sigmoid(a):
    return 1.0 / (1.0 + np.exp(-a))


def _expert_mats(layer: dict, prefix: str, e=None):
    mats = []
    for proj in ("gate_proj", "up_proj", "down_proj"):
        w = layer[f"{prefix}.{proj}.weight"]
        s = layer[f"{prefix}.{proj}.scales"]
        b = layer[f"{prefix}.{proj}.biases"]
        if e is not None:
            w, s, b = w[e], s[e], b[e]
        mats.append(dequant(w, s, b))
    return mats


def _swiglu_mlp(X, mats):
    wg, wu, wd = mats
    g = X @ wg.T
    u = X @ wu.T
    h = silu(g) * u
    return (h @ wd.T).astype(np.float32)


def expert_ffn(x: np.ndarray, layer: dict, idx: np.ndarray, w: np.ndarray,
               shared_gate_w=None) -> np.ndarray:
    """x [T, D] fp32 (values of the bf16 input), layer: numpy arrays named as
    the reference names them ({"switch_mlp.<proj>.<weight|scales|biases>":
    [E, ...]}, optional "shared_expert.*" without the expert axis),
    idx [T, k] int (-1 = slot masked off), w [T, k] fp32.

    out[t] = sum over slots j with idx >= 0, in ascending expert id order, of
    w[t, j] * down(silu(gate(x_t)) * up(x_t)); then, with a shared expert,
    + sigmoid(x_t . shared_gate_w) * shared(x_t) (gate 1 without a weight).
    Computed in fp32, returned in fp32."""
    x = x.astype(np.float32)
    T, D = x.shape
    k = idx.shape[1]
    y = np.zeros((T, k, D), dtype=np.float32)
    for e in sorted(set(int(v) for v in idx.ravel() if v >= 0)):
        tt, jj = np.nonzero(idx == e)
        y[tt, jj] = _swiglu_mlp(x[tt], _expert_mats(layer, "switch_mlp", e))
    out = np.zeros((T, D), dtype=np.float32)
    for t in range(T):
        for j in np.argsort(idx[t], kind="stable"):
            if idx[t, j] >= 0:
                out[t] += np.float32(w[t, j]) * y[t, j]
    if "shared_expert.gate_proj.weight" in layer:
        sh = _swiglu_mlp(x, _expert_mats(layer, "shared_expert"))
        if shared_gate_w is not None:
            gate = sigmoid(x @ np.asarray(shared_gate_w, np.float32)).astype(np.float32)
        else:
            gate = np.ones((T,), np.float32)
        out += gate[:, None] * sh
    return out


def moe_block(x, logits, layer, k, renorm, cache_bias=None, shared_gate_w=None):
    """route + expert_ffn: the MoE part of one layer of make_forward
    (generate.py:122-181). Returns (out fp32 [T, D], idx, w)."""
    idx, w, _ = route(logits, cache_bias, k, renorm)
    return expert_ffn(x, layer, idx, w, shared_gate_w), idx, w


# --------------------------------------------------------------------------- #
# expert-parallel semantics (node.py:142-172, reader.py:278-292, hrw.py)
# --------------------------------------------------------------------------- #

def partial(x, layer, idx, w, partition) -> np.ndarray:
    """One owner's partial: slots whose expert is outside `partition` are
    masked off (weight x 0 in node.py:161-163; here idx -> -1, which is the
    same sum without the zero terms). fp32."""
    part = set(int(e) for e in partition)
    masked = np.where(np.isin(idx, list(part)), idx, -1).astype(np.int32)
    return expert_ffn(x, {k_: v for k_, v in layer.items() if k_.startswith("switch_mlp")},
                      masked, w)


def combine_nodes(partials) -> np.ndarray:
    """Sum of per-owner partials in fixed owner order, fp32 (reader.py:278-286)."""
    total = None
    for p in partials:
        p = np.asarray(p, dtype=np.float32)
        total = p.copy() if total is None else total + p
    return total


def ep_mask(idx: np.ndarray, w: np.ndarray, owner, local_id, world: int):
    """Per-destination routing masks: for rank d, slot j of token t keeps the
    owner-local id of its expert when d owns it, else -1 (the partition mask
    of compute_partial, node.py:158-163). Returns ([world, T, k] int32,
    [world, T, k] fp32)."""
    owner = np.asarray(owner)
    local_id = np.asarray(local_id)
    T, k = idx.shape
    send_idx = np.full((world, T, k), -1, np.int32)
    for d in range(world):
        ok = idx >= 0
        mine = ok & (owner[np.where(ok, idx, 0)] == d)
        send_idx[d] = np.where(mine, local_id[np.where(ok, idx, 0)], -1)
    send_w = np.broadcast_to(w.astype(np.float32), (world, T, k)).copy()
    return send_idx, send_w
