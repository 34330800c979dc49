"""Execute the reference's own MoE-block Python on the MLX stand-in.

Test infrastructure. The reference project's `make_forward`
(src/mlx_expert_sniper/generate.py:92-187) and `run_expert_ffn`
(src/mlx_expert_sniper/engine.py:15-42) are imported from a checkout of the
reference, unmodified, with `tests/mlx_standin` providing `mlx.core`,
`mlx.nn`, `mlx.utils` and `mlx_lm.models.base`. A one-layer fake engine
feeds them:
  * the embedding returns zeros and attention returns zeros, so the residual
    stream before the MoE block is exactly 0 and the layer's output is the
    block's output in the dtype MLX would give it;
  * post_attention_layernorm returns the block input x (bf16);
  * the router `layer.mlp.gate` returns the given bf16 logits;
  * the reader's LRU is the reference's own LRUExpertCache
    (expert_io.py:172-225) holding the cached experts of layer 0, so the
    routing-bias mask is built by the reference's code (generate.py:124-129);
  * with a shared expert, `shared_expert` is a quantised SwiGLU MLP and
    `shared_expert_gate` a bf16 Linear(D, 1), as in mlx_lm's Qwen3-Next block.
`run_expert_ffn` is wrapped (not changed) to record the routing it receives.

Case inputs are seeded and generated on the CPU (torch's CPU generator), so a
case reproduces anywhere from its seeds.
"""
from __future__ import annotations

import contextlib
import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
STANDIN = os.path.join(HERE, "mlx_standin")

_PREFIXES = ("mlx", "mlx_lm", "mlx_expert_sniper")


def reference_root(explicit: str = None):
    """The reference checkout: `explicit`, $EXPERT_SNIPER_REFERENCE, or a
    directory named `reference` beside this repository; None if absent."""
    for c in (explicit, os.environ.get("EXPERT_SNIPER_REFERENCE"),
              os.path.join(ROOT, os.pardir, "reference")):
        if c and os.path.isfile(os.path.join(c, "src", "mlx_expert_sniper", "generate.py")):
            return os.path.abspath(c)
    return None


@contextlib.contextmanager
def reference_modules(ref_root: str):
    """(generate, engine, expert_io, mlx.core, mlx.nn) imported from the
    reference with the stand-in; sys.path and sys.modules are restored."""
    saved_path = list(sys.path)
    saved_mods = {k: v for k, v in sys.modules.items() if k.split(".")[0] in _PREFIXES}
    saved_bc = sys.dont_write_bytecode
    for k in saved_mods:
        del sys.modules[k]
    sys.dont_write_bytecode = True
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, STANDIN)
    try:
        mx = importlib.import_module("mlx.core")
        nn = importlib.import_module("mlx.nn")
        gen = importlib.import_module("mlx_expert_sniper.generate")
        eng = importlib.import_module("mlx_expert_sniper.engine")
        eio = importlib.import_module("mlx_expert_sniper.expert_io")
        assert os.path.dirname(mx.__file__).startswith(STANDIN), "a real mlx shadowed the stand-in"
        yield gen, eng, eio, mx, nn
    finally:
        for k in [k for k in sys.modules if k.split(".")[0] in _PREFIXES]:
            del sys.modules[k]
        sys.modules.update(saved_mods)
        sys.path[:] = saved_path
        sys.dont_write_bytecode = saved_bc


class _Obj:
    pass


def case_inputs(case: dict):
    """Seeded inputs of a case: (cfg, layer tensors, x, logits, shared gate
    weight, cache-bias vector or None, cached ids). With scales "bf16" the
    layer's scales and biases are rounded to bf16 (the dtype of real MLX
    checkpoints); they stay exactly representable in fp16."""
    from expert_sniper_b200 import PRESETS
    from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
    cfg = PRESETS[case["preset"]]
    lay = synthetic_layer(cfg, seed=case["layer_seed"])
    x, _, logits, sg = synthetic_inputs(cfg, case["T"], seed=case["input_seed"])
    if case.get("scales", "f16") == "bf16":
        for name in list(lay):
            if name.endswith(("scales", "biases")):
                lay[name] = lay[name].to(torch.bfloat16)
    bias = float(case.get("bias", 0.0))
    cb, cached = (None, [])
    if bias > 0:
        cb, cached = cache_bias_vector(cfg.num_experts, bias, case.get("cache_seed", 0))
    return cfg, lay, x, logits, sg, cb, cached


def fp16_layer(lay: dict) -> dict:
    """The layer with bf16 scales/biases given as fp16 (exact for these
    values): the form the kernels and the C oracle take."""
    return {k: (v.to(torch.float16) if v.dtype == torch.bfloat16 else v) for k, v in lay.items()}


def run_reference_block(mods, cfg, lay, x, logits, sg, bias: float, cached):
    """One MoE block through the reference's make_forward + run_expert_ffn.
    Returns dict(inds [T, k] int64 as the reference's argpartition left them,
    scores [T, k] float32 values, scores_dtype, out [T, D] float32 values,
    out_dtype)."""
    gen, eng, eio, mx, nn = mods
    T, D = x.shape
    E = cfg.num_experts
    X = mx.array(x[None].clone())
    L = mx.array(logits[None].clone())
    routed = {k: v for k, v in lay.items() if k.startswith("switch_mlp.")}
    expert_cache = {}

    def get_experts(layer_idx, ids):
        out = {}
        for e in ids:
            if e not in expert_cache:
                expert_cache[e] = {k: mx.array(v[e]) for k, v in routed.items()}
            out[e] = expert_cache[e]
        return out

    reader = _Obj()
    reader.lru = eio.LRUExpertCache(max_experts=max(1, len(cached)))
    for e in cached:
        reader.lru.put(0, int(e), None)
    reader.get_experts = get_experts
    reader.prefetch_experts = lambda layer_idx, ids: None

    coact = _Obj()
    coact.ready = False
    coact.record_layer = lambda i, ids: None
    coact.end_token = lambda: None

    mlp = _Obj()
    mlp.gate = lambda n: L
    mlp.top_k = cfg.top_k
    mlp.norm_topk_prob = cfg.norm_topk_prob
    if cfg.has_shared:
        def qproj(name):
            return (mx.array(lay[f"shared_expert.{name}.weight"]),
                    mx.array(lay[f"shared_expert.{name}.scales"]),
                    mx.array(lay[f"shared_expert.{name}.biases"]))
        g_w, u_w, d_w = qproj("gate_proj"), qproj("up_proj"), qproj("down_proj")

        def shared_expert(n):
            g = mx.quantized_matmul(n, *g_w, transpose=True, group_size=64, bits=4)
            u = mx.quantized_matmul(n, *u_w, transpose=True, group_size=64, bits=4)
            return mx.quantized_matmul(nn.silu(g) * u, *d_w, transpose=True, group_size=64,
                                       bits=4)
        sgw = mx.array(sg[:, None].clone())   # Linear(D, 1).weight.T, bf16
        mlp.shared_expert = shared_expert
        mlp.shared_expert_gate = lambda n: n @ sgw

    layer = _Obj()
    layer.input_layernorm = lambda h: h
    layer.self_attn = lambda n, mask=None, cache=None: mx.zeros(n.shape, mx.bfloat16)
    layer.post_attention_layernorm = lambda h: X
    layer.mlp = mlp

    model = _Obj()
    model.model = _Obj()
    model.model.embed_tokens = lambda inp: mx.zeros((1, T, D), mx.bfloat16)
    model.model.layers = [layer]
    model.model.norm = lambda h: h
    model.lm_head = lambda h: h

    engine = _Obj()
    engine.model = model
    engine.num_layers = 1
    engine.num_experts = E
    engine.cache = [None]
    engine.reader = reader
    engine.coact = coact

    rec = {}
    orig = eng.run_expert_ffn

    def recording(x_, expert_data, top_k_indices, top_k_weights):
        out = orig(x_, expert_data, top_k_indices, top_k_weights)
        rec["inds"] = np.array(top_k_indices).reshape(T, -1).astype(np.int64)
        rec["scores"] = np.array(top_k_weights).reshape(T, -1).astype(np.float32)
        rec["scores_dtype"] = top_k_weights.dtype.name
        return out

    eng.run_expert_ffn = recording
    try:
        forward = gen.make_forward(engine, bias=bias)
        h = forward(None)
    finally:
        eng.run_expert_ffn = orig
    rec["out"] = np.array(h).reshape(T, D).astype(np.float32)
    rec["out_dtype"] = h.dtype.name
    return rec


# The cases pinned by tests/golden/reference_block.npz (made by
# tests/golden/make_reference_vectors.py): the reference configurations'
# shapes, with and without the cache bias, fp16 scales (the configurations'
# format) and bf16 scales (real MLX checkpoints: the block's intermediates
# then stay bf16), and the shared expert.
CASES = [
    {"name": "olmoe_T4_f16", "preset": "olmoe-1b-7b", "layer_seed": 11, "input_seed": 12,
     "T": 4, "bias": 0.0, "scales": "f16"},
    {"name": "qwen3_30b_T8_bias_f16", "preset": "qwen3-30b-a3b", "layer_seed": 21,
     "input_seed": 22, "T": 8, "bias": 0.5, "cache_seed": 23, "scales": "f16"},
    {"name": "qwen3_30b_T64_bias_f16", "preset": "qwen3-30b-a3b", "layer_seed": 21,
     "input_seed": 27, "T": 64, "bias": 0.5, "cache_seed": 28, "scales": "f16"},
    {"name": "qwen3_30b_T8_bf16", "preset": "qwen3-30b-a3b", "layer_seed": 21,
     "input_seed": 24, "T": 8, "bias": 0.0, "scales": "bf16"},
    {"name": "qwen3_30b_T4_bias_bf16", "preset": "qwen3-30b-a3b", "layer_seed": 21,
     "input_seed": 25, "T": 4, "bias": 0.5, "cache_seed": 26, "scales": "bf16"},
    {"name": "qwen3_next_T4_shared_f16", "preset": "qwen3-next-80b-a3b", "layer_seed": 31,
     "input_seed": 32, "T": 4, "bias": 0.0, "scales": "f16"},
    {"name": "qwen3_30b_T16_bias_bf16", "preset": "qwen3-30b-a3b", "layer_seed": 21,
     "input_seed": 41, "T": 16, "bias": 0.5, "cache_seed": 42, "scales": "bf16"},
    {"name": "olmoe_T16_f16", "preset": "olmoe-1b-7b", "layer_seed": 11, "input_seed": 43,
     "T": 16, "bias": 0.0, "scales": "f16"},
]
