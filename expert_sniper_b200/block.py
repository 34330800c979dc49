"""Host-side mirror of the reference's MoE-block interface, on the CUDA library.

Reference call surface this mirrors:
  * run_expert_ffn(x, expert_data, top_k_indices, top_k_weights)
      src/mlx_expert_sniper/engine.py:15-42 (same in engine_30b.py,
      engine_next.py, engine_qwen4exp.py)
  * the router of make_forward's layer loop, generate.py:122-136
    (bias mask from reader.lru.cached_ids, softmax(precise), argpartition
    top-k, optional renormalisation)
  * the shared expert add, generate.py:173-178

`MoEBlock` is the fast path: a layer's experts are repacked once into the
device layout and every call is one C-ABI call (es_moe_forward), made
through the registered PyTorch operator torch.ops.expert_sniper.moe_forward_out
(ops.py). The module
level `run_expert_ffn` keeps the reference's per-call signature (a dict of
active experts) for drop-in use; it re-stacks the experts it is given on
every call, exactly like the reference's stack_proj.

Everything runs through libes_moe.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native
from . import ops  # noqa: F401  (registers torch.ops.expert_sniper.*)
from .config import KERNEL_PATHS, MoEConfig
from .quant import PROJS

_DT_CODE = {torch.bfloat16: _native.ES_DTYPE_BF16, torch.float32: _native.ES_DTYPE_F32}


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the MoE block has no CPU path)")


def _proj(weights: dict, prefix: str, proj: str) -> "_native.CMlxProj":
    names = [f"{prefix}.{proj}.{k}" for k in ("weight", "scales", "biases")]
    ts = [weights[n] for n in names]
    for n, t in zip(names, ts):
        _need_cuda(t, n)
        if not t.is_contiguous():
            raise ValueError(f"{n} must be contiguous")
    return _native.CMlxProj(*(t.data_ptr() for t in ts))


def prepare_packed(cfg: MoEConfig, weights: dict, out: torch.Tensor = None) -> torch.Tensor:
    """Repack a layer's MLX tensors ({"switch_mlp.<proj>.<kind>": [E, ...]},
    plus "shared_expert.*" with a shared expert) into the device layout.
    Returns a uint8 tensor of es_moe_packed_bytes bytes."""
    ccfg = cfg.to_c()
    nbytes = _native.packed_bytes(ccfg)
    dev = weights["switch_mlp.gate_proj.weight"].device
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    if out.numel() < nbytes or out.data_ptr() % 256:
        raise ValueError("packed buffer too small or not 256-byte aligned")
    layer = _native.CMlxLayer()
    layer.gate = _proj(weights, "switch_mlp", "gate_proj")
    layer.up = _proj(weights, "switch_mlp", "up_proj")
    layer.down = _proj(weights, "switch_mlp", "down_proj")
    if cfg.has_shared:
        layer.shared_gate_proj = _proj(weights, "shared_expert", "gate_proj")
        layer.shared_up_proj = _proj(weights, "shared_expert", "up_proj")
        layer.shared_down_proj = _proj(weights, "shared_expert", "down_proj")
    with torch.cuda.device(dev):
        _native.check("es_moe_prepare", _native.lib().es_moe_prepare(
            ctypes.byref(ccfg), ctypes.byref(layer), out.data_ptr(), out.numel(), _stream(dev)))
    return out


def uses_tensor_path(cfg: MoEConfig, T: int) -> bool:
    """Whether a call with T tokens runs the tensor-core (tcgen05) expert
    kernels: the rule of es_moe_cfg.kernel_path in include/es_moe.h."""
    return ffn_kernels(cfg, T) != "decode"


# most tokens the fused tiny-batch kernel takes (kSmallMaxTokens, es_kernels.cuh)
SMALL_MAX_TOKENS = 16


def ffn_kernels(cfg: MoEConfig, T: int) -> str:
    """The expert-FFN kernels a call with T tokens runs ("fused", "decode",
    "tensor" or "tensor-small"): the rule of es_moe_cfg.kernel_path in
    include/es_moe.h (automatic: the fused tiny-batch kernel for T <= 16;
    otherwise by the average pairs per routed expert p = T k / E, decode
    below 4, 32-token tiles up to 48, 128-token tiles above, tensor-core
    kernels only from T = 64)."""
    fused_fits = (cfg.x_dtype == "bf16" and 1 <= T <= SMALL_MAX_TOKENS and cfg.hidden <= 4096
                  and T * cfg.top_k <= 512)
    if cfg.kernel_path == "fused":
        return "fused" if fused_fits else "decode"
    if cfg.kernel_path != "auto":
        return cfg.kernel_path
    pk = T * cfg.top_k
    if T >= 64 and pk > 48 * cfg.num_experts:
        return "tensor"
    if T >= 64 and pk >= 4 * cfg.num_experts:
        return "tensor-small"
    if cfg.x_dtype == "f16":
        return "tensor-small"
    return "fused" if fused_fits else "decode"


class MoEBlock:
    """One layer's MoE block with device-resident packed experts.

    forward(x, logits, cache_bias) == the MoE part of one make_forward layer:
    router (+ cache bias) -> top-k -> experts -> combine (+ shared expert).
    """

    def __init__(self, cfg: MoEConfig, weights: dict = None, packed: torch.Tensor = None,
                 shared_gate_w: torch.Tensor = None, max_tokens: int = 64,
                 workspace: torch.Tensor = None):
        if (weights is None) == (packed is None):
            raise ValueError("pass exactly one of weights= or packed=")
        self.cfg = cfg
        self.ccfg = cfg.to_c()
        self.packed = prepare_packed(cfg, weights) if packed is None else packed
        if self.packed.numel() < _native.packed_bytes(self.ccfg):
            raise ValueError("packed tensor smaller than es_moe_packed_bytes")
        self.device = self.packed.device
        _need_cuda(self.packed, "packed")
        self.shared_gate_w = None
        if shared_gate_w is not None:
            self.shared_gate_w = shared_gate_w.to(self.device, torch.bfloat16).contiguous()
        self._ws = None
        self._ws_tokens = -1
        if workspace is not None:
            # a workspace shared by blocks that run one after another on one stream
            if workspace.numel() < _native.workspace_bytes(self.ccfg, max_tokens):
                raise ValueError("workspace smaller than es_moe_workspace_bytes(max_tokens)")
            self._ws = workspace
            self._ws_tokens = max_tokens
        else:
            self.reserve(max_tokens)

    # -- workspace --------------------------------------------------------
    def reserve(self, max_tokens: int) -> None:
        """Grow the workspace to `max_tokens` tokens (zero-filled, as the
        C ABI requires before first use)."""
        if max_tokens <= self._ws_tokens:
            return
        nb = _native.workspace_bytes(self.ccfg, max_tokens)
        self._ws = torch.zeros(nb, dtype=torch.uint8, device=self.device)
        self._ws_tokens = max_tokens

    @staticmethod
    def new_workspace(cfg: MoEConfig, max_tokens: int, device="cuda") -> torch.Tensor:
        nb = _native.workspace_bytes(cfg.to_c(), max_tokens)
        return torch.zeros(nb, dtype=torch.uint8, device=device)

    @property
    def workspace(self) -> torch.Tensor:
        return self._ws

    def read_device_error(self, clear: bool = True) -> int:
        v = ctypes.c_uint32(0)
        _native.check("es_moe_read_error", _native.lib().es_moe_read_error(
            self._ws.data_ptr(), int(clear), ctypes.byref(v), _stream(self.device)))
        return v.value

    # -- calls --------------------------------------------------------------
    def _flat(self, x: torch.Tensor, width: int, name: str) -> torch.Tensor:
        _need_cuda(x, name)
        if x.shape[-1] != width:
            raise ValueError(f"{name}: last dim {x.shape[-1]} != {width}")
        return x.reshape(-1, width).contiguous()

    def route(self, logits: torch.Tensor, cache_bias: torch.Tensor = None):
        """Top-k expert ids [.., k] int32 (descending probability) and weights
        [.., k] fp32 for router logits [.., E] (bf16 or fp32)."""
        cfg = self.cfg
        lg = self._flat(logits, cfg.num_experts, "logits")
        if lg.dtype not in (torch.bfloat16, torch.float32):
            lg = lg.float()
        T = lg.shape[0]
        idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, cfg.top_k), dtype=torch.float32, device=self.device)
        bias = None if cache_bias is None else cache_bias.to(self.device, torch.float32).contiguous()
        _native.check("es_moe_route", _native.lib().es_moe_route(
            ctypes.byref(self.ccfg), lg.data_ptr(), _DT_CODE[lg.dtype], _ptr(bias), T,
            idx.data_ptr(), w.data_ptr(), _stream(self.device)))
        lead = logits.shape[:-1]
        return idx.reshape(*lead, cfg.top_k), w.reshape(*lead, cfg.top_k)

    def forward(self, x: torch.Tensor, logits: torch.Tensor, cache_bias: torch.Tensor = None,
                out_dtype: torch.dtype = torch.bfloat16, return_routing: bool = False,
                out: torch.Tensor = None):
        cfg = self.cfg
        xf = self._flat(x, cfg.hidden, "x")
        want = torch.float16 if cfg.x_dtype == "f16" else torch.bfloat16
        if xf.dtype != want:
            raise ValueError(f"x must be {want} (cfg.x_dtype)")
        lg = self._flat(logits, cfg.num_experts, "logits")
        if lg.dtype not in (torch.bfloat16, torch.float32):
            lg = lg.float()
        T = xf.shape[0]
        if lg.shape[0] != T:
            raise ValueError("x and logits disagree on the number of tokens")
        self.reserve(T)
        if out is None:
            out = torch.empty((T, cfg.hidden), dtype=out_dtype, device=self.device)
        idx = w = None
        if return_routing:
            idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device=self.device)
            w = torch.empty((T, cfg.top_k), dtype=torch.float32, device=self.device)
        bias = None if cache_bias is None else cache_bias.to(self.device, torch.float32).contiguous()
        # the registered operator (ops.py) runs es_moe_forward
        torch.ops.expert_sniper.moe_forward_out(
            xf, lg, bias, self.packed, self.shared_gate_w, self._ws, out, idx, w,
            cfg.num_experts, cfg.top_k, cfg.inter, cfg.norm_topk_prob, cfg.shared_inter,
            KERNEL_PATHS[cfg.kernel_path])
        o = out.reshape(*x.shape[:-1], cfg.hidden)
        if return_routing:
            lead = x.shape[:-1]
            return o, idx.reshape(*lead, cfg.top_k), w.reshape(*lead, cfg.top_k)
        return o

    __call__ = forward

    def forward_timed(self, x: torch.Tensor, logits: torch.Tensor, cache_bias, events,
                      out: torch.Tensor):
        """forward() with six CUDA events recorded around its kernels (router,
        dispatch, gate/up, down, combine, end) on the current stream."""
        cfg = self.cfg
        if len(events) != 6:
            raise ValueError("need 6 events")
        handles = (ctypes.c_void_p * 6)(*[int(e.cuda_event) for e in events])
        T = x.shape[0]
        _native.check("es_moe_forward_timed", _native.lib().es_moe_forward_timed(
            ctypes.byref(self.ccfg), x.data_ptr(), logits.data_ptr(), _DT_CODE[logits.dtype],
            _ptr(cache_bias), _ptr(self.shared_gate_w), self.packed.data_ptr(), out.data_ptr(),
            _DT_CODE[out.dtype], None, None, T, self._ws.data_ptr(), self._ws.numel(),
            _stream(self.device), handles, 6))
        return out

    def expert_ffn(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor,
                   out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor = None,
                   kernel_path: str = None):
        """Experts + combine for given routing (-1 ids are skipped).
        `kernel_path` ("auto", "decode", "tensor", "tensor-small") overrides the block's
        config for this call (e.g. when most slots are masked, the caller
        knows the real number of pairs per expert better than the row count
        does)."""
        cfg = self.cfg
        ccfg = self.ccfg
        if kernel_path is not None and kernel_path != cfg.kernel_path:
            ccfg = cfg.with_(kernel_path=kernel_path).to_c()
        xf = self._flat(x, cfg.hidden, "x")
        want = torch.float16 if cfg.x_dtype == "f16" else torch.bfloat16
        if xf.dtype != want:
            raise ValueError(f"x must be {want} (cfg.x_dtype)")
        idx = self._flat(topk_idx, cfg.top_k, "topk_idx").to(torch.int32)
        w = self._flat(topk_w, cfg.top_k, "topk_w").to(torch.float32)
        T = xf.shape[0]
        self.reserve(T)
        if out is None:
            out = torch.empty((T, cfg.hidden), dtype=out_dtype, device=self.device)
        _native.check("es_moe_expert_ffn", _native.lib().es_moe_expert_ffn(
            ctypes.byref(ccfg), xf.data_ptr(), idx.data_ptr(), w.data_ptr(),
            _ptr(self.shared_gate_w), self.packed.data_ptr(), out.data_ptr(), _DT_CODE[out.dtype],
            T, self._ws.data_ptr(), self._ws.numel(), _stream(self.device)))
        return out.reshape(*x.shape[:-1], cfg.hidden)


def cache_bias_mask(num_experts: int, cached_ids, bias: float, device="cuda") -> torch.Tensor:
    """The reference's routing-bias mask (generate.py:124-129): fp32 [E] with
    `bias` at the cached expert ids. Returns None when bias <= 0, because the
    reference adds no mask then (and keeps its softmax in the logits' dtype)."""
    if bias <= 0:
        return None
    m = torch.zeros(num_experts, dtype=torch.float32)
    ids = list(cached_ids)
    if ids:
        m[ids] = float(bias)
    return m.to(device)


class ExpertPool:
    """Device-resident packed experts for the run_expert_ffn drop-in.

    The reference hands run_expert_ffn a fresh dict of the active experts'
    MLX tensors on every call and re-stacks them (engine.py:22-30). Here
    each distinct expert is repacked once, into a slot of one packed buffer,
    and a call only maps its expert ids to slots. An expert is identified by
    the storage, offset, shape and dtype of its nine tensors; the pool keeps
    a reference to those storages so the memory behind a key cannot be
    reused for other data while the key is cached. Tensors must not be
    modified in place after their first call (or call clear()). At most
    es::kMaxExperts (1024) slots: run_expert_ffn empties a pool that a call
    would take beyond that."""

    MAX_SLOTS = 1024

    def __init__(self, hidden: int, inter: int, device):
        self.hidden, self.inter = hidden, inter
        self.device = torch.device(device)
        self.cfg1 = MoEConfig(hidden, 1, 1, inter, False, name="pool-slot")
        self.slot_bytes = self.cfg1.bytes_per_expert
        self.clear()

    def clear(self):
        self.buf = None
        self.capacity = 0
        self.slots = {}
        self._keep = []
        self._ws = None

    @staticmethod
    def _key(tensors: dict):
        k = []
        for proj in PROJS:
            for kind in ("weight", "scales", "biases"):
                t = tensors[f"switch_mlp.{proj}.{kind}"]
                k.append((t.untyped_storage().data_ptr(), t.storage_offset(), tuple(t.shape),
                          t.dtype))
        return tuple(k)

    def _grow(self, need: int):
        cap = max(16, self.capacity)
        while cap < need:
            cap *= 2
        cap = min(cap, self.MAX_SLOTS)
        buf = torch.empty(cap * self.slot_bytes, dtype=torch.uint8, device=self.device)
        if self.buf is not None:
            buf[:self.buf.numel()].copy_(self.buf)
        self.buf, self.capacity = buf, cap

    def slot(self, tensors: dict) -> int:
        key = self._key(tensors)
        s = self.slots.get(key)
        if s is not None:
            return s
        s = len(self.slots)
        if s >= self.MAX_SLOTS:
            raise RuntimeError("expert pool full: clear() it first")
        if s >= self.capacity:
            self._grow(s + 1)
        one = {}
        for proj in PROJS:
            for kind in ("weight", "scales", "biases"):
                name = f"switch_mlp.{proj}.{kind}"
                t = tensors[name]
                _need_cuda(t, name)
                one[name] = t.contiguous().unsqueeze(0)
        dst = self.buf[s * self.slot_bytes:(s + 1) * self.slot_bytes]
        prepare_packed(self.cfg1, one, out=dst)
        self._keep.append([tensors[f"switch_mlp.{p}.{k}"].untyped_storage()
                           for p in PROJS for k in ("weight", "scales", "biases")])
        self.slots[key] = s
        return s

    def workspace(self, ccfg, T: int) -> torch.Tensor:
        need = _native.workspace_bytes(ccfg, T)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._ws


_POOLS = {}


def expert_pool(hidden: int, inter: int, device) -> ExpertPool:
    """The process-wide pool for experts of one shape on one device."""
    dev = torch.device(device)
    key = (hidden, inter, dev.type, dev.index)
    if key not in _POOLS:
        _POOLS[key] = ExpertPool(hidden, inter, dev)
    return _POOLS[key]


def run_expert_ffn(x: torch.Tensor, expert_data: dict, top_k_indices: torch.Tensor,
                   top_k_weights: torch.Tensor) -> torch.Tensor:
    """Drop-in for the reference's run_expert_ffn (engine.py:15-42).

    expert_data: {expert id: {"switch_mlp.<proj>.<weight|scales|biases>":
    CUDA tensor}} for the active experts; indices not in expert_data map to
    the first active expert, as the reference's id_to_local.get(v, 0) does.
    x [..., D] bf16; returns [..., D] in x's dtype.

    Each distinct expert is repacked once into the shape's ExpertPool; a
    call maps ids to pool slots on the device (no host synchronisation) and
    runs es_moe_expert_ffn on the pool.
    """
    active = sorted(int(e) for e in expert_data.keys())
    first = expert_data[active[0]]
    I, d8 = first["switch_mlp.gate_proj.weight"].shape
    D = d8 * 8
    k = top_k_indices.shape[-1]
    dev = first["switch_mlp.gate_proj.weight"].device
    pool = expert_pool(D, I, dev)
    new = sum(pool._key(expert_data[e]) not in pool.slots for e in active)
    if len(pool.slots) + new > pool.MAX_SLOTS:
        pool.clear()   # start over so that every expert of this call gets a slot
    slots = [pool.slot(expert_data[e]) for e in active]
    hi = active[-1]
    lut = torch.full((hi + 1,), slots[0], dtype=torch.int32)
    lut[torch.tensor(active)] = torch.tensor(slots, dtype=torch.int32)
    lut = lut.to(dev)
    ids = top_k_indices.to(dev).long()
    inside = (ids >= 0) & (ids <= hi)
    local = torch.where(inside, lut[ids.clamp(0, hi)], lut.new_full((), slots[0]))
    cfg = MoEConfig(D, pool.capacity, k, I, False)   # capacity >= 16 >= k
    ccfg = cfg.to_c()
    xf = x.reshape(-1, D).to(torch.bfloat16).contiguous()
    T = xf.shape[0]
    idx = local.reshape(T, k).contiguous()
    w = top_k_weights.to(dev, torch.float32).reshape(T, k).contiguous()
    out = torch.empty((T, D), dtype=torch.float32, device=dev)
    ws = pool.workspace(ccfg, T)
    packed = pool.buf
    with torch.cuda.device(dev):
        _native.check("es_moe_expert_ffn", _native.lib().es_moe_expert_ffn(
            ctypes.byref(ccfg), xf.data_ptr(), idx.data_ptr(), w.data_ptr(), None,
            packed.data_ptr(), out.data_ptr(), _native.ES_DTYPE_F32, T, ws.data_ptr(),
            ws.numel(), _stream(dev)))
    return out.reshape(*x.shape[:-1], D).to(x.dtype)
