"""Expert parallelism across the GPUs of one box.

Replaces the reference's Expert Network exchange (src/expert_network/
reader.py:237-292, node.py:142-198, hrw.py) with NCCL collectives between
one process per GPU:

  placement  experts are assigned to ranks by rendezvous hashing over the
             roster gpu0..gpu{N-1} (hrw.plan, the reference's rule) or its
             capacity-bounded variant (hrw.bounded_plan); every rank derives
             the same table from the roster alone.
  per layer  1. each rank routes its own (home) tokens            [kernel]
             2. per-destination masks: slot -> owner's local expert id or
                -1 (compute_partial's partition mask)             [kernel]
             3. all_gather of the home activations, all_to_all of the masks
             4. each rank runs its shard's experts on every received row,
                producing one fp32 partial per (source rank, token)  [kernels]
             5. all_to_all of the partials back to their home ranks
             6. home sums the partials in fixed rank order (reader.py:278-286),
                plus the shared expert, computed on the home rank [kernel]

Results therefore do not depend on timing, and differ from the one-GPU block
only by fp32 summation order. All ranks must call with the same token count.
The orchestration (`ep_forward`) is written against a small backend so the
same code runs on the CUDA kernels (`CudaEPBackend`) and, in the CPU tests,
on the oracle with gloo.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native, hrw
from .block import MoEBlock, _ptr, _stream, ffn_kernels
from .config import MoEConfig
from .quant import PROJS


@dataclass
class Placement:
    world: int
    roster: list
    owned: list        # owned[r] = sorted global expert ids of rank r
    owner: list        # owner[e] = rank of expert e
    local_id: list     # local_id[e] = index of e in owned[owner[e]]
    policy: str

    @property
    def counts(self):
        return [len(o) for o in self.owned]


def make_placement(num_experts: int, world: int, policy: str = "hrw") -> Placement:
    roster = hrw.gpu_roster(world)
    if policy == "hrw":
        plan = hrw.plan(roster, num_experts)
    elif policy == "bounded":
        plan = hrw.bounded_plan(roster, num_experts)
    else:
        raise ValueError(f"unknown placement policy {policy!r}")
    owned = [sorted(plan[n]) for n in roster]
    owner = [-1] * num_experts
    local = [-1] * num_experts
    for r, es in enumerate(owned):
        for j, e in enumerate(es):
            owner[e] = r
            local[e] = j
    return Placement(world, roster, owned, owner, local, policy)


def shard_layer(layer: dict, experts) -> dict:
    """The owned experts' MLX tensors (stacked in `experts` order); the shared
    expert's tensors are kept whole."""
    out = {}
    ids = None
    for name, t in layer.items():
        if name.startswith("switch_mlp."):
            if ids is None:
                ids = torch.tensor(list(experts), dtype=torch.long, device=t.device)
            out[name] = t.index_select(0, ids).contiguous()
        else:
            out[name] = t
    return out


# --------------------------------------------------------------------------- #
# orchestration
# --------------------------------------------------------------------------- #

def ep_forward(backend, x: torch.Tensor, logits: torch.Tensor, cache_bias=None, group=None):
    """One MoE layer over the home tokens of this rank. x [T, D], logits
    [T, E]. Returns the combined output [T, D] (backend's output dtype)."""
    world = dist.get_world_size(group)
    T, D = x.shape
    idx, w = backend.route(logits, cache_bias)
    send_idx, send_w = backend.mask(idx, w)                 # [world, T, k]
    x_all = backend.empty((world * T, D), x.dtype)
    dist.all_gather_into_tensor(x_all, x.contiguous(), group=group)
    recv_idx = torch.empty_like(send_idx)
    recv_w = torch.empty_like(send_w)
    dist.all_to_all_single(recv_idx, send_idx, group=group)
    dist.all_to_all_single(recv_w, send_w, group=group)
    k = idx.shape[-1]
    partial = backend.ffn(x_all, recv_idx.view(world * T, k),
                          recv_w.view(world * T, k))           # [world * T, D] f32
    recv_part = torch.empty_like(partial)
    dist.all_to_all_single(recv_part, partial, group=group)
    return backend.combine(recv_part.view(world, T, D), backend.shared(x))


class CudaEPBackend:
    """The CUDA kernels behind ep_forward for one rank.

    layer: this layer's full MLX tensors (any device) or None with `packed`
    already built for this rank's shard."""

    def __init__(self, cfg: MoEConfig, placement: Placement, rank: int, layer: dict = None,
                 packed: torch.Tensor = None, shared_gate_w: torch.Tensor = None,
                 max_tokens: int = 64, device=None, workspace: torch.Tensor = None,
                 out_dtype=torch.bfloat16):
        self.cfg = cfg
        self.pl = placement
        self.rank = rank
        self.world = placement.world
        self.device = torch.device(device or "cuda")
        self.out_dtype = out_dtype
        self.route_cfg = cfg.with_(shared_inter=0)
        self.route_ccfg = self.route_cfg.to_c()
        self.owner = torch.tensor(placement.owner, dtype=torch.int32, device=self.device)
        self.local_id = torch.tensor(placement.local_id, dtype=torch.int32, device=self.device)
        owned = placement.owned[rank]
        self.n_local = len(owned)
        rows = self.world * max_tokens
        self.local = None
        if self.n_local:
            lcfg = cfg.with_(num_experts=self.n_local, shared_inter=0, name=f"{cfg.name}:ep{rank}")
            w = None if layer is None else {k: v.to(self.device) for k, v in
                                            shard_layer(layer, owned).items()
                                            if k.startswith("switch_mlp.")}
            self.local = MoEBlock(lcfg, weights=w, packed=packed, max_tokens=rows,
                                  workspace=workspace)
        self.shared_blk = None
        if cfg.has_shared:
            if layer is None:
                raise ValueError("a shared expert needs the layer tensors")
            sw = {}
            for proj in PROJS:
                for kind in ("weight", "scales", "biases"):
                    t = layer[f"shared_expert.{proj}.{kind}"].to(self.device)
                    sw[f"switch_mlp.{proj}.{kind}"] = t.unsqueeze(0).contiguous()
                    sw[f"shared_expert.{proj}.{kind}"] = t.contiguous()
            scfg = MoEConfig(cfg.hidden, 1, 1, cfg.inter, False, shared_inter=cfg.inter,
                             name=f"{cfg.name}:shared")
            self.shared_blk = MoEBlock(scfg, weights=sw, shared_gate_w=shared_gate_w,
                                       max_tokens=max_tokens)

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype, device=self.device)

    def route(self, logits, cache_bias):
        cfg = self.route_cfg
        lg = logits.contiguous()
        if lg.dtype not in (torch.bfloat16, torch.float32):
            lg = lg.float()
        T = lg.shape[0]
        idx = self.empty((T, cfg.top_k), torch.int32)
        w = self.empty((T, cfg.top_k), torch.float32)
        bias = None if cache_bias is None else cache_bias.to(self.device, torch.float32).contiguous()
        code = _native.ES_DTYPE_F32 if lg.dtype == torch.float32 else _native.ES_DTYPE_BF16
        _native.check("es_moe_route", _native.lib().es_moe_route(
            ctypes.byref(self.route_ccfg), lg.data_ptr(), code, _ptr(bias), T, idx.data_ptr(),
            w.data_ptr(), _stream(self.device)))
        return idx, w

    def mask(self, idx, w):
        T, k = idx.shape
        send_idx = self.empty((self.world, T, k), torch.int32)
        send_w = self.empty((self.world, T, k), torch.float32)
        _native.check("es_ep_mask", _native.lib().es_ep_mask(
            idx.data_ptr(), w.data_ptr(), self.owner.data_ptr(), self.local_id.data_ptr(),
            self.cfg.num_experts, k, T, self.world, send_idx.data_ptr(), send_w.data_ptr(),
            _ptr(self.local.workspace if self.local else None), _stream(self.device)))
        return send_idx, send_w

    def ffn(self, x_all, idx, w):
        R, D = x_all.shape
        if self.local is None:  # this rank owns no expert: its partials are zero
            return torch.zeros((R, D), dtype=torch.float32, device=self.device)
        # Most of the R x k slots are masked (-1: another rank's expert), so
        # the row count overstates the work per local expert. Each local
        # expert receives about R k / E_global real pairs, the same per-expert
        # load as a one-GPU call with R tokens: choose the kernels for that.
        path = self.local.cfg.kernel_path
        if path == "auto":
            path = ffn_kernels(self.cfg, R)
        return self.local.expert_ffn(x_all, idx, w, out_dtype=torch.float32, kernel_path=path)

    def shared(self, x):
        if self.shared_blk is None:
            return None
        T = x.shape[0]
        none = torch.full((T, 1), -1, dtype=torch.int32, device=self.device)
        zero = torch.zeros((T, 1), dtype=torch.float32, device=self.device)
        return self.shared_blk.expert_ffn(x, none, zero, out_dtype=torch.float32)

    def combine(self, partials, extra):
        world, T, D = partials.shape
        out = self.empty((T, D), self.out_dtype)
        code = _native.ES_DTYPE_F32 if self.out_dtype == torch.float32 else _native.ES_DTYPE_BF16
        _native.check("es_ep_combine", _native.lib().es_ep_combine(
            partials.data_ptr(), _ptr(extra), world, T, D, out.data_ptr(), code,
            _stream(self.device)))
        return out


# --------------------------------------------------------------------------- #
# peer-to-peer exchange over NVLink (es_ep_dispatch / receive / return /
# combine_p2p): no collective library on the data path
# --------------------------------------------------------------------------- #

def _check(fn: str, status: int):
    _native.check(fn, status)


class EpWindows:
    """This rank's exchange window and the mapped windows of every peer.

    The window is allocated once per rank (es_ep_window_alloc) and shared by
    all layers: the exchange of one layer step completes before the next
    step writes into it. Handles are swapped once with all_gather_object
    over the process group (world > 1); every later exchange is plain
    stores into peer memory made by the kernels."""

    def __init__(self, world: int, rank: int, cap: int, hidden: int, top_k: int, device,
                 group=None, handles=None, local_only: bool = False):
        """local_only: ranks emulated in one process on one device; no
        handles are swapped or opened, and set_peers() supplies the other
        windows' addresses."""
        self.world, self.rank, self.cap = world, rank, cap
        self.hidden, self.top_k = hidden, top_k
        self.device = torch.device(device)
        L = _native.lib()
        nb = ctypes.c_size_t(0)
        _check("es_ep_window_bytes", L.es_ep_window_bytes(world, cap, hidden, top_k,
                                                          ctypes.byref(nb)))
        self.bytes = nb.value
        ptr = ctypes.c_void_p(0)
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            _check("es_ep_window_alloc", L.es_ep_window_alloc(nb.value, ctypes.byref(ptr), handle))
        self.ptr = ptr.value
        self.handle = bytes(handle)
        if local_only:
            handles = None
        elif handles is None:
            handles = [self.handle]
            if world > 1:
                handles = [None] * world
                dist.all_gather_object(handles, self.handle, group=group)
        self.opened = []
        peers = []
        with torch.cuda.device(self.device):
            for r in range(world):
                if r == rank or local_only:
                    peers.append(self.ptr if r == rank else 0)
                    continue
                p = ctypes.c_void_p(0)
                buf = (ctypes.c_char * 64).from_buffer_copy(handles[r])
                _check("es_ep_window_open", L.es_ep_window_open(buf, ctypes.byref(p)))
                peers.append(p.value)
                self.opened.append(p.value)
        self.peers = torch.tensor(peers, dtype=torch.int64, device=self.device)
        self.err = torch.zeros(64, dtype=torch.int32, device=self.device)
        self._rows_offset()

    def set_peers(self, ptrs):
        """Use these window addresses as the peers (ranks emulated in one
        process on one device, whose windows need no IPC mapping)."""
        self.peers.copy_(torch.tensor(ptrs, dtype=torch.int64))

    def _rows_offset(self):
        L = _native.lib()
        off = ctypes.c_size_t(0)
        _check("es_ep_rows_offset", L.es_ep_rows_offset(ctypes.byref(self.plan(None, None, 1)),
                                                        ctypes.byref(off)))
        self.rows_ptr = self.ptr + off.value

    def plan(self, owner: torch.Tensor, local_id: torch.Tensor, num_experts: int):
        return _native.CEpPlan(self.world, self.rank, self.cap, self.hidden, self.top_k,
                               num_experts, _ptr(owner) or self.peers.data_ptr(),
                               _ptr(local_id) or self.peers.data_ptr(), self.peers.data_ptr(),
                               self.ptr, self.err.data_ptr())

    def read_error(self, clear: bool = True) -> int:
        v = int(self.err[0].item())
        if clear:
            self.err.zero_()
        return v & 0xFFFFFFFF

    def close(self):
        """Unmap the peers' windows and free this rank's. Every rank must be
        past its last exchange (synchronise and barrier first)."""
        L = _native.lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p in self.opened:
                L.es_ep_window_close(p)
            self.opened = []
            if self.ptr:
                L.es_ep_window_free(self.ptr)
                self.ptr = 0


class P2PEPBackend:
    """One rank's MoE layer with expert parallelism over NVLink peer memory.

    step(x, logits, cache_bias):
      es_moe_route -> es_ep_dispatch (rows to their owners' windows) ->
      es_ep_receive -> es_moe_expert_ffn (local experts on received rows) ->
      es_ep_return (partials to their home windows) -> shared expert (home) ->
      es_ep_combine_p2p (rank-ordered sum).
    Replaces the reference's per-layer HTTP exchange
    (src/expert_network/reader.py:237-292, node.py:142-172). All launches
    go to the current stream, so a whole step can be captured in one CUDA
    graph; nothing synchronises the host."""

    def __init__(self, cfg: MoEConfig, placement: Placement, rank: int, windows: EpWindows,
                 layer: dict = None, shared_gate_w: torch.Tensor = None,
                 out_dtype=torch.bfloat16, kernel_path: str = "auto",
                 local_workspace: torch.Tensor = None):
        self.cfg = cfg
        self.pl = placement
        self.rank = rank
        self.world = placement.world
        self.win = windows
        self.device = windows.device
        self.cap = windows.cap
        self.out_dtype = out_dtype
        self.route_ccfg = cfg.with_(shared_inter=0).to_c()
        self.owner = torch.tensor(placement.owner, dtype=torch.int32, device=self.device)
        self.local_id = torch.tensor(placement.local_id, dtype=torch.int32, device=self.device)
        self.plan = windows.plan(self.owner, self.local_id, cfg.num_experts)
        owned = placement.owned[rank]
        self.n_local = len(owned)
        R = self.world * self.cap
        self.local = None
        if self.n_local:
            path = kernel_path if kernel_path != "auto" else ffn_kernels(cfg, R)
            lcfg = cfg.with_(num_experts=self.n_local, shared_inter=0, kernel_path=path,
                             name=f"{cfg.name}:ep{rank}")
            w = None if layer is None else {k: v.to(self.device) for k, v in
                                            shard_layer(layer, owned).items()
                                            if k.startswith("switch_mlp.")}
            self.local = MoEBlock(lcfg, weights=w, max_tokens=R, workspace=local_workspace)
        self.shared_blk = None
        if cfg.has_shared:
            sw = {}
            for proj in PROJS:
                for kind in ("weight", "scales", "biases"):
                    t = layer[f"shared_expert.{proj}.{kind}"].to(self.device)
                    sw[f"switch_mlp.{proj}.{kind}"] = t.unsqueeze(0).contiguous()
                    sw[f"shared_expert.{proj}.{kind}"] = t.contiguous()
            scfg = MoEConfig(cfg.hidden, 1, 1, cfg.inter, False, shared_inter=cfg.inter,
                             name=f"{cfg.name}:shared")
            self.shared_blk = MoEBlock(scfg, weights=sw, shared_gate_w=shared_gate_w,
                                       max_tokens=self.cap)
            self._none = torch.full((self.cap, 1), -1, dtype=torch.int32, device=self.device)
            self._zero = torch.zeros((self.cap, 1), dtype=torch.float32, device=self.device)
            self.extra = torch.empty((self.cap, cfg.hidden), dtype=torch.float32,
                                     device=self.device)
        k = cfg.top_k
        self.idx = torch.empty((self.cap, k), dtype=torch.int32, device=self.device)
        self.w = torch.empty((self.cap, k), dtype=torch.float32, device=self.device)
        self.ridx = torch.empty((R, k), dtype=torch.int32, device=self.device)
        self.rw = torch.empty((R, k), dtype=torch.float32, device=self.device)
        self.y = torch.zeros((R, cfg.hidden), dtype=torch.float32, device=self.device)
        self.out = torch.empty((self.cap, cfg.hidden), dtype=out_dtype, device=self.device)

    # each phase on the current stream
    def route(self, logits, cache_bias):
        T = logits.shape[0]
        code = _native.ES_DTYPE_F32 if logits.dtype == torch.float32 else _native.ES_DTYPE_BF16
        _check("es_moe_route", _native.lib().es_moe_route(
            ctypes.byref(self.route_ccfg), logits.data_ptr(), code, _ptr(cache_bias), T,
            self.idx.data_ptr(), self.w.data_ptr(), _stream(self.device)))

    def dispatch(self, x, T):
        _check("es_ep_dispatch", _native.lib().es_ep_dispatch(
            ctypes.byref(self.plan), x.data_ptr(), self.idx.data_ptr(), self.w.data_ptr(), T,
            _stream(self.device)))

    def receive(self):
        _check("es_ep_receive", _native.lib().es_ep_receive(
            ctypes.byref(self.plan), self.ridx.data_ptr(), self.rw.data_ptr(),
            _stream(self.device)))

    def ffn(self):
        if self.local is None:   # no expert here: no token ever sends a row
            return
        blk = self.local
        R = self.world * self.cap
        _check("es_moe_expert_ffn", _native.lib().es_moe_expert_ffn(
            ctypes.byref(blk.ccfg), self.win.rows_ptr, self.ridx.data_ptr(), self.rw.data_ptr(),
            None, blk.packed.data_ptr(), self.y.data_ptr(), _native.ES_DTYPE_F32, R,
            blk.workspace.data_ptr(), blk.workspace.numel(), _stream(self.device)))

    def ret(self):
        _check("es_ep_return", _native.lib().es_ep_return(
            ctypes.byref(self.plan), self.y.data_ptr(), _stream(self.device)))

    def shared(self, x, T):
        if self.shared_blk is None:
            return None
        self.shared_blk.expert_ffn(x, self._none[:T], self._zero[:T], out_dtype=torch.float32,
                                   out=self.extra[:T])
        return self.extra

    def combine(self, extra, T):
        code = _native.ES_DTYPE_F32 if self.out_dtype == torch.float32 else _native.ES_DTYPE_BF16
        _check("es_ep_combine_p2p", _native.lib().es_ep_combine_p2p(
            ctypes.byref(self.plan), self.idx.data_ptr(), _ptr(extra), T, self.out.data_ptr(),
            code, _stream(self.device)))
        return self.out[:T]

    def step(self, x: torch.Tensor, logits: torch.Tensor, cache_bias=None) -> torch.Tensor:
        """One layer for this rank's T home tokens (T <= cap; x [T, D] bf16
        contiguous, logits [T, E]). Every rank of the group must call step
        for the same layer in the same order."""
        T = x.shape[0]
        if T > self.cap or T < 1:
            raise ValueError(f"1 <= T <= {self.cap}")
        self.route(logits, cache_bias)
        self.dispatch(x, T)
        self.receive()
        self.ffn()
        self.ret()
        extra = self.shared(x, T)
        return self.combine(extra, T)
