"""Device-resident cache-aware routing bias, one [E] row per layer.

The reference builds the routing-bias mask on the host for every layer of
every token (src/mlx_expert_sniper/generate.py:124-129): a numpy [E] vector
with `bias` at `reader.lru.cached_ids(i)` (expert_io.py:222-225), uploaded
and added to the router logits. Here the mask for all layers lives on the
GPU as one [L, E] fp32 table; the hot path passes row `i` to the MoE block
as its `cache_bias` (no host work, no upload, safe inside a CUDA graph --
the row's address never changes). The table changes only when the cache
does: `set_cached(layer, ids)` rewrites one row from pinned host memory on a
side stream, ordered before the next forward by an event.

`bias <= 0` means no bias at all (the reference skips the mask then, and its
softmax stays in the logits' dtype): `row()` returns None in that case.
"""
from __future__ import annotations

import numpy as np
import torch


class CacheBiasTable:
    def __init__(self, num_layers: int, num_experts: int, bias: float, device="cuda"):
        self.L, self.E, self.bias = num_layers, num_experts, float(bias)
        self.device = torch.device(device)
        self.table = torch.zeros((num_layers, num_experts), dtype=torch.float32, device=self.device)
        on_gpu = self.device.type == "cuda"
        self._host = torch.zeros((num_layers, num_experts), dtype=torch.float32)
        if on_gpu:
            self._host = self._host.pin_memory()
        self._stream = torch.cuda.Stream(self.device) if on_gpu else None
        self._ready = None

    def sync(self) -> None:
        """Order the current stream after pending row updates (call before
        replaying a graph that reads the table)."""
        if self._ready is not None:
            torch.cuda.current_stream(self.device).wait_event(self._ready)
            self._ready = None

    def row(self, layer: int):
        """The [E] device bias of one layer, or None when bias <= 0. Its
        address is fixed, so a captured graph keeps reading the live row."""
        if self.bias <= 0:
            return None
        self.sync()
        return self.table[layer]

    def set_cached(self, layer: int, cached_ids) -> None:
        """Replace one layer's cached set (LRUExpertCache.cached_ids(layer))."""
        ids = np.asarray(list(cached_ids), dtype=np.int64)
        if ids.size and (ids.min() < 0 or ids.max() >= self.E):
            raise ValueError("expert id out of range")
        h = self._host[layer]
        h.zero_()
        if ids.size:
            h[torch.from_numpy(ids)] = self.bias
        if self._stream is None:
            self.table[layer].copy_(h)
            return
        with torch.cuda.stream(self._stream):
            self.table[layer].copy_(h, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self._stream)
        self._ready = ev

    def host_mask(self, layer: int) -> np.ndarray:
        """The reference's per-layer numpy mask, for checks."""
        return self._host[layer].numpy().copy()
