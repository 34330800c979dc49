"""Expert Sniper's streaming format, read straight into the device layout.

A streaming model keeps each MoE layer's routed experts in one file,
`bin/layer_XX.bin` (src/mlx_expert_sniper/download.py:189-248, the reader
side in src/mlx_expert_sniper/expert_io.py:271-284 and 338-362):

  bytes [0, 16384)      JSON header padded with NULs:
                        {"layer_idx", "num_experts",
                         "layout": {"expert_block_size", "data_start": 16384,
                                    "tensors": {name: {"inner_offset",
                                                       "nbytes",
                                                       "shape_per_expert",
                                                       "dtype"}}}}
  then E expert blocks  each `expert_block_size` bytes (a multiple of 16384):
                        the nine tensors of TENSOR_ORDER back to back at
                        their inner offsets, zero padding after.

`load_layer` reads a layer file into pinned host memory, copies the expert
region to the GPU with one host-to-device copy and repacks it with
es_moe_prepare_blocks, which reads every expert block in place. The shared
expert (not part of the streaming files) comes from ordinary tensors.
`write_layer` produces the same format from MLX-format tensors (used by the
tests and by users converting their own layers).
"""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import torch

from . import _native
from .block import _proj, _stream
from .config import MoEConfig

PAGE_SIZE = 16384

TENSOR_ORDER = [
    "switch_mlp.gate_proj.weight", "switch_mlp.gate_proj.scales", "switch_mlp.gate_proj.biases",
    "switch_mlp.up_proj.weight", "switch_mlp.up_proj.scales", "switch_mlp.up_proj.biases",
    "switch_mlp.down_proj.weight", "switch_mlp.down_proj.scales", "switch_mlp.down_proj.biases",
]

_NP_DTYPES = {"uint32": np.uint32, "float16": np.float16, "bfloat16": np.uint16,
              "float32": np.float32}
_ITEMSIZE = {"uint32": 4, "float16": 2, "bfloat16": 2, "float32": 4}


def _dtype_name(d: str) -> str:
    return d.replace("mlx.core.", "")


def layer_path(model_dir: str, layer_idx: int) -> str:
    """Path of a layer file as the reader opens it (expert_io.py:275)."""
    return os.path.join(model_dir, f"layer_{layer_idx:02d}.bin")


def read_header(path: str) -> dict:
    """The JSON header of a layer file (expert_io.py:276-278)."""
    with open(path, "rb") as f:
        raw = f.read(PAGE_SIZE)
    if len(raw) < PAGE_SIZE:
        raise ValueError(f"{path}: shorter than the {PAGE_SIZE}-byte header")
    return json.loads(raw.rstrip(b"\x00"))


def expected_layout(cfg: MoEConfig) -> dict:
    """Per-expert shape, dtype and byte count of each TENSOR_ORDER tensor for a
    4-bit, group-64 layer of `cfg`."""
    D, I = cfg.hidden, cfg.inter
    shapes = {"gate_proj": (I, D), "up_proj": (I, D), "down_proj": (D, I)}
    out = {}
    for name in TENSOR_ORDER:
        proj, kind = name.split(".")[1], name.split(".")[2]
        n, k = shapes[proj]
        if kind == "weight":
            out[name] = ([n, k // 8], "uint32", n * (k // 8) * 4)
        else:
            out[name] = ([n, k // 64], "float16", n * (k // 64) * 2)
    return out


def check_layout(header: dict, cfg: MoEConfig) -> tuple:
    """Validate a header against `cfg`. Returns (block_bytes, data_start,
    inner offsets in TENSOR_ORDER, scale dtype name). bf16 scales and biases
    (written by some converters, expert_io.py:432) are accepted and converted
    to fp16 on load."""
    lay = header["layout"]
    tensors = lay["tensors"]
    want = expected_layout(cfg)
    offsets, sdtype = [], None
    for name in TENSOR_ORDER:
        if name not in tensors:
            raise ValueError(f"layer file lacks tensor {name}")
        info = tensors[name]
        shape, dt, nbytes = want[name]
        got_dt = _dtype_name(info["dtype"])
        if list(info["shape_per_expert"]) != shape:
            raise ValueError(f"{name}: shape {info['shape_per_expert']} != {shape}")
        if name.endswith("weight"):
            if got_dt != "uint32":
                raise ValueError(f"{name}: dtype {got_dt}, want uint32")
        else:
            if got_dt not in ("float16", "bfloat16"):
                raise ValueError(f"{name}: dtype {got_dt}, want float16 or bfloat16")
            sdtype = sdtype or got_dt
            if got_dt != sdtype:
                raise ValueError("scales and biases must share one dtype")
        if int(info["nbytes"]) != nbytes:
            raise ValueError(f"{name}: nbytes {info['nbytes']} != {nbytes}")
        offsets.append(int(info["inner_offset"]))
    block = int(lay["expert_block_size"])
    data_start = int(lay.get("data_start", PAGE_SIZE))
    ends = [o + want[n][2] for o, n in zip(offsets, TENSOR_ORDER)]
    if max(ends) > block or min(offsets) < 0:
        raise ValueError("tensor extends past its expert block")
    return block, data_start, offsets, sdtype


def write_layer(path: str, layer: dict, layer_idx: int = 0) -> int:
    """Write MLX-format routed-expert tensors ({"switch_mlp.<proj>.<kind>":
    [E, ...]}, numpy or torch) as one streaming-format layer file, in the
    writer's layout (download.py:197-230): tensors in TENSOR_ORDER at
    cumulative inner offsets, blocks padded to a multiple of 16384 bytes.
    Returns the bytes written."""
    arrs = {}
    for name in TENSOR_ORDER:
        t = layer[name]
        a = t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)
        arrs[name] = a
    E = arrs[TENSOR_ORDER[0]].shape[0]
    info, off = {}, 0
    for name in TENSOR_ORDER:
        a = arrs[name]
        per = int(np.prod(a.shape[1:])) * a.dtype.itemsize
        # MLX names; int32 holds the packed uint32 words of torch tensors
        dt = {np.dtype(np.uint32): "uint32", np.dtype(np.int32): "uint32",
              np.dtype(np.float16): "float16"}.get(a.dtype, str(a.dtype))
        info[name] = {"inner_offset": off, "nbytes": per, "shape_per_expert": list(a.shape[1:]),
                      "dtype": dt}
        off += per
    block = (off + PAGE_SIZE - 1) // PAGE_SIZE * PAGE_SIZE
    header = {"layer_idx": layer_idx, "num_experts": E,
              "layout": {"expert_block_size": block, "data_start": PAGE_SIZE, "tensors": info}}
    raw = json.dumps(header).encode()
    if len(raw) >= PAGE_SIZE:
        raise ValueError("header does not fit its page")
    with open(path, "wb") as f:
        f.write(raw.ljust(PAGE_SIZE, b"\x00"))
        for e in range(E):
            blk = bytearray()
            for name in TENSOR_ORDER:
                blk += np.ascontiguousarray(arrs[name][e]).tobytes()
            f.write(bytes(blk).ljust(block, b"\x00"))
    return PAGE_SIZE + E * block


def read_expert(path: str, expert_id: int, header: dict = None) -> dict:
    """One expert's tensors as numpy arrays (expert_io.py:329-362)."""
    header = header or read_header(path)
    lay = header["layout"]
    off = int(lay["data_start"]) + expert_id * int(lay["expert_block_size"])
    with open(path, "rb") as f:
        f.seek(off)
        raw = f.read(int(lay["expert_block_size"]))
    out = {}
    for name, inf in lay["tensors"].items():
        dt = _dtype_name(inf["dtype"])
        a = np.frombuffer(raw, dtype=np.uint8, count=int(inf["nbytes"]),
                          offset=int(inf["inner_offset"]))
        out[name] = a.view(_NP_DTYPES.get(dt, np.float16)).reshape(inf["shape_per_expert"])
    return out


def load_layer(path: str, cfg: MoEConfig, device="cuda", shared: dict = None,
               out: torch.Tensor = None, staging: torch.Tensor = None) -> torch.Tensor:
    """Read one layer file into the packed device layout.

    The expert region (E blocks) goes to the device in one copy from pinned
    host memory (`staging`, reused across layers when given), then
    es_moe_prepare_blocks repacks it in place. `shared` holds the layer's
    "shared_expert.<proj>.<kind>" tensors when cfg has a shared expert.
    Returns the packed uint8 tensor (es_moe_packed_bytes bytes)."""
    device = torch.device(device)
    header = read_header(path)
    block, data_start, offsets, sdtype = check_layout(header, cfg)
    E = int(header.get("num_experts", cfg.num_experts))
    if E != cfg.num_experts:
        raise ValueError(f"layer file holds {E} experts, config has {cfg.num_experts}")
    nbytes = E * block
    if os.path.getsize(path) < data_start + nbytes:
        raise ValueError(f"{path}: truncated")
    if staging is None or staging.numel() < nbytes:
        staging = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    with open(path, "rb", buffering=0) as f:
        f.seek(data_start)
        view = memoryview(staging.numpy())[:nbytes]
        got = 0
        while got < nbytes:
            n = f.readinto(view[got:])
            if not n:
                raise ValueError(f"{path}: short read")
            got += n
    blocks = torch.empty(nbytes, dtype=torch.uint8, device=device)
    blocks.copy_(staging[:nbytes], non_blocking=True)
    if sdtype == "bfloat16":
        blocks = _bf16_scales_to_f16(blocks, cfg, block, offsets)
    ccfg = cfg.to_c()
    pk = _native.packed_bytes(ccfg)
    if out is None:
        out = torch.empty(pk, dtype=torch.uint8, device=device)
    layer = _native.CMlxLayer()
    if cfg.has_shared:
        if shared is None:
            raise ValueError("this config has a shared expert: pass its tensors")
        layer.shared_gate_proj = _proj(shared, "shared_expert", "gate_proj")
        layer.shared_up_proj = _proj(shared, "shared_expert", "up_proj")
        layer.shared_down_proj = _proj(shared, "shared_expert", "down_proj")
    offs = (ctypes.c_int64 * 9)(*offsets)
    with torch.cuda.device(device):
        _native.check("es_moe_prepare_blocks", _native.lib().es_moe_prepare_blocks(
            ctypes.byref(ccfg), blocks.data_ptr(), block, offs,
            ctypes.byref(layer) if cfg.has_shared else None, out.data_ptr(), out.numel(),
            _stream(device)))
    torch.cuda.current_stream(device).synchronize()  # staging and blocks may be reused
    return out


def _bf16_scales_to_f16(blocks: torch.Tensor, cfg: MoEConfig, block: int, offsets) -> torch.Tensor:
    """Rewrite bf16 scales/biases inside the device image as fp16 (in place;
    values beyond the fp16 range saturate)."""
    E = blocks.numel() // block
    rows = blocks.view(E, block)
    want = expected_layout(cfg)
    for name, off in zip(TENSOR_ORDER, offsets):
        if name.endswith("weight"):
            continue
        nb = want[name][2]
        seg = rows[:, off:off + nb].contiguous().view(torch.bfloat16)
        f16 = seg.float().clamp(-65504.0, 65504.0).half()
        rows[:, off:off + nb] = f16.view(torch.uint8)
    return blocks


def load_model(model_dir: str, cfg: MoEConfig, layers, device="cuda", shared_by_layer=None):
    """Packed device tensors for the given layer indices of a streaming model
    directory (the `bin/` folder the reader opens), sharing one pinned staging
    buffer."""
    staging = None
    out = []
    for l in layers:
        p = layer_path(model_dir, l)
        hdr = read_header(p)
        need = int(hdr["num_experts"]) * int(hdr["layout"]["expert_block_size"])
        if staging is None or staging.numel() < need:
            staging = torch.empty(need, dtype=torch.uint8, pin_memory=True)
        sh = None if shared_by_layer is None else shared_by_layer[l]
        out.append(load_layer(p, cfg, device, shared=sh, staging=staging))
    return out


def _bench(argv=None):
    """Time load_layer on a synthetic layer file: file read into pinned
    memory, one host-to-device copy, in-place repack."""
    import argparse
    import tempfile
    import time
    from .config import PRESETS
    from .quant import synthetic_layer
    ap = argparse.ArgumentParser(description="streaming-format layer load throughput")
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args(argv)
    cfg = PRESETS[args.model]
    dev = torch.device("cuda")
    lay = {k: v for k, v in synthetic_layer(cfg, seed=7, device="cpu").items()
           if k.startswith("switch_mlp")}
    with tempfile.TemporaryDirectory() as d:
        p = layer_path(d, 0)
        nb = write_layer(p, lay)
        cfg_r = cfg.with_(shared_inter=0)
        staging = torch.empty(nb, dtype=torch.uint8, pin_memory=True)
        load_layer(p, cfg_r, dev, staging=staging)
        ts = []
        for _ in range(args.reps):
            t0 = time.perf_counter()
            load_layer(p, cfg_r, dev, staging=staging)
            ts.append(time.perf_counter() - t0)
        best = min(ts)
        print(json.dumps({"model": cfg.name, "file_bytes": nb, "best_s": best,
                          "gbs": nb / best / 1e9, "note": "page-cached file; read + H2D + repack"}))


if __name__ == "__main__":
    _bench()
