"""The packed tile layout and the tensor-core kernels' 5-D TMA view of it,
on the CPU.

es_layout.h stores one expert's gate/up tiles as [row-block pair][group]
[block of the pair][gate, up] and its down tiles as [row-block quad][group]
[block of the quad], 576 bytes each, so four tiles sharing a group are one
contiguous 2304-byte run. The tensor-core GEMMs fetch a stage (one unit's
128 rows for kKG consecutive groups) with a single TMA load over a 5-D map
of 8-byte elements: dims {144, 2, group, run, expert}, box {144, 2, kKG,
runs, 1}. These tests restate both and check, for every byte of a box, that
the map reaches the tile byte the dequant warps read at that shared-memory
offset.
"""
from __future__ import annotations

import numpy as np
import pytest

from expert_sniper_b200 import PRESETS

TILE = 576
RUN = 4 * TILE


def expert_bytes(D, I):
    return 3 * D * I * 9 // 16


def gateup_tile_off(GD, rb, G, proj):
    return ((((rb >> 1) * GD + G) * 2 + (rb & 1)) * 2 + proj) * TILE


def down_tile_off(D, I, rb, G):
    return 2 * D * I * 9 // 16 + (((rb >> 2) * (I // 64) + G) * 4 + (rb & 3)) * TILE


def code_map(D, I, E1, gu, runs, kkg):
    """Base, dims, byte strides and box of the code-tile map (the launcher's
    encode_codes_map)."""
    groups = (D if gu else I) // 64
    nruns = I // 32 if gu else D // 64
    base = 0 if gu else 2 * D * I * 9 // 16
    dims = [RUN // 16, 2, groups, nruns, E1]
    strides = [8, RUN // 2, RUN, groups * RUN, expert_bytes(D, I)]   # bytes per step
    box = [RUN // 16, 2, kkg, runs, 1]
    return base, dims, strides, box


def box_bytes_to_global(D, I, E1, gu, runs, kkg, stage, rb, e):
    """Global byte address of every shared-memory byte of one stage's box."""
    base, dims, strides, box = code_map(D, I, E1, gu, runs, kkg)
    start = [0, 0, stage * kkg, runs * rb, e]
    for d in range(5):
        assert 0 <= start[d] and start[d] + box[d] <= dims[d], (d, start, box, dims)
    x, h, g, r, ee = np.meshgrid(*[np.arange(b) for b in box], indexing="ij")
    # shared-memory order: dim 0 fastest (TMA writes the box row-major)
    elem = (((ee * box[3] + r) * box[2] + g) * box[1] + h) * box[0] + x
    addr = (base + (start[0] + x) * strides[0] + (start[1] + h) * strides[1]
            + (start[2] + g) * strides[2] + (start[3] + r) * strides[3]
            + (start[4] + ee) * strides[4])
    order = np.argsort(elem.ravel())
    return addr.ravel()[order]  # element i of shared memory -> global byte address


@pytest.mark.parametrize("name", ["qwen3-30b-a3b", "qwen3-next-80b-a3b", "olmoe-1b-7b"])
@pytest.mark.parametrize("gu", [True, False])
@pytest.mark.parametrize("variant", ["large", "small"])
def test_code_map_reaches_the_dequant_tiles(name, gu, variant):
    cfg = PRESETS[name]
    D, I = cfg.hidden, cfg.inter
    E1 = cfg.num_experts + (1 if cfg.shared_inter else 0)
    kproj = 2 if gu else 1
    kkg = 1 if variant == "large" else (2 if gu else 4)
    tiles_per_group = 8 * kproj                       # 128 rows
    raw_bytes = kkg * tiles_per_group * TILE
    runs = raw_bytes // (RUN * kkg)
    assert runs * RUN * kkg == raw_bytes
    groups = (D if gu else I) // 64
    n_units = (I if gu else D) // 128
    rng = np.random.default_rng(hash((name, gu, variant)) % 2**32)
    for _ in range(4):
        e = int(rng.integers(E1))
        rb = int(rng.integers(n_units))
        stage = int(rng.integers(groups // kkg))
        glob8 = box_bytes_to_global(D, I, E1, gu, runs, kkg, stage, rb, e)
        assert glob8.size * 8 == raw_bytes
        # what the dequant warps read at each shared-memory tile position
        rows_per_run = 4 // kproj
        for b16 in range(8):                           # 16-row tile of the unit
            run, in_run = b16 // rows_per_run, (b16 % rows_per_run) * kproj
            for g2 in range(kkg):
                for pj in range(kproj):
                    smem = (run * kkg + g2) * RUN + (in_run + pj) * TILE
                    G = stage * kkg + g2
                    want = e * expert_bytes(D, I) + (
                        gateup_tile_off(groups, 8 * rb + b16, G, pj) if gu
                        else down_tile_off(D, I, 8 * rb + b16, G))
                    got = glob8[smem // 8] - (smem % 8)
                    assert got == want, (b16, g2, pj, got, want)
                    # the whole tile is one contiguous 576-byte span
                    span = glob8[smem // 8: smem // 8 + TILE // 8]
                    assert np.array_equal(np.diff(span), np.full(TILE // 8 - 1, 8))


def test_map_strides_are_tma_legal():
    """Global strides multiples of 16 bytes, inner box 1152 bytes (a multiple
    of 16), every box dimension at most 256 elements."""
    for name in ("qwen3-30b-a3b", "qwen3-next-80b-a3b", "qwen3-235b-a22b", "olmoe-1b-7b"):
        cfg = PRESETS[name]
        E1 = cfg.num_experts + (1 if cfg.shared_inter else 0)
        for gu in (True, False):
            for kkg in (1, 2, 4):
                base, dims, strides, box = code_map(cfg.hidden, cfg.inter, E1, gu, 2, kkg)
                assert base % 16 == 0
                assert all(s % 16 == 0 for s in strides[1:])
                assert box[0] * 8 % 16 == 0 and max(box) <= 256
