"""The device bias table on the hot path: a graph-captured forward reads
the table row by address, so rewriting the row (the cache changed) changes
the next replay's routing exactly as a fresh host mask would; the
speculative-verify call shape (T = K + 1 tokens, speculative.py:315-318) is
served like any other T."""
from __future__ import annotations

import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig
from expert_sniper_b200.bias_table import CacheBiasTable
from expert_sniper_b200.quant import synthetic_inputs, synthetic_layer

pytestmark = pytest.mark.gpu

CFG = MoEConfig(512, 32, 4, 512, True, name="bias-table")


def test_graph_reads_updated_row(cuda):
    lay = synthetic_layer(CFG, seed=5, device=cuda)
    T = 5  # speculative verify: current token + 4 drafts
    x, _, lg, _ = synthetic_inputs(CFG, T, seed=6, device=cuda)
    blk = MoEBlock(CFG, weights=lay, max_tokens=T)
    table = CacheBiasTable(2, CFG.num_experts, 2.0, device=cuda)
    table.set_cached(1, [0, 1, 2, 3])
    out = torch.empty((T, CFG.hidden), dtype=torch.float32, device=cuda)
    idx = torch.empty((T, CFG.top_k), dtype=torch.int32, device=cuda)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    row = table.row(1)
    with torch.cuda.stream(s):
        blk.forward(x, lg, row, out=out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            o, i, _ = blk.forward(x, lg, row, out_dtype=torch.float32, return_routing=True)
            out.copy_(o)
            idx.copy_(i)
    routed = []
    for cached in ([0, 1, 2, 3], [28, 29, 30, 31]):
        table.set_cached(1, cached)
        table.sync()
        with torch.cuda.stream(s):
            s.wait_stream(torch.cuda.current_stream())
            g.replay()
        torch.cuda.synchronize()
        mask = torch.zeros(CFG.num_experts, device=cuda)
        mask[cached] = 2.0
        want_o, want_i, _ = blk.forward(x, lg, mask, out_dtype=torch.float32, return_routing=True)
        torch.cuda.synchronize()
        assert torch.equal(idx, want_i) and torch.equal(out, want_o)
        routed.append(idx.clone())
    # the replays saw two different cached sets, so the routing moved
    assert not torch.equal(routed[0], routed[1])
