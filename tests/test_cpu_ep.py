"""Expert-parallel orchestration on CPU: two (and four) gloo ranks run
ep_forward with the oracle as the kernel backend and real collectives; the
result must equal the one-process oracle MoE block on every rank's tokens."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from expert_sniper_b200 import ep, hrw
from expert_sniper_b200.config import MoEConfig
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
from oracle import moe_oracle as mo


class OracleEPBackend:
    """ep_forward's backend on the oracle (fp32 numpy)."""

    def __init__(self, cfg, placement, rank, layer_np, sg):
        self.cfg, self.pl, self.rank = cfg, placement, rank
        owned = placement.owned[rank]
        self.local = {k: v[owned] for k, v in layer_np.items() if k.startswith("switch_mlp.")}
        self.shared_layer = {k: v for k, v in layer_np.items() if k.startswith("shared_expert.")}
        self.sg = sg

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype)

    def route(self, logits, bias):
        idx, w, _ = mo.route(logits.float().numpy(), None if bias is None else bias.numpy(),
                             self.cfg.top_k, self.cfg.norm_topk_prob)
        return torch.from_numpy(idx), torch.from_numpy(w)

    def mask(self, idx, w):
        si, sw = mo.ep_mask(idx.numpy(), w.numpy(), self.pl.owner, self.pl.local_id, self.pl.world)
        return torch.from_numpy(si), torch.from_numpy(sw)

    def ffn(self, x_all, idx, w):
        R, D = x_all.shape
        if not self.pl.owned[self.rank]:
            return torch.zeros((R, D), dtype=torch.float32)
        return torch.from_numpy(mo.expert_ffn(x_all.float().numpy(), self.local, idx.numpy(),
                                              w.numpy()))

    def shared(self, x):
        if not self.shared_layer:
            return None
        T = x.shape[0]
        lay = dict(self.shared_layer)
        return torch.from_numpy(mo.expert_ffn(x.float().numpy(), lay, np.full((T, 1), -1, np.int32),
                                              np.zeros((T, 1), np.float32), self.sg))

    def combine(self, partials, extra):
        out = partials[0].clone()
        for r in range(1, partials.shape[0]):
            out += partials[r]
        if extra is not None:
            out += extra
        return out


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cfg, policy, T, q):
    try:
        _work(rank, world, port, cfg, policy, T, q)
    except Exception as exc:  # report instead of leaving the parent waiting
        q.put((rank, f"error: {exc!r}", None))
        raise


def _work(rank, world, port, cfg, policy, T, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lay = {k: v.numpy() for k, v in synthetic_layer(cfg, seed=5).items()}
        x, _, logits, sg = synthetic_inputs(cfg, T, seed=100 + rank)
        sgn = None if sg is None else sg.float().numpy()
        bias = cache_bias_vector(cfg.num_experts, 0.5, 1)[0]
        pl = ep.make_placement(cfg.num_experts, world, policy)
        be = OracleEPBackend(cfg, pl, rank, lay, sgn)
        out = ep.ep_forward(be, x.float(), logits, bias)
        ref, _, _ = mo.moe_block(x.float().numpy(), logits.float().numpy(), lay, cfg.top_k,
                                 cfg.norm_topk_prob, bias.numpy(), sgn)
        rms = float(np.sqrt((ref ** 2).mean()))
        q.put((rank, float(np.abs(out.numpy() - ref).max()) / rms, pl.counts))
    finally:
        dist.destroy_process_group()


def _run(world, cfg, policy="hrw", T=5):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, policy, T, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errors = [r for r in res if isinstance(r[1], str)]
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
    return sorted(res)


@pytest.mark.parametrize("policy", ["hrw", "bounded"])
def test_ep_two_ranks_matches_single_block(policy):
    cfg = MoEConfig(256, 16, 4, 256, True, name="ep-small")
    for rank, rel, counts in _run(2, cfg, policy):
        assert rel < 1e-5, (rank, rel)
        assert sum(counts) == 16


def test_ep_four_ranks_with_shared_expert_and_empty_shard():
    # 3 experts over 4 ranks: at least one rank owns nothing
    cfg = MoEConfig(256, 3, 2, 256, True, shared_inter=256, name="ep-shared")
    res = _run(4, cfg, "hrw", T=3)
    assert any(c == 0 for c in res[0][2])
    for rank, rel, counts in res:
        assert rel < 1e-5, (rank, rel)


def test_placement_tables():
    pl = ep.make_placement(128, 8)
    assert pl.counts == [7, 20, 18, 17, 17, 11, 16, 22]
    for e in range(128):
        assert pl.owned[pl.owner[e]][pl.local_id[e]] == e
    b = ep.make_placement(128, 8, "bounded")
    assert max(b.counts) == 16
    assert pl.roster == hrw.gpu_roster(8)


def test_oracle_ep_mask():
    idx = np.array([[0, 2, -1], [1, 2, 0]], np.int32)
    w = np.array([[.5, .3, .2], [.1, .2, .7]], np.float32)
    si, sw = mo.ep_mask(idx, w, owner=[0, 1, 0], local_id=[0, 0, 1], world=2)
    assert si[0].tolist() == [[0, 1, -1], [-1, 1, 0]]
    assert si[1].tolist() == [[-1, -1, -1], [0, -1, -1]]
    assert (sw[1] == w).all()
