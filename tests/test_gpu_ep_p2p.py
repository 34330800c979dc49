"""Expert parallelism with the peer-to-peer exchange (es_ep_dispatch /
receive / return / combine_p2p; ep.P2PEPBackend) against the one-GPU MoE
block.

With one GPU the ranks are emulated in one process: every rank's window is
ordinary device memory of that GPU, the peers are set to those addresses,
and the ranks' phases run one after another on one stream (all dispatches,
then all receive / FFN / return, then all combines), so every flag a kernel
waits for was set by a kernel that already completed. With two or more GPUs
real ranks run as processes, one per GPU, with CUDA IPC mappings. Either way
the outputs must match the one-GPU block within 1e-3 x RMS (fp32 summation
order of the per-owner partials; fp16 h may round one ulp apart) over
several steps (the step counter advances in the combine), and a captured
CUDA graph of a whole step must replay to the same result.
Reference: src/expert_network/reader.py:237-292, node.py:142-172.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig, PRESETS, ep
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
from tests._helpers import assert_close_rms

pytestmark = pytest.mark.gpu

SMALL = MoEConfig(512, 32, 4, 512, True, shared_inter=512, name="ep-p2p")
EP_REL = 1e-3


def _emulated_step(bes, xs, lgs, bias, T):
    for b, x, lg in zip(bes, xs, lgs):
        b.route(lg, bias)
        b.dispatch(x, T)
    for b in bes:
        b.receive()
        b.ffn()
        b.ret()
    outs = []
    for b, x in zip(bes, xs):
        outs.append(b.combine(b.shared(x, T), T))
    return outs


@pytest.mark.parametrize("cfg,world,policy,T", [(SMALL, 1, "hrw", 5), (SMALL, 2, "hrw", 7),
                                                (SMALL, 4, "bounded", 3),
                                                (PRESETS["qwen3-30b-a3b"], 8, "bounded", 64),
                                                # prefill-sized: the owners run the 128-token
                                                # tensor-core kernels, the full block the
                                                # 32-token ones
                                                (PRESETS["qwen3-next-80b-a3b"], 2, "bounded",
                                                 1024)])
def test_p2p_emulated_ranks(cuda, cfg, world, policy, T):
    lay = synthetic_layer(cfg, seed=3, device=cuda)
    pl = ep.make_placement(cfg.num_experts, world, policy)
    bias = cache_bias_vector(cfg.num_experts, 0.5, 2)[0].to(cuda)
    sg = synthetic_inputs(cfg, 1, seed=49, device=cuda)[3]
    wins = [ep.EpWindows(world, r, T, cfg.hidden, cfg.top_k, cuda, local_only=True)
            for r in range(world)]
    for w in wins:
        w.set_peers([v.ptr for v in wins])
    bes = [ep.P2PEPBackend(cfg, pl, r, wins[r], layer=lay, shared_gate_w=sg,
                           out_dtype=torch.float32) for r in range(world)]
    full = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=T)
    for step in range(3):
        ins = [synthetic_inputs(cfg, T, seed=100 * step + r, device=cuda) for r in range(world)]
        xs = [i[0] for i in ins]
        lgs = [i[2] for i in ins]
        outs = _emulated_step(bes, xs, lgs, bias, T)
        torch.cuda.synchronize()
        for r in range(world):
            assert wins[r].read_error() == 0
            want = full.forward(xs[r], lgs[r], bias, out_dtype=torch.float32)
            assert_close_rms(outs[r].cpu().numpy(), want.cpu().numpy(), rel=EP_REL,
                             what=f"step {step} rank {r}")
    # one CUDA graph holding a whole step of every emulated rank
    xs = [x.clone() for x in xs]
    lgs = [g.clone() for g in lgs]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            outs = _emulated_step(bes, xs, lgs, bias, T)
    torch.cuda.synchronize()
    for step in range(2):
        ins = [synthetic_inputs(cfg, T, seed=7000 + 10 * step + r, device=cuda)
               for r in range(world)]
        for r in range(world):
            xs[r].copy_(ins[r][0])
            lgs[r].copy_(ins[r][2])
        g.replay()
        torch.cuda.synchronize()
        for r in range(world):
            assert wins[r].read_error() == 0
            want = full.forward(ins[r][0], ins[r][2], bias, out_dtype=torch.float32)
            assert_close_rms(outs[r].cpu().numpy(), want.cpu().numpy(), rel=EP_REL,
                             what=f"graph step {step} rank {r}")
    del g
    for w in wins:
        w.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        cfg, T = SMALL, 6
        lay = synthetic_layer(cfg, seed=3, device=dev)
        pl = ep.make_placement(cfg.num_experts, world, "hrw")
        bias = cache_bias_vector(cfg.num_experts, 0.5, 2)[0].to(dev)
        sg = synthetic_inputs(cfg, 1, seed=49, device=dev)[3]
        win = ep.EpWindows(world, rank, T, cfg.hidden, cfg.top_k, dev)
        be = ep.P2PEPBackend(cfg, pl, rank, win, layer=lay, shared_gate_w=sg,
                             out_dtype=torch.float32)
        full = MoEBlock(cfg, weights=lay, shared_gate_w=sg, max_tokens=T)
        worst = 0.0
        for step in range(4):
            x, _, lg, _ = synthetic_inputs(cfg, T, seed=100 * step + rank, device=dev)
            out = be.step(x, lg, bias).clone()
            want = full.forward(x, lg, bias, out_dtype=torch.float32)
            torch.cuda.synchronize()
            rms = float(want.pow(2).mean().sqrt())
            worst = max(worst, float((out - want).abs().max()) / rms)
        err = win.read_error()
        torch.cuda.synchronize()
        dist.barrier()
        win.close()
        dist.barrier()
        q.put((rank, worst, err))
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, f"error: {exc!r}", -1))


def test_p2p_real_ranks(cuda):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs (the emulated ranks cover the kernels on one)")
    import torch.multiprocessing as mp
    world = min(n, 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, rel, err in res:
        assert not isinstance(rel, str), (rank, rel)
        assert err == 0, (rank, err)
        assert rel < EP_REL, (rank, rel)
