"""Expert parallelism on the GPU kernels.

With two or more GPUs: NCCL ranks run ep_forward end to end. With one GPU:
the same backend kernels (router, es_ep_mask, expert FFN on a shard,
es_ep_combine) run for several emulated ranks on one device, with the
collectives replaced by the equivalent tensor moves. Either way the result
must match the one-GPU MoE block. The two differ in fp32 summation order
(per-owner partials summed in rank order, and split-K or not), and h is
rounded to fp16 after the gate/up sums, so an fp16 rounding of h may land one
ulp apart: the bound is 1e-3 x RMS (the parity bar is 1e-2)."""
from __future__ import annotations

import os
import socket

import pytest
import torch

from expert_sniper_b200 import MoEBlock, MoEConfig, ep
from expert_sniper_b200.quant import cache_bias_vector, synthetic_inputs, synthetic_layer
from tests._helpers import assert_close_rms

pytestmark = pytest.mark.gpu

CFG = MoEConfig(512, 32, 4, 512, True, shared_inter=512, name="ep-gpu")
EP_REL = 1e-3


def _emulated(world, policy, T, dev):
    lay = synthetic_layer(CFG, seed=3, device=dev)
    pl = ep.make_placement(CFG.num_experts, world, policy)
    bias = cache_bias_vector(CFG.num_experts, 0.5, 2)[0].to(dev)
    ins = [synthetic_inputs(CFG, T, seed=50 + r, device=dev) for r in range(world)]
    sg = ins[0][3]
    bes = [ep.CudaEPBackend(CFG, pl, r, layer=lay, shared_gate_w=sg, max_tokens=T, device=dev,
                            out_dtype=torch.float32) for r in range(world)]
    # per home rank: route + masks
    masks = [bes[r].mask(*bes[r].route(ins[r][2], bias)) for r in range(world)]
    x_all = torch.cat([ins[r][0] for r in range(world)])                 # all_gather
    partials = []
    for d in range(world):                                                # owner d
        idx = torch.cat([masks[s][0][d] for s in range(world)])          # all_to_all
        w = torch.cat([masks[s][1][d] for s in range(world)])
        partials.append(bes[d].ffn(x_all, idx, w).view(world, T, -1))
    full = MoEBlock(CFG, weights=lay, shared_gate_w=sg, max_tokens=T)
    for r in range(world):
        recv = torch.stack([partials[d][r] for d in range(world)])        # all_to_all back
        out = bes[r].combine(recv, bes[r].shared(ins[r][0]))
        want = full.forward(ins[r][0], ins[r][2], bias, out_dtype=torch.float32)
        assert_close_rms(out.cpu().numpy(), want.cpu().numpy(), rel=EP_REL, what=f"rank {r}")
    return pl


@pytest.mark.parametrize("world,policy", [(2, "hrw"), (4, "bounded"), (8, "hrw")])
def test_ep_kernels_emulated_ranks(cuda, world, policy):
    _emulated(world, policy, T=6, dev=cuda)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        lay = synthetic_layer(CFG, seed=3, device=dev)
        pl = ep.make_placement(CFG.num_experts, world, "hrw")
        bias = cache_bias_vector(CFG.num_experts, 0.5, 2)[0].to(dev)
        x, _, logits, sg = synthetic_inputs(CFG, 5, seed=50 + rank, device=dev)
        sg0 = synthetic_inputs(CFG, 5, seed=50, device=dev)[3]
        be = ep.CudaEPBackend(CFG, pl, rank, layer=lay, shared_gate_w=sg0, max_tokens=5,
                              device=dev, out_dtype=torch.float32)
        out = ep.ep_forward(be, x, logits, bias)
        full = MoEBlock(CFG, weights=lay, shared_gate_w=sg0, max_tokens=5)
        want = full.forward(x, logits, bias, out_dtype=torch.float32)
        torch.cuda.synchronize()
        rms = float(want.pow(2).mean().sqrt())
        q.put((rank, float((out - want).abs().max()) / rms))
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, f"error: {exc!r}"))


def test_ep_nccl_ranks(cuda):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs (the one-GPU emulation covers the kernels)")
    import torch.multiprocessing as mp
    world = min(n, 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, rel in res:
        assert not isinstance(rel, str), (rank, rel)
        assert rel < EP_REL, (rank, rel)
