"""Two NCCL ranks on two GPUs (skipped with fewer): the one all-reduce of
dconv_bases / drouter returns the sum over ranks of each rank's own gradients, eagerly
and inside a CUDA graph (how bench.py runs it).  Ranks are child processes (127.0.0.1) with
NVLS off and a short process-group timeout."""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from moc import MoC, dp

        torch.manual_seed(5)
        m = MoC(dim=256, z_dim=192, kernel_size=4, k=16, init_std=0.02).to(dev, torch.bfloat16)
        with torch.no_grad():
            m.router.normal_(0, 0.02, generator=torch.Generator(device=dev).manual_seed(6))
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(2, 128, 256, generator=g).bfloat16().to(dev).requires_grad_()
        z = torch.randn(2, 128, 192, generator=g).bfloat16().to(dev).requires_grad_()
        dy = torch.randn(2, 128, 256, generator=g).bfloat16().to(dev)

        def step(reducer=None):
            y, _ = m(x, z)
            grads = torch.autograd.grad(y, (m.conv_bases, m.router), dy)
            if reducer is not None:
                reducer(grads)
            return grads

        own = [t.float() for t in step()]
        expect = []
        for t in own:
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            expect.append(sum(parts))
        reducer = dp.GradAllReduce([m.conv_bases, m.router])
        eager = [t.float() for t in step(reducer)]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            captured = step(reducer)
        graph.replay()
        torch.cuda.synchronize()
        graphed = [t.float() for t in captured]
        del graph
        res = []
        for e, a, b in zip(expect, eager, graphed):
            scale = e.abs().max().item()
            res.append(((a - e).abs().max().item() / scale, (b - e).abs().max().item() / scale))
        out[rank] = res
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_allreduce_sums_parameter_gradients_over_two_gpus():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        for eager_err, graph_err in res[r]:
            # bf16 gradients summed in fp32 and rounded once to bf16
            assert eager_err <= 1e-2 and graph_err <= 1e-2, res[r]
