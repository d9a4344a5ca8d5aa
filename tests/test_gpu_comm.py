"""The NVLink gradient all-reduce (moc_comm_* / moc.dp.NVLinkGradAllReduce).

* One rank on one GPU: the sum over one rank is the data itself (bf16 and fp32 segments
  through the fp32 exchange buffer), over repeated calls (the buffer halves alternate) and
  replays of a CUDA graph that holds the call.
* Two NCCL ranks on two GPUs (skipped with fewer): every rank gets the sum of both ranks'
  tensors, the same bits on both ranks, eagerly and from a graph replay.  Ranks are child
  processes (127.0.0.1) with NVLS off and a short process-group timeout; every wait in the
  kernel is bounded, and the device status must show no timeout.
"""
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


def _tensors(rank: int, dev):
    g = torch.Generator().manual_seed(40 + rank)
    a = torch.randn(16, 4, 300, generator=g).bfloat16().to(dev)   # dconv_bases-shaped
    b = torch.randn(16, 520, generator=g).to(dev)                  # fp32
    c = torch.randn(7, generator=g).bfloat16().to(dev)
    return [a, b, c]


def test_single_rank_is_identity_eager_and_graphed():
    from moc import _lib, dp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        dev = torch.device("cuda", 0)
        ts = _tensors(0, dev)
        ref = [t.clone() for t in ts]
        red = dp.NVLinkGradAllReduce(ts)
        for _ in range(3):
            red(ts)
        torch.cuda.synchronize()
        for t, r in zip(ts, ref):
            assert torch.equal(t, r)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            red(ts)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        for t, r in zip(ts, ref):
            assert torch.equal(t, r)
        del graph
        assert _lib.device_status(clear=True) == 0
        red.close()
    finally:
        dist.destroy_process_group()


def _rank_main(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from moc import _lib, dp

        ts = _tensors(rank, dev)
        expect = []
        for t in ts:
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            total = torch.zeros_like(t, dtype=torch.float32)
            for p in parts:
                total += p.float()
            expect.append(total.to(t.dtype))
        red = dp.NVLinkGradAllReduce(ts)
        mine = [t.clone() for t in ts]
        red(mine)
        torch.cuda.synchronize()
        eager_ok = all(torch.equal(m, e) for m, e in zip(mine, expect))
        # graph replays: three sums of fresh copies of the original tensors
        work = [t.clone() for t in ts]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            red(work)
        graph_ok = True
        for _ in range(3):
            for w, t in zip(work, ts):
                w.copy_(t)
            graph.replay()
            torch.cuda.synchronize()
            graph_ok &= all(torch.equal(w, e) for w, e in zip(work, expect))
        del graph
        # bitwise the same on both ranks
        same = True
        for m in mine:
            parts = [torch.empty_like(m) for _ in range(world)]
            dist.all_gather(parts, m)
            same &= all(torch.equal(p, parts[0]) for p in parts)
        status = _lib.device_status(clear=True)
        dist.barrier()
        red.close()
        out[rank] = (eager_ok, graph_ok, same, status)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_sum_and_agree():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        assert res[r] == (True, True, True, 0), res


def _skip_rank_main(rank: int, world: int, port: int, out):
    """Rank 1 skips one call of the all-reduce (between steps: none of its kernels is in
    flight).  Rank 0's call gives up after a short poll limit; the step-boundary check
    raises CommTimeout on both ranks and resets both communicators; the next call sums."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from moc import dp

        ts = _tensors(rank, dev)
        expect = []
        for t in ts:
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            total = torch.zeros_like(t, dtype=torch.float32)
            for p in parts:
                total += p.float()
            expect.append(total.to(t.dtype))
        red = dp.NVLinkGradAllReduce(ts)
        red.set_poll_limit(1 << 14)
        skipped = [t.clone() for t in ts]
        if rank == 0:
            red(skipped)  # rank 1 makes no matching call
        raised = False
        try:
            red.check()
        except dp.CommTimeout:
            raised = True
        unchanged = all(torch.equal(s, t) for s, t in zip(skipped, ts))
        red.set_poll_limit(0)
        again = [t.clone() for t in ts]
        red(again)
        red.check()
        summed = all(torch.equal(a, e) for a, e in zip(again, expect))
        dist.barrier()
        red.close()
        out[rank] = (raised, unchanged, summed)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_skipped_call_times_out_raises_on_every_rank_and_recovers():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_skip_rank_main, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        assert res[r] == (True, True, True), res
