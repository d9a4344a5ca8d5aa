"""Data-parallel host logic on the CPU: the sequence sharding and the one all-reduce of
the parameter gradients, run as two gloo ranks (127.0.0.1) against the float64 oracle of
the whole batch.  Sharding whole sequences and summing dbasis / drouter over ranks must
reproduce the single-process gradients, since sequences share nothing but parameters."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from moc import dp
from oracle import moc_oracle as O


def test_shard_fixed_partitions_the_batch():
    for batch in (0, 1, 4, 5, 8, 13):
        for world in (1, 2, 3, 4, 8):
            got = [dp.shard_fixed(batch, r, world) for r in range(world)]
            assert got[0].start == 0 and got[-1].stop == batch
            for a, b in zip(got, got[1:]):
                assert a.stop == b.start
            sizes = [s.stop - s.start for s in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        dp.shard_fixed(4, 2, 2)


def test_shard_varlen_covers_balances_and_rebases():
    g = torch.Generator().manual_seed(3)
    for world in (1, 2, 3, 4, 8):
        lens = torch.randint(1, 300, (17,), generator=g)
        cu = torch.cat((torch.zeros(1, dtype=torch.int64), lens.cumsum(0)))
        total = int(cu[-1])
        prev = 0
        for r in range(world):
            t0, t1, local = dp.shard_varlen(cu, r, world)
            assert t0 == prev and t1 >= t0
            prev = t1
            assert int(local[0]) == 0 and int(local[-1]) == t1 - t0
            # rank boundaries fall on sequence boundaries
            assert t0 in cu.tolist() and t1 in cu.tolist()
            # balanced to within the longest sequence
            assert abs((t1 - t0) - total / world) <= 2 * int(lens.max())
        assert prev == total
    with pytest.raises(ValueError):
        dp.shard_varlen([1, 4], 0, 1)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(varlen: bool):
    g = torch.Generator().manual_seed(11)
    B, T, D, Dz, K, S = 4, 24, 16, 12, 4, 3
    x = torch.randn(B * T, D, generator=g)
    z = torch.randn(B * T, Dz, generator=g)
    dy = torch.randn(B * T, D, generator=g)
    w = torch.randn(K, Dz, generator=g) * 0.3
    basis = torch.randn(K, S, D, generator=g) * 0.3
    cu = torch.tensor([0, 5, 30, 31, 60, 96]) if varlen else None
    return B, T, x, z, dy, w, basis, cu


def _rank_main(rank: int, world: int, port: int, varlen: bool, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, T, x, z, dy, w, basis, cu = _inputs(varlen)
        if varlen:
            t0, t1, local_cu = dp.shard_varlen(cu, rank, world)
            rows = slice(t0, t1)
        else:
            seqs = dp.shard_fixed(B, rank, world)
            rows, local_cu = slice(seqs.start * T, seqs.stop * T), None
        xs, zs, dys = x[rows], z[rows], dy[rows]
        if not varlen:
            xs, zs, dys = (t.reshape(-1, T, t.shape[-1]) for t in (xs, zs, dys))
        got = O.module_grads(xs, zs, w, basis, dys, "softmax", "silu", cu_seqlens=local_cu)
        params = [torch.zeros_like(basis, dtype=torch.float64), torch.zeros_like(w, dtype=torch.float64)]
        reducer = dp.GradAllReduce(params)
        dbasis, drouter = reducer([got["dbasis"].clone(), got["drouter"].clone()])
        out[rank] = (dbasis, drouter, rows, got["dx"].reshape(-1, x.shape[1]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("varlen", [False, True], ids=["fixed", "varlen"])
def test_two_gloo_ranks_reproduce_the_whole_batch_gradients(varlen):
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(world, _free_port(), varlen, out), nprocs=world, join=True)
        res = dict(out)
    B, T, x, z, dy, w, basis, cu = _inputs(varlen)
    if not varlen:
        x, z, dy = (t.reshape(B, T, -1) for t in (x, z, dy))
    full = O.module_grads(x, z, w, basis, dy, "softmax", "silu", cu_seqlens=cu)
    # the summed parameter gradients agree on every rank, up to float64 summation order
    for r in range(world):
        dbasis, drouter, _, _ = res[r]
        torch.testing.assert_close(dbasis, full["dbasis"], rtol=1e-10, atol=1e-12)
        torch.testing.assert_close(drouter, full["drouter"], rtol=1e-10, atol=1e-12)
    # and the activation gradients of each shard are its rows of the whole-batch ones
    dx_full = full["dx"].reshape(-1, x.shape[-1])
    for r in range(world):
        _, _, rows, dx = res[r]
        torch.testing.assert_close(dx, dx_full[rows], rtol=1e-10, atol=1e-12)


class _FakeComm(dp.NVLinkGradAllReduce):
    """The step-boundary check of NVLinkGradAllReduce with the device calls replaced: each
    rank reports the status bits `fail` says, and counts its resets."""

    def __init__(self, bits: int):
        self.group, self.device, self._comm = None, torch.device("cpu"), None
        self.bits, self.resets = bits, 0

    def _sync(self):
        pass

    def status(self, clear=False):
        bits = self.bits
        if clear:
            self.bits = 0
        return bits

    def reset(self):
        self.resets += 1
        self.bits = 0


def _check_main(rank: int, world: int, port: int, failing: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = _FakeComm(1 if rank == failing else 0)
        first = "ok"
        try:
            comm.check()
        except dp.CommTimeout:
            first = "raised"
        second = "ok"
        try:
            comm.check()  # after the reset every rank is consistent again
        except dp.CommTimeout:
            second = "raised"
        out[rank] = (first, second, comm.resets)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("failing", [-1, 0, 1], ids=["none", "rank0", "rank1"])
def test_allreduce_timeout_raises_on_every_rank_and_resets_all(failing):
    """A timeout seen by one rank makes every rank raise CommTimeout and reset (so the
    ranks' call counters pair up again); with no timeout nobody raises or resets."""
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_check_main, args=(world, _free_port(), failing, out), nprocs=world, join=True)
        res = dict(out)
    want = ("ok", "ok", 0) if failing < 0 else ("raised", "ok", 1)
    assert all(res[r] == want for r in range(world)), res
