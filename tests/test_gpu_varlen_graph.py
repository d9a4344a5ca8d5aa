"""Packed varlen without host offsets: no stream synchronisation, capturable in a CUDA graph.

The reference builds its chunk table with ``repeat_interleave`` on ``cu_seqlens``, which
waits for the device unless ``cu_seqlens_cpu`` is given (moc/ops.py:82-97).  Here, without
``cu_seqlens_cpu``, the module sizes the table by the bound n_tokens // 64 + n_seqs and
fills it on the device (padding rows (-1, -1) are skipped by the kernels), so
``MoC.forward(..., cu_seqlens=...)`` and its backward run with no host read and can be
captured in a CUDA graph.  The checks:

* the bound-sized table starts with the reference's table and pads with (-1, -1);
* forward + backward without ``cu_seqlens_cpu`` raise under torch's sync-debug mode "error";
  i.e. they issue no synchronising call;
* a graph of that step replays to bitwise the eager results;
* the eager results equal those with the exact table (``cu_seqlens_cpu`` given) bitwise for
  y, dx, dz and drouter; dbasis sums its per-CTA partials over a different number of CTA
  groups, so it agrees to fp32 rounding (<= 1e-5 relative) instead;
* and they match the float64 oracle within the bf16 tolerance (2e-2).
"""
from __future__ import annotations

import pytest
import torch

import moc.ops as ops
from conftest import rel_err
from moc import MoC
from oracle import moc_oracle as O

pytestmark = pytest.mark.gpu

LENS = [100, 64, 136, 1, 3, 119, 64, 200, 2]


def _setup(seed=5):
    torch.manual_seed(seed)
    m = MoC(dim=256, z_dim=192, kernel_size=4, k=16, activation="silu", init_std=0.05, router_activation="exp")
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        m.router.copy_(torch.randn(16, 192, generator=g) * 0.05)
    m = m.to(device="cuda", dtype=torch.bfloat16)
    cu_cpu = torch.tensor([0] + torch.tensor(LENS).cumsum(0).tolist(), dtype=torch.int32)
    n = int(cu_cpu[-1])
    x = torch.randn(n, 256, generator=g).bfloat16()
    z = torch.randn(n, 192, generator=g).bfloat16()
    dy = torch.randn(n, 256, generator=g).bfloat16()
    return m, cu_cpu, x, z, dy


def _step(m, x, z, dy, cu, cu_cpu=None):
    y, _ = m(x, z, cu_seqlens=cu, max_seqlen=max(LENS), cu_seqlens_cpu=cu_cpu)
    grads = torch.autograd.grad(y, (x, z, m.conv_bases, m.router), dy)
    # y detached: a kept output would keep its autograd graph (and the leaves' gradient
    # accumulators, made on the eager stream) alive into the capture
    return (y.detach(),) + grads


NAMES = ("y", "dx", "dz", "dbasis", "drouter")


def test_bound_sized_table_pads_the_reference_table():
    _, cu_cpu, x, _, _ = _setup()
    cu = cu_cpu.cuda()
    exact = ops.prepare_chunk_indices(cu, cu_seqlens_cpu=cu_cpu)
    bound = ops.chunk_indices_upper_bound(cu, x.shape[0])
    assert bound.shape[0] == x.shape[0] // 64 + len(LENS) >= exact.shape[0]
    assert torch.equal(bound[: exact.shape[0]], exact)
    assert bool((bound[exact.shape[0]:] == -1).all())
    ref = torch.tensor(O.chunk_indices(cu_cpu, 64), dtype=torch.int64)
    assert torch.equal(exact.cpu().long(), ref)


def test_varlen_without_host_offsets_is_sync_free_and_graph_capturable():
    m, cu_cpu, x, z, dy = _setup()
    cu = cu_cpu.cuda()
    xd, zd, dyd = x.cuda().requires_grad_(), z.cuda().requires_grad_(), dy.cuda()

    ops.clear_chunk_index_cache()
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        eager = _step(m, xd, zd, dyd, cu)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    exact = _step(m, xd, zd, dyd, cu, cu_cpu)

    # warm-up on a side stream, then capture the step (no cu_seqlens_cpu) and replay it
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _step(m, xd, zd, dyd, cu)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = _step(m, xd, zd, dyd, cu)
    graph.replay()
    torch.cuda.synchronize()
    for name, a, b in zip(NAMES, captured, eager):
        assert torch.equal(a, b), f"graph replay differs from eager: {name}"
    del graph

    for name, a, b in zip(NAMES, eager, exact):
        if name == "dbasis":
            assert rel_err(a, b) <= 1e-5, name
        else:
            assert torch.equal(a, b), f"bound-sized table changed {name}"

    ref = O.module_grads(x, z, m.router.detach().cpu(), m.conv_bases.detach().cpu(), dy,
                         router_activation="exp", activation="silu", cu_seqlens=cu_cpu)
    for name, got in zip(NAMES, eager):
        assert rel_err(got, ref[name]) <= 2e-2, name
