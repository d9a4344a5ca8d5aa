"""moc_router_backward_noalloc: the router backward for callers that cannot allocate.

Some users of this library never get to call cudaMalloc: a host that reaches the
kernels only through the C ABI and holds nothing but the tensors it was handed, or a
server that fixes all of its device memory at start-up and must not allocate while it
runs.  For them the no-allocation entry point keeps its scratch (the per-CTA dweight
partials) in a fixed device array inside the library instead of a caller workspace.
These tests call it through the C ABI and check that, on two calls in a row on
different problems (the second reusing the array the first one wrote), it returns what
moc_router_backward returns with a workspace: within the bf16 tolerance of the other GPU
tests (max|err| / max|ref| <= 2e-2), and in fact bitwise, since both run the same kernels
and the same fixed-order reduction.  The file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import moc.ops as ops
from conftest import rel_err
from moc import _lib

pytestmark = pytest.mark.gpu

BF16 = 2
TOL = 2e-2


def _inputs(N, Dz, K, seed):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(N, Dz, generator=g).bfloat16().cuda()
    w = (torch.randn(K, Dz, generator=g) * 0.02).bfloat16().cuda()
    dalpha = torch.randn(N, K, generator=g).bfloat16().cuda()
    return z, w, dalpha


@pytest.mark.parametrize("router", ["softmax", "exp"])
def test_noalloc_matches_workspace_entry_point_twice(router):
    """Two calls in a row on different problems: the second reuses the array the first
    one filled, so a partial it failed to rewrite would carry the first call's values.
    Both calls run the same kernels and the same fixed-order reduction as the workspace
    entry point, so the results must be bitwise equal to it (which is within the 2e-2
    tolerance of the other GPU tests, also asserted)."""
    lib = _lib.load()
    act = ops.ROUTER_ACTIVATIONS[router]
    stream = torch.cuda.current_stream().cuda_stream
    for N, Dz, K, seed in ((4096, 2048, 16, 21), (1000, 1536, 32, 22)):
        z, w, dalpha = _inputs(N, Dz, K, seed)
        alpha = ops.launch_router_forward(z, w, router)
        ref_dz, ref_dw = ops.launch_router_backward(z, w, alpha, dalpha, router)
        dz = torch.full_like(z, float("nan"))
        dw = torch.full_like(w, float("nan"))
        rc = lib.moc_router_backward_noalloc(
            N, Dz, K, BF16, act, z.data_ptr(), w.data_ptr(), alpha.data_ptr(), dalpha.data_ptr(), BF16,
            dz.data_ptr(), dw.data_ptr(), stream,
        )
        assert rc == 0, lib.moc_error_string(rc).decode()
        torch.cuda.synchronize()
        assert rel_err(dz, ref_dz) <= TOL
        assert rel_err(dw, ref_dw) <= TOL
        assert torch.equal(dz, ref_dz), f"dz differs from the workspace entry point ({N}, {Dz}, {K})"
        assert torch.equal(dw, ref_dw), f"dweight differs from the workspace entry point ({N}, {Dz}, {K})"
    assert _lib.device_status(clear=True) == 0, "a staging wait ran out"


def test_noalloc_rejects_what_it_cannot_serve():
    lib = _lib.load()
    t = torch.zeros(16, device="cuda", dtype=torch.bfloat16)
    p = t.data_ptr()
    # partials of a 32-base router over 131072 columns need 16 MiB > MOC_NOALLOC_SCRATCH_BYTES
    assert lib.moc_router_backward_noalloc(64, 131072, 32, BF16, 0, p, p, p, p, BF16, p, p, None) == 7
    assert "scratch" in lib.moc_error_string(7).decode()
    # fp32 routers run on the workspace entry point only
    assert lib.moc_router_backward_noalloc(64, 64, 16, 0, 0, p, p, p, p, 0, p, p, None) == 2
    # shapes outside the tensor-core router
    assert lib.moc_router_backward_noalloc(64, 64, 12, BF16, 0, p, p, p, p, BF16, p, p, None) == 3
    torch.cuda.synchronize()
