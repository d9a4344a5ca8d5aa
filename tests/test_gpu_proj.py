"""GPU parity of the fused projection + convolution forward (moc_proj_forward).

The reference: the projection in float64 from the same bf16 inputs, rounded to bf16 (the
reference's bf16 qkv tensor), then the oracle convolution; tolerance as for the bf16
convolution, max|err| / max|ref| <= 2e-2.  The unfused GPU path (torch matmul, then
moc_forward) is compared the same way.
"""
from __future__ import annotations

import pytest
import torch

from conftest import rel_err
from moc import MoC, _lib
from moc import fused
from oracle import moc_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _case(B, T, Dm, D, K, S, act, router_act="softmax", seed=0):
    torch.manual_seed(seed)
    m = MoC(dim=D, z_dim=Dm, kernel_size=S, k=K, activation=act, init_std=0.1, router_activation=router_act)
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        m.router.copy_(torch.randn(K, Dm, generator=g) * 0.05)
    m = m.to(device="cuda", dtype=torch.bfloat16)
    h = torch.randn(B, T, Dm, generator=g).bfloat16().cuda()
    w = (torch.randn(D, Dm, generator=g) / Dm ** 0.5).bfloat16().cuda()
    return m, h, w


def _reference(m, h, w, alpha):
    x = (h.cpu().double() @ w.cpu().double().T).bfloat16().double()
    return O.conv(x, alpha.cpu().double(), m.conv_bases.detach().cpu().double(), activation=m.activation)


@pytest.mark.parametrize("B,T,Dm,D,K,S,act", [
    (2, 300, 256, 256, 16, 4, None),     # several tiles per sequence, two sequences
    (1, 120, 128, 128, 16, 4, "silu"),   # exactly one tile
    (3, 5, 64, 64, 8, 3, None),          # sequences shorter than the halo
    (1, 257, 200, 200, 16, 8, "silu"),   # ragged in_dim (k-block) and dim (channel tile)
    (2, 130, 512, 384, 16, 1, None),
    (1, 1000, 1024, 512, 16, 2, "silu"),
])
def test_proj_matches_reference(B, T, Dm, D, K, S, act):
    m, h, w = _case(B, T, Dm, D, K, S, act)
    z = h
    import moc.ops as ops

    alpha = ops.launch_router_forward(z, m.router.detach(), m.router_activation)
    y = fused.proj_forward(h, w, m, alpha=alpha)
    ref = _reference(m, h, w, alpha)
    assert rel_err(y, ref) <= TOL
    # the unfused GPU path on the same inputs
    y2, _ = m(h @ w.T, z)
    assert rel_err(y, y2.detach()) <= TOL
    assert _lib.device_status(clear=True) == 0


def test_proj_routes_from_z_and_rejects_bad_arguments():
    m, h, w = _case(1, 64, 128, 128, 16, 4, None, router_act="exp")
    y = fused.proj_forward(h, w, m, z=h)
    y2, _ = m(h @ w.T, h)
    assert rel_err(y, y2.detach()) <= TOL
    with pytest.raises(ValueError):
        fused.proj_forward(h, w, m)                       # neither z nor alpha
    with pytest.raises(ValueError):
        fused.proj_forward(h, w[:64], m, z=h)             # weight rows != module.dim
    with pytest.raises(ValueError):
        fused.proj_forward(h.float(), w, m, z=h)          # not bf16


def test_proj_is_deterministic():
    m, h, w = _case(2, 500, 256, 256, 16, 4, "silu", seed=3)
    a = fused.proj_forward(h, w, m, z=h)
    b = fused.proj_forward(h, w, m, z=h)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dims,acts", [((512, 128, 128), (None, None, None)),
                                       ((256, 200, 64), ("silu", None, "silu")),
                                       ((384,), (None,))])
def test_proj_multi_matches_per_module_calls(dims, acts):
    """One launch over the concatenated weight gives each module bitwise what its own
    moc_proj_forward gives (same tiles, same sums)."""
    torch.manual_seed(5)
    B, T, Dm, S = 2, 250, 256, 4
    g = torch.Generator().manual_seed(6)
    mods = []
    for D, act in zip(dims, acts):
        m = MoC(dim=D, z_dim=Dm, kernel_size=S, k=16, activation=act, init_std=0.1, router_activation="exp")
        with torch.no_grad():
            m.router.copy_(torch.randn(16, Dm, generator=g) * 0.05)
        mods.append(m.to(device="cuda", dtype=torch.bfloat16))
    h = torch.randn(B, T, Dm, generator=g).bfloat16().cuda()
    w = (torch.randn(sum(dims), Dm, generator=g) / Dm ** 0.5).bfloat16().cuda()
    ys = fused.proj_forward_multi(h, w, mods, z=h)
    off = 0
    for m, y, D in zip(mods, ys, dims):
        ref = fused.proj_forward(h, w[off:off + D], m, z=h)
        assert torch.equal(y, ref)
        y2, _ = m(h @ w[off:off + D].T, h)
        assert rel_err(y, y2.detach()) <= TOL
        off += D
    assert _lib.device_status(clear=True) == 0
    with pytest.raises(ValueError):
        fused.proj_forward_multi(h, w[:-8], mods, z=h)  # weight rows != sum of dims
