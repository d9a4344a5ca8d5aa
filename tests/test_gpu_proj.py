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
    y = fused.proj_forward(h, w, m, alpha=alpha)  # the module's parameters require grad: training launch
    ref = _reference(m, h, w, alpha)
    assert rel_err(y, ref) <= TOL
    with torch.no_grad():  # the inference launch (no x copy) gives the same y
        assert torch.equal(fused.proj_forward(h, w, m, alpha=alpha), y.detach())
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


# ---------------------------------------------------------------------------- training

def _oracle_proj_grads(m, h, w, dy):
    """float64 reference of the projection + module training step with z = h (the reference's
    attention block routes by the projection's own input): x = h . w^T rounded to bf16 (its
    gradient passes straight through, as autograd treats the bf16 qkv tensor), then the
    oracle module backward; dh = dx . w + dz, dw = dx^T . h."""
    h64, w64 = h.detach().cpu().double(), w.detach().cpu().double()
    x = (h64 @ w64.T).bfloat16().double()
    g = O.module_grads(x, h64, m.router.detach().cpu(), m.conv_bases.detach().cpu(), dy.cpu(),
                       router_activation=m.router_activation, activation=m.activation)
    B, T, Dm = h.shape
    dx = g["dx"].reshape(B * T, -1)
    return {"y": g["y"], "dh": (dx @ w64).reshape(B, T, Dm) + g["dz"], "dw": dx.T @ h64.reshape(B * T, Dm),
            "dbasis": g["dbasis"], "drouter": g["drouter"]}


def _train_grads(run, h, w, mods, dys):
    hq = h.detach().clone().requires_grad_()
    wq = w.detach().clone().requires_grad_()
    for m in mods:
        m.zero_grad(set_to_none=True)
    ys = run(hq, wq)
    torch.autograd.backward([y for y, d in zip(ys, dys) if d is not None], [d for d in dys if d is not None])
    out = {"ys": [y.detach() for y in ys], "dh": hq.grad, "dw": wq.grad}
    for i, m in enumerate(mods):
        out[f"dbasis{i}"] = None if m.conv_bases.grad is None else m.conv_bases.grad.clone()
        out[f"drouter{i}"] = None if m.router.grad is None else m.router.grad.clone()
    return out


@pytest.mark.parametrize("B,T,Dm,D,K,S,act", [
    (2, 300, 256, 256, 16, 4, None),
    (1, 257, 200, 200, 16, 8, "silu"),   # ragged in_dim and dim, several tiles
    (3, 5, 64, 64, 8, 3, "silu"),        # sequences shorter than the halo
])
def test_proj_training_matches_oracle(B, T, Dm, D, K, S, act):
    """proj_forward under autograd: y and every gradient (h, weight, conv_bases, router) against
    the float64 reference, and against the unfused GPU path (projection GEMM, then the module)."""
    m, h, w = _case(B, T, Dm, D, K, S, act, seed=11)
    g = torch.Generator().manual_seed(12)
    dy = torch.randn(B, T, D, generator=g).bfloat16().cuda()
    got = _train_grads(lambda hq, wq: [fused.proj_forward(hq, wq, m, z=hq)], h, w, [m], [dy])
    ref = _oracle_proj_grads(m, h, w, dy)
    assert rel_err(got["ys"][0], ref["y"]) <= TOL
    for key, gk in (("dh", "dh"), ("dw", "dw"), ("dbasis", "dbasis0"), ("drouter", "drouter0")):
        assert rel_err(got[gk], ref[key]) <= TOL, key
    unf = _train_grads(lambda hq, wq: [m(hq @ wq.T, hq)[0]], h, w, [m], [dy])
    for key in ("dh", "dw", "dbasis0", "drouter0"):
        assert rel_err(got[key], unf[key]) <= TOL, key
    assert _lib.device_status(clear=True) == 0


def test_proj_multi_training_matches_unfused():
    """proj_forward_multi under autograd (q / k / v over one weight, routed by h) against the
    unfused path (one projection GEMM, split, each module on its slice); the k output takes no
    part in the loss, so its bases and router get no gradient and its dx is zero."""
    torch.manual_seed(21)
    B, T, Dm, S = 2, 250, 256, 4
    dims, acts, racts = (256, 128, 128), ("silu", None, None), ("exp", "exp", "softmax")
    g = torch.Generator().manual_seed(22)
    mods = []
    for D, act, ra in zip(dims, acts, racts):
        m = MoC(dim=D, z_dim=Dm, kernel_size=S, k=16, activation=act, init_std=0.1, router_activation=ra)
        with torch.no_grad():
            m.router.copy_(torch.randn(16, Dm, generator=g) * 0.05)
        mods.append(m.to(device="cuda", dtype=torch.bfloat16))
    h = torch.randn(B, T, Dm, generator=g).bfloat16().cuda()
    w = (torch.randn(sum(dims), Dm, generator=g) / Dm ** 0.5).bfloat16().cuda()
    dys = [torch.randn(B, T, D, generator=g).bfloat16().cuda() for D in dims]
    dys[1] = None
    offs = [0, dims[0], dims[0] + dims[1], sum(dims)]

    def unfused(hq, wq):
        qkv = hq @ wq.T
        return [m(qkv[..., offs[i]:offs[i + 1]], hq)[0] for i, m in enumerate(mods)]

    got = _train_grads(lambda hq, wq: fused.proj_forward_multi(hq, wq, mods, z=hq), h, w, mods, dys)
    ref = _train_grads(unfused, h, w, mods, dys)
    for a, b in zip(got["ys"], ref["ys"]):
        assert rel_err(a, b) <= TOL
    for key in ("dh", "dw", "dbasis0", "drouter0", "dbasis2", "drouter2"):
        assert rel_err(got[key], ref[key]) <= TOL, key
    assert got["dbasis1"] is None and got["drouter1"] is None
    assert torch.count_nonzero(got["dw"][offs[1]:offs[2]]) == 0  # rows of the unused module
    assert _lib.device_status(clear=True) == 0


def test_proj_training_saves_the_rounded_projection():
    """The training launch writes x = bf16(h . w^T) next to y: y equals the inference launch's
    bitwise, x matches the float64 projection to bf16 rounding, and moc_forward on x gives y
    back within the convolution's bf16 tolerance."""
    import ctypes
    import moc.ops as ops

    m, h, w = _case(2, 300, 256, 256, 16, 4, "silu", seed=31)
    alpha = ops.launch_router_forward(h, m.router.detach(), m.router_activation)
    with torch.no_grad():
        y_inf = fused.proj_forward(h, w, m, alpha=alpha)
    B, T, Dm = h.shape
    out = torch.empty(B, T, m.dim, dtype=torch.bfloat16, device="cuda")
    x = torch.full((B, T, m.dim), float("nan"), dtype=torch.bfloat16, device="cuda")
    basis = m.conv_bases.detach().contiguous()
    prob = _lib.MocProjProblem(batch=B, seq_len=T, in_dim=Dm, dim=m.dim, n_bases=m.k, kernel_size=m.kernel_size,
                               activation=1, h=h.data_ptr(), weight=w.data_ptr(), alpha=alpha.data_ptr(),
                               basis=basis.data_ptr(), out=out.data_ptr())
    rc = _lib.load().moc_proj_forward_save(ctypes.byref(prob), x.data_ptr(), _lib.stream_of(h.device))
    _lib.check(rc, "moc_proj_forward_save")
    assert torch.equal(out, y_inf)
    x_ref = (h.double() @ w.double().T)
    assert not torch.isnan(x).any()
    assert rel_err(x, x_ref) <= 1e-2
    y_again = ops.launch_forward(x, alpha, basis, activation_flag=1)
    assert rel_err(y_again, out) <= 1e-2
    assert _lib.device_status(clear=True) == 0
