"""Fused multi-module decode (moc.fused.decode_step / moc_decode_step_multi) against the
unfused per-module path (router + moc_step, the reference's MoC.step lines) and the float64
oracle.  MoC.step itself takes the fused kernel with one module where it covers the shapes;
it is checked here against the same unfused path.

Modules sharing z, with caches prefilled from a prompt, decode several tokens.  Per step:
* the caches are bitwise equal to the per-module path's (they only move stored values);
* y agrees with the per-module path within 2e-2 of max|y| (that path rounds each
  alpha*basis product to bf16 like the reference's decode kernel; the fused one sums the
  exact products in fp32 on the tensor cores, and sums the router logits in another order);
* y agrees within 2e-2 with the oracle step (bf16 products, float64 sums) fed the float64
  router's alpha rounded to bf16, and the oracle's new cache is bitwise the fused one.
"""
from __future__ import annotations

import pytest
import torch

import moc.ops as ops
from conftest import rel_err
from moc import MoC, _lib, moc_triton
from moc.fused import decode_step
from oracle import moc_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _modules(specs, z_dim, ks, seed):
    torch.manual_seed(seed)
    mods = []
    g = torch.Generator().manual_seed(seed + 1)
    for dim, k, ract, act in specs:
        m = MoC(dim=dim, z_dim=z_dim, kernel_size=ks, k=k, init_std=0.05, router_activation=ract,
                activation=act)
        with torch.no_grad():
            m.router.copy_(torch.randn(k, z_dim, generator=g) * 0.05)
        mods.append(m.cuda().bfloat16())
    return mods


def _unfused_step(m, x, z, cache):
    """The reference's step lines (moc/api.py:383-388, 242-259): the router launch, then
    the cache update (moc_step), without the fused kernel."""
    alpha = ops.launch_router_forward(z, m.router.detach(), m.router_activation)
    return moc_triton(x, alpha, m.conv_bases.detach(), cache=cache, activation=m.activation)[0]


def _run(specs, B, z_dim, ks, steps=4, prompt=9, seed=3):
    _lib.device_status(clear=True)
    mods = _modules(specs, z_dim, ks, seed)
    g = torch.Generator().manual_seed(seed + 2)
    zp = torch.randn(B, prompt, z_dim, generator=g).bfloat16().cuda()
    caches = []
    with torch.no_grad():
        for m in mods:
            xp = torch.randn(B, prompt, m.dim, generator=g).bfloat16().cuda()
            caches.append(m(xp, zp, output_final_state=True)[1].contiguous())
        ref_caches = [c.clone() for c in caches]
        for _ in range(steps):
            z = torch.randn(B, 1, z_dim, generator=g).bfloat16().cuda()
            xs = [torch.randn(B, 1, m.dim, generator=g).bfloat16().cuda() for m in mods]
            before = [c.clone() for c in caches]
            ys = decode_step(mods, xs, z, caches)
            refs = [_unfused_step(m, x, z, c) for m, x, c in zip(mods, xs, ref_caches)]
            for i, (m, x, y, r) in enumerate(zip(mods, xs, ys, refs)):
                assert y.shape == x.shape
                assert torch.equal(caches[i], ref_caches[i]), f"module {i}: cache differs"
                assert rel_err(y, r) <= TOL, f"module {i}: {rel_err(y, r):.3e}"
                # the oracle on the same inputs
                a64 = O.router(z[:, 0].double().cpu(), m.router.detach().double().cpu(), m.router_activation)
                yo, so = O.step(x[:, 0].double().cpu(), a64.bfloat16().double(),
                                m.conv_bases.detach().double().cpu(), before[i].double().cpu(),
                                m.activation, bf16_products=True)
                assert rel_err(y[:, 0], yo) <= TOL
                assert torch.equal(caches[i].double().cpu(), so)
    assert _lib.device_status() == 0, "a decode wait ran out of polls"


def test_qkv_shaped_modules():
    # q / k / v as in the reference's attention block: exp, exp, softmax routers
    _run([(512, 16, "exp", None), (128, 16, "exp", None), (128, 16, "softmax", None)], B=37, z_dim=256, ks=4)


@pytest.mark.parametrize("ks", [1, 2, 3, 4])
def test_kernel_sizes_bases_and_silu(ks):
    _run([(96, 8, "softmax", "silu"), (264, 16, "exp", None), (40, 5, "exp", "silu")], B=5, z_dim=520, ks=ks,
         seed=ks)


def test_dims_off_the_8_channel_grid_take_the_per_module_path():
    _run([(258, 16, "exp", None), (37, 5, "softmax", "silu")], B=5, z_dim=64, ks=4, steps=2)


def test_single_module_and_single_sequence():
    _run([(64, 4, "softmax", None)], B=1, z_dim=64, ks=4, steps=3)


def test_four_modules_and_large_batch():
    _run([(256, 16, "softmax", None)] * 4, B=130, z_dim=128, ks=4, steps=2)


def test_long_routing_input():
    # z_dim spans more chunks than the router cluster has CTAs
    _run([(128, 16, "softmax", None), (64, 16, "exp", None)], B=20, z_dim=8200, ks=4, steps=2)


def test_unfusable_modules_take_the_per_module_path():
    # more than 16 bases: decode_step falls back to MoC.step and still agrees
    _run([(64, 32, "softmax", None), (64, 16, "exp", None)], B=3, z_dim=64, ks=4, steps=2)


def test_wide_modules_span_several_clusters():
    # more than 1024 channels: several clusters per 16-token group, each routing the tokens
    # itself; the last cluster of the first module has CTAs without channels
    _run([(2056, 16, "exp", "silu"), (1160, 12, "softmax", None)], B=18, z_dim=264, ks=4, steps=2)


def test_config4_shapes():
    # the decode benchmark's modules: q D=4096, k / v D=1024, z_dim 4096, batch 128
    _run([(4096, 16, "exp", None), (1024, 16, "exp", None), (1024, 16, "softmax", None)], B=128, z_dim=4096,
         ks=4, steps=1)


def test_fused_path_is_one_launch():
    mods = _modules([(512, 16, "exp", None), (128, 16, "exp", None), (128, 16, "softmax", None)], 256, 4, 9)
    B = 8
    caches = [torch.zeros(B, m.dim, 4, dtype=torch.bfloat16, device="cuda") for m in mods]
    xs = [torch.randn(B, 1, m.dim, device="cuda").bfloat16() for m in mods]
    z = torch.randn(B, 1, 256, device="cuda").bfloat16()
    n0 = _lib.launch_count()
    decode_step(mods, xs, z, caches)
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 == 1


@pytest.mark.parametrize("act,ract", [(None, "exp"), ("silu", "softmax")])
def test_module_step_is_one_fused_launch(act, ract):
    """MoC.step (the call unmodified reference code makes per module) runs the router and
    the update as one launch, agrees with the unfused path within 2e-2 and moves the cache
    bit for bit."""
    m = _modules([(1024, 16, ract, act)], 512, 4, 21)[0]
    B = 33
    g = torch.Generator().manual_seed(22)
    with torch.no_grad():
        xp = torch.randn(B, 7, m.dim, generator=g).bfloat16().cuda()
        zp = torch.randn(B, 7, 512, generator=g).bfloat16().cuda()
        cache = m(xp, zp, output_final_state=True)[1].contiguous()
        ref_cache = cache.clone()
        for _ in range(3):
            x = torch.randn(B, 1, m.dim, generator=g).bfloat16().cuda()
            z = torch.randn(B, 1, 512, generator=g).bfloat16().cuda()
            torch.cuda.synchronize()
            n0 = _lib.launch_count()
            y, out_cache = m.step(x, z, cache, output_final_state=True)
            torch.cuda.synchronize()
            assert _lib.launch_count() - n0 == 1
            assert out_cache is cache and y.shape == x.shape
            ref = _unfused_step(m, x, z, ref_cache)
            assert torch.equal(cache, ref_cache)
            assert rel_err(y, ref) <= TOL
    assert _lib.device_status() == 0
