"""Argument checks of the fused entry points (moc.fused), on CPU: every rejection happens in
Python before any library call, so none of these needs a GPU."""
from __future__ import annotations

import pytest
import torch

from moc import MoC, fused


def _mod(D=64, Dz=32, S=4, K=16):
    return MoC(dim=D, z_dim=Dz, kernel_size=S, k=K).bfloat16()


def test_proj_forward_rejects_cpu_or_non_bf16_inputs():
    m = _mod()
    h = torch.randn(1, 8, 32).bfloat16()
    w = torch.randn(64, 32).bfloat16()
    with pytest.raises(ValueError, match="CUDA bf16"):
        fused.proj_forward(h, w, m, z=h)
    with pytest.raises(ValueError, match="CUDA bf16"):
        fused.proj_forward(h.float(), w, m, z=h)
    with pytest.raises(ValueError, match=r"\[B, T, in_dim\]"):
        fused.proj_forward(h[0], w, m, z=h)


def test_proj_forward_multi_checks_modules_and_weight_before_launch():
    mods = [_mod(64), _mod(32)]
    h = torch.randn(1, 8, 32).bfloat16()
    with pytest.raises(ValueError, match="1 to 4 modules"):
        fused.proj_forward_multi(h, torch.randn(96, 32).bfloat16(), [], z=h)
    with pytest.raises(ValueError, match="1 to 4 modules"):
        fused.proj_forward_multi(h, torch.randn(96, 32).bfloat16(), [_mod()] * 5, z=h)
    with pytest.raises(ValueError, match="CUDA bf16"):
        fused.proj_forward_multi(h, torch.randn(96, 32).bfloat16(), mods, z=h)


def test_proj_training_launch_only_when_autograd_records():
    """The fused projection keeps each module's projection for a backward only when a gradient can
    flow: grad mode on, and h, the weight, the routing input (or the router outputs) or a module's
    parameters requiring grad.  Otherwise it is the inference launch."""
    m = _mod()
    h = torch.randn(1, 8, 32).bfloat16()
    w = torch.randn(64, 32).bfloat16()
    assert fused._wants_grad(h, w, [m], h, None)  # conv_bases and router are parameters
    with torch.no_grad():
        assert not fused._wants_grad(h, w, [m], h, None)
    m.requires_grad_(False)
    assert not fused._wants_grad(h, w, [m], h, None)
    assert not fused._wants_grad(h, w, [m], None, [torch.zeros(1, 8, 16)])
    assert fused._wants_grad(h, w, [m], None, [torch.zeros(1, 8, 16, requires_grad=True)])
    assert fused._wants_grad(h.clone().requires_grad_(), w, [m], h, None)
    assert fused._wants_grad(h, w.clone().requires_grad_(), [m], h, None)


def test_decode_step_shape_checks():
    m = _mod()
    x = torch.randn(2, 1, 64).bfloat16()
    z = torch.randn(2, 1, 32).bfloat16()
    cache = torch.zeros(2, 64, 4).bfloat16()
    with pytest.raises(ValueError, match="one x and one cache per module"):
        fused.decode_step([m], [x, x], z, [cache])
    with pytest.raises(ValueError, match="one token per sequence"):
        fused.decode_step([m], [torch.randn(2, 3, 64).bfloat16()], z, [cache])
    with pytest.raises(ValueError, match="cache must be"):
        fused.decode_step([m], [x], z, [torch.zeros(2, 64, 3).bfloat16()])
    with pytest.raises(ValueError, match="z_dim"):
        fused.decode_step([m], [x], torch.randn(2, 1, 16).bfloat16(), [cache])
    with pytest.raises(ValueError, match="CUDA"):
        fused.decode_step([m], [x], z, [cache])
    with pytest.raises(TypeError, match="moc.MoC"):
        fused.decode_step([torch.nn.Linear(2, 2)], [x], z, [cache])
