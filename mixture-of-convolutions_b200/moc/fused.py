"""Fused paths around MoC modules: the decode step of modules that share their routing
input, and the projection that feeds a module with the convolution as its epilogue.

In the reference's attention block (README.md:120-129) the q, k and v short convolutions
are three MoC modules routed by the same ``x_norm``.  Decoding one token through them one
by one costs, per module, a router GEMM, its softmax / exp and the update kernel
(moc/api.py:383-388, moc/ops.py:341-362).  ``decode_step`` runs all of them in one
launch of ``moc_decode_step_multi``: clusters of CTAs compute each module's router, pass
the routing weights between their CTAs on chip, then mix, convolve and shift every
module's cache.

Results match calling ``module.step(x, z, cache)`` for each module; shapes the fused
kernels do not cover (fp32 or fp16 modules, more than 16 bases, kernel sizes above 4,
mixed kernel sizes, dims that are not a multiple of 8, more than four modules) take that
per-module path.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch
from torch.autograd.function import once_differentiable

from . import _lib
from .api import MoC

_ROUTER_ACTS = {"softmax": 0, "exp": 1}


def _as_2d(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.ndim == 3:
        if t.shape[1] != 1:
            raise ValueError(f"{name} must have one token per sequence, got shape {tuple(t.shape)}")
        return t[:, 0]
    if t.ndim != 2:
        raise ValueError(f"{name} must be [B, 1, D] or [B, D], got shape {tuple(t.shape)}")
    return t


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _fusable(modules: Sequence[MoC], xs, z, caches) -> bool:
    if not 1 <= len(modules) <= _lib.DECODE_MAX_MODULES:
        return False
    S = modules[0].kernel_size
    for m, x, c in zip(modules, xs, caches):
        if m.conv_bases.dtype != torch.bfloat16 or m.router.dtype != torch.bfloat16:
            return False
        if x.dtype != torch.bfloat16 or c.dtype != torch.bfloat16 or not c.is_contiguous():
            return False
        if m.k > 16 or m.kernel_size != S or S > 4 or m.dim % 8 != 0:
            return False
        if c.data_ptr() % 16 != 0:
            return False
    return z.dtype == torch.bfloat16 and z.shape[-1] % 8 == 0


def decode_step(modules: Sequence[MoC], xs: Sequence[torch.Tensor], z: torch.Tensor,
                caches: Sequence[torch.Tensor]) -> list[torch.Tensor]:
    """One decode token through every module in ``modules``.

    modules: MoC modules with the same z_dim, on one CUDA device.
    xs:      per module, the token's input [B, 1, D_i] (or [B, D_i]).
    z:       the shared routing input [B, 1, z_dim] (or [B, z_dim]).
    caches:  per module, its conv cache [B, D_i, kernel_size]; updated in place, as
             ``MoC.step`` does (slots shift left, x enters the last slot).

    Returns the outputs y_i, shaped like xs[i]."""
    if not (len(modules) == len(xs) == len(caches)) or not modules:
        raise ValueError("decode_step needs one x and one cache per module")
    z2 = _as_2d(z, "z")
    x2 = [_as_2d(x, "x") for x in xs]
    B = z2.shape[0]
    for m, x, c in zip(modules, x2, caches):
        if not isinstance(m, MoC):
            raise TypeError("decode_step expects moc.MoC modules")
        if x.shape != (B, m.dim):
            raise ValueError(f"x must be [B, {m.dim}] for this module, got {tuple(x.shape)}")
        if c.shape != (B, m.dim, m.kernel_size):
            raise ValueError(f"cache must be [B, {m.dim}, {m.kernel_size}], got {tuple(c.shape)}")
        if z2.shape[1] != m.z_dim:
            raise ValueError(f"z must have z_dim={m.z_dim}, got {z2.shape[1]}")
        if not (x.is_cuda and c.is_cuda and z2.is_cuda and m.conv_bases.is_cuda):
            raise ValueError("decode_step runs on CUDA tensors")
    if not _fusable(modules, x2, z2, caches):
        zs = z2.unsqueeze(1)
        return [m.step(x.unsqueeze(1), zs, c)[0].reshape(xo.shape)
                for m, x, c, xo in zip(modules, x2, caches, xs)]

    z2 = _aligned(z2)
    keep = [z2]
    mods = (_lib.MocDecodeModule * len(modules))()
    ys, alphas = [], []
    for i, (m, x, c) in enumerate(zip(modules, x2, caches)):
        x = _aligned(x)
        w = _aligned(m.router.detach())
        b = _aligned(m.conv_bases.detach())
        y = torch.empty_like(x)
        alpha = torch.empty(B, m.k, dtype=torch.bfloat16, device=x.device)
        keep += [x, w, b]
        ys.append(y)
        alphas.append(alpha)
        mods[i] = _lib.MocDecodeModule(
            dim=m.dim, n_bases=m.k, kernel_size=m.kernel_size, activation=int(m.activation is not None),
            router_act=_ROUTER_ACTS[m.router_activation], weight=w.data_ptr(), basis=b.data_ptr(),
            x=x.data_ptr(), cache=c.data_ptr(), alpha=alpha.data_ptr(), out=y.data_ptr())
    with torch.cuda.device(z2.device):
        rc = _lib.load().moc_decode_step_multi(len(modules), mods, B, z2.shape[1], z2.data_ptr(),
                                               _lib.stream_of(z2.device))
    _lib.check(rc, "moc_decode_step_multi")
    return [y.reshape(xo.shape) for y, xo in zip(ys, xs)]


def step_one(module: MoC, x: torch.Tensor, z: torch.Tensor, cache: torch.Tensor) -> torch.Tensor | None:
    """``module``'s decode step (x [B, 1, D], z [B, 1, z_dim], cache [B, D, S] updated in
    place) as one launch of the fused kernel: the router and the update in the same CTAs,
    where the per-module path launches the router, then the update.  Returns y [B, 1, D],
    or None when the shapes are outside the fused kernel (the caller then takes the
    per-module path).  Like the reference's step (moc/api.py:242-259), y carries no
    gradient."""
    if x.ndim != 3 or z.ndim != 3 or x.shape[1] != 1 or z.shape[1] != 1 or x.shape[0] != z.shape[0]:
        return None
    if x.shape[2] != module.dim or z.shape[2] != module.z_dim or cache.ndim != 3:
        return None
    if tuple(cache.shape) != (x.shape[0], module.dim, module.kernel_size):
        return None
    if not (x.is_cuda and z.is_cuda and cache.is_cuda and module.conv_bases.is_cuda):
        return None
    dev = x.device
    if z.device != dev or cache.device != dev or module.conv_bases.device != dev or module.router.device != dev:
        return None
    if not _fusable([module], [x[:, 0]], z[:, 0], [cache]):
        return None
    return decode_step([module], [x], z, [cache])[0]


def _proj_alpha(h: torch.Tensor, module: MoC, z: torch.Tensor | None, alpha: torch.Tensor | None,
                train: bool = False) -> torch.Tensor:
    """The module's router output for the fused projection: ``alpha`` as given, or routed from z
    (through the router's autograd function when ``train``, so dalpha reaches z and the router)."""
    B, T = h.shape[:2]
    from . import ops
    from .api import _route

    if alpha is None:
        if z is None or z.shape[:2] != (B, T):
            raise ValueError(f"z must be [{B}, {T}, z_dim], got {None if z is None else tuple(z.shape)}")
        if train:
            alpha = _route(z, module.router, module.router_activation)
        else:
            alpha = ops.launch_router_forward(z.detach(), module.router.detach(), module.router_activation)
    if alpha.shape != (B, T, module.k) or alpha.dtype != torch.bfloat16:
        raise ValueError(f"alpha must be bf16 [{B}, {T}, {module.k}], got {tuple(alpha.shape)} {alpha.dtype}")
    return alpha if train else _aligned(alpha.detach())


def _wants_grad(h, weight, modules, z, alphas) -> bool:
    if not torch.is_grad_enabled():
        return False
    ts = [h, weight] + [p for m in modules for p in (m.conv_bases, m.router)]
    ts += [z] if z is not None else list(alphas or ())
    return any(t is not None and t.requires_grad for t in ts)


class _ProjConvFunction(torch.autograd.Function):
    """Training form of the fused projection + convolution, for one or more modules over one
    projection weight (the reference's ``qkv_proj`` then ``q_conv`` / ``k_conv`` / ``v_conv``
    under autograd, README.md:115-129).

    Forward: one ``moc_proj_forward_multi_save`` launch gives each module's y and keeps its
    rounded projection x (the tensor the unfused path's projection GEMM writes), so the
    convolution reads no x back from memory.  Backward: each module's convolution backward on
    its saved x (``moc_backward``: dx, dalpha, dbasis; reference moc/api.py:148-195), then the
    projection's gradients as two library GEMMs over the modules' dx side by side:
    dh = dx . weight and dweight = dx^T . h."""

    @staticmethod
    def forward(ctx, h, weight, spec, *alpha_basis):
        # spec: per module (dim, activation flag); alpha_basis: alpha_0, basis_0, alpha_1, ...
        B, T, Dm = h.shape
        n = len(spec)
        h2, w2 = _aligned(h), _aligned(weight)
        alphas = [_aligned(a) for a in alpha_basis[0::2]]
        bases = [_aligned(b) for b in alpha_basis[1::2]]
        arr = (_lib.MocProjModule * n)()
        x_ptrs = (ctypes.c_void_p * n)()
        outs, xs = [], []
        off = 0
        for i, ((D, act), a, b) in enumerate(zip(spec, alphas, bases)):
            out = torch.empty(B, T, D, dtype=torch.bfloat16, device=h.device)
            x = torch.empty(B, T, D, dtype=torch.bfloat16, device=h.device)
            outs.append(out)
            xs.append(x)
            x_ptrs[i] = x.data_ptr()
            arr[i] = _lib.MocProjModule(dim=D, row_offset=off, n_bases=a.shape[-1], activation=act,
                                        alpha=a.data_ptr(), basis=b.data_ptr(), out=out.data_ptr())
            off += D
        with torch.cuda.device(h.device):
            rc = _lib.load().moc_proj_forward_multi_save(n, arr, x_ptrs, B, T, Dm, bases[0].shape[1], h2.data_ptr(),
                                                         w2.data_ptr(), weight.shape[0], _lib.stream_of(h.device))
        _lib.check(rc, "moc_proj_forward_multi_save")
        ctx.save_for_backward(h2, w2, *xs, *alphas, *bases)
        ctx.spec = spec
        ctx.set_materialize_grads(False)  # an output outside the loss arrives as None: its module is skipped
        return tuple(outs)

    @staticmethod
    @once_differentiable
    def backward(ctx, *dys):
        from . import ops

        n = len(ctx.spec)
        saved = ctx.saved_tensors
        h2, w2 = saved[0], saved[1]
        xs, alphas, bases = saved[2:2 + n], saved[2 + n:2 + 2 * n], saved[2 + 2 * n:]
        B, T, Dm = h2.shape
        N = B * T
        need_proj = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        dxs, grads = [], []
        for i, ((D, act), dy) in enumerate(zip(ctx.spec, dys)):
            if dy is None:  # this module's output took no part in the loss
                dxs.append(torch.zeros(B, T, D, dtype=torch.bfloat16, device=h2.device))
                grads += [None, None]
                continue
            dx, dalpha, dbasis = ops.launch_backward(xs[i], alphas[i], bases[i], dy.contiguous(), dy,
                                                     activation_flag=act, need_x=need_proj)
            dxs.append(dx)
            grads += [dalpha, dbasis]
        dh = dw = None
        if need_proj:
            dx_all = (dxs[0] if n == 1 else torch.cat(dxs, dim=-1)).view(N, -1)
            if ctx.needs_input_grad[0]:
                dh = torch.mm(dx_all, w2).view(B, T, Dm)
            if ctx.needs_input_grad[1]:
                dw = torch.mm(dx_all.t(), h2.view(N, Dm))
        return (dh, dw, None, *grads)


def proj_forward_multi(h: torch.Tensor, weight: torch.Tensor, modules: Sequence[MoC], z: torch.Tensor | None = None,
                       alphas: Sequence[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """The reference's attention-block pattern (README.md:115-129) in one kernel:

        q, k, v = qkv_proj(x_norm).split([q_dim, k_dim, v_dim], dim=-1)
        q, _ = q_conv(q, x_norm); k, _ = k_conv(k, x_norm); v, _ = v_conv(v, x_norm)

    h:       [B, T, in_dim] bf16 (x_norm), fixed-length sequences (no cache, no packing).
    weight:  [sum of module dims, in_dim] bf16 (qkv_proj.weight), module i's rows following
             module i-1's.
    modules: up to four bf16 MoC modules with one kernel size (K % 8 == 0, K <= 16).
    z:       the routing input for every module, or ``alphas``: each module's router output.

    h is read once for all modules; each module's projection is rounded to bf16 and
    convolved on chip.  Returns the modules' outputs.  When autograd records (grad enabled and
    h, weight, z / alphas or a module's parameters require grad) the launch also keeps each
    module's projection for the backward, and the outputs carry the graph: gradients reach h,
    weight, z (through the routers) and every module's conv_bases and router."""
    if not 1 <= len(modules) <= _lib.PROJ_MAX_MODULES:
        raise ValueError(f"proj_forward_multi takes 1 to {_lib.PROJ_MAX_MODULES} modules, got {len(modules)}")
    if h.ndim != 3 or h.dtype != torch.bfloat16 or not h.is_cuda:
        raise ValueError(f"h must be a CUDA bf16 tensor [B, T, in_dim], got {tuple(h.shape)} {h.dtype}")
    B, T, Dm = h.shape
    rows = sum(m.dim for m in modules)
    if weight.shape != (rows, Dm) or weight.dtype != torch.bfloat16:
        raise ValueError(f"weight must be bf16 [{rows}, {Dm}], got {tuple(weight.shape)} {weight.dtype}")
    if any(not isinstance(m, MoC) or m.conv_bases.dtype != torch.bfloat16 for m in modules):
        raise ValueError("proj_forward_multi needs bf16 moc.MoC modules")
    if len({m.kernel_size for m in modules}) != 1:
        raise ValueError("all modules must have one kernel_size")
    if (alphas is None) == (z is None):
        raise ValueError("pass exactly one of z (routing input) or alphas (router outputs)")
    if alphas is not None and len(alphas) != len(modules):
        raise ValueError("one alpha per module")
    if _wants_grad(h, weight, modules, z, alphas):
        ab = []
        for i, m in enumerate(modules):
            ab += [_proj_alpha(h, m, z, None if alphas is None else alphas[i], train=True), m.conv_bases]
        spec = tuple((m.dim, int(m.activation is not None)) for m in modules)
        return list(_ProjConvFunction.apply(h, weight, spec, *ab))
    h2, w2 = _aligned(h.detach()), _aligned(weight.detach())
    keep, outs = [h2, w2], []
    arr = (_lib.MocProjModule * len(modules))()
    off = 0
    for i, m in enumerate(modules):
        a2 = _proj_alpha(h, m, z, None if alphas is None else alphas[i])
        basis = _aligned(m.conv_bases.detach())
        out = torch.empty(B, T, m.dim, dtype=torch.bfloat16, device=h.device)
        keep += [a2, basis]
        outs.append(out)
        arr[i] = _lib.MocProjModule(dim=m.dim, row_offset=off, n_bases=m.k, activation=int(m.activation is not None),
                                    alpha=a2.data_ptr(), basis=basis.data_ptr(), out=out.data_ptr())
        off += m.dim
    with torch.cuda.device(h.device):
        rc = _lib.load().moc_proj_forward_multi(len(modules), arr, B, T, Dm, modules[0].kernel_size, h2.data_ptr(),
                                                w2.data_ptr(), rows, _lib.stream_of(h.device))
    _lib.check(rc, "moc_proj_forward_multi")
    return outs


def proj_forward(h: torch.Tensor, weight: torch.Tensor, module: MoC, z: torch.Tensor | None = None,
                 alpha: torch.Tensor | None = None) -> torch.Tensor:
    """``module(h @ weight.T, z)[0]`` in one kernel: the projection runs on the tensor cores and
    the convolution is its epilogue, so the projected tensor never reaches memory.

    h:      [B, T, in_dim] bf16, fixed-length sequences (no cache, no packing).
    weight: [module.dim, in_dim] bf16, the module's slice of the projection (nn.Linear layout:
            for the reference's attention block, the q, k or v rows of qkv_proj.weight).
    z:      the routing input [B, T, z_dim]; or ``alpha`` [B, T, module.k], the router output.

    The projection is rounded to bf16 before the convolution, as a bf16 qkv tensor is; the
    result matches the unfused path up to the order of the projection's fp32 sums.  Under
    autograd (grad enabled and an input or the module's parameters require grad) the launch
    also keeps the projection for the backward, as ``proj_forward_multi`` does."""
    if h.ndim != 3 or h.dtype != torch.bfloat16 or not h.is_cuda:
        raise ValueError(f"h must be a CUDA bf16 tensor [B, T, in_dim], got {tuple(h.shape)} {h.dtype}")
    B, T, Dm = h.shape
    if weight.shape != (module.dim, Dm) or weight.dtype != torch.bfloat16:
        raise ValueError(f"weight must be bf16 [{module.dim}, {Dm}], got {tuple(weight.shape)} {weight.dtype}")
    if module.conv_bases.dtype != torch.bfloat16:
        raise ValueError("proj_forward needs a bf16 module")
    if (alpha is None) == (z is None):
        raise ValueError("pass exactly one of z (routing input) or alpha (router output)")
    if _wants_grad(h, weight, [module], z, None if alpha is None else [alpha]):
        a2 = _proj_alpha(h, module, z, alpha, train=True)
        spec = ((module.dim, int(module.activation is not None)),)
        return _ProjConvFunction.apply(h, weight, spec, a2, module.conv_bases)[0]
    a2 = _proj_alpha(h, module, z, alpha)
    h2, w2 = _aligned(h.detach()), _aligned(weight.detach())
    basis = _aligned(module.conv_bases.detach())
    out = torch.empty(B, T, module.dim, dtype=torch.bfloat16, device=h.device)
    prob = _lib.MocProjProblem(batch=B, seq_len=T, in_dim=Dm, dim=module.dim, n_bases=module.k,
                               kernel_size=module.kernel_size, activation=int(module.activation is not None),
                               h=h2.data_ptr(), weight=w2.data_ptr(), alpha=a2.data_ptr(),
                               basis=basis.data_ptr(), out=out.data_ptr())
    with torch.cuda.device(h.device):
        rc = _lib.load().moc_proj_forward(ctypes.byref(prob), _lib.stream_of(h.device))
    _lib.check(rc, "moc_proj_forward")
    return out
