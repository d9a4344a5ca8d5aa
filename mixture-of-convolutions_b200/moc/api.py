"""Public API: ``moc_triton`` (functional), ``MoC`` (module) and their autograd.

The names, signatures, accepted inputs and error messages are those of the
reference's moc/api.py, so code written against it runs unchanged.  Two things sit
behind the same interface but differ in how they run:

* every kernel is a hand-written sm_100a CUDA kernel reached through the C ABI
  (``moc.ops`` -> ``libmoc_b200.so``), never Triton and never a CPU fallback;
* ``MoC.forward`` computes the router (``z @ router^T`` then softmax/exp) in one
  kernel with fp32 logits, and its backward (softmax/exp Jacobian, ``dz``, ``drouter``)
  in the library too, instead of ``F.linear`` + ``torch.softmax`` + PyTorch autograd
  (reference: moc/api.py:383-388).
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
from torch.autograd.function import once_differentiable

from . import ops
from .optim import moc_fan_in_std

SUPPORTED_DTYPES = (torch.bfloat16, torch.float32)


# ----------------------------------------------------------------------------- checks
# Messages and exception types follow moc/api.py:18-92 and 198-215 word for word: they
# are part of the interface callers may match on.

def activation_flag(activation: str | None) -> int:
    if activation is None:
        return 0
    if activation in ("silu", "swish"):
        return 1
    raise ValueError(f"unsupported activation: {activation}")


def check_router_activation(router_activation: str) -> None:
    if router_activation in ("softmax", "exp"):
        return
    raise ValueError(
        f"unsupported router activation: {router_activation}; expected 'softmax' or 'exp'"
    )


def check_common_dtypes(x: torch.Tensor, alpha: torch.Tensor, basis: torch.Tensor) -> None:
    if not all(t.is_cuda for t in (x, alpha, basis)):
        raise ValueError("x, alpha, and basis must all be CUDA tensors")
    if alpha.device != x.device or basis.device != x.device:
        raise ValueError("x, alpha, and basis must be on the same CUDA device")
    if x.dtype not in SUPPORTED_DTYPES:
        raise TypeError(f"unsupported x dtype: {x.dtype}")
    for name, t in (("alpha", alpha), ("basis", basis)):
        if not t.is_floating_point():
            raise TypeError(f"{name} must be floating point, got {t.dtype}")


def _check_bank(alpha_k: int, basis: torch.Tensor, dim: int) -> tuple[int, int]:
    n_bases, kernel_size, basis_dim = basis.shape
    if (alpha_k, dim) != (n_bases, basis_dim):
        raise ValueError(
            f"alpha/basis dimensions disagree: K,D={(alpha_k, dim)} vs {(n_bases, basis_dim)}"
        )
    return n_bases, kernel_size


def check_fixed_inputs(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
) -> tuple[int, int, int, int, int]:
    check_common_dtypes(x, alpha, basis)
    if (x.ndim, alpha.ndim, basis.ndim) != (3, 3, 3):
        raise ValueError("fixed-length inputs must have x/alpha/basis ranks 3/3/3")
    B, T, D = x.shape
    if tuple(alpha.shape[:2]) != (B, T):
        raise ValueError(
            f"x and alpha batch/time shapes differ: {(B, T)} vs {tuple(alpha.shape[:2])}"
        )
    K, KS = _check_bank(alpha.shape[2], basis, D)
    if min(B, T, D, K, KS) <= 0:
        raise ValueError("B, T, D, K, and KS must all be positive")
    return B, T, D, K, KS


def check_packed_inputs(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
) -> tuple[int, int, int, int, int]:
    check_common_dtypes(x, alpha, basis)
    if (x.ndim, alpha.ndim, basis.ndim) != (2, 2, 3):
        raise ValueError("packed inputs must have x/alpha/basis ranks 2/2/3 internally")
    N, D = x.shape
    if alpha.shape[0] != N:
        raise ValueError(f"x and alpha token counts differ: {N} vs {alpha.shape[0]}")
    K, KS = _check_bank(alpha.shape[1], basis, D)
    if min(N, D, K, KS) <= 0:
        raise ValueError("total tokens, D, K, and KS must all be positive")
    if not cu_seqlens.is_cuda or cu_seqlens.device != x.device:
        raise ValueError("cu_seqlens must be a CUDA tensor on the same device as x")
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be rank-1 with at least two entries")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError("cu_seqlens must have dtype torch.int32 or torch.int64")
    if not isinstance(max_seqlen, int) or max_seqlen <= 0:
        raise ValueError("max_seqlen must be a positive Python int")
    return N, cu_seqlens.numel() - 1, D, K, KS


# ----------------------------------------------------------------------------- autograd

class _MoCFunction(torch.autograd.Function):
    """Convolution autograd (reference: moc/api.py:95-195).

    Backward is one library call: dx (when x needs a gradient), dalpha and dbasis, with
    the SiLU pre-activation recomputed inside the kernels rather than materialised by an
    extra forward pass.
    """

    @staticmethod
    def forward(
        ctx,
        x: torch.Tensor,
        alpha: torch.Tensor,
        basis: torch.Tensor,
        activation: str | None,
        cu_seqlens: Optional[torch.Tensor],
        max_seqlen: Optional[int],
        cu_seqlens_cpu: Optional[torch.Tensor],
        chunk_indices: Optional[torch.Tensor],
        halo: Optional[torch.Tensor] = None,
    ) -> torch.Tensor:
        x, alpha, basis = x.contiguous(), alpha.contiguous(), basis.contiguous()
        varlen = cu_seqlens is not None
        if varlen:
            if max_seqlen is None:
                raise ValueError("max_seqlen is required when cu_seqlens is provided")
            cu_seqlens = cu_seqlens.contiguous()
            if cu_seqlens_cpu is not None:
                cu_seqlens_cpu = cu_seqlens_cpu.contiguous()
            check_packed_inputs(x, alpha, basis, cu_seqlens, max_seqlen)
            if chunk_indices is None:
                if cu_seqlens_cpu is not None:
                    chunk_indices = ops.prepare_chunk_indices(cu_seqlens, cu_seqlens_cpu=cu_seqlens_cpu)
                else:
                    # the reference reads cu_seqlens on the host here (a stream sync,
                    # moc/ops.py:82-97); a table sized by an upper bound needs no sync
                    chunk_indices = ops.chunk_indices_upper_bound(cu_seqlens, x.shape[0])
            else:
                chunk_indices = chunk_indices.contiguous()
        else:
            if max_seqlen is not None:
                raise ValueError("max_seqlen must be None when cu_seqlens is None")
            if cu_seqlens_cpu is not None or chunk_indices is not None:
                raise ValueError("cu_seqlens_cpu and chunk_indices require cu_seqlens")
            check_fixed_inputs(x, alpha, basis)

        act = activation_flag(activation)
        out = ops.launch_forward(
            x, alpha, basis, activation_flag=act, cu_seqlens=cu_seqlens, chunk_indices=chunk_indices, halo=halo,
        )
        saved = (x, alpha, basis, cu_seqlens) if varlen else (x, alpha, basis)
        ctx.save_for_backward(*saved)
        ctx.activation_flag = act
        ctx.is_varlen = varlen
        ctx.chunk_indices = chunk_indices
        ctx.halo = halo
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, dy: torch.Tensor):
        if ctx.is_varlen:
            x, alpha, basis, cu_seqlens = ctx.saved_tensors
        else:
            (x, alpha, basis), cu_seqlens = ctx.saved_tensors, None
        dy = dy.contiguous()
        dx, dalpha, dbasis = ops.launch_backward(
            x, alpha, basis, dy, dy,
            activation_flag=ctx.activation_flag,
            need_x=ctx.needs_input_grad[0],
            cu_seqlens=cu_seqlens,
            chunk_indices=ctx.chunk_indices,
            halo=ctx.halo,
        )
        return dx, dalpha, dbasis, None, None, None, None, None, None


class _RouterFunction(torch.autograd.Function):
    """alpha = softmax/exp(z @ router^T) and its backward, both in the library."""

    @staticmethod
    def forward(ctx, z: torch.Tensor, router: torch.Tensor, router_activation: str) -> torch.Tensor:
        z = z.contiguous()
        router = router.contiguous()
        alpha = ops.launch_router_forward(z, router, router_activation)
        ctx.save_for_backward(z, router, alpha)
        ctx.router_activation = router_activation
        ctx.set_materialize_grads(False)
        return alpha

    @staticmethod
    @once_differentiable
    def backward(ctx, dalpha: torch.Tensor | None):
        if dalpha is None:  # alpha reached the loss through no path: z and the router get no gradient
            return None, None, None
        z, router, alpha = ctx.saved_tensors
        dz, drouter = ops.launch_router_backward(
            z, router, alpha, dalpha.contiguous(), ctx.router_activation,
            need_z=ctx.needs_input_grad[0], need_weight=ctx.needs_input_grad[1],
        )
        return dz, drouter, None


def _route(z: torch.Tensor, router: torch.Tensor, router_activation: str) -> torch.Tensor:
    # F.linear's own preconditions, checked before any launch.
    if z.shape[-1] != router.shape[-1]:
        raise RuntimeError(
            f"mat1 and mat2 shapes cannot be multiplied "
            f"({z.numel() // max(z.shape[-1], 1)}x{z.shape[-1]} and {router.shape[1]}x{router.shape[0]})"
        )
    if z.dtype != router.dtype:
        raise RuntimeError(
            f"expected m1 and m2 to have the same dtype, but got: {z.dtype} != {router.dtype}"
        )
    if not z.is_cuda:
        # The reference computes alpha on z's device and then rejects non-CUDA alpha.
        raise ValueError("x, alpha, and basis must all be CUDA tensors")
    if router.device != z.device:
        raise RuntimeError(
            f"Expected all tensors to be on the same device, but found at least two devices, "
            f"{z.device} and {router.device}!"
        )
    return _RouterFunction.apply(z, router, router_activation)


# ----------------------------------------------------------------------------- functional

def _canonicalize_packed_input(
    x: torch.Tensor,
    alpha: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor, bool]:
    if x.ndim == 2 and alpha.ndim == 2:
        return x, alpha, False
    if x.ndim == 3 and alpha.ndim == 3 and x.shape[0] == 1 and alpha.shape[0] == 1:
        # views, as the reference's squeeze(0) (moc/api.py:204-205): their backward is a view
        # too, where x[0]'s would zero-fill a [1, N, D] gradient and copy dx into it
        return x.squeeze(0), alpha.squeeze(0), True
    raise ValueError("varlen x/alpha must be [N,D]/[N,K] or [1,N,D]/[1,N,K]")


def _check_cache(x: torch.Tensor, basis: torch.Tensor, cache: torch.Tensor) -> None:
    want = (x.shape[0], x.shape[2], basis.shape[1])
    if tuple(cache.shape) != want:
        raise ValueError(f"cache must have shape {want}, got {tuple(cache.shape)}")
    if cache.device != x.device or cache.dtype != x.dtype:
        raise ValueError("cache must have the same device and dtype as x")


def _final_state(x: torch.Tensor, cache: torch.Tensor | None, kernel_size: int) -> torch.Tensor:
    """Last kernel_size tokens as [B, D, S] (reference: moc/api.py:218-227)."""
    B, T, D = x.shape
    recent = x.transpose(1, 2)
    if T >= kernel_size:
        return recent[:, :, T - kernel_size:].contiguous()
    older = x.new_zeros(B, D, kernel_size - T) if cache is None else cache[:, :, T:]
    return torch.cat((older, recent), dim=-1)


def _fixed_moc(x, alpha, basis, activation):
    check_fixed_inputs(x, alpha, basis)
    return _MoCFunction.apply(x, alpha, basis, activation, None, None, None, None)


def _step_moc(x, alpha, basis, cache, activation):
    T = check_fixed_inputs(x, alpha, basis)[1]
    if T != 1:
        raise ValueError(f"step expects sequence length 1, got {T}")
    _check_cache(x, basis, cache)
    y = ops.launch_update(
        x[:, 0].contiguous(), alpha[:, 0].contiguous(), basis.contiguous(), cache,
        activation_flag=activation_flag(activation),
    )
    return y[:, None]


def moc_triton(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    cache: torch.Tensor | None = None,
    output_final_state: bool = False,
    activation: str | None = None,
    cu_seqlens: Optional[torch.Tensor] = None,
    max_seqlen: Optional[int] = None,
    cu_seqlens_cpu: Optional[torch.Tensor] = None,
    chunk_indices: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Mixture-of-convolutions over fixed-length or packed sequences, or one decode step.

    Same dispatch as the reference (moc/api.py:262-335): a cache with T == 1 is a decode
    step (cache updated in place, no autograd); a cache with T > 1 prepends the cached
    tokens with zero routing weights; ``cu_seqlens`` selects the packed varlen path.
    """
    activation_flag(activation)

    if cu_seqlens is None:
        if cu_seqlens_cpu is not None or chunk_indices is not None:
            raise ValueError("cu_seqlens_cpu and chunk_indices require cu_seqlens")
        B, T, D, K, KS = check_fixed_inputs(x, alpha, basis)
        if cache is not None:
            _check_cache(x, basis, cache)
            if T == 1:
                y = _step_moc(x, alpha, basis, cache, activation)
                return y, (cache if output_final_state else None)
            if cache.requires_grad and torch.is_grad_enabled():
                # the reference's form, which also differentiates the cache
                prefix_x = cache.transpose(1, 2)
                prefix_alpha = alpha.new_zeros(B, KS, K)
                y = _fixed_moc(
                    torch.cat((prefix_x, x), dim=1), torch.cat((prefix_alpha, alpha), dim=1), basis, activation,
                )[:, KS:]
            else:
                # the kernels read the cache as the sequences' causal halo (no concatenation)
                y = _MoCFunction.apply(x, alpha, basis, activation, None, None, None, None, cache.detach())
        else:
            y = _fixed_moc(x, alpha, basis, activation)
        return y, (_final_state(x, cache, KS) if output_final_state else None)

    if cache is not None or output_final_state:
        raise ValueError("cache and output_final_state are only supported for fixed-length inputs")
    if max_seqlen is None:
        raise ValueError("max_seqlen is required for varlen inputs")
    x_packed, alpha_packed, batched = _canonicalize_packed_input(x, alpha)
    check_packed_inputs(x_packed, alpha_packed, basis, cu_seqlens, max_seqlen)
    y = _MoCFunction.apply(
        x_packed, alpha_packed, basis, activation, cu_seqlens, max_seqlen, cu_seqlens_cpu, chunk_indices,
    )
    return (y[None] if batched else y), None


# ----------------------------------------------------------------------------- module

class MoC(nn.Module):
    """Token-routed depthwise causal convolution (reference: moc/api.py:338-425).

    Parameters ``conv_bases`` [k, kernel_size, dim] (uniform in +-init_std*sqrt(3)) and
    ``router`` [k, z_dim] (zeros) keep the reference's names, shapes and initialisation,
    so state dicts interchange.
    """

    def __init__(
        self,
        dim: int,
        z_dim: int,
        kernel_size: int,
        k: int,
        activation: str | None = None,
        init_std: float | None = None,
        router_activation: str = "softmax",
    ) -> None:
        super().__init__()
        activation_flag(activation)
        check_router_activation(router_activation)
        self.dim = dim
        self.z_dim = z_dim
        self.kernel_size = kernel_size
        self.k = k
        self.activation = activation
        self.router_activation = router_activation
        self.conv_bases = nn.Parameter(torch.empty(k, kernel_size, dim))
        self.router = nn.Parameter(torch.zeros(k, z_dim))
        std = moc_fan_in_std(k, kernel_size) if init_std is None else init_std
        bound = std * math.sqrt(3)
        nn.init.uniform_(self.conv_bases, a=-bound, b=bound)

    def forward(
        self,
        x: torch.Tensor,
        z: torch.Tensor,
        cache: torch.Tensor | None = None,
        output_final_state: bool = False,
        cu_seqlens: Optional[torch.Tensor] = None,
        max_seqlen: Optional[int] = None,
        cu_seqlens_cpu: Optional[torch.Tensor] = None,
        chunk_indices: Optional[torch.Tensor] = None,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        if (cache is not None and cu_seqlens is None and cu_seqlens_cpu is None and chunk_indices is None
                and x.ndim == 3 and x.shape[1] == 1):
            # a decode step: router and cache update in one launch where the fused kernel
            # covers the shapes (bf16, k <= 16, kernel_size <= 4), else the path below
            from .fused import step_one

            y = step_one(self, x, z, cache)
            if y is not None:
                return y, (cache if output_final_state else None)
        alpha = _route(z, self.router, self.router_activation)
        return moc_triton(
            x,
            alpha,
            self.conv_bases,
            cache=cache,
            output_final_state=output_final_state,
            activation=self.activation,
            cu_seqlens=cu_seqlens,
            max_seqlen=max_seqlen,
            cu_seqlens_cpu=cu_seqlens_cpu,
            chunk_indices=chunk_indices,
        )

    def step(
        self,
        x: torch.Tensor,
        z: torch.Tensor,
        cache: torch.Tensor | None = None,
        output_final_state: bool = False,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        if x.ndim != 3 or x.shape[1] != 1:
            raise ValueError(f"step expects x with shape [B, 1, D], got {tuple(x.shape)}")
        if z.ndim != 3 or z.shape[:2] != x.shape[:2]:
            raise ValueError(f"step expects z with shape [B, 1, Z], got {tuple(z.shape)}")
        if cache is None:
            cache = x.new_zeros(x.shape[0], self.dim, self.kernel_size)
        return self.forward(x, z, cache=cache, output_final_state=output_final_state)

    @property
    def state_size(self) -> int:
        return self.dim * self.kernel_size


__all__ = ["MoC", "moc_triton"]
