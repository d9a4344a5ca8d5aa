"""Dense PyTorch statement of the operator, kept for users of ``moc.reference``.

Materialises the per-token kernels ([B, T, D, S]) and runs on any device; it is a
readable definition, not a code path of ``moc_triton`` (which always runs the CUDA
kernels).  Interface of the reference's moc/reference.py:19-59.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _activate(out: torch.Tensor, activation: str | None) -> torch.Tensor:
    if activation is None:
        return out
    if activation not in ("silu", "swish"):
        raise ValueError(f"unsupported activation: {activation}")
    return F.silu(out)


def moc_ref(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    activation: str | None = None,
) -> torch.Tensor:
    """y[b,t,d] = sum_s (sum_k alpha[b,t,k] basis[k,s,d]) * x[b, t-(S-1-s), d]."""
    S = basis.shape[1]
    T = x.shape[1]
    kernels = torch.einsum("btk,ksd->btsd", alpha, basis)
    padded = torch.cat((x.new_zeros(x.shape[0], S - 1, x.shape[2]), x), dim=1)
    out = sum(kernels[:, :, s] * padded[:, s:s + T] for s in range(S))
    return _activate(out, activation)


def moc_varlen_ref(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    cu_seqlens: torch.Tensor,
    activation: str | None = None,
) -> torch.Tensor:
    """moc_ref applied to each packed sequence [cu[i], cu[i+1]) of x ([N,D] or [1,N,D])."""
    batched = x.ndim == 3
    if batched:
        x, alpha = x[0], alpha[0]
    offsets = [int(v) for v in cu_seqlens.detach().cpu().tolist()]
    parts = [
        moc_ref(x[a:b][None], alpha[a:b][None], basis, activation=activation)[0]
        for a, b in zip(offsets[:-1], offsets[1:])
    ]
    out = torch.cat(parts, dim=0)
    return out[None] if batched else out


__all__ = ["moc_ref", "moc_varlen_ref"]
