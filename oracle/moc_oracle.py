"""CPU oracle for the Mixture-of-Convolutions hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module, and only as the checker (or, for the baseline, as the timed CPU
port of the reference's PyTorch path).  The product (the ``moc`` package and
``libmoc_b200.so``) never imports it.

It restates the reference's algorithm in plain PyTorch CPU code (float64 by default):

* ``conv``            — moc/reference.py:19-33 (tap s reads x[t-(S-1-s)], zeros before
                        the sequence start; per-token kernel = alpha . basis[:, s])
* ``conv_varlen``     — moc/reference.py:36-59 (``conv`` per packed sequence)
* ``router``          — moc/api.py:383-388 (``z @ W^T`` then softmax over K or exp)
* ``step``            — the decode kernel moc/kernels.py:442-550 (state = cache slots
                        1..S-1 plus x; cache shifted left, x appended)
* ``final_state``     — moc/api.py:218-227
* ``chunk_indices``   — moc/ops.py:82-97 (pure-Python loops)

Gradients come from torch autograd through these definitions, as the reference's
verify.py obtains them from moc/reference.py.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against
``tests/golden/moc_golden.npz``, produced by ``tests/golden/make_golden.py`` from the
reference's own code (moc/reference.py, moc/api.py, moc/ops.py) run on CPU.
"""
from __future__ import annotations

import torch

__all__ = [
    "conv",
    "conv_varlen",
    "router",
    "step",
    "final_state",
    "chunk_indices",
    "conv_grads",
    "module_grads",
]


def _silu(v: torch.Tensor) -> torch.Tensor:
    return v * torch.sigmoid(v)


def _shift_back(x: torch.Tensor, shift: int) -> torch.Tensor:
    """x[:, t - shift] along dim 1, zero where t - shift < 0."""
    if shift == 0:
        return x
    out = torch.zeros_like(x)
    if shift < x.shape[1]:
        out[:, shift:] = x[:, : x.shape[1] - shift]
    return out


def conv(x: torch.Tensor, alpha: torch.Tensor, basis: torch.Tensor, activation: str | None = None) -> torch.Tensor:
    """x [B,T,D], alpha [B,T,K], basis [K,S,D] -> [B,T,D]."""
    S = basis.shape[1]
    y = torch.zeros_like(x)
    for s in range(S):
        tap_weight = alpha @ basis[:, s, :]  # [B,T,D]: sum_k alpha[t,k] basis[k,s,d]
        y = y + tap_weight * _shift_back(x, S - 1 - s)
    return _silu(y) if activation is not None else y


def conv_varlen(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    cu_seqlens,
    activation: str | None = None,
) -> torch.Tensor:
    """x [N,D], alpha [N,K]; sequences are rows [cu[i], cu[i+1])."""
    offs = [int(v) for v in (cu_seqlens.tolist() if hasattr(cu_seqlens, "tolist") else cu_seqlens)]
    pieces = []
    for a, b in zip(offs[:-1], offs[1:]):
        pieces.append(conv(x[None, a:b], alpha[None, a:b], basis, activation)[0])
    return torch.cat(pieces, dim=0) if pieces else x.new_zeros(0, x.shape[1])


def router(z: torch.Tensor, weight: torch.Tensor, router_activation: str = "softmax") -> torch.Tensor:
    """alpha = softmax(z W^T) over K, or exp(z W^T)."""
    logits = z @ weight.transpose(0, 1)
    if router_activation == "softmax":
        return torch.softmax(logits, dim=-1)
    if router_activation == "exp":
        return torch.exp(logits)
    raise ValueError(router_activation)


def step(
    x_t: torch.Tensor,
    alpha_t: torch.Tensor,
    basis: torch.Tensor,
    cache: torch.Tensor,
    activation: str | None = None,
    bf16_products: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """One decode step: x_t [B,D], alpha_t [B,K], cache [B,D,S] -> (y [B,D], new cache).

    ``bf16_products`` reproduces the bf16 mode's rounding of each alpha*basis product.
    """
    states = torch.cat((cache[:, :, 1:], x_t[:, :, None]), dim=2)  # [B,D,S]
    prods = alpha_t[:, :, None, None] * basis[None]  # [B,K,S,D]
    if bf16_products:
        prods = prods.to(torch.bfloat16).to(x_t.dtype)
    tap_weight = prods.sum(dim=1)  # [B,S,D]
    y = (states * tap_weight.transpose(1, 2)).sum(dim=2)
    if activation is not None:
        y = _silu(y)
    return y, states


def final_state(x: torch.Tensor, cache: torch.Tensor | None, kernel_size: int) -> torch.Tensor:
    """Last kernel_size tokens of x as [B,D,S]; missing slots from cache[:, :, T:] or zeros."""
    B, T, D = x.shape
    out = torch.zeros(B, D, kernel_size, dtype=x.dtype)
    for slot in range(kernel_size):
        t = T - kernel_size + slot
        if t >= 0:
            out[:, :, slot] = x[:, t, :]
        elif cache is not None:
            out[:, :, slot] = cache[:, :, T + slot]
    return out


def chunk_indices(cu_seqlens, chunk_size: int) -> list[tuple[int, int]]:
    """(seq_id, chunk_in_seq) for every chunk_size-token chunk, sequences in order."""
    offs = [int(v) for v in cu_seqlens]
    table = []
    for seq, (a, b) in enumerate(zip(offs[:-1], offs[1:])):
        n = -(-(b - a) // chunk_size) if b > a else 0
        table.extend((seq, c) for c in range(n))
    return table


def conv_grads(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    dy: torch.Tensor,
    activation: str | None = None,
    cu_seqlens=None,
    dtype: torch.dtype = torch.float64,
) -> dict[str, torch.Tensor]:
    """Forward + autograd backward of ``conv`` (or ``conv_varlen``) in ``dtype``."""
    xr = x.detach().to(dtype).requires_grad_()
    ar = alpha.detach().to(dtype).requires_grad_()
    br = basis.detach().to(dtype).requires_grad_()
    if cu_seqlens is None:
        y = conv(xr, ar, br, activation)
    else:
        y = conv_varlen(xr, ar, br, cu_seqlens, activation)
    y.backward(dy.detach().to(dtype))
    return {"y": y.detach(), "dx": xr.grad, "dalpha": ar.grad, "dbasis": br.grad}


def module_grads(
    x: torch.Tensor,
    z: torch.Tensor,
    weight: torch.Tensor,
    basis: torch.Tensor,
    dy: torch.Tensor,
    router_activation: str = "softmax",
    activation: str | None = None,
    cu_seqlens=None,
    dtype: torch.dtype = torch.float64,
) -> dict[str, torch.Tensor]:
    """Router + convolution forward and backward (the MoC module's training step)."""
    xr = x.detach().to(dtype).requires_grad_()
    zr = z.detach().to(dtype).requires_grad_()
    wr = weight.detach().to(dtype).requires_grad_()
    br = basis.detach().to(dtype).requires_grad_()
    alpha = router(zr, wr, router_activation)
    if cu_seqlens is None:
        y = conv(xr, alpha, br, activation)
    else:
        y = conv_varlen(xr, alpha, br, cu_seqlens, activation)
    y.backward(dy.detach().to(dtype))
    return {
        "y": y.detach(),
        "alpha": alpha.detach(),
        "dx": xr.grad,
        "dz": zr.grad,
        "drouter": wr.grad,
        "dbasis": br.grad,
    }
