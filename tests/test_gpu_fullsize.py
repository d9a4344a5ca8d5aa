"""Parity at the BASELINE configs' own sizes, element by element.

The other GPU tests run the reference's verify.py matrix (verify.py:16-23, 242-285) at
small sizes.  These run the CUDA path at the sizes the benchmarks use, so the paths that
only appear there (multi-wave grids, the 32-bit item index, config 5's two-pass backward
with K*S = 256, long sequences) are compared with the float64 oracle too:

* config 2 in full: B=4, T=4096, D=z_dim=2048, K=16, S=4, softmax router, no SiLU;
* config 3: 16384 packed tokens, lengths uniform in [64, 4096] (seeded, the last one
  truncated), D=z_dim=2048, K=16, S=4, exp router, fused SiLU;
* config 5 on one GPU: one full sequence (B=1) of T=8192, D=z_dim=4096, K=32, S=8, softmax
  router, bases at the fan-in std sqrt(K / 3S).

Each runs twice: the MoC module (y, dx, dz, dconv_bases, drouter) and the convolution with
the router's alpha as a leaf tensor (y, dx, dalpha, dconv_bases).  Inputs are bf16; the
oracle computes in float64 on the same bf16 values.  Two bounds, both stated here:

* norm-wise, as the other tests: max|got - ref| / max|ref| <= 2e-2;
* element-wise: |got - ref| <= 2e-2 * |ref| + ATOL_FRAC * max|ref| for every element, with
  ATOL_FRAC = 5e-3.  The absolute part covers elements that are small only because their
  terms cancel: the reference's bf16 rounding points (alpha, basis and dz*x rounded to bf16
  before the contractions, moc/kernels.py:92-95, 390-392) leave each of the up to 16384
  summed terms a 2^-9 relative error, about 2^-9 * sqrt(n) * term size in the sum, which is
  below 1e-3 of the tensor's largest element at these sizes.
"""
from __future__ import annotations

import pytest
import torch

import moc.ops as ops
from moc import MoC, moc_triton
from oracle import moc_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 2e-2
ATOL_FRAC = 5e-3

CONFIGS = {
    "config2": dict(B=4, T=4096, D=2048, Dz=2048, K=16, S=4, act=None, ract="softmax", init_std=0.002),
    "config3": dict(total=16384, D=2048, Dz=2048, K=16, S=4, act="silu", ract="exp", init_std=0.002),
    "config5": dict(B=1, T=8192, D=4096, Dz=4096, K=32, S=8, act=None, ract="softmax",
                    init_std=(32 / (3 * 8)) ** 0.5),
}


def varlen_lengths(total: int, seed: int) -> list[int]:
    """Lengths uniform in [64, 4096] from a seeded generator, the last one truncated so that
    they add up to `total` (config 3's packing)."""
    g = torch.Generator().manual_seed(seed)
    lens, acc = [], 0
    while acc < total:
        n = min(int(torch.randint(64, 4097, (1,), generator=g)), total - acc)
        lens.append(n)
        acc += n
    return lens


def _make(name: str, seed: int = 2024):
    c = CONFIGS[name]
    torch.manual_seed(seed)
    m = MoC(dim=c["D"], z_dim=c["Dz"], kernel_size=c["S"], k=c["K"], activation=c["act"], init_std=c["init_std"],
            router_activation=c["ract"])
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        m.router.copy_(torch.randn(c["K"], c["Dz"], generator=g) * 0.02)
    m = m.to(device="cuda", dtype=torch.bfloat16)
    if "total" in c:
        lens = varlen_lengths(c["total"], seed)
        cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
        shape = (c["total"],)
        kw = {"cu_seqlens": cu, "max_seqlen": max(lens)}
    else:
        shape = (c["B"], c["T"])
        kw = {}
    x = torch.randn(*shape, c["D"], generator=g).bfloat16()
    z = torch.randn(*shape, c["Dz"], generator=g).bfloat16()
    dy = torch.randn(*shape, c["D"], generator=g).bfloat16()
    return m, x, z, dy, kw


def _check(what: str, got: torch.Tensor, ref: torch.Tensor) -> None:
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    assert got.shape == ref.shape, what
    assert torch.isfinite(got).all(), f"{what}: non-finite values"
    scale = ref.abs().max().item() or 1.0
    err = (got - ref).abs()
    assert err.max().item() / scale <= RTOL, f"{what}: norm-wise {err.max().item() / scale:.3e}"
    bound = RTOL * ref.abs() + ATOL_FRAC * scale
    bad = err > bound
    if bad.any():
        worst = torch.argmax((err - bound).reshape(-1)).item()
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {ref.numel()} elements outside |err| <= {RTOL}|ref| + "
            f"{ATOL_FRAC} max|ref|; worst: got {got.reshape(-1)[worst]:.6g} ref {ref.reshape(-1)[worst]:.6g}"
        )


def _kw_cuda(kw):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in kw.items()}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_module_at_full_size(name):
    m, x, z, dy, kw = _make(name)
    kx = x.cuda().requires_grad_()
    kz = z.cuda().requires_grad_()
    y, _ = m(kx, kz, **_kw_cuda(kw))
    y.backward(dy.cuda())
    got = {"y": y, "dx": kx.grad, "dz": kz.grad, "drouter": m.router.grad, "dbasis": m.conv_bases.grad}
    got = {k: v.detach().cpu() for k, v in got.items()}
    del y, kx, kz
    torch.set_num_threads(max(torch.get_num_threads(), 8))
    ref = O.module_grads(x, z, m.router.detach().cpu(), m.conv_bases.detach().cpu(), dy,
                         router_activation=m.router_activation, activation=m.activation,
                         cu_seqlens=kw.get("cu_seqlens"))
    for k, v in got.items():
        _check(f"{name} module {k}", v, ref[k])


@pytest.mark.parametrize("name", list(CONFIGS))
def test_conv_at_full_size(name):
    """The convolution alone, alpha and the bases as leaves: adds dalpha to the checked outputs."""
    m, x, z, dy, kw = _make(name)
    with torch.no_grad():
        alpha = ops.launch_router_forward(z.cuda(), m.router.detach(), m.router_activation)
    kx = x.cuda().requires_grad_()
    ka = alpha.clone().requires_grad_()
    kb = m.conv_bases.detach().clone().requires_grad_()
    y, _ = moc_triton(kx, ka, kb, activation=m.activation, **_kw_cuda(kw))
    y.backward(dy.cuda())
    got = {"y": y.detach().cpu(), "dx": kx.grad.cpu(), "dalpha": ka.grad.cpu(), "dbasis": kb.grad.cpu()}
    del y, kx, ka, kb
    ref = O.conv_grads(x, alpha.cpu(), m.conv_bases.detach().cpu(), dy, activation=m.activation,
                       cu_seqlens=kw.get("cu_seqlens"))
    for k, v in got.items():
        _check(f"{name} conv {k}", v, ref[k])
