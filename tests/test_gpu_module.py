"""GPU parity of the full MoC module (router + convolution, forward and backward) and of
decode, against the CPU oracle and the golden vectors.  Tolerances as in
test_gpu_conv.py: fp32 <= 1e-4, bf16 <= 2e-2 (max|err| / max|ref|); decode caches are
compared bit-exactly."""
from __future__ import annotations

import pytest
import torch

import moc.ops as ops
from conftest import rel_err
from moc import MoC, _lib, moc_triton
from oracle import moc_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def _module(D, Dz, S, K, act, router_act, dtype, init_std=0.1, seed=0):
    torch.manual_seed(seed)
    m = MoC(dim=D, z_dim=Dz, kernel_size=S, k=K, activation=act, init_std=init_std,
            router_activation=router_act)
    g = torch.Generator().manual_seed(seed + 100)
    with torch.no_grad():
        m.router.copy_(torch.randn(K, Dz, generator=g) * 0.02 * (Dz ** 0.5) / 4)
    return m.to(device="cuda", dtype=dtype)


def _step_and_compare(m, x, z, dy, dtype, cu=None, max_seqlen=None):
    kx = x.to(dtype).cuda().requires_grad_()
    kz = z.to(dtype).cuda().requires_grad_()
    kw = {} if cu is None else {"cu_seqlens": cu.cuda(), "max_seqlen": max_seqlen}
    y, _ = m(kx, kz, **kw)
    y.backward(dy.to(dtype).cuda())
    ref = O.module_grads(kx.detach().cpu(), kz.detach().cpu(), m.router.detach().cpu(), m.conv_bases.detach().cpu(),
                         dy.to(dtype), router_activation=m.router_activation, activation=m.activation,
                         cu_seqlens=None if cu is None else cu)
    got = {"y": y, "dx": kx.grad, "dz": kz.grad, "drouter": m.router.grad, "dbasis": m.conv_bases.grad}
    for name, t in got.items():
        err = rel_err(t, ref[name])
        assert err <= TOL[dtype], f"{name}: {err:.3e}"


def test_config1_fp32_module():
    """BASELINE config 1 shape (B=2, T=256, D=Dz=128, K=4, S=4, fp32, softmax, no SiLU)."""
    m = _module(128, 128, 4, 4, None, "softmax", torch.float32, init_std=0.002)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 256, 128, generator=g)
    z = torch.randn(2, 256, 128, generator=g)
    dy = torch.randn(2, 256, 128, generator=g)
    _step_and_compare(m, x, z, dy, torch.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
@pytest.mark.parametrize("router_act,act", [("softmax", None), ("exp", "silu"), ("softmax", "silu")])
def test_module_fixed(dtype, router_act, act):
    m = _module(192, 160, 4, 16, act, router_act, dtype)
    g = torch.Generator().manual_seed(12)
    x, z, dy = torch.randn(2, 130, 192, generator=g), torch.randn(2, 130, 160, generator=g), \
        torch.randn(2, 130, 192, generator=g)
    _step_and_compare(m, x, z, dy, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
def test_module_varlen_exp_silu(dtype):
    """BASELINE config 3 semantics (packed varlen, exp router, fused SiLU) at test size."""
    m = _module(256, 256, 4, 16, "silu", "exp", dtype, init_std=0.05)
    cu = torch.tensor([0, 100, 164, 300, 301, 420], dtype=torch.int32)
    g = torch.Generator().manual_seed(13)
    x, z, dy = torch.randn(420, 256, generator=g), torch.randn(420, 256, generator=g), \
        torch.randn(420, 256, generator=g)
    _step_and_compare(m, x, z, dy, dtype, cu=cu, max_seqlen=136)


def test_golden_module_cases(golden):
    for case in golden.meta["module_cases"]:
        key = f"module/{case['name']}"
        xin = golden.t(f"{key}/in_x")
        m = MoC(dim=xin.shape[-1], z_dim=case["z_dim"], kernel_size=4, k=8, activation=case["activation"],
                router_activation=case["router_activation"]).cuda()
        with torch.no_grad():
            m.router.copy_(golden.t(f"{key}/in_router"))
            m.conv_bases.copy_(golden.t(f"{key}/in_conv_bases"))
        kx = xin.cuda().requires_grad_()
        kz = golden.t(f"{key}/in_z").cuda().requires_grad_()
        kw = {"cu_seqlens": golden.t("in/cu_seqlens").cuda(), "max_seqlen": 13} if case["varlen"] else {}
        y, _ = m(kx, kz, **kw)
        y.backward(golden.t(f"{key}/in_dy").cuda())
        for name, t in (("y", y), ("dx", kx.grad), ("dz", kz.grad), ("drouter", m.router.grad),
                        ("dbasis", m.conv_bases.grad)):
            assert rel_err(t, golden.t(f"{key}/{name}")) <= 1e-4, (case["name"], name)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
@pytest.mark.parametrize("K", [4, 16, 32])
@pytest.mark.parametrize("router_act", ["softmax", "exp"])
def test_router_forward_backward(dtype, K, router_act):
    g = torch.Generator().manual_seed(14)
    z = torch.randn(3, 97, 320, generator=g)
    w = torch.randn(K, 320, generator=g) * 0.05
    da = torch.randn(3, 97, K, generator=g)
    kz, kw = z.to(dtype).cuda(), w.to(dtype).cuda()
    alpha = ops.launch_router_forward(kz, kw, router_act)
    dz, dw = ops.launch_router_backward(kz, kw, alpha, da.to(dtype).cuda(), router_act)
    zr = kz.cpu().double().requires_grad_()
    wr = kw.cpu().double().requires_grad_()
    ar = O.router(zr, wr, router_act)
    ar.backward(da.to(dtype).double())
    assert rel_err(alpha, ar) <= TOL[dtype]
    assert rel_err(dz, zr.grad) <= TOL[dtype]
    assert rel_err(dw, wr.grad) <= TOL[dtype]


@pytest.mark.parametrize("K", [16, 32])
@pytest.mark.parametrize("router_act", ["softmax", "exp"])
def test_router_backward_scalar_and_vector_paths_agree(K, router_act):
    """bf16 alpha / dalpha are fetched with vector loads and dz leaves through 16-byte
    stores when aligned; fp32 dalpha and a dz that is only 4-byte aligned take the
    per-element paths.  Same arithmetic, so the results are bitwise equal."""
    g = torch.Generator().manual_seed(15)
    N, Dz = 2 * 97, 320
    kz = torch.randn(N, Dz, generator=g).bfloat16().cuda()
    kw = (torch.randn(K, Dz, generator=g) * 0.05).bfloat16().cuda()
    da = torch.randn(N, K, generator=g).bfloat16().cuda()
    alpha = ops.launch_router_forward(kz, kw, router_act)
    dz_ref, dw_ref = ops.launch_router_backward(kz, kw, alpha, da, router_act)
    dz32, dw32 = ops.launch_router_backward(kz, kw, alpha, da.float(), router_act)
    assert torch.equal(dz32, dz_ref) and torch.equal(dw32, dw_ref)

    lib = _lib.load()
    buf = torch.empty(N * Dz + 2, dtype=torch.bfloat16, device="cuda")
    dz = buf[2:].view(N, Dz)  # 4-byte, not 16-byte, aligned
    dw = torch.empty_like(kw)
    code = _lib.dtype_code(kz)
    ws_bytes = lib.moc_router_backward_workspace_bytes(N, Dz, K, code)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    rc = lib.moc_router_backward(N, Dz, K, code, ops.ROUTER_ACTIVATIONS[router_act], _lib.ptr(kz), _lib.ptr(kw),
                                 _lib.ptr(alpha), _lib.ptr(da), code, _lib.ptr(dz), _lib.ptr(dw), _lib.ptr(ws),
                                 ws_bytes, _lib.stream_of(kz.device))
    _lib.check(rc, "moc_router_backward")
    assert torch.equal(dz, dz_ref) and torch.equal(dw, dw_ref)


# ------------------------------------------------------------------ decode

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
@pytest.mark.parametrize("ks", [2, 4])
@pytest.mark.parametrize("act", [None, "silu"])
def test_decode_steps_match_full_sequence(dtype, ks, act):
    """verify.py:173-213: 8 single-token steps equal the full-sequence conv; the final
    cache holds exactly the last S inputs (bitwise)."""
    g = torch.Generator().manual_seed(15)
    B, T, D, K = 2, 8, 64, 8
    x = (torch.randn(B, T, D, generator=g) * 0.5).to(dtype)
    a = torch.softmax(torch.randn(B, T, K, generator=g), -1).to(dtype)
    basis = (torch.randn(K, ks, D, generator=g) * 0.1).to(dtype)
    ref = O.conv(x.double(), a.double(), basis.double(), act)
    cache = torch.zeros(B, D, ks, device="cuda", dtype=dtype)
    ys = []
    for t in range(T):
        y, cache = moc_triton(x[:, t:t + 1].cuda(), a[:, t:t + 1].cuda(), basis.cuda(), cache=cache,
                              output_final_state=True, activation=act)
        ys.append(y)
    assert rel_err(torch.cat(ys, 1), ref) <= TOL[dtype]
    assert torch.equal(cache.cpu(), x[:, -ks:].transpose(1, 2))


def test_decode_step_against_oracle_step_and_strided_cache():
    g = torch.Generator().manual_seed(16)
    B, D, K, S = 5, 300, 16, 4
    cache_full = torch.randn(B, S, D, generator=g).bfloat16()
    cache = cache_full.cuda().transpose(1, 2)  # [B, D, S] with non-contiguous strides
    x = torch.randn(B, D, generator=g).bfloat16()
    a = torch.softmax(torch.randn(B, K, generator=g), -1).bfloat16()
    basis = (torch.randn(K, S, D, generator=g) * 0.1).bfloat16()
    before = cache.cpu().clone()
    y = ops.launch_update(x.cuda(), a.cuda(), basis.cuda(), cache, activation_flag=1)
    ref_y, ref_cache = O.step(x.double(), a.double(), basis.double(), before.double(), activation="silu",
                              bf16_products=True)
    assert rel_err(y, ref_y) <= 2e-2
    assert torch.equal(cache.cpu(), ref_cache.bfloat16())  # shift + append, bit-exact
    assert torch.equal(cache.cpu()[:, :, :S - 1], before[:, :, 1:])


def test_module_prefill_then_step():
    m = _module(128, 96, 4, 16, None, "exp", torch.bfloat16)
    g = torch.Generator().manual_seed(17)
    x = torch.randn(3, 20, 128, generator=g).bfloat16()
    z = torch.randn(3, 20, 96, generator=g).bfloat16()
    with torch.no_grad():
        y_full, _ = m(x.cuda(), z.cuda())
        y_pre, cache = m(x[:, :12].cuda(), z[:, :12].cuda(), output_final_state=True)
        ys = [y_pre]
        for t in range(12, 20):
            y, cache = m.step(x[:, t:t + 1].cuda(), z[:, t:t + 1].cuda(), cache=cache, output_final_state=True)
            ys.append(y)
    assert rel_err(torch.cat(ys, 1), y_full) <= 2e-2
    assert torch.equal(cache, x[:, -4:].cuda().transpose(1, 2))


def test_step_without_cache_allocates_zero_cache():
    m = _module(64, 32, 4, 8, None, "softmax", torch.float32)
    x = torch.randn(2, 1, 64, device="cuda")
    z = torch.randn(2, 1, 32, device="cuda")
    y, cache = m.step(x, z, output_final_state=True)
    assert cache.shape == (2, 64, 4)
    assert torch.equal(cache[:, :, -1], x[:, 0]) and torch.count_nonzero(cache[:, :, :-1]) == 0


def test_c_abi_workspace_too_small_is_an_error():
    x = torch.randn(1, 64, 64, device="cuda").bfloat16()
    a = torch.softmax(torch.randn(1, 64, 8, device="cuda"), -1).bfloat16()
    b = torch.randn(8, 4, 64, device="cuda").bfloat16()
    p, _ = ops._problem(x, a, b, 0, None, None, None, 64)
    import ctypes
    lib = _lib.load()
    need = lib.moc_backward_workspace_bytes(ctypes.byref(p))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    out = [torch.empty_like(t) for t in (x, a, b)]
    rc = lib.moc_backward(ctypes.byref(p), x.data_ptr(), a.data_ptr(), b.data_ptr(), x.data_ptr(),
                          out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(), ws.data_ptr(), need - 1, None)
    assert rc == 5
