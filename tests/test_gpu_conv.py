"""GPU parity of the convolution kernels against the CPU oracle and the golden vectors.

Tolerances (north star), as max|got - ref| / max|ref| per tensor, with the oracle run
in float64 on the same inputs rounded the way the kernels see them (the reference's
verify.py:54-64 convention):
  * fp32 inputs: <= 1e-4
  * bf16 inputs: <= 2e-2
Decode caches and varlen boundaries are checked bit-exactly.
"""
from __future__ import annotations

import pytest
import torch

import moc.ops as ops
from conftest import DTYPES, rel_err
from moc import _lib, moc_triton
from oracle import moc_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}
# an output stored in a narrower dtype than the compute dtype carries that dtype's rounding
STORE_TOL = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 2e-2}
DEV = "cuda"


def _inputs(B, T, D, K, S, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g) * 0.5
    a = torch.softmax(torch.randn(B, T, K, generator=g), dim=-1)
    dy = torch.randn(B, T, D, generator=g) * 0.1
    basis = torch.randn(K, S, D, generator=g) * 0.1
    return x, a, dy, basis


def _run(x, a, basis, dy, xdt, adt, bdt, act, cu=None, max_seqlen=None, **kw):
    kx = x.to(xdt).to(DEV).requires_grad_()
    ka = a.to(adt).to(DEV).requires_grad_()
    kb = basis.to(bdt).to(DEV).requires_grad_()
    y, _ = moc_triton(kx, ka, kb, activation=act, cu_seqlens=None if cu is None else cu.to(DEV),
                      max_seqlen=max_seqlen, **kw)
    y.backward(dy.to(xdt).to(DEV))
    got = {"y": y, "dx": kx.grad, "dalpha": ka.grad, "dbasis": kb.grad}
    # oracle input: what the kernel computes with (alpha/basis rounded to the x dtype)
    ref = O.conv_grads(kx.detach().cpu().double(), ka.detach().cpu().to(xdt).double(),
                       kb.detach().cpu().to(xdt).double(), dy.to(xdt).double(), activation=act,
                       cu_seqlens=None if cu is None else cu.cpu())
    return got, ref


def _assert_close(got, ref, xdt, label):
    for name in ("y", "dx", "dalpha", "dbasis"):
        tol = max(TOL[xdt], STORE_TOL[got[name].dtype])
        err = rel_err(got[name], ref[name])
        assert err <= tol, f"{label} {name}: rel err {err:.3e} > {tol}"


@pytest.fixture(params=[0, 1, 2], ids=["auto", "generic", "warp_bwd"])
def kernel_path(request):
    _lib.set_kernel_path(request.param)
    yield request.param
    _lib.set_kernel_path(0)


# ------------------------------------------------------------- the reference's verify matrix

@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
@pytest.mark.parametrize("ks", [2, 4])
@pytest.mark.parametrize("act", [None, "silu"])
def test_verify_matrix_fixed(kernel_path, xdt, ks, act):
    x, a, dy, basis = _inputs(2, 64, 64, 8, ks)
    got, ref = _run(x, a, basis, dy, xdt, xdt, xdt, act)
    _assert_close(got, ref, xdt, f"fixed {xdt} ks={ks} {act}")


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
@pytest.mark.parametrize("ks", [2, 4])
@pytest.mark.parametrize("act", [None, "silu"])
def test_verify_matrix_varlen(kernel_path, xdt, ks, act):
    lengths = [31, 17, 5, 23]
    cu = torch.tensor([0, 31, 48, 53, 76], dtype=torch.int32)
    x, a, dy, basis = _inputs(1, 76, 64, 8, ks, seed=1)
    got, ref = _run(x[0], a[0], basis, dy[0], xdt, xdt, xdt, act, cu=cu, max_seqlen=max(lengths))
    _assert_close(got, ref, xdt, f"varlen {xdt} ks={ks} {act}")
    # the [1, N, D] form gives the same output
    y3, _ = moc_triton(x.to(xdt).to(DEV), a.to(xdt).to(DEV), basis.to(xdt).to(DEV), activation=act,
                       cu_seqlens=cu.to(DEV), max_seqlen=max(lengths))
    assert y3.shape == (1, 76, 64)
    assert torch.equal(y3[0], got["y"].detach())


@pytest.mark.parametrize("xdt,adt,bdt", [(torch.bfloat16, torch.float32, torch.float16),
                                         (torch.float32, torch.bfloat16, torch.float16)])
def test_mixed_storage_dtypes(kernel_path, xdt, adt, bdt):
    x, a, dy, basis = _inputs(2, 64, 64, 8, 4, seed=2)
    got, ref = _run(x, a, basis, dy, xdt, adt, bdt, None)
    _assert_close(got, ref, xdt, "mixed")
    assert got["dalpha"].dtype == adt and got["dbasis"].dtype == bdt and got["dx"].dtype == xdt


# ------------------------------------------------------------- golden vectors

def test_golden_conv_cases(golden):
    for case in golden.meta["conv_cases"]:
        v = case["varlen"]
        xdt = DTYPES[case["x_dtype"]]
        x = golden.t("in/xv" if v else "in/x")
        a = golden.t("in/av" if v else "in/alpha")
        dy = golden.t("in/dyv" if v else "in/dy")
        basis = golden.t(f"in/{case['basis']}")
        cu = golden.t("in/cu_seqlens") if v else None
        kx = x.to(xdt).to(DEV).requires_grad_()
        ka = a.to(DTYPES[case["alpha_dtype"]]).to(DEV).requires_grad_()
        kb = basis.to(DTYPES[case["basis_dtype"]]).to(DEV).requires_grad_()
        y, _ = moc_triton(kx, ka, kb, activation=case["activation"],
                          cu_seqlens=None if cu is None else cu.to(DEV), max_seqlen=13 if v else None)
        y.backward(dy.to(xdt).to(DEV))
        for name, t in (("y", y), ("dx", kx.grad), ("dalpha", ka.grad), ("dbasis", kb.grad)):
            err = rel_err(t, golden.t(f"conv/{case['name']}/{name}"))
            assert err <= max(TOL[xdt], STORE_TOL[t.dtype]), (case["name"], name, err)


# ------------------------------------------------------------- determinism and options

def test_backward_is_bitwise_deterministic():
    x, a, dy, basis = _inputs(4, 256, 256, 16, 4, seed=3)
    outs = []
    for _ in range(2):
        dx, da, db = ops.launch_backward(
            x.bfloat16().cuda(), a.bfloat16().cuda(), basis.bfloat16().cuda(), dy.bfloat16().cuda(),
            dy.bfloat16().cuda(), activation_flag=1, need_x=True)
        outs.append((dx, da, db))
    for t1, t2 in zip(*outs):
        assert torch.equal(t1, t2)


def test_first_call_on_a_fresh_thread():
    """A thread whose first CUDA work is this library's call (as the autograd engine's
    device thread can be) gets the same results as the thread that made the earlier calls."""
    import threading

    x, a, dy, basis = _inputs(2, 128, 256, 32, 8, seed=5)
    args = [t.bfloat16().cuda() for t in (x, a, basis, dy, dy)]
    ref = ops.launch_backward(*args, activation_flag=0, need_x=True)
    torch.cuda.synchronize()
    box = {}

    def work():
        try:
            box["out"] = ops.launch_backward(*args, activation_flag=0, need_x=True)
            torch.cuda.synchronize()
        except Exception as e:  # re-raised on the test thread
            box["err"] = e

    t = threading.Thread(target=work)
    t.start()
    t.join()
    if "err" in box:
        raise box["err"]
    for t1, t2 in zip(ref, box["out"]):
        assert torch.equal(t1, t2)


def test_need_x_false_skips_dx():
    x, a, dy, basis = _inputs(2, 64, 64, 8, 4)
    dx, da, db = ops.launch_backward(x.cuda(), a.cuda(), basis.cuda(), dy.cuda(), dy.cuda(),
                                     activation_flag=0, need_x=False)
    assert dx is None and da.shape == a.shape and db.shape == basis.shape


def test_preact_matches_forward_without_activation():
    x, a, _, basis = _inputs(2, 64, 64, 8, 4)
    p = ops.launch_preact(x.cuda(), a.cuda(), basis.cuda())
    y = ops.launch_forward(x.cuda(), a.cuda(), basis.cuda(), activation_flag=0)
    assert torch.equal(p, y)


# ------------------------------------------------------------- varlen edge cases

@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
def test_varlen_ragged_lengths_and_boundaries(kernel_path, xdt):
    # lengths around the kernel size and the 64-token chunk; int64 offsets
    lengths = [1, 3, 4, 63, 64, 65, 130, 2]
    cu = torch.tensor([0] + torch.tensor(lengths).cumsum(0).tolist(), dtype=torch.int64)
    N = int(cu[-1])
    x, a, dy, basis = _inputs(1, N, 96, 16, 4, seed=4)
    got, ref = _run(x[0], a[0], basis, dy[0], xdt, xdt, xdt, "silu", cu=cu, max_seqlen=max(lengths))
    _assert_close(got, ref, xdt, "ragged")


@pytest.mark.parametrize("K,S,path", [(16, 4, 0), (32, 8, 2)], ids=["k16s4", "k32s8_warp_bwd"])
@pytest.mark.parametrize("lengths", [None, [1024, 960, 64, 1000, 1048], [70, 2000, 2026]],
                         ids=["fixed", "aligned", "ragged"])
def test_silu_backward_hands_dz_rows_between_items(lengths, K, S, path):
    """With SiLU a CTA of the warp-level backward runs its 64-token items last to first, and each
    item hands its first S - 1 dz rows to the item before it.  At D = 2048 a CTA takes several
    items (16 channel slices share the SMs), so hand-overs happen inside sequences. They must not
    happen across sequence boundaries, whether those fall on item boundaries (fixed: 1088 = 17
    items, so one CTA holds the last item of sequence 0 and the first of sequence 1; aligned:
    1024, 1984, 2048, ...) or inside items (ragged).  32 bases with 8 taps take the two-pass
    warp-level kernel here (moc_set_kernel_path(MOC_PATH_WARP_BACKWARD)); both passes hand over."""
    D = 2048
    _lib.set_kernel_path(path)
    try:
        if lengths is None:
            x, a, dy, basis = _inputs(2, 1088, D, K, S, seed=41)
            got, ref = _run(x, a, basis, dy, torch.bfloat16, torch.bfloat16, torch.bfloat16, "silu")
        else:
            cu = torch.tensor([0] + torch.tensor(lengths).cumsum(0).tolist(), dtype=torch.int32)
            x, a, dy, basis = _inputs(1, int(cu[-1]), D, K, S, seed=42)
            got, ref = _run(x[0], a[0], basis, dy[0], torch.bfloat16, torch.bfloat16, torch.bfloat16, "silu",
                            cu=cu, max_seqlen=max(lengths))
    finally:
        _lib.set_kernel_path(0)
    _assert_close(got, ref, torch.bfloat16, "hand-over")
    assert _lib.device_status(clear=True) == 0


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
def test_varlen_boundaries_are_bit_exact(kernel_path, xdt):
    """Poisoning every other sequence (x, dy times 1000) leaves the outputs of one
    sequence bitwise unchanged: no tap or gradient crosses a cu_seqlens boundary."""
    lengths = [5, 64, 3, 70, 1, 66]
    cu = torch.tensor([0] + torch.tensor(lengths).cumsum(0).tolist(), dtype=torch.int32)
    N = int(cu[-1])
    x, a, dy, basis = _inputs(1, N, 64, 8, 4, seed=9)
    kb = basis.to(xdt).cuda()
    ka = a[0].to(xdt).cuda()

    def run(xx, dd):
        kx = xx.to(xdt).cuda()
        y = ops.launch_forward(kx, ka, kb, activation_flag=1, cu_seqlens=cu.cuda())
        dx, da, _ = ops.launch_backward(kx, ka, kb, dd.to(xdt).cuda(), None, activation_flag=1, need_x=True,
                                        cu_seqlens=cu.cuda())
        return y, dx, da

    clean = run(x[0], dy[0])
    for s in range(len(lengths)):
        lo, hi = int(cu[s]), int(cu[s + 1])
        scale = torch.full((N, 1), 1000.0)
        scale[lo:hi] = 1.0
        poisoned = run(x[0] * scale, dy[0] * scale)
        for c, p in zip(clean, poisoned):
            assert torch.equal(c[lo:hi], p[lo:hi]), s


def test_varlen_explicit_chunk_indices_and_cpu_offsets():
    lengths = [70, 5, 129]
    cu = torch.tensor([0, 70, 75, 204], dtype=torch.int32)
    x, a, _, basis = _inputs(1, 204, 64, 8, 4, seed=5)
    args = (x[0].bfloat16().cuda(), a[0].bfloat16().cuda(), basis.bfloat16().cuda())
    ref = ops.launch_forward(*args, activation_flag=1, cu_seqlens=cu.cuda())
    ops.clear_chunk_index_cache()
    table = ops.prepare_chunk_indices(cu.cuda(), cu_seqlens_cpu=cu)
    assert table.tolist() == [list(p) for p in O.chunk_indices(cu.tolist(), 64)]
    via_table, _ = moc_triton(*args, activation="silu", cu_seqlens=cu.cuda(), max_seqlen=max(lengths),
                              chunk_indices=table)
    via_cpu, _ = moc_triton(*args, activation="silu", cu_seqlens=cu.cuda(), max_seqlen=max(lengths),
                            cu_seqlens_cpu=cu)
    assert torch.equal(ref, via_table) and torch.equal(ref, via_cpu)


def test_device_chunk_builder_matches_host_table(golden):
    for case in golden.meta["chunk_cases"]:
        ops.clear_chunk_index_cache()
        cu = torch.tensor(case["cu_seqlens"], dtype=torch.int32, device=DEV)
        assert ops.prepare_chunk_indices(cu, case["chunk_size"]).cpu().tolist() == case["table"]


# ------------------------------------------------------------- multi-token with a cache

@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
def test_prefill_continuation_with_cache(xdt):
    B, T, D, K, S = 2, 24, 64, 8, 4
    x, a, _, basis = _inputs(B, T + 10, D, K, S, seed=6)
    full = O.conv(x.to(xdt).double(), a.to(xdt).double(), basis.to(xdt).double())
    kx, ka, kb = x.to(xdt).cuda(), a.to(xdt).cuda(), basis.to(xdt).cuda()
    y1, state = moc_triton(kx[:, :10], ka[:, :10], kb, output_final_state=True)
    y2, state2 = moc_triton(kx[:, 10:], ka[:, 10:], kb, cache=state, output_final_state=True)
    assert rel_err(torch.cat((y1, y2), 1), full) <= TOL[xdt]
    assert torch.equal(state2, kx[:, -S:].transpose(1, 2))


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
@pytest.mark.parametrize("S,act", [(4, None), (3, "silu"), (2, None), (1, "silu")])
def test_prefill_with_cache_reads_the_cache_as_halo(kernel_path, xdt, S, act):
    """A cache with T > 1: the kernels read the cache as each sequence's causal halo.  y and
    the gradients of x, alpha and basis equal the reference's form (cache prepended with
    zero routing weights, moc/api.py:299-309) in the float64 oracle, and the GPU result of
    that form (taken when the cache needs a gradient)."""
    B, T, D, K = 2, 70, 192, 16
    g = torch.Generator().manual_seed(30 + S)
    x = torch.randn(B, T, D, generator=g) * 0.5
    a = torch.softmax(torch.randn(B, T, K, generator=g), dim=-1)
    basis = torch.randn(K, S, D, generator=g) * 0.2
    cache = torch.randn(B, D, S, generator=g) * 0.5
    dy = torch.randn(B, T, D, generator=g) * 0.1
    # oracle of the prepended form, rows t >= 0
    px = torch.cat((cache.to(xdt).double().transpose(1, 2), x.to(xdt).double()), 1)
    pa = torch.cat((torch.zeros(B, S, K, dtype=torch.float64), a.to(xdt).double()), 1)
    pdy = torch.cat((torch.zeros(B, S, D, dtype=torch.float64), dy.to(xdt).double()), 1)
    ref = O.conv_grads(px, pa, basis.to(xdt).double(), pdy, activation=act)
    ref = {"y": ref["y"][:, S:], "dx": ref["dx"][:, S:], "dalpha": ref["dalpha"][:, S:], "dbasis": ref["dbasis"]}
    kx = x.to(xdt).cuda().requires_grad_()
    ka = a.to(xdt).cuda().requires_grad_()
    kb = basis.to(xdt).cuda().requires_grad_()
    kc = cache.to(xdt).cuda().transpose(1, 2).contiguous().transpose(1, 2)  # a strided [B, D, S] view
    y, _ = moc_triton(kx, ka, kb, cache=kc, activation=act)
    y.backward(dy.to(xdt).cuda())
    got = {"y": y, "dx": kx.grad, "dalpha": ka.grad, "dbasis": kb.grad}
    _assert_close(got, ref, xdt, f"prefill S={S} {act}")
    # the reference's form on the GPU (cache with requires_grad) agrees as well
    kx2, ka2, kb2 = (t.detach().clone().requires_grad_() for t in (kx, ka, kb))
    kc2 = kc.detach().clone().requires_grad_()
    y2, _ = moc_triton(kx2, ka2, kb2, cache=kc2, activation=act)
    y2.backward(dy.to(xdt).cuda())
    for name, t1, t2 in (("y", y, y2), ("dx", kx.grad, kx2.grad), ("dalpha", ka.grad, ka2.grad),
                         ("dbasis", kb.grad, kb2.grad)):
        assert rel_err(t1, t2) <= max(TOL[xdt], STORE_TOL[t1.dtype]), name
    assert kc2.grad is not None


# ------------------------------------------------------------- larger shapes

@pytest.mark.parametrize("B,T,D,K,S", [(2, 300, 520, 16, 4), (1, 130, 256, 32, 8), (3, 77, 192, 4, 3),
                                       (1, 64, 2048, 16, 4), (3, 333, 384, 16, 4), (2, 256, 2048, 8, 2),
                                       (1, 129, 96, 16, 3), (2, 200, 160, 16, 1)])
def test_larger_shapes_bf16(kernel_path, B, T, D, K, S):
    x, a, dy, basis = _inputs(B, T, D, K, S, seed=7)
    got, ref = _run(x, a, basis, dy, torch.bfloat16, torch.bfloat16, torch.bfloat16, "silu")
    _assert_close(got, ref, torch.bfloat16, f"shape {(B, T, D, K, S)}")


@pytest.mark.parametrize("K,S,act", [(32, 8, None), (32, 8, "silu"), (32, 5, "silu"), (24, 6, None),
                                     (32, 7, None), (17, 8, "silu")])
def test_many_bases_long_kernels(kernel_path, K, S, act):
    """Up to 32 bases with up to 8 taps (the large data-parallel config is K=32, S=8): the
    basis sits in shared memory and the forward / backward run one CTA per SM."""
    x, a, dy, basis = _inputs(2, 160, 384, K, S, seed=11)
    got, ref = _run(x, a, basis, dy, torch.bfloat16, torch.bfloat16, torch.bfloat16, act)
    _assert_close(got, ref, torch.bfloat16, f"K={K} S={S} act={act}")


def test_many_bases_long_kernels_varlen(kernel_path):
    lengths = [5, 70, 1, 8, 130, 64]
    cu = torch.tensor([0] + torch.tensor(lengths).cumsum(0).tolist(), dtype=torch.int32)
    x, a, dy, basis = _inputs(1, int(cu[-1]), 256, 32, 8, seed=12)
    got, ref = _run(x[0], a[0], basis, dy[0], torch.bfloat16, torch.bfloat16, torch.bfloat16, None, cu=cu,
                    max_seqlen=max(lengths))
    _assert_close(got, ref, torch.bfloat16, "varlen K=32 S=8")


@pytest.mark.parametrize("S", [5, 8])
@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("form", ["fixed", "varlen", "halo", "no_dx"])
def test_tcgen05_and_warp_level_backward_agree(S, act, form):
    """The two tensor-core backward kernels of 17..32 bases with 5..8 taps (the tcgen05 one,
    MOC_PATH_AUTO, and the warp-level one, MOC_PATH_WARP_BACKWARD) on the same inputs: dx is
    formed the same way in both (W_s on mma.sync, FFMA2 taps) and dalpha / dbasis differ only
    in the order of their fp32 sums, so they agree to the rounding of the bf16 outputs."""
    x, a, dy, basis = _inputs(2, 200, 384, 24, S, seed=31 + S)
    kw, cu = {}, None
    if form == "varlen":
        cu = torch.tensor([0, 3, 70, 71, 199, 260, 400], dtype=torch.int32).cuda()
        x, a, dy = x.reshape(1, 400, 384)[0], a.reshape(1, 400, 24)[0], dy.reshape(1, 400, 384)[0]
        kw = {"cu_seqlens": cu}
    if form == "halo":
        kw = {"halo": torch.randn(2, 384, S).bfloat16().cuda()}
    args = [t.bfloat16().cuda() for t in (x, a, basis)]
    res = []
    for path in (0, 2):
        _lib.set_kernel_path(path)
        try:
            res.append(ops.launch_backward(*args, dy.bfloat16().cuda(), None, activation_flag=act,
                                           need_x=form != "no_dx", **kw))
        finally:
            _lib.set_kernel_path(0)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    (dx5, da5, db5), (dxw, daw, dbw) = res
    if form == "no_dx":
        assert dx5 is None and dxw is None
    else:
        assert rel_err(dx5, dxw) <= 1e-2
    assert rel_err(da5, daw) <= 1e-2
    assert rel_err(db5, dbw) <= 1e-2


def test_generic_and_tensor_core_paths_agree():
    x, a, dy, basis = _inputs(2, 256, 512, 16, 4, seed=8)
    res = []
    for path in (0, 1):
        _lib.set_kernel_path(path)
        try:
            args = (x.bfloat16().cuda(), a.bfloat16().cuda(), basis.bfloat16().cuda())
            y = ops.launch_forward(*args, activation_flag=1)
            grads = ops.launch_backward(*args, dy.bfloat16().cuda(), None, activation_flag=1, need_x=True)
            res.append((y, *grads))
        finally:
            _lib.set_kernel_path(0)
    for t0, t1 in zip(*res):
        assert rel_err(t0, t1) <= TOL[torch.bfloat16]
