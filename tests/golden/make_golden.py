"""Generate the golden fixtures in this folder from the reference implementation.

    python tests/golden/make_golden.py --reference <path to the reference checkout>

Runs the reference's own CPU-capable code — moc/reference.py (``moc_ref``,
``moc_varlen_ref``), ``MoC.forward`` of moc/api.py (its router lines, with
``moc_triton`` pointed at ``moc_ref`` because the Triton path needs a GPU),
``_final_state`` (moc/api.py:218-227), ``prepare_chunk_indices`` (moc/ops.py:47-104),
the moc/optim.py helpers and the CPU-reachable validation errors — on seeded CPU
inputs, and writes:

* ``moc_golden.npz``         inputs (float32 masters) and reference outputs
* ``moc_golden_meta.json``   case list, dtypes, shapes, errors, optim values

Case matrix mirrors the reference's verify.py:9-23,242-285 (x dtype in {fp32, bf16},
kernel size in {2, 4}, activation in {None, silu}, fixed and varlen, a mixed-storage
case per dtype, decode steps) at reduced sizes so the fixtures stay small.  Only this
script reads the reference; the tests read the fixtures.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

B, T, D, K = 2, 32, 32, 8
VARLEN_LENGTHS = [13, 7, 1, 11]
STEP_T = 8
DT = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MOC_REFERENCE"),
                    help="the reference checkout (default: $MOC_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set MOC_REFERENCE to the reference checkout")
    sys.path.insert(0, args.reference)
    import moc as ref  # noqa: E402  (the reference package)
    import moc.api as ref_api  # noqa: E402
    import moc.ops as ref_ops  # noqa: E402
    import moc.optim as ref_optim  # noqa: E402
    from moc.reference import moc_ref, moc_varlen_ref  # noqa: E402

    arrays: dict[str, np.ndarray] = {}
    meta: dict = {"shapes": {"B": B, "T": T, "D": D, "K": K, "varlen_lengths": VARLEN_LENGTHS,
                             "step_t": STEP_T}, "conv_cases": [], "step_cases": [], "module_cases": []}

    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, T, D, generator=g) * 0.5
    alpha = torch.softmax(torch.randn(B, T, K, generator=g), dim=-1)
    dy = torch.randn(B, T, D, generator=g) * 0.1
    offsets = np.cumsum([0] + VARLEN_LENGTHS).tolist()
    N = offsets[-1]
    xv = torch.randn(N, D, generator=g) * 0.5
    av = torch.softmax(torch.randn(N, K, generator=g), dim=-1)
    dyv = torch.randn(N, D, generator=g) * 0.1
    bases = {ks: torch.randn(K, ks, D, generator=g) * 0.1 for ks in (2, 4)}
    basis_mixed = torch.randn(K, 4, D, generator=g) * 0.1
    for name, t in (("x", x), ("alpha", alpha), ("dy", dy), ("xv", xv), ("av", av), ("dyv", dyv),
                    ("basis2", bases[2]), ("basis4", bases[4]), ("basis_mixed", basis_mixed)):
        arrays[f"in/{name}"] = _np(t)
    arrays["in/cu_seqlens"] = np.asarray(offsets, dtype=np.int64)

    # ---------------------------------------------------------------- convolution cases
    def run_conv(case: str, varlen: bool, xdt: str, adt: str, bdt: str, ks: int, act):
        basis = basis_mixed if case.startswith("mixed") else bases[ks]
        xs, als, dys = (xv, av, dyv) if varlen else (x, alpha, dy)
        kx, ka, kb = xs.to(DT[xdt]), als.to(DT[adt]), basis.to(DT[bdt])
        # verify.py:54-64: the oracle sees the inputs rounded to the compute dtype
        rx = kx.float().detach().clone().requires_grad_()
        ra = ka.to(DT[xdt]).float().detach().clone().requires_grad_()
        rb = kb.to(DT[xdt]).float().detach().clone().requires_grad_()
        if varlen:
            y = moc_varlen_ref(rx, ra, rb, torch.tensor(offsets, dtype=torch.int32), activation=act)
        else:
            y = moc_ref(rx, ra, rb, activation=act)
        y.backward(dys.to(DT[xdt]).float())
        key = f"conv/{case}"
        arrays[f"{key}/y"] = _np(y)
        arrays[f"{key}/dx"] = _np(rx.grad)
        arrays[f"{key}/dalpha"] = _np(ra.grad)
        arrays[f"{key}/dbasis"] = _np(rb.grad)
        meta["conv_cases"].append({"name": case, "varlen": varlen, "x_dtype": xdt, "alpha_dtype": adt,
                                   "basis_dtype": bdt, "kernel_size": ks, "activation": act,
                                   "basis": "basis_mixed" if case.startswith("mixed") else f"basis{ks}"})

    for xdt in ("fp32", "bf16"):
        for ks in (2, 4):
            for act in (None, "silu"):
                for varlen in (False, True):
                    run_conv(f"{'varlen' if varlen else 'fixed'}_{xdt}_ks{ks}_{act or 'plain'}", varlen,
                             xdt, xdt, xdt, ks, act)
        adt, bdt = ("fp32", "fp16") if xdt == "bf16" else ("bf16", "fp16")
        for varlen in (False, True):
            run_conv(f"mixed_{'varlen' if varlen else 'fixed'}_{xdt}", varlen, xdt, adt, bdt, 4, None)

    # ---------------------------------------------------------------- decode steps
    for xdt in ("fp32", "bf16"):
        for ks in (2, 4):
            for act in (None, "silu"):
                kx = x[:, :STEP_T].to(DT[xdt])
                ka = alpha[:, :STEP_T].to(DT[xdt])
                kb = bases[ks].to(DT[xdt])
                y = moc_ref(kx.float(), ka.float(), kb.float(), activation=act)
                key = f"step/{xdt}_ks{ks}_{act or 'plain'}"
                arrays[f"{key}/y"] = _np(y)
                arrays[f"{key}/final_cache"] = _np(kx[:, -ks:].transpose(1, 2))
                meta["step_cases"].append({"name": f"{xdt}_ks{ks}_{act or 'plain'}", "x_dtype": xdt,
                                           "kernel_size": ks, "activation": act})

    # ---------------------------------------------------------------- module (router + conv)
    def cpu_moc_triton(x_, alpha_, basis_, cache=None, output_final_state=False, activation=None,
                       cu_seqlens=None, max_seqlen=None, cu_seqlens_cpu=None, chunk_indices=None):
        if cu_seqlens is not None:
            return moc_varlen_ref(x_, alpha_, basis_, cu_seqlens, activation=activation), None
        return moc_ref(x_, alpha_, basis_, activation=activation), None

    original_moc_triton = ref_api.moc_triton
    ref_api.moc_triton = cpu_moc_triton  # MoC.forward resolves moc_triton from module globals
    z_dim = 24
    for name, router_act, act, varlen in (("softmax_plain", "softmax", None, False),
                                          ("exp_silu", "exp", "silu", False),
                                          ("softmax_silu_varlen", "softmax", "silu", True)):
        torch.manual_seed(1)
        m = ref.MoC(dim=D, z_dim=z_dim, kernel_size=4, k=K, activation=act, init_std=0.1,
                    router_activation=router_act)
        with torch.no_grad():
            m.router.copy_(torch.randn(K, z_dim, generator=g) * 0.2)
        shape = (N, D) if varlen else (B, T, D)
        xm = (torch.randn(*shape, generator=g) * 0.5).requires_grad_()
        zm = torch.randn(*shape[:-1], z_dim, generator=g).requires_grad_()
        dym = torch.randn(*shape, generator=g) * 0.1
        kwargs = {"cu_seqlens": torch.tensor(offsets, dtype=torch.int32), "max_seqlen": max(VARLEN_LENGTHS)} \
            if varlen else {}
        y, _ = m(xm, zm, **kwargs)
        y.backward(dym)
        key = f"module/{name}"
        for k_, v_ in (("x", xm), ("z", zm), ("dy", dym), ("router", m.router), ("conv_bases", m.conv_bases)):
            arrays[f"{key}/in_{k_}"] = _np(v_)
        arrays[f"{key}/y"] = _np(y)
        arrays[f"{key}/dx"] = _np(xm.grad)
        arrays[f"{key}/dz"] = _np(zm.grad)
        arrays[f"{key}/drouter"] = _np(m.router.grad)
        arrays[f"{key}/dbasis"] = _np(m.conv_bases.grad)
        meta["module_cases"].append({"name": name, "router_activation": router_act, "activation": act,
                                     "varlen": varlen, "z_dim": z_dim})

    ref_api.moc_triton = original_moc_triton

    # ---------------------------------------------------------------- final state
    meta["final_state_cases"] = []
    for i, (tt, ks, with_cache) in enumerate(((6, 4, False), (2, 4, False), (2, 4, True), (3, 3, True),
                                              (1, 2, True))):
        xs = torch.randn(B, tt, 5, generator=g)
        cache = torch.randn(B, 5, ks, generator=g) if with_cache else None
        st = ref_api._final_state(xs, cache, ks)
        arrays[f"final_state/{i}/x"] = _np(xs)
        if cache is not None:
            arrays[f"final_state/{i}/cache"] = _np(cache)
        arrays[f"final_state/{i}/out"] = _np(st)
        meta["final_state_cases"].append({"T": tt, "kernel_size": ks, "cache": with_cache})

    # ---------------------------------------------------------------- chunk indices
    meta["chunk_cases"] = []
    for cu in ([0, 31, 48, 53, 76], [0, 64, 128], [0, 1], [0, 0, 5, 5, 70], [0, 65, 65, 129, 4000]):
        for cs in (1, 3, 16, 64):
            if cu[-1] // cs > 600:
                continue
            tab = ref_ops.prepare_chunk_indices(torch.tensor(cu, dtype=torch.int64), cs)
            meta["chunk_cases"].append({"cu_seqlens": cu, "chunk_size": cs, "table": tab.tolist()})
            ref_ops.clear_chunk_index_cache()

    # ---------------------------------------------------------------- optim helpers
    meta["optim"] = {
        "fan_in_16_4": ref_optim.moc_fan_in_std(16, 4),
        "fan_in_32_8": ref_optim.moc_fan_in_std(32, 8),
        "lr": ref_optim.match_lr_to_init_std(ref_optim.moc_fan_in_std(16, 4), reference_std=0.01,
                                             reference_lr=1e-3),
        "lr_default": ref_optim.match_lr_to_init_std(0.05),
        "wd": ref_optim.match_weight_decay_to_lr(0.1155, reference_lr=1e-3, reference_weight_decay=0.1),
        "wd_default": ref_optim.match_weight_decay_to_lr(3e-4),
    }

    # ---------------------------------------------------------------- CPU-reachable errors
    errors = []

    def record(name, fn):
        try:
            fn()
        except Exception as exc:  # noqa: BLE001
            errors.append({"name": name, "type": type(exc).__name__, "message": str(exc)})
        else:
            errors.append({"name": name, "type": None, "message": None})

    xc, ac, bc = torch.zeros(1, 4, 8), torch.zeros(1, 4, 2), torch.zeros(2, 3, 8)
    record("bad_activation", lambda: ref_api.activation_flag("gelu"))
    record("bad_router_activation", lambda: ref_api.check_router_activation("sigmoid"))
    record("module_bad_activation", lambda: ref.MoC(8, 8, 3, 2, activation="relu"))
    record("module_bad_router", lambda: ref.MoC(8, 8, 3, 2, router_activation="relu"))
    record("cpu_tensors", lambda: ref_api.check_common_dtypes(xc, ac, bc))
    record("cpu_fixed", lambda: ref_api.check_fixed_inputs(xc, ac, bc))
    record("moc_triton_cpu", lambda: ref_api.moc_triton(xc, ac, bc))
    record("moc_triton_bad_activation", lambda: ref_api.moc_triton(xc, ac, bc, activation="tanh"))
    record("cpu_seqlens_without_cu", lambda: ref_api.moc_triton(xc, ac, bc, cu_seqlens_cpu=torch.zeros(2)))
    record("chunk_indices_without_cu",
           lambda: ref_api.moc_triton(xc, ac, bc, chunk_indices=torch.zeros(1, 2, dtype=torch.int32)))
    record("packed_bad_rank", lambda: ref_api._canonicalize_packed_input(torch.zeros(2, 4, 8), torch.zeros(2, 4, 2)))
    record("cache_shape", lambda: ref_api._check_cache(xc, bc, torch.zeros(1, 8, 2)))
    record("cache_dtype", lambda: ref_api._check_cache(xc, bc, torch.zeros(1, 8, 3, dtype=torch.float64)))
    record("step_x_shape", lambda: ref.MoC(8, 8, 3, 2).step(torch.zeros(1, 2, 8), torch.zeros(1, 2, 8)))
    record("step_z_shape", lambda: ref.MoC(8, 8, 3, 2).step(torch.zeros(1, 1, 8), torch.zeros(1, 2, 8)))
    record("chunk_size_zero", lambda: ref_ops.prepare_chunk_indices(torch.tensor([0, 4]), 0))
    record("chunk_size_float", lambda: ref_ops.prepare_chunk_indices(torch.tensor([0, 4]), 2.0))
    record("cu_rank", lambda: ref_ops.prepare_chunk_indices(torch.tensor([[0, 4]]), 2))
    record("cu_short", lambda: ref_ops.prepare_chunk_indices(torch.tensor([4]), 2))
    record("cu_dtype", lambda: ref_ops.prepare_chunk_indices(torch.tensor([0.0, 4.0]), 2))
    record("cu_cpu_dtype",
           lambda: ref_ops.prepare_chunk_indices(torch.tensor([0, 4]), 2, torch.tensor([0.0, 4.0])))
    record("cu_cpu_shape",
           lambda: ref_ops.prepare_chunk_indices(torch.tensor([0, 4]), 2, torch.tensor([0, 2, 4])))
    meta["errors"] = errors

    np.savez_compressed(os.path.join(HERE, "moc_golden.npz"), **arrays)
    with open(os.path.join(HERE, "moc_golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(f"wrote {len(arrays)} arrays, {len(meta['conv_cases'])} conv cases, {len(errors)} errors")


if __name__ == "__main__":
    main()
