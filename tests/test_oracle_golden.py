"""Pins the CPU oracle to the reference: every golden vector made from the reference's
own code (tests/golden/make_golden.py) must be reproduced by oracle/moc_oracle.py."""
from __future__ import annotations

import pytest
import torch

from conftest import DTYPES, rel_err
from oracle import moc_oracle as O

TOL = 2e-5  # oracle (float64) vs reference (float32), same rounded inputs


def _conv_inputs(g, case):
    varlen = case["varlen"]
    x = g.t("in/xv" if varlen else "in/x")
    a = g.t("in/av" if varlen else "in/alpha")
    dy = g.t("in/dyv" if varlen else "in/dy")
    basis = g.t(f"in/{case['basis']}")
    xdt = DTYPES[case["x_dtype"]]
    kx = x.to(xdt)
    ka = a.to(DTYPES[case["alpha_dtype"]]).to(xdt)
    kb = basis.to(DTYPES[case["basis_dtype"]]).to(xdt)
    return kx.double(), ka.double(), kb.double(), dy.to(xdt).double()


def test_golden_has_full_matrix(golden):
    names = {c["name"] for c in golden.meta["conv_cases"]}
    assert len(names) == 20
    assert {"fixed_bf16_ks4_silu", "varlen_fp32_ks2_plain", "mixed_fixed_bf16", "mixed_varlen_fp32"} <= names


@pytest.mark.parametrize("idx", range(20))
def test_conv_matches_reference(golden, idx):
    case = golden.meta["conv_cases"][idx]
    x, a, b, dy = _conv_inputs(golden, case)
    cu = golden.t("in/cu_seqlens") if case["varlen"] else None
    got = O.conv_grads(x, a, b, dy, activation=case["activation"], cu_seqlens=cu)
    for name in ("y", "dx", "dalpha", "dbasis"):
        err = rel_err(got[name], golden.t(f"conv/{case['name']}/{name}"))
        assert err < TOL, (case["name"], name, err)


def test_step_matches_reference(golden):
    S_T = golden.meta["shapes"]["step_t"]
    for case in golden.meta["step_cases"]:
        xdt = DTYPES[case["x_dtype"]]
        ks = case["kernel_size"]
        x = golden.t("in/x")[:, :S_T].to(xdt).double()
        a = golden.t("in/alpha")[:, :S_T].to(xdt).double()
        b = golden.t(f"in/basis{ks}").to(xdt).double()
        cache = torch.zeros(x.shape[0], x.shape[2], ks, dtype=torch.float64)
        ys = []
        for t in range(S_T):
            y, cache = O.step(x[:, t], a[:, t], b, cache, activation=case["activation"])
            ys.append(y)
        key = f"step/{case['name']}"
        assert rel_err(torch.stack(ys, 1), golden.t(f"{key}/y")) < TOL, case["name"]
        assert torch.equal(cache.float(), golden.t(f"{key}/final_cache")), case["name"]


@pytest.mark.parametrize("idx", range(3))
def test_module_matches_reference(golden, idx):
    case = golden.meta["module_cases"][idx]
    key = f"module/{case['name']}"
    cu = golden.t("in/cu_seqlens") if case["varlen"] else None
    got = O.module_grads(
        golden.t(f"{key}/in_x"), golden.t(f"{key}/in_z"), golden.t(f"{key}/in_router"),
        golden.t(f"{key}/in_conv_bases"), golden.t(f"{key}/in_dy"),
        router_activation=case["router_activation"], activation=case["activation"], cu_seqlens=cu,
    )
    for name in ("y", "dx", "dz", "drouter", "dbasis"):
        err = rel_err(got[name], golden.t(f"{key}/{name}"))
        assert err < TOL, (case["name"], name, err)


def test_final_state_matches_reference(golden):
    for i, case in enumerate(golden.meta["final_state_cases"]):
        x = golden.t(f"final_state/{i}/x")
        cache = golden.t(f"final_state/{i}/cache") if case["cache"] else None
        assert torch.equal(O.final_state(x, cache, case["kernel_size"]), golden.t(f"final_state/{i}/out"))


def test_chunk_indices_match_reference(golden):
    for case in golden.meta["chunk_cases"]:
        got = [list(p) for p in O.chunk_indices(case["cu_seqlens"], case["chunk_size"])]
        assert got == case["table"], case


def test_oracle_detects_a_planted_tap_error(golden):
    """A wrong tap convention (x[t-s] instead of x[t-(S-1-s)]) must fail the golden check."""
    case = golden.meta["conv_cases"][2]  # fixed fp32 ks2 silu
    x, a, b, dy = _conv_inputs(golden, case)
    flipped = O.conv_grads(x, a, b.flip(1), dy, activation=case["activation"])
    assert rel_err(flipped["y"], golden.t(f"conv/{case['name']}/y")) > 1e-2
