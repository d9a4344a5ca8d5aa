"""Host-side behaviour of the drop-in ``moc`` package that needs no GPU: validation
messages, helpers and bookkeeping, each compared with what the reference produced
(tests/golden/moc_golden_meta.json)."""
from __future__ import annotations

import pytest
import torch

import moc
import moc.api as api
import moc.ops as ops
import moc.optim as optim
from conftest import rel_err
from moc.reference import moc_ref, moc_varlen_ref


def test_exports_match_reference():
    assert moc.__all__ == ["MoC", "moc_triton", "moc_fan_in_std", "match_lr_to_init_std",
                           "match_weight_decay_to_lr"]
    for name in ("launch_forward", "launch_preact", "launch_backward", "launch_update",
                 "prepare_chunk_indices", "clear_chunk_index_cache"):
        assert callable(getattr(ops, name))
    assert ops.VARLEN_BLOCK_T == 64


def _replay(name):
    xc, ac, bc = torch.zeros(1, 4, 8), torch.zeros(1, 4, 2), torch.zeros(2, 3, 8)
    calls = {
        "bad_activation": lambda: api.activation_flag("gelu"),
        "bad_router_activation": lambda: api.check_router_activation("sigmoid"),
        "module_bad_activation": lambda: moc.MoC(8, 8, 3, 2, activation="relu"),
        "module_bad_router": lambda: moc.MoC(8, 8, 3, 2, router_activation="relu"),
        "cpu_tensors": lambda: api.check_common_dtypes(xc, ac, bc),
        "cpu_fixed": lambda: api.check_fixed_inputs(xc, ac, bc),
        "moc_triton_cpu": lambda: api.moc_triton(xc, ac, bc),
        "moc_triton_bad_activation": lambda: api.moc_triton(xc, ac, bc, activation="tanh"),
        "cpu_seqlens_without_cu": lambda: api.moc_triton(xc, ac, bc, cu_seqlens_cpu=torch.zeros(2)),
        "chunk_indices_without_cu": lambda: api.moc_triton(
            xc, ac, bc, chunk_indices=torch.zeros(1, 2, dtype=torch.int32)),
        "packed_bad_rank": lambda: api._canonicalize_packed_input(torch.zeros(2, 4, 8), torch.zeros(2, 4, 2)),
        "cache_shape": lambda: api._check_cache(xc, bc, torch.zeros(1, 8, 2)),
        "cache_dtype": lambda: api._check_cache(xc, bc, torch.zeros(1, 8, 3, dtype=torch.float64)),
        "step_x_shape": lambda: moc.MoC(8, 8, 3, 2).step(torch.zeros(1, 2, 8), torch.zeros(1, 2, 8)),
        "step_z_shape": lambda: moc.MoC(8, 8, 3, 2).step(torch.zeros(1, 1, 8), torch.zeros(1, 2, 8)),
        "chunk_size_zero": lambda: ops.prepare_chunk_indices(torch.tensor([0, 4]), 0),
        "chunk_size_float": lambda: ops.prepare_chunk_indices(torch.tensor([0, 4]), 2.0),
        "cu_rank": lambda: ops.prepare_chunk_indices(torch.tensor([[0, 4]]), 2),
        "cu_short": lambda: ops.prepare_chunk_indices(torch.tensor([4]), 2),
        "cu_dtype": lambda: ops.prepare_chunk_indices(torch.tensor([0.0, 4.0]), 2),
        "cu_cpu_dtype": lambda: ops.prepare_chunk_indices(torch.tensor([0, 4]), 2, torch.tensor([0.0, 4.0])),
        "cu_cpu_shape": lambda: ops.prepare_chunk_indices(torch.tensor([0, 4]), 2, torch.tensor([0, 2, 4])),
    }
    try:
        calls[name]()
    except Exception as exc:  # noqa: BLE001
        return type(exc).__name__, str(exc)
    return None, None


def test_error_messages_match_reference(golden):
    for err in golden.meta["errors"]:
        got = _replay(err["name"])
        assert got == (err["type"], err["message"]), err["name"]


def test_module_on_cpu_raises_like_reference():
    m = moc.MoC(16, 12, 4, 4)
    with pytest.raises(ValueError, match="x, alpha, and basis must all be CUDA tensors"):
        m(torch.zeros(1, 3, 16), torch.zeros(1, 3, 12))


def test_optim_helpers_match_reference(golden):
    o = golden.meta["optim"]
    assert optim.moc_fan_in_std(16, 4) == o["fan_in_16_4"]
    assert optim.moc_fan_in_std(32, 8) == o["fan_in_32_8"]
    assert optim.match_lr_to_init_std(optim.moc_fan_in_std(16, 4), reference_std=0.01,
                                      reference_lr=1e-3) == o["lr"]
    assert optim.match_lr_to_init_std(0.05) == o["lr_default"]
    assert optim.match_weight_decay_to_lr(0.1155, reference_lr=1e-3, reference_weight_decay=0.1) == o["wd"]
    assert optim.match_weight_decay_to_lr(3e-4) == o["wd_default"]


def test_module_parameters_and_init():
    torch.manual_seed(0)
    m = moc.MoC(dim=64, z_dim=32, kernel_size=4, k=16, init_std=0.002)
    assert m.conv_bases.shape == (16, 4, 64) and m.router.shape == (16, 32)
    assert torch.count_nonzero(m.router) == 0
    bound = 0.002 * 3 ** 0.5
    assert m.conv_bases.abs().max() <= bound and m.conv_bases.abs().max() > 0.8 * bound
    assert m.state_size == 64 * 4
    assert set(m.state_dict()) == {"conv_bases", "router"}
    m2 = moc.MoC(dim=8, z_dim=8, kernel_size=4, k=16)  # fan-in init
    assert m2.conv_bases.abs().max() <= optim.moc_fan_in_std(16, 4) * 3 ** 0.5


def test_final_state_matches_reference(golden):
    for i, case in enumerate(golden.meta["final_state_cases"]):
        x = golden.t(f"final_state/{i}/x")
        cache = golden.t(f"final_state/{i}/cache") if case["cache"] else None
        assert torch.equal(api._final_state(x, cache, case["kernel_size"]), golden.t(f"final_state/{i}/out"))


def test_prepare_chunk_indices_host_offsets_match_reference(golden):
    for case in golden.meta["chunk_cases"]:
        for dt in (torch.int32, torch.int64):
            ops.clear_chunk_index_cache()
            cu = torch.tensor(case["cu_seqlens"], dtype=dt)
            tab = ops.prepare_chunk_indices(cu, case["chunk_size"])
            assert tab.dtype == torch.int32 and tab.is_contiguous()
            assert tab.tolist() == case["table"], case


def test_chunk_index_cache_is_lru_keyed_on_identity_and_version():
    ops.clear_chunk_index_cache()
    cu = torch.tensor([0, 5, 9], dtype=torch.int32)
    t1 = ops.prepare_chunk_indices(cu, 2)
    assert ops.prepare_chunk_indices(cu, 2) is t1
    assert ops.prepare_chunk_indices(cu.clone(), 2) is not t1  # identity, not value
    cu.add_(0)  # bumps _version
    t2 = ops.prepare_chunk_indices(cu, 2)
    assert t2 is not t1 and torch.equal(t1, t2)
    for c in range(2, 10):
        ops.prepare_chunk_indices(cu, c)
    assert len(ops._chunk_index_cache) == 4


def test_public_reference_module_matches_golden(golden):
    for case in golden.meta["conv_cases"]:
        if case["x_dtype"] != "fp32" or case["alpha_dtype"] != "fp32":
            continue
        v = case["varlen"]
        x = golden.t("in/xv" if v else "in/x")
        a = golden.t("in/av" if v else "in/alpha")
        b = golden.t(f"in/{case['basis']}")
        if v:
            y = moc_varlen_ref(x, a, b, golden.t("in/cu_seqlens"), activation=case["activation"])
        else:
            y = moc_ref(x, a, b, activation=case["activation"])
        assert rel_err(y, golden.t(f"conv/{case['name']}/y")) < 1e-5
