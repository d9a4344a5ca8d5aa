"""The C ABI library loads without a GPU, exports every function declared in
include/moc_b200.h, and rejects malformed arguments before touching the device."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT
from moc import _lib

HEADER = os.path.join(ROOT, "include", "moc_b200.h")


def _declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moc_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_functions()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), name
    # the ctypes prototypes cover exactly the declared surface
    assert sorted(_lib.SIGNATURES) == declared


def test_version_and_error_strings():
    lib = _lib.load()
    assert lib.moc_version().decode().startswith("moc_b200")
    assert lib.moc_error_string(0).decode() == "ok"
    assert "workspace" in lib.moc_error_string(5).decode()
    assert lib.moc_last_cuda_error().decode() == ""


def _problem(**kw):
    p = _lib.MocProblem()
    p.batch, p.seq_len, p.n_tokens, p.dim = 2, 8, 16, 32
    p.n_bases, p.kernel_size = 4, 4
    p.x_dtype = p.alpha_dtype = p.basis_dtype = 2
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize(
    "fields,code",
    [
        ({"x_dtype": 1}, 2),          # f16 x is not a compute dtype
        ({"alpha_dtype": 7}, 2),
        ({"dim": 0}, 1),
        ({"n_bases": 0}, 1),
        ({"n_bases": 129}, 3),
        ({"kernel_size": 65}, 3),
        ({"n_tokens": 15}, 1),        # batch*seq_len mismatch
        ({"activation": 2}, 1),
    ],
)
def test_forward_rejects_bad_problems(fields, code):
    lib = _lib.load()
    p = _problem(**fields)
    assert lib.moc_forward(ctypes.byref(p), 1, 1, 1, 1, None) == code


def test_null_problem_and_pointers_rejected():
    lib = _lib.load()
    assert lib.moc_forward(None, 1, 1, 1, 1, None) == 1
    p = _problem()
    assert lib.moc_forward(ctypes.byref(p), None, 1, 1, 1, None) == 1
    assert lib.moc_backward_workspace_bytes(None) == 0


def test_varlen_problem_checks():
    lib = _lib.load()
    p = _problem(batch=0, seq_len=0, cu_seqlens=1, n_seqs=0, chunk_size=64)
    assert lib.moc_forward(ctypes.byref(p), 1, 1, 1, 1, None) == 1
    p = _problem(batch=0, seq_len=0, cu_seqlens=1, n_seqs=2, chunk_size=64, n_chunks=3, chunk_indices=None)
    assert lib.moc_forward(ctypes.byref(p), 1, 1, 1, 1, None) == 1
    p = _problem(batch=0, seq_len=0, cu_seqlens=1, n_seqs=2, chunk_size=64, n_chunks=0, cu_seqlens_dtype=5)
    assert lib.moc_forward(ctypes.byref(p), 1, 1, 1, 1, None) == 2


def test_workspace_query_needs_no_gpu():
    lib = _lib.load()
    p = _problem()
    assert lib.moc_backward_workspace_bytes(ctypes.byref(p)) > 0
    assert lib.moc_router_backward_workspace_bytes(16, 32, 4, 2) > 0


def test_step_router_and_chunk_checks():
    lib = _lib.load()
    strides = (ctypes.c_int64 * 3)(32, 4, 1)
    assert lib.moc_step(2, 8, 4, 4, 1, 2, 2, 0, 1, 1, 1, 1, strides, 1, None) == 2
    assert lib.moc_step(2, 0, 4, 4, 2, 2, 2, 0, 1, 1, 1, 1, strides, 1, None) == 1
    assert lib.moc_step(0, 8, 4, 4, 2, 2, 2, 0, 1, 1, 1, 1, strides, 1, None) == 0  # empty batch: no work
    assert lib.moc_router_forward(4, 8, 4, 9, 0, 1, 1, 1, None) == 2
    assert lib.moc_router_forward(4, 8, 4, 2, 3, 1, 1, 1, None) == 1
    assert lib.moc_prepare_chunk_indices(1, 0, 1, 0, 1, 1, None) == 1
    assert lib.moc_set_kernel_path(5) == 1
