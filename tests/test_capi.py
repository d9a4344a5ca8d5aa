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


def test_misaligned_workspace_rejected_before_any_launch():
    """The conv backward writes its dalpha partials to the workspace 16 bytes at a time,
    so a workspace that does not start on a 16-byte boundary is refused on the host
    (MOC_ERR_MISALIGNED = 4), before any device call."""
    lib = _lib.load()
    p = _problem()
    assert lib.moc_backward(ctypes.byref(p), 16, 16, 16, 16, 16, 16, 16, 4, 1 << 20, None) == 4
    assert lib.moc_router_backward(16, 32, 8, 2, 0, 16, 16, 16, 16, 2, 16, 16, 8, 1 << 20, None) == 4


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


def _c_layout(struct: str, fields: list[str]) -> dict[str, int]:
    """sizeof / offsetof of a header struct, compiled with the host C compiler."""
    import shutil
    import subprocess
    import tempfile

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    body = "".join(f'printf("{f} %zu\\n", offsetof({struct}, {f}));' for f in fields)
    src = (f'#include <stddef.h>\n#include <stdio.h>\n#include "{HEADER}"\n'
           f'int main(void) {{ printf("sizeof %zu\\n", sizeof({struct})); {body} return 0; }}\n')
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "l.c"), "w") as f:
            f.write(src)
        exe = os.path.join(d, "l")
        subprocess.run([cc, "-I", os.path.join(ROOT, "include"), os.path.join(d, "l.c"), "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.splitlines())}


@pytest.mark.parametrize("struct,mirror", [("moc_problem", _lib.MocProblem),
                                           ("moc_decode_module", _lib.MocDecodeModule),
                                           ("moc_proj_problem", _lib.MocProjProblem),
                                           ("moc_proj_module", _lib.MocProjModule)])
def test_ctypes_structs_match_the_header_layout(struct, mirror):
    names = [f[0] for f in mirror._fields_]
    layout = _c_layout(struct, names)
    assert layout["sizeof"] == ctypes.sizeof(mirror)
    for n in names:
        assert layout[n] == getattr(mirror, n).offset, n


def test_decode_multi_checks():
    lib = _lib.load()

    def mods(n, **kw):
        arr = (_lib.MocDecodeModule * n)()
        for i in range(n):
            f = dict(dim=64, n_bases=16, kernel_size=4, activation=0, router_act=0, weight=256, basis=512,
                     x=768, cache=1024, alpha=1280, out=1536)
            f.update(kw)
            arr[i] = _lib.MocDecodeModule(**f)
        return arr

    assert lib.moc_decode_step_multi(0, mods(1), 4, 64, 2048, None) == 1
    assert lib.moc_decode_step_multi(5, mods(5), 4, 64, 2048, None) == 1
    assert lib.moc_decode_step_multi(1, mods(1, n_bases=17), 4, 64, 2048, None) == 3
    assert lib.moc_decode_step_multi(1, mods(1, kernel_size=5), 4, 64, 2048, None) == 3
    assert lib.moc_decode_step_multi(1, mods(1, dim=0), 4, 64, 2048, None) == 1
    assert lib.moc_decode_step_multi(1, mods(1, dim=60), 4, 64, 2048, None) == 3  # dim % 8
    assert lib.moc_decode_step_multi(1, mods(1), 4, 60, 2048, None) == 3  # z_dim % 8
    assert lib.moc_decode_step_multi(1, mods(1, router_act=2), 4, 64, 2048, None) == 1
    assert lib.moc_decode_step_multi(1, mods(1, cache=1030), 4, 64, 2048, None) == 4
    assert lib.moc_decode_step_multi(1, mods(1, x=0), 4, 64, 2048, None) == 1
    two = mods(2)
    two[1].kernel_size = 2
    assert lib.moc_decode_step_multi(2, two, 4, 64, 2048, None) == 3  # one kernel size for all modules
    assert lib.moc_decode_step_multi(2, mods(2), 0, 64, 2048, None) == 0  # empty batch: no work


def test_proj_checks():
    lib = _lib.load()

    def prob(**kw):
        f = dict(batch=2, seq_len=64, in_dim=256, dim=128, n_bases=16, kernel_size=4, activation=0, h=256,
                 weight=512, alpha=768, basis=1024, out=1280)
        f.update(kw)
        return ctypes.byref(_lib.MocProjProblem(**f))

    assert lib.moc_proj_forward(None, None) == 1
    assert lib.moc_proj_forward(prob(n_bases=32), None) == 3    # at most 16 bases
    assert lib.moc_proj_forward(prob(n_bases=12), None) == 3    # n_bases % 8
    assert lib.moc_proj_forward(prob(kernel_size=9), None) == 3
    assert lib.moc_proj_forward(prob(in_dim=100), None) == 3    # in_dim % 8
    assert lib.moc_proj_forward(prob(dim=132), None) == 3       # dim % 8
    assert lib.moc_proj_forward(prob(dim=0), None) == 1
    assert lib.moc_proj_forward(prob(activation=2), None) == 1
    assert lib.moc_proj_forward(prob(seq_len=1 << 40), None) == 3  # 32-bit tensor-map coordinates
    assert lib.moc_proj_forward(prob(weight=0), None) == 1
    assert lib.moc_proj_forward(prob(out=1288), None) == 4      # 16-byte alignment
    assert lib.moc_proj_forward(prob(batch=0), None) == 0       # no tokens: no work


def test_proj_multi_checks():
    lib = _lib.load()

    def mods(n, **kw):
        arr = (_lib.MocProjModule * n)()
        for i in range(n):
            f = dict(dim=128, row_offset=128 * i, n_bases=16, activation=0, alpha=256, basis=512, out=768)
            f.update(kw)
            arr[i] = _lib.MocProjModule(**f)
        return arr

    def call(n, m, rows=384, **kw):
        f = dict(batch=2, seq_len=64, in_dim=256, kernel_size=4, h=1024, weight=1280)
        f.update(kw)
        return lib.moc_proj_forward_multi(n, m, f["batch"], f["seq_len"], f["in_dim"], f["kernel_size"], f["h"],
                                          f["weight"], rows, None)

    assert call(0, mods(1)) == 1
    assert call(5, mods(5)) == 1                       # at most 4 modules
    assert call(3, mods(3), rows=300) == 1             # rows past the weight
    assert call(1, mods(1, row_offset=-8)) == 1
    assert call(1, mods(1, n_bases=24)) == 3
    assert call(1, mods(1, dim=100)) == 3
    assert call(1, mods(1), kernel_size=9) == 3
    assert call(1, mods(1, activation=3)) == 1
    assert call(1, mods(1, out=776)) == 4              # 16-byte alignment
    assert call(1, mods(1), h=1032) == 4
    assert call(3, mods(3), batch=0) == 0              # no tokens: no work


def test_comm_checks():
    lib = _lib.load()
    comm = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    assert lib.moc_comm_create(0, 0, 16, ctypes.byref(comm), handle) == 1
    assert lib.moc_comm_create(2, 2, 16, ctypes.byref(comm), handle) == 1
    assert lib.moc_comm_create(0, 9, 16, ctypes.byref(comm), handle) == 1  # more than 8 ranks
    assert lib.moc_comm_create(0, 1, 0, ctypes.byref(comm), handle) == 1
    assert lib.moc_comm_connect(None, handle) == 1
    assert lib.moc_comm_allreduce(None, 0, None, None, None, None) == 1
    assert lib.moc_comm_destroy(None) == 1
