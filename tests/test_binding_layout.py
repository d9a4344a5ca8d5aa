"""The published ctypes binding of ``struct moc_problem`` matches the C header.

INTEGRATION.md shows the stub a maintainer of the reference would paste into its
moc/ops.py (the launch it replaces is moc/ops.py:129-194).  A stub that is shorter than
the C struct makes the library read past its end (the trailing ``halo`` pointer), so the
documented field list, ``moc._lib.MocProblem`` and the header must agree field by field,
in order, by C type, offset and total size.  The C side is measured by compiling a tiny
program against include/moc_b200.h with the host C compiler.
"""
from __future__ import annotations

import ctypes
import os
import re
import shutil
import subprocess
import tempfile

import pytest

from conftest import ROOT
from moc import _lib

HEADER = os.path.join(ROOT, "include", "moc_b200.h")
INTEGRATION = os.path.join(ROOT, "INTEGRATION.md")

_CTYPE_OF_C = {"int64_t": ctypes.c_int64, "int32_t": ctypes.c_int32, "const void*": ctypes.c_void_p,
               "void*": ctypes.c_void_p}


def _header_fields() -> list[tuple[str, str, int]]:
    """(name, C type, array length or 0) of struct moc_problem, in declaration order."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct moc_problem \{(.*?)\} moc_problem;", text, flags=re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        m = re.fullmatch(r"((?:const )?\w+\*?) (\w+)(?:\[(\d+)\])?", decl)
        assert m, f"unparsed declaration: {decl!r}"
        fields.append((m.group(2), m.group(1), int(m.group(3) or 0)))
    return fields


def _integration_stub() -> type:
    """Executes the MocProblem class of INTEGRATION.md's ctypes stub."""
    text = open(INTEGRATION).read()
    start = text.index("class MocProblem(ctypes.Structure)")
    end = text.index("]", text.index("_fields_", start))
    # the class statement through the closing bracket of _fields_ (the list holds no "]"
    # other than its own: array types are written `ctypes.c_int64 * 3`)
    src = text[start:end + 1]
    ns: dict = {"ctypes": ctypes}
    exec(src, ns)  # noqa: S102 - documentation code under test
    return ns["MocProblem"]


def _same_ctype(a, b) -> bool:
    if hasattr(a, "_length_") or hasattr(b, "_length_"):
        return (getattr(a, "_length_", None) == getattr(b, "_length_", None)
                and a._type_ is b._type_)
    return a is b


@pytest.mark.parametrize("which", ["integration_md", "moc._lib"])
def test_binding_matches_header(which):
    cls = _integration_stub() if which == "integration_md" else _lib.MocProblem
    header = _header_fields()
    got = cls._fields_
    assert [f[0] for f in got] == [h[0] for h in header], f"{which}: field names or order differ"
    for (name, ct), (_, ctype_c, n) in zip(got, header):
        want = _CTYPE_OF_C[ctype_c]
        if n:
            want = want * n
        assert _same_ctype(ct, want), f"{which}.{name}: {ct} vs {ctype_c}[{n}]"


def test_stub_size_and_offsets_equal_the_c_struct():
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    names = [h[0] for h in _header_fields()]
    prog = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {",
            'printf("sizeof %zu\\n", sizeof(moc_problem));']
    prog += [f'printf("{n} %zu\\n", offsetof(moc_problem, {n}));' for n in names]
    prog += ["return 0; }"]
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "layout.c"), os.path.join(d, "layout")
        with open(src, "w") as f:
            f.write("\n".join(prog))
        subprocess.run([cc, src, "-o", exe], check=True, capture_output=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    c = {k: int(v) for k, v in (line.split() for line in out.splitlines())}
    for cls in (_integration_stub(), _lib.MocProblem):
        assert ctypes.sizeof(cls) == c["sizeof"]
        for n in names:
            assert getattr(cls, n).offset == c[n], n
