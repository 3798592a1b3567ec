"""The ctypes mirrors in rollfast_b200/_lib.py against the C header: every
field's offset and every struct's size, from a C program compiled here with
gcc against include/rollfast_b200.h (no GPU, no CUDA headers needed)."""

import ctypes
import os
import shutil
import subprocess

import pytest

from rollfast_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

STRUCTS = [
    ("rf_muon_leaf", _lib.RfMuonLeaf),
    ("rf_muon_params", _lib.RfMuonParams),
    ("rf_tail_leaf", _lib.RfTailLeaf),
    ("rf_adam_leaf", _lib.RfAdamLeaf),
    ("rf_adam_params", _lib.RfAdamParams),
    ("rf_ipc_handle", _lib.RfIpcHandle),
]


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    d = tmp_path_factory.mktemp("abi")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "rollfast_b200.h"', "int main(void) {"]
    for cname, cls in STRUCTS:
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = d / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = d / "layout"
    subprocess.run([cc, "-std=c99", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {(a, b): int(c) for a, b, c in (ln.split() for ln in out.splitlines())}


@pytest.mark.parametrize("cname,cls", STRUCTS, ids=[s[0] for s in STRUCTS])
def test_ctypes_mirror_matches_header(c_layout, cname, cls):
    assert ctypes.sizeof(cls) == c_layout[(cname, "sizeof")]
    for fname, _ in cls._fields_:
        assert getattr(cls, fname).offset == c_layout[(cname, fname)], (cname, fname)


def test_enum_values_match_header():
    src = open(os.path.join(ROOT, "include", "rollfast_b200.h")).read()
    for name, value in [("RF_PRECOND_FROBENIUS", _lib.RF_PRECOND_FROBENIUS), ("RF_PRECOND_SPECTRAL", _lib.RF_PRECOND_SPECTRAL),
                        ("RF_PRECOND_AOL", _lib.RF_PRECOND_AOL), ("RF_PRECOND_SCHATTEN", _lib.RF_PRECOND_SCHATTEN),
                        ("RF_NS_F16", _lib.RF_NS_F16), ("RF_NS_BF16", _lib.RF_NS_BF16), ("RF_NS_F32", _lib.RF_NS_F32)]:
        assert f"{name} = {value}" in src, name
