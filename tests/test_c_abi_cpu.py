"""The C ABI from C: tests/c/abi_consumer.c compiled with gcc against
include/rollfast_b200.h and linked to the built librollfast_b200.so (no GPU:
it calls the planning and validation entry points only)."""

import os
import shutil
import subprocess

import pytest

from rollfast_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_c_consumer_links_and_runs(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    libdir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "abi_consumer"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "abi_consumer.c"), "-o", str(exe),
                    "-L", libdir, "-lrollfast_b200", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "0 failures" in out.stdout
