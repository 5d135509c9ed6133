"""The C ABI used from a plain C program: tests/c/abi_from_c.c is compiled
with gcc against include/b2x.h, linked to libb2x.so and run (no GPU needed:
it exercises only argument checks, queries and default configuration)."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_abi_from_plain_c():
    from b2x import _lib as L
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    libdir = os.path.dirname(L.LIB_PATH)
    if not os.path.exists(L.LIB_PATH):
        L.build()
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "abi_from_c")
        subprocess.run([cc, "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "c", "abi_from_c.c"), "-L", libdir, "-l:libb2x.so",
                        f"-Wl,-rpath,{libdir}", "-o", exe], check=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout
