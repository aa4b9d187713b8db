"""The C ABI from plain C: tests/c/abi_check.c compiled with gcc as C99 (-Wall -Werror)
against include/w4a16_b200.h and linked with libw4a16_b200.so, then run; it only calls
entries that answer on the host (validation, sizes, strings), so no GPU is needed."""
import os
import shutil
import subprocess

import pytest

from w4a16 import _lib
from w4a16 import build as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_and_library_from_c(tmp_path):
    B.build()
    lib = _lib.lib_path()
    exe = tmp_path / "abi_check"
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", "abi_check.c"), "-o", str(exe), lib,
           "-Wl,-rpath," + os.path.dirname(lib)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "c abi ok" in out.stdout
