# SPDX-License-Identifier: Apache-2.0
"""The C ABI from a plain-C host: tests/c_host/kf_c_host_check.c includes
include/kotflash_b200.h, is compiled by gcc as C99 (so the header must be
valid C, not only C++) and linked against the in-tree shared library, then
run.  It calls only host-side entry points and argument checks, so it runs
without a GPU -- the situation of an FFI embedder (cgo, JNI, a C runtime)
that binds the library directly instead of through Python."""
import shutil
import subprocess
from pathlib import Path

import pytest

from kotflash_b200 import _ext

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_plain_c_host_links_and_passes_host_checks(tmp_path):
    _ext.load()  # the library must be built
    exe = tmp_path / "kf_c_host_check"
    lib_dir = _ext.LIB_PATH.parent
    subprocess.run(
        ["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"),
         str(ROOT / "tests" / "c_host" / "kf_c_host_check.c"), "-L", str(lib_dir), "-lkotflash_b200",
         f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
        check=True, capture_output=True, text=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "all C-host checks passed" in run.stdout
