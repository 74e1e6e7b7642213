# SPDX-License-Identifier: Apache-2.0
"""Build ``kotflash_b200/_lib/libkotflash_b200.so`` from the .cu sources here.

    python -m kotflash_b200.csrc.build [--verbose]

Compiles every ``*.cu`` in this directory for sm_100a with nvcc, links a
shared library with the static CUDA runtime, and skips the rebuild when the
library is newer than every source and header.  Needs only nvcc (no GPU).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libkotflash_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-I", str(ROOT / "include")]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def sources():
    return sorted(HERE.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    newest = max(p.stat().st_mtime for p in list(HERE.glob("*.cu")) + list(HERE.glob("*.cuh"))
                 + list(HERE.glob("*.h")) + list((ROOT / "include").glob("*.h")) + [Path(__file__)])
    return newest > LIB.stat().st_mtime


def build(force: bool = False, verbose: bool = False, jobs: int = 0) -> Path:
    if not force and not _stale():
        return LIB
    nvcc = _nvcc()
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose else []
    with tempfile.TemporaryDirectory(prefix="kf_build_") as tmp:
        objs = []
        procs = []
        for src in sources():
            obj = Path(tmp) / (src.stem + ".o")
            cmd = [nvcc, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
            objs.append(obj)
        failed = False
        for src, proc in procs:
            out, _ = proc.communicate()
            text = out.decode(errors="replace")
            if proc.returncode != 0:
                failed = True
                sys.stderr.write(f"--- nvcc failed on {src.name}\n{text}\n")
            elif verbose and text.strip():
                sys.stdout.write(f"--- {src.name}\n{text}\n")
        if failed:
            raise RuntimeError("nvcc compilation failed")
        tmp_lib = Path(tmp) / LIB.name
        link = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp_lib), *map(str, objs)]
        res = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
        if res.returncode != 0:
            raise RuntimeError("link failed:\n" + res.stdout.decode(errors="replace"))
        shutil.copy2(tmp_lib, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
