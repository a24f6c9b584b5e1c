"""Build libenl_b200.so in-tree with nvcc for sm_100a.

Usage: ``python -m enilnets_b200.build [--force]``. The library is one
translation unit (csrc/enl_lib.cu) compiled with
``-gencode arch=compute_100a,code=sm_100a``; the resulting .so sits next to
this file so that it travels with the source tree.

The build reports registers and spills per kernel (-Xptxas -v).
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_NAME = "libenl_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libenl_b200.so")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    lib_mtime = LIB_PATH.stat().st_mtime
    return all(src.stat().st_mtime <= lib_mtime for src in _sources())


def _check_ptxas_report(report: str) -> dict:
    """Parse the -Xptxas -v report: per-kernel registers and spill bytes."""
    info = {}
    current = None
    for line in report.splitlines():
        m = re.search(r"Compiling entry function '(\w+)'", line)
        if m:
            current = m.group(1)
            info[current] = {"regs": None, "spill": 0}
            continue
        if current is None:
            continue
        m = re.search(r"(\d+) bytes spill stores", line)
        if m:
            info[current]["spill"] = int(m.group(1))
        m = re.search(r"Used (\d+) registers", line)
        if m:
            info[current]["regs"] = int(m.group(1))
    return info


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", f"-I{INCLUDE}",
           "-Xcompiler", "-fPIC", "-shared", "-Xptxas", "-v", "-o", str(tmp),
           str(CSRC / "enl_lib.cu")]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"nvcc failed ({proc.returncode}) building {LIB_NAME}")
    info = _check_ptxas_report(proc.stderr)
    if verbose:
        for name, rec in sorted(info.items()):
            print(f"{name}: {rec['regs']} regs, {rec['spill']} B spill")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    path = build(force="--force" in argv, verbose=True)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
