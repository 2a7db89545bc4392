"""Compile librepercep_b200.so (sm_100a) in-tree with nvcc.

    python -m repercep_runtime_b200.build [--force] [--verbose]

The library is written next to this file so that it travels with the source
tree; it is rebuilt when any source under csrc/ or include/ is newer.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_NAME = "librepercep_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = ("capi.cu", "quantize.cu", "quantize_noalloc.cu", "attention.cu", "gemm.cu")

ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps += list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > built for p in deps)


def compile_command(verbose: bool = False) -> list[str]:
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-O3",
        "-std=c++17",
        "-lineinfo",
        "-Xcompiler",
        "-fPIC,-O2",
        "-shared",
        "-I",
        str(INCLUDE),
        "-o",
        str(LIB_PATH),
        *(str(CSRC / s) for s in SOURCES),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    return cmd


def build(force: bool = False, verbose: bool = False) -> Path:
    """Build the shared library if it is missing or stale; return its path."""
    if not force and not _stale():
        return LIB_PATH
    cmd = compile_command(verbose)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd[cmd.index("-o") + 1] = str(tmp)
    proc = subprocess.run(cmd, cwd=str(PKG_DIR), capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
