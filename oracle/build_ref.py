"""Build the reference's own CPU attention kernel into oracle/_ref/.

Test/baseline infrastructure only.  Compiles, from the reference source tree
where it lies (never copied), the AMX BF16 flash-attention extension
``kernels/cpu/amx_attn/flash_attn_amx.cpp`` with the compile flags of the
reference's own ``kernels/cpu/amx_attn/setup.py``, through
``torch.utils.cpp_extension`` (the reference builds it the same way).  The
resulting ``oracle/_ref/repercep_amx_ref*.so`` is git-ignored but travels to
the GPU box, where ``bench.py --impl reference`` times it on the host cores.

    python -m oracle.build_ref [--reference <reference source tree>]
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
MODULE = "repercep_amx_ref"
REL_SOURCE = Path("kernels/cpu/amx_attn/flash_attn_amx.cpp")
# Flags of kernels/cpu/amx_attn/setup.py (EXTRA_COMPILE_ARGS / EXTRA_LINK_ARGS).
CFLAGS = [
    "-std=c++17", "-O3", "-fopenmp", "-march=sapphirerapids", "-mamx-bf16", "-mamx-tile",
    "-mamx-int8", "-mavx512bf16", "-mavx512fp16", "-mavx512f", "-mavx512vl", "-mavx512dq",
    "-mavx512bw", "-funroll-loops", "-fno-strict-aliasing", "-Wno-unused-function",
    "-Wno-unused-variable",
]
LDFLAGS = ["-fopenmp"]


def built_module_path() -> Path | None:
    for p in sorted(REF_DIR.glob(f"{MODULE}*.so")):
        return p
    return None


def host_has_amx() -> bool:
    try:
        text = Path("/proc/cpuinfo").read_text()
    except OSError:
        return False
    for line in text.splitlines():
        if line.startswith("flags"):
            return "amx_bf16" in line.split()
    return False


def load_reference_kernel():  # type: ignore[no-untyped-def]
    """Import the prebuilt reference AMX module, or return None."""
    path = built_module_path()
    if path is None or not host_has_amx():
        return None
    spec = importlib.util.spec_from_file_location(MODULE, path)
    if spec is None or spec.loader is None:
        return None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def build(reference: Path) -> Path | None:
    src = reference / REL_SOURCE
    if not src.exists():
        return None
    from torch.utils import cpp_extension

    REF_DIR.mkdir(exist_ok=True)
    # /usr/bin/g++ links OpenMP correctly in this image (the /opt toolchain lacks libgomp.spec).
    if Path("/usr/bin/g++").exists():
        os.environ["CXX"] = "/usr/bin/g++"
    cpp_extension.load(
        name=MODULE,
        sources=[str(src)],
        extra_cflags=CFLAGS,
        extra_ldflags=LDFLAGS,
        build_directory=str(REF_DIR),
        verbose=False,
    )
    # Keep only the module: the object files and ninja state stay out of the tree's payload.
    for p in REF_DIR.iterdir():
        if p.suffix in (".o", ".ninja_deps", ".ninja_log") or p.name in ("build.ninja", ".ninja_log"):
            p.unlink()
    return built_module_path()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    out = build(Path(args.reference))
    print(out if out else "reference source not found; nothing built", file=sys.stderr)


if __name__ == "__main__":
    main()
