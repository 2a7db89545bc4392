"""Build the reference's own CPU attention kernel into oracle/_ref/, and
install the reference's Python package into baseline/_ref/.

Test/baseline infrastructure only.

* Compiles, from the reference source tree where it lies, the AMX BF16
  flash-attention extension ``kernels/cpu/amx_attn/flash_attn_amx.cpp`` with
  the compile flags of the reference's own ``kernels/cpu/amx_attn/setup.py``,
  through ``torch.utils.cpp_extension`` (the reference builds it the same way).
  The resulting ``oracle/_ref/repercep_amx_ref*.so`` is git-ignored but travels
  to the GPU box, where ``bench.py --impl reference`` times it on the host cores.
* Installs the reference's pure-Python package (``src/repercep``) and its Triton
  kernels module (``kernels/triton_kernels``) unmodified into ``baseline/_ref``
  (git-ignored, travels to the GPU box): the files ``pip install --target
  baseline/_ref`` would place there.  pip itself cannot do it offline, because
  the reference's build backend (hatchling) is not in the wheelhouse.  The
  binding tests import the reference's registries, protocols and diffusers
  bridge from there, and the bench runs the reference's own CPU op and Triton
  kernel from there.

The reference tree is found through the ``REPERCEP_REFERENCE_ROOT`` environment
variable, else as a ``reference`` directory beside this repository.

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
REPO = HERE.parent
# Where the reference's Python package is installed (what pip --target would write).
REF_PKG_DIR = REPO / "baseline" / "_ref"
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


def reference_root() -> Path | None:
    """The reference source tree: $REPERCEP_REFERENCE_ROOT, else ../reference."""
    env = os.environ.get("REPERCEP_REFERENCE_ROOT")
    cands = [Path(env)] if env else []
    cands.append(REPO.parent / "reference")
    for c in cands:
        if (c / "src" / "repercep").is_dir():
            return c
    return None


def install_reference_package(reference: Path) -> Path | None:
    """Copy the reference's ``src/repercep`` package and ``kernels/triton_kernels``
    module, unmodified, into baseline/_ref (the ``pip install --target`` layout)."""
    pkg = reference / "src" / "repercep"
    tk = reference / "kernels" / "triton_kernels"
    if not pkg.is_dir():
        return None
    REF_PKG_DIR.mkdir(parents=True, exist_ok=True)
    for src_dir, name in ((pkg, "repercep"), (tk, "triton_kernels")):
        if not src_dir.is_dir():
            continue
        dst = REF_PKG_DIR / name
        if dst.exists():
            shutil.rmtree(dst)
        # plain file copies (no permission bits): the installed tree stays
        # writable, so Python can cache bytecode and a later install can replace it
        shutil.copytree(src_dir, dst, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"),
                        copy_function=shutil.copyfile)
        for d in [dst, *dst.rglob("*")]:
            if d.is_dir():
                d.chmod(0o755)
    return REF_PKG_DIR


def installed_reference_path() -> Path | None:
    """sys.path entry holding the installed reference package, or None."""
    return REF_PKG_DIR if (REF_PKG_DIR / "repercep" / "__init__.py").exists() else None


def build(reference: Path) -> Path | None:
    install_reference_package(reference)
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
    ap.add_argument("--reference", default=None,
                    help="reference source tree (default: $REPERCEP_REFERENCE_ROOT or ../reference)")
    args = ap.parse_args()
    ref = Path(args.reference) if args.reference else reference_root()
    out = build(ref) if ref is not None else None
    print(out if out else "reference source not found; nothing built", file=sys.stderr)


if __name__ == "__main__":
    main()
