"""Build the sm_100a shared library ``libchol_b200.so`` in-tree with nvcc.

The reference JIT-compiles its CUDA strings with ``torch.utils.cpp_extension.load_inline``
per shape (cholesky/cholesky.py:79-111). Here one C-ABI library is built ahead of time
from ``csrc/*.cu`` so that it ships with the source tree and needs no compiler at run time.

Usage: ``python -m linalg_kernels_b200.build [--force] [--verbose]``.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_NAME = "libchol_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME
STAMP = PKG_DIR / ".libchol_b200.hash"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin directory on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _digest() -> str:
    h = hashlib.sha256()
    files = (sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.c"))
             + sorted(INCLUDE.glob("*.h")))
    for f in files:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every csrc/*.cu into LIB_PATH unless it is up to date."""
    digest = _digest()
    if (not force and LIB_PATH.exists() and STAMP.exists()
            and STAMP.read_text().strip() == digest):
        return LIB_PATH
    nvcc = _nvcc()
    objdir = PKG_DIR / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src),
               "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    _build_pyext(verbose)
    STAMP.write_text(digest + "\n")
    return LIB_PATH


def _build_pyext(verbose: bool) -> Path:
    """gcc the CPython fast-call binding (csrc/chol_pyext.c) against libchol_b200.so."""
    import sysconfig

    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = PKG_DIR / ("_cholpy" + suffix)
    tmp = out.with_name(out.name + ".tmp")
    cmd = ["gcc", "-O2", "-shared", "-fPIC", "-I", sysconfig.get_paths()["include"],
           "-I", str(INCLUDE), str(CSRC / "chol_pyext.c"), "-o", str(tmp),
           "-L", str(PKG_DIR), "-lchol_b200", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true",
                    help="print per-kernel registers / spills / shared memory")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
