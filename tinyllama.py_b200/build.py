"""Build libtinyllama_b200.so, the C-ABI library of the sm_100a decode kernels.

Every ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) as relocatable device code, then
linked into one shared library next to the ``cscr`` package, where the op
modules load it. The library lives in-tree, so a copy of the repository
carries it as built.

Usage: ``python tinyllama.py_b200/build.py [--force] [--verbose]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = PKG_ROOT.parent / "include"
BUILD_DIR = PKG_ROOT.parent / "_build"
LIB_PATH = PKG_ROOT / "cscr" / "libtinyllama_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "--use_fast_math",
    "-std=c++17",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(
        INCLUDE.glob("*.h")
    )


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _deps())


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-dc", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the kernels and link the shared library; returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    workers = min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
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
