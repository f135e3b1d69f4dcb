"""Build the reference's own CUDA ops into ``oracle/_ref/`` — TEST INFRASTRUCTURE ONLY.

The reference (CodeClaper/tinyllama.py) ships three pybind11 torch extensions,
``cscr.attention``, ``cscr.cache`` and ``cscr.pos_encoding`` (setup.py:4-41),
compiled with ``-O3`` for the host and ``-O3 --use_fast_math`` for nvcc. This
recipe compiles those same source files, unchanged and where they lie in the
reference tree, with the same flags for sm_100a (``TORCH_CUDA_ARCH_LIST=10.0a``)
through torch's extension builder. It does not run the reference's setup.py.

Each module gets a name of its own (``tlref_attention``, ``tlref_cache``,
``tlref_pos_encoding``: the sources take the module name from
``TORCH_EXTENSION_NAME``), so loading one can never shadow the product
``cscr`` package. Outputs go to ``oracle/_ref/`` only, which git ignores; the
built ``.so`` files travel with a copy of the repository to a GPU host, where
the parity tests load them by file path (``load_ref_module``).

Only the test suite uses these modules, as a second checker of the product
kernels (the reference's own RoPE and paged-attention kernels run on the same
inputs). Nothing on the product path loads them.

Usage: ``python oracle/build_ref.py [--reference DIR] [--force]``.
"""

from __future__ import annotations

import argparse
import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
DEFAULT_REFERENCE = Path("/root/reference")

# (module name here, reference sources under cscr/) — setup.py:5-39.
MODULES = {
    "tlref_attention": ("attention.cpp", "attention_kernel.cu"),
    "tlref_cache": ("cache.cpp", "cache_kernel.cu"),
    "tlref_pos_encoding": ("pos_encoding.cpp", "pos_encoding_kernel.cu"),
}
# setup.py:11-14 (the same for all three extensions) plus the target.
CXX_FLAGS = ["-O3"]
NVCC_FLAGS = ["-O3", "--use_fast_math"]
ARCH_LIST = "10.0a"


def so_path(name: str) -> Path:
    return OUT / f"{name}.so"


def built() -> bool:
    return all(so_path(n).exists() for n in MODULES)


def _up_to_date(name: str, srcs: list[Path]) -> bool:
    so = so_path(name)
    return so.exists() and all(s.stat().st_mtime <= so.stat().st_mtime for s in srcs)


def build(reference: Path = DEFAULT_REFERENCE, force: bool = False, verbose: bool = False) -> bool:
    """Compile the three reference modules; False when the reference tree is absent."""
    cscr = Path(reference) / "cscr"
    if not cscr.is_dir():
        return False
    os.environ["TORCH_CUDA_ARCH_LIST"] = ARCH_LIST
    from torch.utils import cpp_extension

    OUT.mkdir(parents=True, exist_ok=True)
    for name, files in MODULES.items():
        srcs = [cscr / f for f in files]
        if not force and _up_to_date(name, srcs):
            continue
        bdir = OUT / f"build_{name}"
        bdir.mkdir(parents=True, exist_ok=True)
        cpp_extension.load(
            name=name,
            sources=[str(s) for s in srcs],
            extra_cflags=CXX_FLAGS,
            extra_cuda_cflags=NVCC_FLAGS,
            extra_include_paths=[str(cscr)],
            build_directory=str(bdir),
            verbose=verbose,
            is_python_module=True,
        )
        os.replace(bdir / f"{name}.so", so_path(name))
    return True


def load_ref_module(name: str):
    """Import one built reference module from ``oracle/_ref/`` by file path.

    ``name`` is one of ``tlref_attention``, ``tlref_cache``,
    ``tlref_pos_encoding``. torch must be imported first (the modules link
    against the torch libraries already loaded in the process).
    """
    import torch  # noqa: F401  (loads libtorch / libc10 into the process)

    path = so_path(name)
    if not path.exists():
        raise FileNotFoundError(f"{path} not built (run oracle/build_ref.py where the "
                                "reference sources are present)")
    if name in sys.modules:
        return sys.modules[name]
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_file_location(name, str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    ok = build(args.reference, force=args.force, verbose=args.verbose)
    print("built" if ok else f"reference sources not found under {args.reference}",
          *(str(so_path(n)) for n in MODULES if so_path(n).exists()), sep="\n")


if __name__ == "__main__":
    main()
