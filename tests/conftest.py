"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs everywhere (oracle vs golden fixtures, host logic, the
C-ABI library's exports and argument checks, gloo multi-rank logic);
``-m gpu`` needs a CUDA device and compares the sm_100a kernels, called
through the C ABI, with the CPU oracle.
"""

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "tinyllama.py_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def built_lib():
    """Path of libtinyllama_b200.so, building it first when nvcc is available."""
    import build as tlb_build  # tinyllama.py_b200/build.py

    if not tlb_build.up_to_date():
        try:
            tlb_build.build()
        except Exception as exc:  # no toolkit: use what is there
            if not tlb_build.LIB_PATH.exists():
                pytest.fail(f"library not built and build failed: {exc}")
    return tlb_build.LIB_PATH
