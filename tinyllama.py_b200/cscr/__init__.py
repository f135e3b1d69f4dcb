"""cscr — B200 (sm_100a) drop-in for tinyllama.py's native op modules.

The reference ships three pybind11 extensions, ``cscr.attention``,
``cscr.cache`` and ``cscr.pos_encoding`` (setup.py:4-41). This package
provides the same module names, functions, keyword names and error messages,
backed by libtinyllama_b200.so, so ``from cscr import attention as _C`` in
src/model_executor/layers/attention.py:4-5 and ``from cscr import cache`` in
src/core/cache_engine.py:7 resolve here unchanged. Importing the package does
not load the CUDA library; the first op call does.
"""

__all__ = ["attention", "cache", "pos_encoding"]
