"""The C-ABI library without a GPU: it loads, exports every symbol the header
declares, and rejects bad arguments with the reference's messages before any
CUDA call. The cscr op modules raise the reference's errors on CPU tensors."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import REPO

HEADER = REPO / "include" / "tinyllama_b200.h"


def header_symbols():
    text = HEADER.read_text()
    return re.findall(r"TLB_API\s+[\w\s\*]+?\b(tlb_\w+)\s*\(", text)


def test_header_declares_expected_entry_points():
    syms = header_symbols()
    for name in ("tlb_paged_attention", "tlb_rotary_embedding_neox", "tlb_reshape_and_cache",
                 "tlb_write_kv_cache", "tlb_rotary_embedding_neox_with_cache", "tlb_copy_blocks",
                 "tlb_swap_blocks", "tlb_decode_metadata", "tlb_last_error"):
        assert name in syms


def test_library_exports_every_declared_symbol(built_lib):
    lib = ctypes.CDLL(str(built_lib))
    for name in header_symbols():
        assert hasattr(lib, name), name


def test_binding_covers_header(built_lib):
    from cscr import _lib

    assert set(header_symbols()) == set(_lib.EXPORTS)
    _lib.load()
    assert b"sm_100a" in _lib.load().tlb_version()


def test_argument_errors_without_gpu(built_lib):
    from cscr import _lib

    lib = _lib.load()
    rc = lib.tlb_paged_attention(1, 1, 1, 1, 1, 1, 0, 16, 2, 128, 10, 16, 4, 1.0, 2, None, 0, 0, None)
    assert rc == 1 and "at least one sequence" in _lib.last_error()
    rc = lib.tlb_paged_attention(1, 1, 1, 1, 1, 1, 4, 15, 2, 128, 10, 16, 4, 1.0, 2, None, 0, 0, None)
    assert rc == 1 and "divisible" in _lib.last_error()
    rc = lib.tlb_paged_attention(1, 1, 1, 1, 1, 1, 4, 16, 2, 2048, 10, 16, 4, 1.0, 2, None, 0, 0, None)
    assert rc == 1 and "head_dim too large" in _lib.last_error()
    rc = lib.tlb_paged_attention(1, 1, 1, 1, 1, 1, 4, 16, 2, 128, 10, 16, 4, 1.0, 7, None, 0, 0, None)
    assert rc == 1 and "dtype" in _lib.last_error()
    rc = lib.tlb_rotary_embedding_neox(1, 1, 4, 1, 1, 4, 2, 1, 64, 1, 10, 63, 128, 64, 128, 2, None)
    assert rc == 1 and "even" in _lib.last_error()
    rc = lib.tlb_rotary_embedding_neox(1, 1, 4, 1, 1, 4, 2, 1, 64, 1, 10, 128, 128, 64, 128, 2, None)
    assert rc == 1 and "must not exceed head_size" in _lib.last_error()
    rc = lib.tlb_rotary_embedding_neox(1, 1, 9, 1, 1, 4, 2, 1, 64, 1, 10, 64, 128, 64, 128, 2, None)
    assert rc == 1 and "int32 or int64" in _lib.last_error()
    size = ctypes.c_size_t()
    assert lib.tlb_paged_attention_workspace_zeroed_bytes(64, 2, ctypes.byref(size)) == 0
    assert size.value >= 64 * 2 * 4


def test_no_alloc_checks_arguments_before_touching_its_scratch(built_lib):
    """The allocation-free entry point runs every argument check of the
    workspace entry point before it clears or uses its static array: a bad
    call (here a null output, with far more sequences than the array could
    serve, fp32 and bf16) is refused with no CUDA call at all, so it also
    fails cleanly on a host without a GPU."""
    from cscr import _lib

    lib = _lib.load()
    for dtype in (0, 2):
        rc = lib.tlb_paged_attention_no_alloc(None, 256, 256, 256, 256, 256, 5_000_000, 16, 2,
                                              128, 10, 16, 4, 0.1, dtype, 0, None)
        assert rc == 1 and "must not be null" in _lib.last_error()
    rc = lib.tlb_paged_attention_no_alloc(256, 256, 256, 256, 256, 256, 4, 16, 2, 128, 10, 16, 4,
                                          0.1, 2, 0x80, None)
    assert rc == 1 and "unknown flags" in _lib.last_error()


def test_reference_messages_on_cpu_tensors():
    from cscr import attention as A
    from cscr import pos_encoding as PE
    from cscr import cache as C

    q = torch.zeros(1, 2, 64)
    kc = torch.zeros(1, 2, 8, 64)
    with pytest.raises(RuntimeError, match="^query must be a CUDA tensor$"):
        A.paged_attention(q, kc, kc, torch.zeros(1, 1, dtype=torch.int32),
                          torch.ones(1, dtype=torch.int32), 0.125)
    with pytest.raises(RuntimeError, match="^positions must be a CUDA tensor$"):
        PE.rotary_embedding_neox(torch.zeros(1, dtype=torch.int64), q.view(1, -1),
                                 q.view(1, -1).clone(), 64, torch.zeros(4, 64))
    with pytest.raises(RuntimeError, match="^src and dst must have the same element size$"):
        C.swap_blocks(torch.zeros(2, 4), torch.zeros(2, 4, dtype=torch.float16), {0: 1})
    with pytest.raises(RuntimeError, match=r"^dst block index 5 is out of range \[0, 2\)$"):
        C.swap_blocks(torch.zeros(2, 4), torch.zeros(2, 4), {0: 5})


def test_swap_blocks_host_to_host_runs_on_cpu(built_lib):
    """CPU<->CPU swaps are memcpys in the reference too (cache_kernel.cu:144-152)."""
    from cscr import cache as C
    from oracle import decode_oracle as O

    src = torch.arange(6 * 32, dtype=torch.float32).view(6, 2, 16)
    dst = torch.zeros(8, 2, 16)
    mapping = {0: 7, 5: 0, 2: 3}
    ref = dst.numpy().copy()
    O.swap_blocks(src.numpy(), ref, mapping)
    C.swap_blocks(src, dst, mapping)
    assert np.array_equal(dst.numpy(), ref)


def test_build_flags_target_sm100a_only():
    import build as B

    assert B.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert "-lineinfo" in B.NVCC_FLAGS


def test_fused_step_argument_errors_without_gpu(built_lib):
    """tlb_paged_attention_with_rope rejects bad arguments, and shapes the
    fused kernel does not serve, before any CUDA call."""
    from cscr import _lib

    lib = _lib.load()
    p = 1 << 12  # stands in for 16-byte aligned device pointers; nothing is dereferenced

    def call(num_seqs=4, head_dim=128, dtype=2, cache_rows=4096, key_stride=256):
        return lib.tlb_paged_attention_with_rope(
            p, p, p, p, p, p, p, p, p, cache_rows, num_seqs, 16, 2, head_dim, 10, 16, 4,
            key_stride, 256, 0.125, dtype, None, 0, 0, None)

    assert call(num_seqs=0) == 1 and "at least one sequence" in _lib.last_error()
    assert call(cache_rows=0) == 1 and "at least one row" in _lib.last_error()
    assert call(key_stride=100) == 1
    # fp32 and head dim 96 are served by the two-launch form, which the op falls back to
    assert call(dtype=0) == _lib.TLB_ERR_UNSUPPORTED and "tensor-core path" in _lib.last_error()
    assert call(head_dim=96, key_stride=192) == _lib.TLB_ERR_UNSUPPORTED
