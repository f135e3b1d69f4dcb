"""KV pool sizing and allocation (host logic, CPU)."""

import pytest
import torch

from paged_decode import pool as KP


def test_block_bytes_matches_the_engine_formula():
    # cache_engine.py:110-115: layers * (K + V) * bs * KVH * D * element size
    assert KP.block_bytes(36, 2, 128, 16, torch.bfloat16) == 36 * 2 * 16 * 2 * 128 * 2
    assert KP.block_bytes(1, 2, 64, 8, torch.float32) == 2 * 8 * 2 * 64 * 4


def test_long_tail_pool_of_150_gb():
    # Qwen2.5-3B-shaped cache, block_size 32, bf16: 32 KB of K+V per block and layer
    n = KP.blocks_for_budget(150 * 10**9, 1, 2, 128, 32, torch.bfloat16)
    assert KP.block_bytes(1, 2, 128, 32, torch.bfloat16) == 32 * 1024
    assert n == 150 * 10**9 // (32 * 1024)
    assert 4_500_000 < n < 4_600_000


def test_allocation_layout_is_what_the_ops_read():
    caches = KP.allocate_kv_cache(3, 10, 2, 64, 16, torch.float16, device="cpu")
    assert len(caches) == 3
    for k, v in caches:
        assert k.shape == v.shape == (10, 2, 16, 64)
        assert k.is_contiguous() and v.is_contiguous() and k.dtype == torch.float16


def test_empty_pool_is_refused_like_the_engine():
    with pytest.raises(ValueError, match="No KV cache blocks"):
        KP.allocate_kv_cache(1, 0, 2, 64, 16, torch.float16, device="cpu")
    with pytest.raises(ValueError):
        KP.blocks_for_budget(-1, 1, 2, 64, 16, torch.float16)
