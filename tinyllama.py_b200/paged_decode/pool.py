"""KV pool allocation in the layout the decode ops read.

The reference engine (src/core/cache_engine.py:55-108) allocates per layer a
key cache in an x-packed layout ``[NB, KVH, D/x, bs, x]`` and a value cache
``[NB, KVH, D, bs]``, which its own attention kernel cannot read
(cscr/attention.h:10-11 and tests/test_paged_attention.py index
``[NB, KVH, bs, D]``). Here both caches of every layer are
``[num_blocks, num_kv_heads, block_size, head_size]`` — the layout
``cscr.attention.paged_attention``, ``cscr.cache`` and the RoPE + cache-write
op use — and the pool is sized per GPU from a byte budget or from the free
device memory, the way ``CacheEngine.calculate_cache_block_size``
(cache_engine.py:110-115) sizes blocks.
"""

from __future__ import annotations

import torch

KVCache = tuple[torch.Tensor, torch.Tensor]


def block_bytes(num_layers: int, num_kv_heads: int, head_size: int, block_size: int,
                dtype: torch.dtype) -> int:
    """Bytes one block number costs across all layers, K and V
    (cache_engine.py:110-115)."""
    per_cache = block_size * num_kv_heads * head_size
    return num_layers * 2 * per_cache * torch.tensor([], dtype=dtype).element_size()


def blocks_for_budget(budget_bytes: int, num_layers: int, num_kv_heads: int, head_size: int,
                      block_size: int, dtype: torch.dtype) -> int:
    """Largest block count whose pool fits in ``budget_bytes``."""
    if budget_bytes < 0:
        raise ValueError("budget_bytes must not be negative")
    return budget_bytes // block_bytes(num_layers, num_kv_heads, head_size, block_size, dtype)


def blocks_for_free_memory(fraction: float, num_layers: int, num_kv_heads: int,
                           head_size: int, block_size: int, dtype: torch.dtype,
                           device: torch.device | int | None = None) -> int:
    """Block count that takes ``fraction`` of the device's currently free
    memory (the reference profiles free memory before sizing its pool)."""
    if not 0.0 < fraction <= 1.0:
        raise ValueError("fraction must be in (0, 1]")
    free, _ = torch.cuda.mem_get_info(device)
    return blocks_for_budget(int(free * fraction), num_layers, num_kv_heads, head_size,
                             block_size, dtype)


def allocate_kv_cache(num_layers: int, num_blocks: int, num_kv_heads: int, head_size: int,
                      block_size: int, dtype: torch.dtype,
                      device: torch.device | str = "cuda") -> list[KVCache]:
    """One ``(key_cache, value_cache)`` pair per layer, both
    ``[num_blocks, num_kv_heads, block_size, head_size]``, uninitialised
    (cache_engine.py:55-82 allocates with ``torch.empty`` as well)."""
    if num_blocks <= 0:
        raise ValueError(
            "No KV cache blocks allocated. Profile the available memory before creating "
            "the cache.")
    shape = (num_blocks, num_kv_heads, block_size, head_size)
    return [(torch.empty(shape, dtype=dtype, device=device),
             torch.empty(shape, dtype=dtype, device=device)) for _ in range(num_layers)]
