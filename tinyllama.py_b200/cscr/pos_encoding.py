"""cscr.pos_encoding — drop-in for the reference's pybind module of the same name.

``rotary_embedding_neox(postions, query, key, head_size, cos_sin_cache)`` keeps
the reference's signature (including the ``postions`` keyword spelling of
cscr/pos_encoding.cpp:20-25), its checks and messages
(cscr/pos_encoding_kernel.cu:79-104) and its effects: returns the rotated
query as a new tensor and rotates ``key`` in place.

``rotary_embedding_neox_with_cache`` additionally writes the rotated key and
the value into the paged KV cache in the same launch (the reference's RoPE
followed by its KV write, attention.py:151-157).
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import DTYPE_CODE, torch_check

_INDEX_TYPES = (torch.int32, torch.int64)


def _check_rope(postions, query, key, head_size, cos_sin_cache, out):
    torch_check(postions.is_cuda, "positions must be a CUDA tensor")
    torch_check(query.is_cuda, "query must be a CUDA tensor")
    torch_check(key.is_cuda, "key must be a CUDA tensor")
    torch_check(cos_sin_cache.is_cuda, "cos_sin_cache must be a CUDA tensor")
    torch_check(query.is_contiguous(), "query must be contiguous")
    torch_check(key.is_contiguous(), "key must be contiguous")
    torch_check(out.is_contiguous(), "out must be contiguous")
    torch_check(cos_sin_cache.is_contiguous(), "cos_sin_cache must be contiguous")
    torch_check(query.dtype == key.dtype, "query and key must share dtype")
    torch_check(query.dtype == cos_sin_cache.dtype, "query and cos_sin_cache must share dtype")
    torch_check(query.dtype == out.dtype, "query and out must share dtype")
    torch_check(query.dim() == 2, "query must be [num_tokens, num_heads * head_size]")
    torch_check(key.dim() == 2, "key must be [num_tokens, num_kv_heads * head_size]")
    torch_check(postions.dim() == 1, "positions must be [num_tokens]")
    num_tokens = postions.numel()
    torch_check(num_tokens > 0, "positions must contain at least one token")
    torch_check(query.size(0) == num_tokens, "query must have one row per token")
    torch_check(key.size(0) == num_tokens, "key must have one row per token")
    torch_check(head_size > 0, "head_size must be positive")
    torch_check(query.size(1) % head_size == 0, "query size must be divisible by head_size")
    torch_check(key.size(1) % head_size == 0, "key size must be divisible by head_size")
    rot_dim = cos_sin_cache.size(1)
    torch_check(rot_dim > 0 and rot_dim % 2 == 0, "rotary dimension must be even and positive")
    torch_check(rot_dim <= head_size, "rotary dimension must not exceed head_size")
    torch_check(postions.dtype in _INDEX_TYPES, "positions must be int32 or int64")
    torch_check(query.dtype in (torch.float16, torch.bfloat16, torch.float32),
                "dtype must be float16, bfloat16 or float32")
    dev = query.device
    torch_check(key.device == dev and postions.device == dev and cos_sin_cache.device == dev,
                "all tensors must be on the same CUDA device")
    return num_tokens, rot_dim


def rotary_embedding_neox(postions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                          head_size: int, cos_sin_cache: torch.Tensor) -> torch.Tensor:
    """Apply GPT-NeoX style rotary embedding to query (returned) and key (in place)."""
    out = torch.empty_like(query)
    num_tokens, rot_dim = _check_rope(postions, query, key, head_size, cos_sin_cache, out)
    dev = query.device
    with _lib.device_guard(dev):
        rc = _lib.load().tlb_rotary_embedding_neox(
            out.data_ptr(), postions.data_ptr(), DTYPE_CODE[postions.dtype], query.data_ptr(),
            key.data_ptr(), num_tokens, query.size(1) // head_size, key.size(1) // head_size,
            head_size, cos_sin_cache.data_ptr(), cos_sin_cache.size(0), rot_dim,
            query.stride(0), key.stride(0), out.stride(0), DTYPE_CODE[query.dtype],
            _lib.stream_of(dev))
        _lib.check(rc)
    return out


def rotary_embedding_neox_with_cache(postions: torch.Tensor, query: torch.Tensor,
                                     key: torch.Tensor, value: torch.Tensor,
                                     key_cache: torch.Tensor, value_cache: torch.Tensor,
                                     slot_mapping: torch.Tensor | None, head_size: int,
                                     cos_sin_cache: torch.Tensor,
                                     block_tables: torch.Tensor | None = None, *,
                                     overlap_previous: bool = False) -> torch.Tensor:
    """RoPE on query/key plus the KV-cache write of the rotated key and the value.

    query [T, H * head_size], key [T, KVH * head_size] (rotated in place),
    value [T, KVH, head_size] or [T, KVH * head_size], caches
    [num_blocks, KVH, block_size, head_size]. The destination of token t is
    slot_mapping[t] (int32/int64, slot = block * block_size + offset, negative =
    no write) or, when slot_mapping is None, block_tables[t, pos // block_size]
    at offset pos % block_size as src/model_executor/layers/attention.py:96-116
    addresses it (negative block id = no write).

    overlap_previous=True launches the kernel programmatically so that it
    starts while the kernel before it on the stream finishes; until then it
    reads only positions, slots, block tables and the cos/sin table. Use it
    only when that kernel writes none of those (an attention launch or a QKV
    projection).
    """
    out = torch.empty_like(query)
    num_tokens, rot_dim = _check_rope(postions, query, key, head_size, cos_sin_cache, out)
    torch_check(value.is_cuda and key_cache.is_cuda and value_cache.is_cuda,
                "value and caches must be CUDA tensors")
    torch_check(key_cache.dim() == 4 and value_cache.shape == key_cache.shape,
                "key_cache and value_cache must be [num_blocks, num_kv_heads, block_size, head_size]")
    torch_check(key_cache.is_contiguous() and value_cache.is_contiguous(),
                "key_cache and value_cache must be contiguous")
    torch_check(key_cache.dtype == query.dtype and value_cache.dtype == query.dtype
                and value.dtype == query.dtype, "value and caches must share the query dtype")
    num_kv_heads = key.size(1) // head_size
    torch_check(key_cache.size(1) == num_kv_heads and key_cache.size(3) == head_size,
                "cache heads / head_size must match key")
    v2 = value.reshape(num_tokens, -1)
    torch_check(v2.size(1) == num_kv_heads * head_size and v2.stride(1) == 1,
                "value must be [num_tokens, num_kv_heads, head_size] with unit inner stride")
    if slot_mapping is not None:
        torch_check(slot_mapping.is_cuda and slot_mapping.dim() == 1
                    and slot_mapping.numel() == num_tokens
                    and slot_mapping.dtype in _INDEX_TYPES and slot_mapping.is_contiguous(),
                    "slot_mapping must be a contiguous [num_tokens] int32/int64 CUDA tensor")
        slots_ptr, slots_code, bt_ptr, bt_cols = slot_mapping.data_ptr(), \
            DTYPE_CODE[slot_mapping.dtype], None, 0
    else:
        torch_check(block_tables is not None, "either slot_mapping or block_tables is required")
        torch_check(block_tables.is_cuda and block_tables.dim() == 2
                    and block_tables.dtype == torch.int32 and block_tables.is_contiguous()
                    and block_tables.size(0) >= num_tokens,
                    "block_tables must be a contiguous int32 CUDA tensor with a row per token")
        slots_ptr, slots_code, bt_ptr, bt_cols = None, DTYPE_CODE[torch.int64], \
            block_tables.data_ptr(), block_tables.size(1)
    dev = query.device
    with _lib.device_guard(dev):
        rc = _lib.load().tlb_rotary_embedding_neox_with_cache(
            out.data_ptr(), postions.data_ptr(), DTYPE_CODE[postions.dtype], query.data_ptr(),
            key.data_ptr(), v2.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            slots_ptr, slots_code, bt_ptr, bt_cols, num_tokens,
            query.size(1) // head_size, num_kv_heads, head_size, cos_sin_cache.data_ptr(),
            cos_sin_cache.size(0), rot_dim, key_cache.size(0), key_cache.size(2),
            query.stride(0), key.stride(0), v2.stride(0), out.stride(0),
            DTYPE_CODE[query.dtype], 1 if overlap_previous else 0, _lib.stream_of(dev))
        _lib.check(rc)
    return out
