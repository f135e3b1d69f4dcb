"""cscr.cache — drop-in for the reference's pybind module of the same name.

* ``swap_blocks(src, dst, block_mapping)`` and ``copy_blocks(key_caches,
  value_caches, block_mapping)`` keep the signatures, checks and messages of
  cscr/cache.cpp:94-151 (bound at :153-162). ``copy_blocks`` issues one launch
  for all layers and passes the block pairs in the kernel parameters, so it
  neither allocates nor waits on a host-to-device upload.
* ``reshape_and_cache(key, value, key_cache, value_cache, slot_mapping)`` is
  the KV-cache write the reference performs with torch indexing in
  src/model_executor/layers/attention.py:96-116, as one kernel addressed by a
  slot mapping (slot = block * block_size + offset; negative slots skipped).
* ``write_kv_cache(key, value, positions, key_cache, value_cache,
  block_tables)`` is that write addressed exactly as the reference addresses
  it (block_tables[row, position // block_size]), without its host sync.
"""

from __future__ import annotations

import ctypes
import itertools

import numpy as np

import torch

from . import _lib
from ._lib import DTYPE_CODE, torch_check

_INDEX_TYPES = (torch.int32, torch.int64)


def _block_bytes(cache: torch.Tensor) -> int:
    torch_check(cache.dim() >= 1, "cache tensors must have at least one dimension")
    torch_check(cache.size(0) > 0, "cache tensors must contain at least one block")
    return cache.element_size() * (cache.numel() // cache.size(0))


def _pairs_array(pairs):
    """(src, dst) pairs as a ctypes int64 array (kept alive by the caller)."""
    n = len(pairs)
    arr = np.ascontiguousarray(np.asarray(pairs, dtype=np.int64).reshape(-1)) if n else \
        np.zeros(2, np.int64)
    return arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), n, arr


def _check_mapping_range(block_mapping, nb: int, lo: int, hi: int) -> None:
    """The reference's per-index range checks (cache.cpp:35-45), in its order;
    the loop (and its message formatting) only runs when an index is out of
    range."""
    if lo >= 0 and hi < nb:
        return
    for s, dsts in block_mapping.items():
        torch_check(0 <= int(s) < nb, f"src block index {int(s)} is out of range [0, {nb})")
        for d in dsts:
            torch_check(0 <= int(d) < nb, f"dst block index {int(d)} is out of range [0, {nb})")


def swap_blocks(src: torch.Tensor, dst: torch.Tensor, block_mapping: dict[int, int]) -> None:
    """Copy KV cache blocks src[s] -> dst[d] for every (s, d) of block_mapping."""
    src_cuda, dst_cuda = src.is_cuda, dst.is_cuda
    torch_check(src_cuda or src.device.type == "cpu", "src must be a CPU or CUDA tensor")
    torch_check(dst_cuda or dst.device.type == "cpu", "dst must be a CPU or CUDA tensor")
    torch_check(not (src_cuda and dst_cuda) or src.device.index == dst.device.index,
                "src and dst must be on the same GPU")
    torch_check(src.is_contiguous(), "src must be contiguous")
    torch_check(dst.is_contiguous(), "dst must be contiguous")
    torch_check(src.element_size() == dst.element_size(),
                "src and dst must have the same element size")
    if not block_mapping:
        return
    torch_check(_block_bytes(src) == _block_bytes(dst), "src and dst blocks must have the same size")
    ns, nd = src.size(0), dst.size(0)
    pairs = []
    for s, d in block_mapping.items():
        s, d = int(s), int(d)
        torch_check(0 <= s < ns, f"src block index {s} is out of range [0, {ns})")
        torch_check(0 <= d < nd, f"dst block index {d} is out of range [0, {nd})")
        pairs.append((s, d))
    arr, n, _keep = _pairs_array(pairs)
    lib = _lib.load()
    if not src_cuda and not dst_cuda:
        _lib.check(lib.tlb_swap_blocks(src.data_ptr(), 0, dst.data_ptr(), 0, arr, n,
                                       _block_bytes(src), None))
        return
    dev = src.device if src_cuda else dst.device
    with _lib.device_guard(dev):
        _lib.check(lib.tlb_swap_blocks(src.data_ptr(), int(src_cuda), dst.data_ptr(),
                                       int(dst_cuda), arr, n, _block_bytes(src),
                                       _lib.stream_of(dev)))


def copy_blocks(key_caches: list[torch.Tensor], value_caches: list[torch.Tensor],
                block_mapping: dict[int, list[int]]) -> None:
    """In-place block copies src -> each dst, in every layer's key and value cache."""
    torch_check(len(key_caches) == len(value_caches),
                "key_caches and value_caches must have the same number of layers")
    if not key_caches or not block_mapping:
        return
    device = key_caches[0].device
    dev_index = key_caches[0].get_device()
    pairs = [(int(s), int(d)) for s, dsts in block_mapping.items() for d in dsts]
    idx = [int(s) for s in block_mapping] + [d for _, d in pairs]
    lo, hi = min(idx), max(idx)
    # One pass over the caches: the reference's per-cache checks in its order
    # (cache.cpp:48-105), then the cache's pointer into the group of its block
    # size (one launch per distinct block size; key and value caches normally
    # agree). A list of 72 caches costs ~1 us of Python per cache, so each
    # tensor attribute is read once.
    groups: dict[int, list[int]] = {}
    for cache in itertools.chain(key_caches, value_caches):
        torch_check(cache.is_cuda, "cache tensors must be CUDA tensors")
        torch_check(cache.get_device() == dev_index, "all cache tensors must be on the same GPU")
        shape = cache.shape
        torch_check(len(shape) >= 1, "cache tensors must have at least one dimension")
        nb = shape[0]
        torch_check(nb > 0, "cache tensors must contain at least one block")
        torch_check(cache.is_contiguous(), "cache tensors must be contiguous")
        _check_mapping_range(block_mapping, nb, lo, hi)
        groups.setdefault(cache.element_size() * (cache.numel() // nb), []).append(
            cache.data_ptr())
    if not pairs:
        return
    arr, n, _keep = _pairs_array(pairs)
    lib = _lib.load()
    with _lib.device_guard(device):
        stream = _lib.stream_of(device)
        for block_bytes, ptrs in groups.items():
            parr = (ctypes.c_void_p * len(ptrs))(*ptrs)
            _lib.check(lib.tlb_copy_blocks(parr, len(ptrs), arr, n, block_bytes, stream))


def _check_cache_pair(key_cache, value_cache, dtype):
    torch_check(key_cache.is_cuda and value_cache.is_cuda, "cache tensors must be CUDA tensors")
    torch_check(key_cache.dim() == 4,
                "key_cache must be [num_blocks, num_kv_heads, block_size, head_size]")
    torch_check(value_cache.shape == key_cache.shape,
                "value_cache must have the same shape as key_cache")
    torch_check(key_cache.is_contiguous() and value_cache.is_contiguous(),
                "cache tensors must be contiguous")
    torch_check(key_cache.dtype == value_cache.dtype,
                "key_cache and value_cache must share the same dtype")


def _rows(x: torch.Tensor, num_tokens: int, width: int, dtype: torch.dtype) -> torch.Tensor:
    """[T, KVH, D] or [T, KVH * D] view with unit inner stride, in the cache dtype."""
    if x.dtype != dtype:
        x = x.to(dtype)  # the reference casts the same way (attention.py:110-113)
    x2 = x.reshape(num_tokens, width)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    return x2


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor,
                      value_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Scatter key/value rows [T, KVH, D] into the paged caches at slot_mapping."""
    _check_cache_pair(key_cache, value_cache, key.dtype)
    torch_check(key.is_cuda and value.is_cuda and slot_mapping.is_cuda,
                "key, value and slot_mapping must be CUDA tensors")
    torch_check(slot_mapping.dim() == 1 and slot_mapping.dtype in _INDEX_TYPES,
                "slot_mapping must be a [num_tokens] int32 or int64 tensor")
    num_blocks, kvh, block_size, head_size = key_cache.shape
    T = slot_mapping.numel()
    width = kvh * head_size
    torch_check(key.numel() == T * width and value.numel() == T * width,
                "key and value must be [num_tokens, num_kv_heads, head_size]")
    if T == 0:
        return
    k2 = _rows(key, T, width, key_cache.dtype)
    v2 = _rows(value, T, width, key_cache.dtype)
    slots = slot_mapping.contiguous()
    dev = key_cache.device
    with _lib.device_guard(dev):
        _lib.check(_lib.load().tlb_reshape_and_cache(
            k2.data_ptr(), v2.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            slots.data_ptr(), DTYPE_CODE[slots.dtype], T, kvh, head_size, num_blocks, block_size,
            k2.stride(0), v2.stride(0), DTYPE_CODE[key_cache.dtype], _lib.stream_of(dev)))


def write_kv_cache(key: torch.Tensor, value: torch.Tensor, positions: torch.Tensor,
                   key_cache: torch.Tensor, value_cache: torch.Tensor,
                   block_tables: torch.Tensor) -> None:
    """KV write of attention.py:82-116: row r -> block_tables[r, pos // bs], pos % bs."""
    _check_cache_pair(key_cache, value_cache, key.dtype)
    torch_check(key.is_cuda and value.is_cuda and positions.is_cuda and block_tables.is_cuda,
                "key, value, positions and block_tables must be CUDA tensors")
    torch_check(positions.dtype in _INDEX_TYPES, "positions must be int32 or int64")
    torch_check(block_tables.dim() == 2, "block_tables must be [num_seqs, max_blocks_per_seq]")
    num_blocks, kvh, block_size, head_size = key_cache.shape
    T = positions.numel()
    torch_check(block_tables.size(0) >= T, "block_tables must have one row per token")
    width = kvh * head_size
    torch_check(key.numel() == T * width and value.numel() == T * width,
                "key and value must be [num_tokens, num_kv_heads, head_size]")
    if T == 0:
        return
    k2 = _rows(key, T, width, key_cache.dtype)
    v2 = _rows(value, T, width, key_cache.dtype)
    pos = positions.contiguous()
    bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    bt = bt.contiguous()
    dev = key_cache.device
    with _lib.device_guard(dev):
        _lib.check(_lib.load().tlb_write_kv_cache(
            k2.data_ptr(), v2.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            pos.data_ptr(), DTYPE_CODE[pos.dtype], bt.data_ptr(), bt.size(1), T, kvh, head_size,
            num_blocks, block_size, k2.stride(0), v2.stride(0), DTYPE_CODE[key_cache.dtype],
            _lib.stream_of(dev)))
