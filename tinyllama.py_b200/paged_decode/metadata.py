"""Decode-step metadata built on the device.

The reference's worker (src/worker/worker.py:84-169) walks Python lists every
step to form positions, slot mappings and context lengths, then discards all
but the positions (:166-169). Here the block tables and context lengths the
block manager hands out are packed once into a pinned host buffer, moved with
one host-to-device copy, and the positions and slot mapping are derived on
the GPU by ``tlb_decode_metadata`` (position = context_len - 1,
slot = block_table[position // block_size] * block_size + position %
block_size, as worker.py:144-159).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from cscr import _lib


@dataclass
class DecodeMetadata:
    block_tables: torch.Tensor   # [S, max_blocks] int32
    context_lens: torch.Tensor   # [S] int32
    positions: torch.Tensor      # [S] int64
    slot_mapping: torch.Tensor   # [S] int64


def pack_block_tables(block_tables: list[list[int]], context_lens: list[int],
                      pad: int = 0) -> np.ndarray:
    """[S, 1 + max_blocks] int32 host array: context length, then the table row."""
    S = len(block_tables)
    width = max([1] + [len(t) for t in block_tables])
    buf = np.full((S, 1 + width), pad, np.int32)
    for r, (row, L) in enumerate(zip(block_tables, context_lens)):
        buf[r, 0] = L
        buf[r, 1:1 + len(row)] = row
    return buf


def decode_metadata(block_tables: list[list[int]], context_lens: list[int], block_size: int,
                    device: torch.device | str = "cuda") -> DecodeMetadata:
    """Device tensors for one decode step from the block manager's lists."""
    dev = torch.device(device)
    packed = torch.from_numpy(pack_block_tables(block_tables, context_lens)).pin_memory()
    S = packed.shape[0]
    on_dev = packed.to(dev, non_blocking=True)
    lens = on_dev[:, 0].contiguous()
    tables = on_dev[:, 1:].contiguous()
    positions = torch.empty(S, dtype=torch.int64, device=dev)
    slots = torch.empty(S, dtype=torch.int64, device=dev)
    if S:
        with _lib.device_guard(dev):
            _lib.check(_lib.load().tlb_decode_metadata(
                lens.data_ptr(), tables.data_ptr(), S, tables.size(1), block_size,
                positions.data_ptr(), slots.data_ptr(), _lib.stream_of(dev)))
    return DecodeMetadata(tables, lens, positions, slots)


def decode_metadata_from_tensors(context_lens: torch.Tensor, block_tables: torch.Tensor,
                                 block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """positions, slot_mapping for device-resident context_lens / block_tables."""
    _lib.torch_check(context_lens.is_cuda and block_tables.is_cuda,
                     "context_lens and block_tables must be CUDA tensors")
    _lib.torch_check(context_lens.dtype == torch.int32 and block_tables.dtype == torch.int32,
                     "context_lens and block_tables must be int32")
    lens = context_lens.contiguous()
    tables = block_tables.contiguous()
    S = lens.numel()
    dev = lens.device
    positions = torch.empty(S, dtype=torch.int64, device=dev)
    slots = torch.empty(S, dtype=torch.int64, device=dev)
    if S:
        with _lib.device_guard(dev):
            _lib.check(_lib.load().tlb_decode_metadata(
                lens.data_ptr(), tables.data_ptr(), S, tables.size(1), block_size,
                positions.data_ptr(), slots.data_ptr(), _lib.stream_of(dev)))
    return positions, slots
