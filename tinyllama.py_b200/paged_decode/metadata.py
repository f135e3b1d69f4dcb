"""Decode-step and packed-step metadata built on the device.

The reference's worker (src/worker/worker.py:84-169) walks Python lists every
step to form positions, slot mappings and context lengths, then discards all
but the positions (:166-169). Here the block tables and context lengths the
block manager hands out are packed once into a pinned host buffer, moved with
one host-to-device copy, and the positions and slot mapping are derived on
the GPU by ``tlb_decode_metadata`` (position = context_len - 1,
slot = block_table[position // block_size] * block_size + position %
block_size, as worker.py:144-159).

``step_metadata`` does the same for a continuous-batching step that also
carries prompts (worker.py:95-124): the prompts' tokens first, then one token
per decode sequence, positions padded with 0 to a multiple of 8 (:163-164),
from one host-to-device copy and one launch (``tlb_step_metadata``).
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


@dataclass
class StepMetadata:
    positions: torch.Tensor      # [padded] int64 (0 past num_tokens)
    slot_mapping: torch.Tensor   # [padded] int64 (-1 past num_tokens)
    num_tokens: int              # sum(prompt_lens) + num_decode
    prompt_lens: torch.Tensor    # [P] int32
    prompt_tables: torch.Tensor  # [P, maxBp] int32
    context_lens: torch.Tensor   # [S] int32
    block_tables: torch.Tensor   # [S, maxB] int32 (decode sequences)


def _table_array(rows: list[list[int]], pad: int = -1) -> np.ndarray:
    out = np.full((len(rows), max([1] + [len(r) for r in rows])), pad, np.int32)
    for r, row in enumerate(rows):
        out[r, : len(row)] = row
    return out


def step_metadata(prompt_tables: list[list[int]], prompt_lens: list[int],
                  decode_tables: list[list[int]], context_lens: list[int], block_size: int,
                  device: torch.device | str = "cuda", alignment: int = 8) -> StepMetadata:
    """Device metadata of one packed step from the block manager's lists.

    The four int32 arrays go to the device in one pinned host-to-device copy;
    positions and the slot mapping are derived there by one launch.
    """
    dev = torch.device(device)
    P, S = len(prompt_lens), len(context_lens)
    _lib.torch_check(len(prompt_tables) == P and len(decode_tables) == S,
                     "one block table per prompt and per decode sequence")
    pt = _table_array(prompt_tables)
    dt = _table_array(decode_tables)
    parts = [np.asarray(prompt_lens, np.int32).ravel(), pt.ravel(),
             np.asarray(context_lens, np.int32).ravel(), dt.ravel()]
    host = torch.from_numpy(np.concatenate(parts)).pin_memory()
    on_dev = host.to(dev, non_blocking=True)
    views, off = [], 0
    for a in parts:
        views.append(on_dev[off:off + a.size])
        off += a.size
    plens, ptab = views[0], views[1].view(pt.shape)
    clens, dtab = views[2], views[3].view(dt.shape)
    T = int(sum(max(int(L), 0) for L in prompt_lens)) + S
    padded = -(-T // alignment) * alignment
    positions = torch.empty(padded, dtype=torch.int64, device=dev)
    slots = torch.empty(padded, dtype=torch.int64, device=dev)
    with _lib.device_guard(dev):
        _lib.check(_lib.load().tlb_step_metadata(
            plens.data_ptr() if P else None, ptab.data_ptr() if P else None, P, pt.shape[1],
            clens.data_ptr() if S else None, dtab.data_ptr() if S else None, S, dt.shape[1],
            block_size, T, alignment, positions.data_ptr() if padded else None,
            slots.data_ptr() if padded else None, _lib.stream_of(dev)))
    return StepMetadata(positions, slots, T, plens, ptab, clens, dtab)
