"""Layer glue of the decode step on the sm_100a ops.

``PagedAttention`` and ``PagedAttentionWithRoPE`` keep the constructors,
buffers and forward signatures of src/model_executor/layers/attention.py:7-166,
so a model built against the reference's layers runs on these unchanged.
The forward of ``PagedAttentionWithRoPE`` does the reference's three steps —
RoPE (:151-153), the KV-cache write (:155-157) and paged attention (:160-166) —
in two launches: one fused RoPE + cache-write kernel addressed through the
block tables exactly as ``_write_kv_cache`` addresses it, then the attention
kernel. Unlike the reference it does not synchronise the host (the
``valid.any()`` of :103) and converts the cos/sin table once per device and
dtype instead of on every call (:148-150).

``positions=None`` states the decode invariant the reference's worker builds
(src/worker/worker.py:144-146,154: a decode token sits at position
``context_len - 1`` and ``seq_lens`` holds the context lengths), so the
position of every token is ``seq_lens - 1``; with full-width rotary
(``rotary_dim == head_size``) the whole step then runs as ONE launch
(``cscr.attention.paged_attention_with_rope``).
"""

from __future__ import annotations

import torch
from torch import nn

from cscr import attention as _C
from cscr import cache as _Cache
from cscr import pos_encoding as _PE


class PagedAttention(nn.Module):
    def __init__(self, num_heads: int, head_size: int, scale: float):
        super().__init__()
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = scale

    def forward(self, query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                block_tables: torch.Tensor, seq_lens: torch.Tensor) -> torch.Tensor:
        """query [S, H, D]; caches [NB, KVH, bs, D]; block_tables [S, maxB] int32;
        seq_lens [S] int32 -> [S, H, D]."""
        return _C.paged_attention(query=query, key_cache=key_cache, value_cache=value_cache,
                                  block_tables=block_tables, seq_lens=seq_lens, scale=self.scale)


class PagedAttentionWithRoPE(PagedAttention):
    def __init__(self, num_heads: int, head_size: int, scale: float, rotary_dim: int,
                 max_position: int = 8192, base: int = 10000):
        super().__init__(num_heads, head_size, scale)
        if rotary_dim <= 0 or rotary_dim % 2 != 0:
            raise ValueError("rotary_dim must be a positive even number")
        if rotary_dim > head_size:
            raise ValueError("rotary_dim must not exceed head_size")
        self.rotary_dim = rotary_dim
        # Same expression, same default-dtype dependence as attention.py:71-79.
        inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2) / rotary_dim))
        t = torch.arange(max_position).float()
        freqs = torch.einsum("i,j -> ij", t, inv_freq.float())
        cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1)
        cache = cache.to(torch.get_default_dtype())
        self.register_buffer("cos_sin_cache", cache, persistent=False)
        self._cs_cast: dict[tuple, torch.Tensor] = {}

    def _table(self, device: torch.device, dtype: torch.dtype) -> torch.Tensor:
        key = (device, dtype, self.cos_sin_cache.data_ptr(), self.cos_sin_cache._version)
        t = self._cs_cast.get(key)
        if t is None:
            self._cs_cast.clear()
            t = self.cos_sin_cache.to(device=device, dtype=dtype).contiguous()
            self._cs_cast[key] = t
        return t

    def _write_kv_cache(self, key, value, positions, key_cache, value_cache, block_tables):
        """attention.py:82-116 as one kernel (no host sync)."""
        _Cache.write_kv_cache(key, value, positions, key_cache, value_cache,
                              block_tables.to(torch.int32))

    def forward(self, positions: torch.Tensor | None, query: torch.Tensor, key: torch.Tensor,
                value: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                block_tables: torch.Tensor, seq_lens: torch.Tensor) -> torch.Tensor:
        if query.dim() != 3:
            raise ValueError("query must be [num_tokens, num_heads, head_dim]")
        if key.dim() != 3:
            raise ValueError("key must be [num_tokens, num_kv_heads, head_dim]")
        if value.dim() != 3:
            raise ValueError("value must be [num_tokens, num_kv_heads, head_dim]")
        num_tokens, num_heads, head_size = query.shape
        if head_size != self.head_size:
            raise ValueError("query head_dim must match head_size")
        if num_tokens != block_tables.size(0):
            raise NotImplementedError(
                "PagedAttentionWithRoPE only supports decode: there must be one token per sequence")

        cos_sin_cache = self._table(query.device, query.dtype)
        tables = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
        tables = tables.contiguous()
        if positions is None:
            if self.rotary_dim == head_size:
                # RoPE, cache write and attention in one launch; the key is
                # rotated in place, as rotary_embedding_neox does to it
                return _C.paged_attention_with_rope(
                    query.contiguous(), key, value, key_cache, value_cache, tables, seq_lens,
                    cos_sin_cache, self.scale)
            positions = seq_lens.to(torch.int64) - 1
        query_2d = query.reshape(num_tokens, num_heads * head_size).contiguous()
        key_2d = key.reshape(num_tokens, -1).contiguous()
        fused = key_cache.dtype == query.dtype and value.dtype == query.dtype
        if fused:
            query_2d = _PE.rotary_embedding_neox_with_cache(
                positions, query_2d, key_2d, value, key_cache, value_cache, None,
                self.head_size, cos_sin_cache, block_tables=tables)
        else:
            query_2d = _PE.rotary_embedding_neox(positions, query_2d, key_2d, self.head_size,
                                                 cos_sin_cache)
            self._write_kv_cache(key_2d, value, positions, key_cache, value_cache, tables)
        query = query_2d.view(num_tokens, num_heads, head_size)
        # The kernel just launched (RoPE + cache write) writes neither the
        # block tables nor seq_lens, so attention may overlap its prologue.
        return _C.paged_attention(query=query, key_cache=key_cache, value_cache=value_cache,
                                  block_tables=tables, seq_lens=seq_lens, scale=self.scale,
                                  overlap_prologue=fused)
