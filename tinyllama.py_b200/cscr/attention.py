"""cscr.attention — drop-in for the reference's pybind module of the same name.

``paged_attention(query, key_cache, value_cache, block_tables, seq_lens, scale)``
keeps the signature, keyword names, checks and error messages of
cscr/attention.cpp:7-48 (bound at :50-56) and returns a new
``[num_seqs, num_heads, head_dim]`` tensor, computed asynchronously on the
current CUDA stream by the sm_100a kernels of libtinyllama_b200.so.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import DTYPE_CODE, torch_check

_FLOAT_TYPES = (torch.float16, torch.bfloat16, torch.float32)

class _Workspace:
    """Scratch of one (device, stream) and the length of its zero-at-rest prefix.

    The kernel needs the arrival-counter prefix of the workspace to be zero
    when it starts and leaves exactly that prefix zero when it ends; the bytes
    after it hold partial results. A call whose counter prefix is longer than
    the one currently known to be clean therefore zeroes it first (an async
    memset on the same stream); calls of a steady shape never do.
    """

    __slots__ = ("buf", "clean")

    def __init__(self, buf: torch.Tensor):
        self.buf = buf
        self.clean = buf.numel()


# (device index, stream handle) -> workspace
_workspaces: dict[tuple[int, int], _Workspace] = {}
_ws_sizes: dict[tuple, tuple[int, int]] = {}


def invalidate_workspaces(device_index: int) -> None:
    """Forget which counter prefixes of this device's workspaces are zero, so
    that the next call on each re-zeroes its prefix (after a kernel reported
    a wait that gave up, TLB_STATUS_WAIT_TIMEOUT)."""
    for (dev, _stream), ws in _workspaces.items():
        if dev == device_index:
            ws.clean = 0


def workspace_bytes(num_seqs: int, num_heads: int, num_kv_heads: int, head_dim: int,
                    dtype: torch.dtype, device_index: int) -> tuple[int, int]:
    """(total bytes, zero-at-rest prefix bytes) of scratch for this shape on this device."""
    key = (num_seqs, num_heads, num_kv_heads, head_dim, dtype, device_index)
    n = _ws_sizes.get(key)
    if n is None:
        lib = _lib.load()
        total, zeroed = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.check(lib.tlb_paged_attention_workspace_size(
            num_seqs, num_heads, num_kv_heads, head_dim, DTYPE_CODE[dtype], ctypes.byref(total)))
        _lib.check(lib.tlb_paged_attention_workspace_zeroed_bytes(
            num_seqs, num_kv_heads, ctypes.byref(zeroed)))
        n = (total.value, zeroed.value)
        _ws_sizes[key] = n
    return n


def _workspace(device: torch.device, stream: int, nbytes: int, zeroed: int) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    key = (device.index, stream)
    ws = _workspaces.get(key)
    if ws is None or ws.buf.numel() < nbytes:
        ws = _Workspace(torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device))
        _workspaces[key] = ws
    if zeroed > ws.clean:
        ws.buf[:zeroed].zero_()
    ws.clean = zeroed
    return ws.buf


def paged_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                    block_tables: torch.Tensor, seq_lens: torch.Tensor,
                    scale: float, *, overlap_prologue: bool = False) -> torch.Tensor:
    """PagedAttention decode forward (CUDA, sm_100a).

    query [num_seqs, num_heads, head_dim]; key_cache / value_cache
    [num_blocks, num_kv_heads, block_size, head_dim]; block_tables
    [num_seqs, max_blocks_per_seq] int32; seq_lens [num_seqs] int32.

    ``overlap_prologue`` (keyword only, not in the reference API) lets the
    kernel start while the kernel launched just before it on this stream is
    finishing; set it only when that kernel writes neither block_tables nor
    seq_lens — e.g. right after ``rotary_embedding_neox_with_cache``.
    """
    torch_check(query.is_cuda, "query must be a CUDA tensor")
    torch_check(key_cache.is_cuda, "key_cache must be a CUDA tensor")
    torch_check(value_cache.is_cuda, "value_cache must be a CUDA tensor")
    torch_check(block_tables.is_cuda, "block_tables must be a CUDA tensor")
    torch_check(seq_lens.is_cuda, "seq_lens must be a CUDA tensor")
    torch_check(query.dim() == 3, "query must be [num_seqs, num_heads, head_dim]")
    torch_check(key_cache.dim() == 4,
                "key_cache must be [num_blocks, num_kv_heads, block_size, head_dim]")
    torch_check(value_cache.shape == key_cache.shape,
                "value_cache must have the same shape as key_cache")
    torch_check(block_tables.dim() == 2, "block_tables must be [num_seqs, max_blocks_per_seq]")
    torch_check(seq_lens.dim() == 1, "seq_lens must be [num_seqs]")
    torch_check(query.is_contiguous(), "query must be contiguous")
    torch_check(key_cache.is_contiguous(), "key_cache must be contiguous")
    torch_check(value_cache.is_contiguous(), "value_cache must be contiguous")
    torch_check(block_tables.is_contiguous(), "block_tables must be contiguous")
    torch_check(seq_lens.is_contiguous(), "seq_lens must be contiguous")
    torch_check(block_tables.dtype == torch.int32, "block_tables must be int32")
    torch_check(seq_lens.dtype == torch.int32, "seq_lens must be int32")
    torch_check(query.dtype == key_cache.dtype and query.dtype == value_cache.dtype,
                "query, key_cache and value_cache must share the same dtype")
    torch_check(query.dtype in _FLOAT_TYPES, "dtype must be float16, bfloat16 or float32")

    num_seqs, num_heads, head_dim = query.shape
    num_blocks, num_kv_heads, block_size, cache_head_dim = key_cache.shape
    torch_check(num_seqs > 0, "query must contain at least one sequence")
    torch_check(head_dim == cache_head_dim, "query head_dim must match the cache head_dim")
    torch_check(num_heads % num_kv_heads == 0, "num_heads must be divisible by num_kv_heads")
    torch_check(block_tables.size(0) == num_seqs, "block_tables must have one row per sequence")
    torch_check(seq_lens.size(0) == num_seqs, "seq_lens must have one entry per sequence")
    torch_check(head_dim <= 1024, "head_dim too large for the reference kernel")
    dev = query.device
    torch_check(key_cache.device == dev and value_cache.device == dev
                and block_tables.device == dev and seq_lens.device == dev,
                "all tensors must be on the same CUDA device")

    out = torch.empty_like(query)
    if num_blocks == 0 or block_tables.size(1) == 0:
        # No cache to read: every softmax is empty, which the kernel defines as 0.
        out.zero_()
        return out
    lib = _lib.load()
    with _lib.device_guard(dev):
        stream = _lib.stream_of(dev)
        nbytes, zeroed = workspace_bytes(num_seqs, num_heads, num_kv_heads, head_dim,
                                         query.dtype, dev.index)
        ws = _workspace(dev, stream, nbytes, zeroed)
        rc = lib.tlb_paged_attention(
            out.data_ptr(), query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            block_tables.data_ptr(), seq_lens.data_ptr(), num_seqs, num_heads, num_kv_heads,
            head_dim, num_blocks, block_size, block_tables.size(1), float(scale),
            DTYPE_CODE[query.dtype], ws.data_ptr() if ws is not None else None,
            ws.numel() if ws is not None else 0, 1 if overlap_prologue else 0, stream)
        _lib.check(rc)
    return out


def paged_attention_with_rope(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                              key_cache: torch.Tensor, value_cache: torch.Tensor,
                              block_tables: torch.Tensor, seq_lens: torch.Tensor,
                              cos_sin_cache: torch.Tensor, scale: float, *,
                              overlap_prologue: bool = False) -> torch.Tensor:
    """A decode step in one launch (not in the reference API): NeoX RoPE of the
    raw ``query`` and ``key`` at position ``seq_lens[s] - 1``, the cache write
    of that token's rotated key and ``value`` through ``block_tables``, and
    paged attention with the rotated query — what
    ``rotary_embedding_neox_with_cache(seq_lens - 1, query, key, value, ...,
    block_tables=block_tables)`` followed by ``paged_attention`` computes
    (src/model_executor/layers/attention.py:151-166 for a decode batch).

    query [num_seqs, num_heads, head_dim] (left as is), key
    [num_seqs, num_kv_heads * head_dim] or [num_seqs, num_kv_heads, head_dim]
    (rotated in place), value likewise, cos_sin_cache [rows, head_dim] in the
    query dtype. Shapes the tensor-core kernel does not serve run as those two
    launches.

    ``overlap_prologue`` has the contract of ``paged_attention``'s: set it
    only when the kernel launched just before on this stream writes neither
    block_tables nor seq_lens (query, key, value and the caches are read only
    after that kernel has finished).
    """
    torch_check(query.is_cuda and key.is_cuda and value.is_cuda and cos_sin_cache.is_cuda,
                "query, key, value and cos_sin_cache must be CUDA tensors")
    torch_check(query.dim() == 3 and query.is_contiguous(),
                "query must be a contiguous [num_seqs, num_heads, head_dim] tensor")
    num_seqs, num_heads, head_dim = query.shape
    k2 = key.reshape(num_seqs, -1) if key.dim() == 3 else key
    v2 = value.reshape(num_seqs, -1)
    torch_check(k2.dim() == 2 and k2.size(0) == num_seqs and k2.stride(1) == 1,
                "key must be [num_seqs, num_kv_heads * head_dim] with unit inner stride")
    torch_check(v2.size(1) == k2.size(1) and v2.stride(1) == 1,
                "value must match key: [num_seqs, num_kv_heads, head_dim]")
    torch_check(key.dtype == query.dtype and value.dtype == query.dtype
                and cos_sin_cache.dtype == query.dtype,
                "key, value and cos_sin_cache must share the query dtype")
    torch_check(cos_sin_cache.dim() == 2 and cos_sin_cache.is_contiguous()
                and cos_sin_cache.size(1) == head_dim,
                "cos_sin_cache must be a contiguous [rows, head_dim] tensor")
    torch_check(key_cache.dim() == 4 and k2.size(1) == key_cache.size(1) * head_dim,
                "key must hold num_kv_heads * head_dim values per token")
    torch_check(seq_lens.dim() == 1 and seq_lens.size(0) == num_seqs,
                "seq_lens must have one entry per sequence")
    out = torch.empty_like(query)
    if key_cache.size(0) > 0 and block_tables.dim() == 2 and block_tables.size(1) > 0 \
            and block_tables.dtype == torch.int32 and seq_lens.dtype == torch.int32 \
            and block_tables.is_contiguous() and seq_lens.is_contiguous() \
            and key_cache.is_contiguous() and value_cache.is_contiguous() \
            and key_cache.shape == value_cache.shape and key_cache.dtype == query.dtype:
        lib = _lib.load()
        dev = query.device
        with _lib.device_guard(dev):
            stream = _lib.stream_of(dev)
            nbytes, zeroed = workspace_bytes(num_seqs, num_heads, key_cache.size(1), head_dim,
                                             query.dtype, dev.index)
            ws = _workspace(dev, stream, nbytes, zeroed)
            rc = lib.tlb_paged_attention_with_rope(
                out.data_ptr(), query.data_ptr(), k2.data_ptr(), v2.data_ptr(),
                key_cache.data_ptr(), value_cache.data_ptr(), block_tables.data_ptr(),
                seq_lens.data_ptr(), cos_sin_cache.data_ptr(), cos_sin_cache.size(0), num_seqs,
                num_heads, key_cache.size(1), head_dim, key_cache.size(0), key_cache.size(2),
                block_tables.size(1), k2.stride(0), v2.stride(0), float(scale),
                DTYPE_CODE[query.dtype], ws.data_ptr() if ws is not None else None,
                ws.numel() if ws is not None else 0, 1 if overlap_prologue else 0, stream)
            if rc != _lib.TLB_ERR_UNSUPPORTED:
                _lib.check(rc)
                return out
    # Shapes outside the fused kernel: the same step as two launches.
    from . import pos_encoding as _PE
    positions = (seq_lens.to(torch.int64) - 1)
    q_rot = _PE.rotary_embedding_neox_with_cache(
        positions, query.reshape(num_seqs, -1), k2, v2, key_cache, value_cache, None, head_dim,
        cos_sin_cache, block_tables=block_tables)
    return paged_attention(q_rot.view(num_seqs, num_heads, head_dim), key_cache, value_cache,
                           block_tables, seq_lens, scale)


def paged_prefill_attention(query: torch.Tensor, key_cache: torch.Tensor,
                            value_cache: torch.Tensor, block_tables: torch.Tensor,
                            query_start: torch.Tensor, context_lens: torch.Tensor, scale: float,
                            max_query_len: int | None = None,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal paged attention of prompt chunks (not in the reference API, whose
    layer is decode-only: src/model_executor/layers/attention.py:139-143).

    query [num_tokens, num_heads, head_dim]: chunk c owns rows
    query_start[c] .. query_start[c + 1] - 1, the last tokens of the first
    context_lens[c] tokens of its sequence, whose keys and values are already
    in the caches (run the RoPE + cache write over the packed step first).
    block_tables [num_chunks, max_blocks] int32, query_start [num_chunks + 1]
    int32, context_lens [num_chunks] int32. ``max_query_len`` (the longest
    chunk) sizes the launch; when omitted it is read from query_start (a
    device-to-host read). Returns ``out`` (a new tensor unless given); rows
    outside every chunk are left as they were.
    """
    torch_check(query.is_cuda and key_cache.is_cuda and value_cache.is_cuda
                and block_tables.is_cuda and query_start.is_cuda and context_lens.is_cuda,
                "all tensors must be CUDA tensors")
    torch_check(query.dim() == 3 and query.is_contiguous(),
                "query must be a contiguous [num_tokens, num_heads, head_dim] tensor")
    torch_check(key_cache.dim() == 4 and key_cache.shape == value_cache.shape
                and key_cache.is_contiguous() and value_cache.is_contiguous(),
                "key_cache and value_cache must be contiguous [num_blocks, num_kv_heads, "
                "block_size, head_dim] tensors of one shape")
    torch_check(query.dtype in (torch.float16, torch.bfloat16)
                and key_cache.dtype == query.dtype and value_cache.dtype == query.dtype,
                "prefill attention supports float16 and bfloat16 (query and caches alike)")
    torch_check(block_tables.dtype == torch.int32 and query_start.dtype == torch.int32
                and context_lens.dtype == torch.int32,
                "block_tables, query_start and context_lens must be int32")
    num_chunks = context_lens.numel()
    torch_check(block_tables.dim() == 2 and block_tables.size(0) == num_chunks
                and query_start.numel() == num_chunks + 1,
                "one block-table row and one context length per chunk, num_chunks + 1 starts")
    T, H, D = query.shape
    torch_check(key_cache.size(3) == D, "query head_dim must match the cache head_dim")
    if out is None:
        out = torch.empty_like(query)
    if max_query_len is None:
        max_query_len = int((query_start[1:] - query_start[:-1]).max().item()) if num_chunks else 0
    dev = query.device
    with _lib.device_guard(dev):
        rc = _lib.load().tlb_paged_prefill_attention(
            out.data_ptr(), query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            block_tables.contiguous().data_ptr(), query_start.contiguous().data_ptr(),
            context_lens.contiguous().data_ptr(), num_chunks, H, key_cache.size(1), D,
            key_cache.size(0), key_cache.size(2), block_tables.size(1), int(max_query_len),
            float(scale), DTYPE_CODE[query.dtype], _lib.stream_of(dev))
        _lib.check(rc)
    return out
