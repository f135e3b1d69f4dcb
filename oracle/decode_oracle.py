"""CPU restatement of tinyllama.py's decode hot path — TEST INFRASTRUCTURE ONLY.

This module is the parity oracle: the test suite, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg use it to check or to time the reference
algorithm on the host. Nothing on the product path imports it.

Every function restates a piece of the reference (CodeClaper/tinyllama.py) in
numpy, fp32 arithmetic on storage-dtype inputs, citing the file:line it
follows. Parity is pinned by ``tests/test_oracle_golden.py`` against fixtures
produced from the reference's own Python code (``tests/golden/make_golden.py``):

* paged attention   — tests/test_paged_attention.py:42-57 (the reference test's
  own oracle), with the kernel's skip rule for negative block ids
  (cscr/attention_kernel.cu:70-72) and zero output for an empty softmax (:102);
* KV-cache write    — src/model_executor/layers/attention.py:96-116 (bit-exact);
* decode metadata   — src/worker/worker.py:139-159;
* cos/sin table     — src/model_executor/layers/attention.py:71-80 (pinned in
  the tests through the layer glue that rebuilds it with torch).

The NeoX rotation restates cscr/pos_encoding_kernel.cu:24-65. The reference
has no CPU path for it, so that restatement is not pinned by a reference run
here (see the golden-fixture script for what is).

Storage dtypes are "float32", "float16" and "bfloat16"; bfloat16 arrays are
carried as ``np.uint16`` bit patterns.
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

DTYPES = ("float32", "float16", "bfloat16")


# ----------------------------------------------------------------- dtypes
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (NaN kept NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    rounded = ((u + (0x7FFF + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return bf16_bits_to_f32(a)
    return np.asarray(a, dtype=np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return f32_to_bf16_bits(x)
    if dtype == "float16":
        return np.asarray(x, dtype=np.float32).astype(np.float16)
    return np.asarray(x, dtype=np.float32)


def storage_np_dtype(dtype: str):
    return {"float32": np.float32, "float16": np.float16, "bfloat16": np.uint16}[dtype]


# ------------------------------------------------------------ attention
def _attend_one(q32, kc, vc, dtype, block_table, seq_len, block_size, num_kv_heads, group, scale):
    """One sequence: q32 [H, D] fp32 -> [H, D] fp32 (pre-cast)."""
    H, D = q32.shape
    max_blocks = block_table.shape[0]
    L = min(max(int(seq_len), 0), max_blocks * block_size)
    out = np.zeros((H, D), np.float32)
    if L == 0:
        return out
    tok = np.arange(L)
    blk = block_table[tok // block_size].astype(np.int64)
    valid = (blk >= 0) & (blk < kc.shape[0])
    if not valid.any():
        return out
    blk, off = blk[valid], (tok % block_size)[valid]
    # gather [Lv, KVH, D] rows, then fp32 — tests/test_paged_attention.py:45-50
    keys = to_f32(kc[blk, :, off, :], dtype)
    values = to_f32(vc[blk, :, off, :], dtype)
    # group folding == repeat_interleave(group, dim=1) of the test (:51-52)
    q = q32.reshape(num_kv_heads, group, D)
    kT = np.ascontiguousarray(keys.transpose(1, 2, 0))  # [KVH, D, Lv]
    v = np.ascontiguousarray(values.transpose(1, 0, 2))  # [KVH, Lv, D]
    scores = np.matmul(q, kT) * np.float32(scale)  # [KVH, G, Lv]   (:54)
    m = scores.max(axis=-1, keepdims=True)
    p = np.exp(scores - m)
    p /= p.sum(axis=-1, keepdims=True)  # softmax (:55)
    return np.matmul(p, v).reshape(H, D)  # einsum("hl,lhd->hd") (:56)


def paged_attention(query, key_cache, value_cache, block_tables, seq_lens, scale, dtype,
                    threads: int | None = None) -> np.ndarray:
    """Decode attention over paged K/V; returns [S, H, D] in the storage dtype.

    Restates tests/test_paged_attention.py:42-57 for each sequence: gather the
    sequence's blocks, keep its first seq_len tokens, fold query heads onto
    their KV head (h // (H / KVH)), fp32 softmax(scale q K^T) V, cast once.
    """
    return from_f32(paged_attention_f32(query, key_cache, value_cache, block_tables, seq_lens,
                                        scale, dtype, threads), dtype)


def paged_attention_f32(query, key_cache, value_cache, block_tables, seq_lens, scale, dtype,
                        threads: int | None = None) -> np.ndarray:
    """paged_attention's fp32 result before the final cast (the tolerance reference)."""
    S, H, D = query.shape
    NB, KVH, BS, Dk = key_cache.shape
    assert Dk == D and H % KVH == 0
    group = H // KVH
    q32 = to_f32(query, dtype)
    out = np.empty((S, H, D), np.float32)

    def work(s):
        out[s] = _attend_one(q32[s], key_cache, value_cache, dtype, block_tables[s],
                             seq_lens[s], BS, KVH, group, scale)

    threads = threads or 1
    if threads == 1 or S == 1:
        for s in range(S):
            work(s)
    else:
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(work, range(S)))
    return out


def paged_attention_threads(query, key_cache, value_cache, block_tables, seq_lens, scale, dtype,
                            threads: int | None = None):
    """paged_attention on all host cores (BLAS pinned to one thread per worker)."""
    threads = threads or os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        return paged_attention(query, key_cache, value_cache, block_tables, seq_lens, scale,
                               dtype, threads)
    with threadpool_limits(limits=1):
        return paged_attention(query, key_cache, value_cache, block_tables, seq_lens, scale,
                               dtype, threads)


def paged_prefill_attention_f32(query, key_cache, value_cache, block_tables, query_start,
                                context_lens, scale, dtype, threads: int | None = None):
    """Causal attention of prompt chunks over their paged context, fp32.

    The reference has no prefill op (its layer is decode-only,
    src/model_executor/layers/attention.py:139-143). This is the reference
    test's math (tests/test_paged_attention.py:42-57: gather the sequence's
    blocks, fold query heads onto their kv head, fp32 softmax(scale q K^T) V)
    with a causal mask: row j of chunk c, at position
    p = context_lens[c] - n_c + j, sees tokens 0..p of its sequence. Blocks
    with a negative id are skipped; an empty softmax gives zeros.
    Returns [T, H, D] fp32; rows outside every chunk stay zero.
    """
    T, H, D = query.shape
    NB, KVH, BS, _ = key_cache.shape
    G = H // KVH
    q32 = to_f32(query, dtype)
    out = np.zeros((T, H, D), np.float32)
    qs = np.asarray(query_start, np.int64)

    def chunk(c):
        n = int(qs[c + 1] - qs[c])
        ctx = int(context_lens[c])
        if n <= 0:
            return
        first = ctx - n
        L = max(0, min(ctx, block_tables.shape[1] * BS))
        tok = np.arange(L)
        blk = np.asarray(block_tables[c], np.int64)[tok // BS]
        valid = (blk >= 0) & (blk < NB)
        keys = np.zeros((L, KVH, D), np.float32)
        vals = np.zeros((L, KVH, D), np.float32)
        keys[valid] = to_f32(key_cache[blk[valid], :, (tok % BS)[valid], :], dtype)
        vals[valid] = to_f32(value_cache[blk[valid], :, (tok % BS)[valid], :], dtype)
        q = q32[qs[c]:qs[c] + n].reshape(n, KVH, G, D)
        pos = first + np.arange(n)
        allowed = valid[None, :] & (tok[None, :] <= pos[:, None])  # [n, L]
        for h in range(KVH):
            qh = np.ascontiguousarray(q[:, h].transpose(1, 0, 2))        # [G, n, D]
            sc = np.matmul(qh, np.ascontiguousarray(keys[:, h].T)) * np.float32(scale)
            sc = np.where(allowed[None], sc, np.float32(-np.inf))       # [G, n, L]
            m = sc.max(axis=-1, keepdims=True)
            m = np.where(np.isfinite(m), m, np.float32(0.0))
            pr = np.exp(sc - m)
            den = pr.sum(axis=-1, keepdims=True)
            pr = np.divide(pr, den, out=np.zeros_like(pr), where=den > 0)
            o = np.matmul(pr, np.ascontiguousarray(vals[:, h]))         # [G, n, D]
            out[qs[c]:qs[c] + n, h * G:(h + 1) * G] = o.transpose(1, 0, 2)

    nchunks = len(context_lens)
    if (threads or 1) > 1 and nchunks > 1:
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(chunk, range(nchunks)))
    else:
        for c in range(nchunks):
            chunk(c)
    return out


# ------------------------------------------------------------------ RoPE
def rotary_embedding_neox(positions, query, key, head_size, cos_sin_cache, dtype):
    """NeoX rotary embedding; returns (out, key_rotated) in the storage dtype.

    Restates cscr/pos_encoding_kernel.cu:24-65: for pair (i, i + rot/2),
    x' = x*cos - y*sin, y' = y*cos + x*sin in fp32 with cos/sin read from the
    (dtype-rounded) cache row of the token's position, one rounding to dtype.
    The query goes to a new array, the key is returned rotated (the kernel
    rewrites it in place). Query elements >= rot are passed through.
    """
    T = positions.shape[0]
    rot = cos_sin_cache.shape[1]
    half = rot // 2
    cs = to_f32(cos_sin_cache, dtype)[np.asarray(positions, np.int64)]  # [T, rot]
    cos = cs[:, None, :half]
    sin = cs[:, None, half:rot]

    def rotate(x2d):
        x = to_f32(x2d, dtype).reshape(T, -1, head_size).copy()
        a = x[..., :half].copy()
        b = x[..., half:rot].copy()
        x[..., :half] = a * cos - b * sin
        x[..., half:rot] = b * cos + a * sin
        return x.reshape(T, -1)

    out = from_f32(rotate(query), dtype)
    k_rot = from_f32(rotate(key), dtype)
    # pass-through elements keep their exact bits
    if rot < head_size:
        qv = out.reshape(T, -1, head_size)
        qv[..., rot:] = np.asarray(query).reshape(T, -1, head_size)[..., rot:]
        kv = k_rot.reshape(T, -1, head_size)
        kv[..., rot:] = np.asarray(key).reshape(T, -1, head_size)[..., rot:]
    return out, k_rot


def cos_sin_cache(rotary_dim: int, max_position: int, base: float) -> np.ndarray:
    """fp32 cos/sin table of attention.py:71-77 evaluated with an fp32 default dtype.

    The layer casts it to the default dtype afterwards (:78-79); with a
    half-precision default dtype the reference also rounds the frequency
    exponent, which the layer glue reproduces with torch (pinned by tests).
    """
    inv_freq = (1.0 / (np.float32(base) ** (np.arange(0, rotary_dim, 2, dtype=np.float32)
                                              / np.float32(rotary_dim)))).astype(np.float32)
    t = np.arange(max_position, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    return np.concatenate([np.cos(freqs), np.sin(freqs)], axis=-1).astype(np.float32)


# ------------------------------------------------------------ cache write
def write_kv_cache(key, value, positions, key_cache, value_cache, block_tables):
    """In-place KV write exactly as attention.py:96-116 addresses it.

    Token r goes to block block_tables[r, positions[r] // bs] at offset
    positions[r] % bs; rows whose block id is negative are skipped. Bit copy.
    """
    bs = key_cache.shape[2]
    kvh, D = key_cache.shape[1], key_cache.shape[3]
    T = positions.shape[0]
    pos = np.asarray(positions, np.int64)
    logical = pos // bs
    slots = pos % bs
    rows = np.arange(T)
    phys = np.asarray(block_tables, np.int64)[rows, logical]
    valid = phys >= 0
    k = np.asarray(key).reshape(T, kvh, D)
    v = np.asarray(value).reshape(T, kvh, D)
    for r in rows[valid]:
        key_cache[phys[r], :, slots[r], :] = k[r]
        value_cache[phys[r], :, slots[r], :] = v[r]


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping):
    """Slot-addressed form of the same write: slot = block*bs + offset; <0 skips."""
    bs = key_cache.shape[2]
    kvh, D = key_cache.shape[1], key_cache.shape[3]
    T = slot_mapping.shape[0]
    k = np.asarray(key).reshape(T, kvh, D)
    v = np.asarray(value).reshape(T, kvh, D)
    for t in range(T):
        slot = int(slot_mapping[t])
        if slot < 0:
            continue
        key_cache[slot // bs, :, slot % bs, :] = k[t]
        value_cache[slot // bs, :, slot % bs, :] = v[t]


# ------------------------------------------------------------- metadata
def decode_metadata(context_lens, block_tables, block_size):
    """positions and slots of decode tokens, as worker.py:139-159 computes them.

    position = context_len - 1; slot = block_table[position // bs] * bs +
    position % bs (-1 when the context is empty or the block id is negative).
    """
    ctx = np.asarray(context_lens, np.int64)
    pos = ctx - 1
    slots = np.full(pos.shape, -1, np.int64)
    for r, p in enumerate(pos):
        if p < 0:
            continue
        blk = int(block_tables[r][p // block_size])
        if blk >= 0:
            slots[r] = blk * block_size + p % block_size
    return pos, slots


def step_metadata(prompt_lens, prompt_tables, context_lens, decode_tables, block_size,
                  alignment: int = 8):
    """positions and slots of a packed continuous-batching step, as
    worker.py:84-169 forms them: every prompt's tokens first (position i of
    prompt p at slot prompt_table[p][i // bs] * bs + i % bs, :95-124), then one
    token per decode sequence (position context_len - 1, slot as
    decode_metadata, :126-159). Positions are padded with 0 to a multiple of
    ``alignment`` (:163-164); the slots are returned unpadded, as the worker
    forms them. A negative block id gives slot -1 (the decode rule here; the
    reference's block manager never hands out one for a prompt).
    """
    pos, slots = [], []
    for L, table in zip(prompt_lens, prompt_tables):
        for i in range(int(L)):
            blk = int(table[i // block_size])
            pos.append(i)
            slots.append(blk * block_size + i % block_size if blk >= 0 else -1)
    dpos, dslots = decode_metadata(context_lens, decode_tables, block_size)
    pos.extend(int(p) for p in dpos)
    slots.extend(int(s) for s in dslots)
    padded = pos + [0] * ((-len(pos)) % alignment)
    return np.asarray(padded, np.int64), np.asarray(slots, np.int64)


# ------------------------------------------------------------ block copies
def copy_blocks(caches, block_mapping):
    """cscr/cache_kernel.cu:124-212 (copy_blocks): src block -> each dst, every cache."""
    for c in caches:
        for src, dsts in block_mapping.items():
            for dst in dsts:
                c[dst] = c[src]


def swap_blocks(src, dst, block_mapping):
    """cscr/cache_kernel.cu:124-178 (swap_blocks): dst[d] = src[s] for each pair."""
    for s, d in block_mapping.items():
        dst[d] = src[s]


def ceil_div(a, b):
    return -(-a // b)


__all__ = [
    "DTYPES", "bf16_bits_to_f32", "f32_to_bf16_bits", "to_f32", "from_f32", "storage_np_dtype",
    "paged_attention", "paged_attention_f32", "paged_attention_threads",
    "paged_prefill_attention_f32", "rotary_embedding_neox", "cos_sin_cache",
    "write_kv_cache", "reshape_and_cache", "decode_metadata", "step_metadata", "copy_blocks", "swap_blocks",
    "ceil_div",
]
