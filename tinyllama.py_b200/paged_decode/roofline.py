"""Algorithmic byte counts of the decode-step kernels (the roofline numerators).

attention    2*L*KVH*D*e per sequence (K and V of every context token)
             + 2*S*H*D*e (query read, output write)
             + 4*ceil(L/bs) per sequence (block-table entries) + 4*S (seq_lens)
rope         2*T*(H+KVH)*D*e (q, k read and written) + T*rot*e (cos/sin row) + T*8
cache write  2*(2*T*KVH*D*e) (k, v read, then written) + 8*T (slot)
"""

from __future__ import annotations

import numpy as np


def attention_bytes(seq_lens, block_size, num_heads, num_kv_heads, head_dim, elem_bytes):
    L = np.clip(np.asarray(seq_lens, np.int64), 0, None)
    S = L.shape[0]
    kv = int((2 * L * num_kv_heads * head_dim * elem_bytes).sum())
    qo = 2 * S * num_heads * head_dim * elem_bytes
    tables = int((4 * np.ceil(L / block_size)).sum()) + 4 * S
    return kv + qo + tables


def rope_bytes(num_tokens, num_heads, num_kv_heads, head_dim, rot_dim, elem_bytes, pos_bytes=8):
    return (2 * num_tokens * (num_heads + num_kv_heads) * head_dim * elem_bytes
            + num_tokens * rot_dim * elem_bytes + num_tokens * pos_bytes)


def cache_write_bytes(num_tokens, num_kv_heads, head_dim, elem_bytes):
    return 2 * (2 * num_tokens * num_kv_heads * head_dim * elem_bytes) + 8 * num_tokens
