"""Shared helpers of the GPU parity tests: run the kernels through the cscr
C-ABI ops and compare with the CPU oracle on the same seeded inputs."""

from __future__ import annotations

import numpy as np
import torch

from oracle import decode_oracle as O
from paged_decode import workloads as W

# North-star tolerance for half-precision outputs against the fp32 oracle.
HALF_TOL = dict(atol=2e-3, rtol=1e-2)
# The reference test's fp32 tolerance (tests/test_paged_attention.py:59-60).
F32_TOL = dict(atol=1e-4, rtol=1e-4)


def tol_for(dtype: str) -> dict:
    return F32_TOL if dtype == "float32" else HALF_TOL


def oracle_attention_f32(query, kc, vc, tables, lens, scale, dtype, threads=None):
    """fp32 oracle output (before the final rounding) on host arrays."""
    S, H, D = query.shape
    KVH = kc.shape[1]
    q32 = O.to_f32(query, dtype)
    out = np.zeros((S, H, D), np.float32)
    import os
    from concurrent.futures import ThreadPoolExecutor

    def work(s):
        out[s] = O._attend_one(q32[s], kc, vc, dtype, tables[s], lens[s], kc.shape[2], KVH,
                               H // KVH, scale)

    with ThreadPoolExecutor(max_workers=threads or os.cpu_count()) as ex:
        list(ex.map(work, range(S)))
    return out


def check_attention(batch: W.DecodeBatch, out: torch.Tensor, seqs=None, query=None):
    """Compare `out` ([S, H, D] on device) with the oracle for the given sequences."""
    dtype = batch.spec.dtype
    kc, vc, tables, lens = W.compact_for_oracle(batch) if seqs is None else _subset(batch, seqs)
    q = W.to_numpy(batch.query[batch.decode_rows] if query is None else query)
    got = W.to_numpy(out)
    if seqs is not None:
        q, got = q[seqs], got[seqs]
    ref = oracle_attention_f32(q, kc, vc, tables, lens, batch.scale, dtype)
    np.testing.assert_allclose(O.to_f32(got, dtype), ref, **tol_for(dtype))


def oracle_f32_from_tensors(query, key_cache, value_cache, block_tables, seq_lens, scale, dtype):
    """fp32 oracle output for device tensors of one attention call (pool compacted)."""
    from types import SimpleNamespace

    view = SimpleNamespace(block_tables=block_tables, seq_lens=seq_lens, key_cache=key_cache,
                           value_cache=value_cache,
                           spec=SimpleNamespace(block_size=key_cache.shape[2]))
    kc, vc, tables, lens = W.compact_for_oracle(view)
    return oracle_attention_f32(W.to_numpy(query), kc, vc, tables, lens, scale, dtype)


def _subset(batch: W.DecodeBatch, seqs):
    sub = W.DecodeBatch(**{**batch.__dict__})
    sub.block_tables = batch.block_tables[list(seqs)]
    sub.seq_lens = batch.seq_lens[list(seqs)]
    return W.compact_for_oracle(sub)
