"""The fused decode step (RoPE + cache write + attention in one launch) against
the same step as separate launches, and through them against the oracle.

The separate launches are rotary_embedding_neox_with_cache (positions
seq_lens - 1, block-table addressing) followed by paged_attention; both are
checked against the oracle elsewhere. Here: the cache rows and the rotated key
the fused launch leaves must be the same bits, and so must the attention
output (the query is rotated by the same function, the caches hold the same
rows, and the work partition and merge order are the same), and edge cases (negative block ids,
positions outside the cos/sin table, empty sequences, many splits) behave as
the separate launches do.
"""

import math

import pytest
import torch

from cscr import _lib
from cscr import attention as A
from cscr import pos_encoding as PE
from helpers import check_attention, tol_for
from paged_decode import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_status():
    torch.cuda.set_device(0)
    _lib.device_status(clear=True)
    yield
    torch.cuda.synchronize()


def _batch(lens, H, KVH, D, bs, dtype, seed=0, max_position=None):
    spec = W.DecodeSpec("fused", list(lens), H, KVH, D, bs, dtype,
                        num_blocks=sum(math.ceil(max(L, 0) / bs) for L in lens) + 8,
                        rope_theta=1e6, max_position=max_position, seed=seed)
    return W.make_batch(spec)


def _two_launches(b, kc, vc, key):
    S = b.num_decode
    H, D = b.spec.num_heads, b.spec.head_dim
    positions = b.seq_lens.to(torch.int64) - 1
    q = PE.rotary_embedding_neox_with_cache(positions, b.query[:S].reshape(S, -1), key,
                                            b.value[:S], kc, vc, None, D, b.cos_sin_cache,
                                            block_tables=b.block_tables)
    return A.paged_attention(q.view(S, H, D), kc, vc, b.block_tables, b.seq_lens, b.scale)


def _fused(b, kc, vc, key):
    S = b.num_decode
    return A.paged_attention_with_rope(b.query[:S].contiguous(), key, b.value[:S], kc, vc,
                                       b.block_tables, b.seq_lens, b.cos_sin_cache, b.scale)


def _compare(b, repeats=2):
    S = b.num_decode
    k0 = b.key[:S].reshape(S, -1).clone()
    kc0, vc0 = b.key_cache.clone(), b.value_cache.clone()
    k_ref, kc_ref, vc_ref = k0.clone(), kc0.clone(), vc0.clone()
    ref = _two_launches(b, kc_ref, vc_ref, k_ref)
    torch.cuda.synchronize()
    _lib.device_status(clear=True)  # the status below is the fused launches' own
    for _ in range(repeats):
        k, kc, vc = k0.clone(), kc0.clone(), vc0.clone()
        out = _fused(b, kc, vc, k)
        torch.cuda.synchronize()
        assert torch.equal(k.view(torch.int16), k_ref.view(torch.int16)), "rotated key"
        assert torch.equal(kc.view(torch.int16), kc_ref.view(torch.int16)), "key cache"
        assert torch.equal(vc.view(torch.int16), vc_ref.view(torch.int16)), "value cache"
        tol = tol_for(b.spec.dtype)
        torch.testing.assert_close(out.float(), ref.float(), atol=tol["atol"], rtol=tol["rtol"])
        # same query bits (one rotation function), same cache rows, same work
        # partition and merge order: the very same output bits
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), "attention output"
    return out, kc, vc, _lib.device_status()


def test_qwen3b_decode_step(built_lib):
    b = W.make_batch(W.qwen3b_decode(11, batch=64))
    out, kc, vc, status = _compare(b)
    assert status == 0
    # and against the oracle on the caches the step left
    b.key_cache, b.value_cache = kc, vc
    S = b.num_decode
    q_rot = PE.rotary_embedding_neox(b.seq_lens.to(torch.int64) - 1,
                                     b.query[:S].reshape(S, -1).contiguous(),
                                     b.key[:S].reshape(S, -1).clone(), b.spec.head_dim,
                                     b.cos_sin_cache)
    check_attention(b, out, query=q_rot.view_as(b.query[:S]))


@pytest.mark.parametrize("H,KVH,D,bs,dtype", [
    (14, 2, 64, 8, "float16"),
    (14, 2, 64, 16, "bfloat16"),
    (16, 2, 128, 32, "float16"),
    (16, 1, 128, 64, "bfloat16"),
    (32, 2, 128, 16, "bfloat16"),   # group 16: two head tiles
    (8, 8, 128, 16, "float16"),     # group 1
])
def test_head_shapes_and_block_sizes(H, KVH, D, bs, dtype, built_lib):
    b = _batch([1, 2, 15, 16, 17, 100, 333, 1024, 77, 4000], H, KVH, D, bs, dtype)
    assert _compare(b)[3] == 0


def test_one_long_sequence_cut_into_many_pieces(built_lib):
    b = _batch([30000], 16, 2, 128, 16, "bfloat16", seed=3)
    _compare(b)


def test_empty_sequences_and_skipped_blocks(built_lib):
    b = _batch([0, 40, 1, 0, 700, 33], 14, 2, 64, 16, "bfloat16", seed=5)
    # a sequence whose last block (the new token's) is not mapped: no write, no read
    b.block_tables[4, (700 - 1) // 16] = -1
    b.block_tables[1, 0] = -1
    assert _compare(b)[3] == 0  # empty sequences have no new token: nothing to flag


def test_position_outside_the_table_passes_through_and_is_flagged(built_lib):
    # cos/sin table of 256 rows; the 600-token sequence's new token is at 599
    b = _batch([100, 600, 30], 16, 2, 128, 16, "bfloat16", seed=7, max_position=256)
    assert _compare(b, repeats=1)[3] & 0x4


def test_fp32_runs_as_two_launches(built_lib):
    b = _batch([5, 64, 300], 16, 2, 128, 16, "float32", seed=9)
    _compare(b, repeats=1)


def test_counters_at_rest_after_fused_steps(built_lib):
    b = _batch([512], 14, 2, 64, 8, "bfloat16", seed=13)
    for _ in range(3):
        S = b.num_decode
        A.paged_attention_with_rope(b.query[:S].contiguous(), b.key[:S].reshape(S, -1).clone(),
                                    b.value[:S], b.key_cache, b.value_cache, b.block_tables,
                                    b.seq_lens, b.cos_sin_cache, b.scale)
    torch.cuda.synchronize()
    ws = A._workspaces[(torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)]
    assert int(ws.buf[:ws.clean].count_nonzero()) == 0
