"""Prefill (causal, multi-token) paged attention on the GPU against the oracle.

The reference has no prefill op (its layer is decode-only), so the oracle is
the reference test's attention math with a causal mask
(oracle.decode_oracle.paged_prefill_attention_f32). Its last row of every
chunk is the decode attention of that sequence, which ties it to the pinned
decode oracle; the CPU tests check that.
"""

import math

import numpy as np
import pytest
import torch

from cscr import _lib
from cscr import attention as A
from cscr import pos_encoding as PE
from helpers import HALF_TOL
from oracle import decode_oracle as O
from paged_decode import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device():
    torch.cuda.set_device(0)
    _lib.device_status(clear=True)
    yield
    torch.cuda.synchronize()


def _check(q, kc, vc, bt, qs, ctx, scale, dtype, out):
    ref = O.paged_prefill_attention_f32(W.to_numpy(q), W.to_numpy(kc), W.to_numpy(vc),
                                        W.to_numpy(bt), W.to_numpy(qs), W.to_numpy(ctx), scale,
                                        dtype, threads=8)
    qs_np = W.to_numpy(qs)
    rows = np.concatenate([np.arange(qs_np[c], qs_np[c + 1]) for c in range(len(qs_np) - 1)])
    got = O.to_f32(W.to_numpy(out), dtype)
    np.testing.assert_allclose(got[rows], ref[rows], **HALF_TOL)


def test_ragged_batch_prompt_chunks(built_lib):
    """Config 3's four prompt chunks (U[256, 2048] tokens, fp16, 16/2 heads, hd
    128): RoPE + cache write of the whole packed step, then causal attention of
    each prompt over itself."""
    spec = W.ragged_batch(0)
    b = W.make_batch(spec)
    T = b.query.shape[0]
    q_rot = PE.rotary_embedding_neox_with_cache(b.positions, b.query.view(T, -1),
                                                b.key.view(T, -1), b.value, b.key_cache,
                                                b.value_cache, b.slot_mapping, 128,
                                                b.cos_sin_cache)
    lens = spec.prefill_lens
    starts = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tables = torch.stack([b.token_block_tables[int(starts[c])] for c in range(len(lens))])
    qs = torch.from_numpy(starts).cuda()
    ctx = torch.tensor(lens, dtype=torch.int32, device="cuda")
    qp = q_rot.view(T, 16, 128)[: starts[-1]].contiguous()
    out = A.paged_prefill_attention(qp, b.key_cache, b.value_cache, tables, qs, ctx, b.scale,
                                    max_query_len=max(lens))
    torch.cuda.synchronize()
    _check(qp, b.key_cache, b.value_cache, tables, qs, ctx, b.scale, "float16", out)
    assert _lib.device_status() == 0


def _chunks_case(chunk_lens, ctx_lens, H, KVH, D, bs, dtype, seed=0, nb_extra=8):
    """Random pool with one sequence per chunk of ctx_lens[c] tokens; the chunk
    is the last chunk_lens[c] tokens."""
    g = torch.Generator().manual_seed(seed)
    tdt = W.TORCH_DTYPES[dtype]
    nblk = [math.ceil(L / bs) for L in ctx_lens]
    NB = sum(nblk) + nb_extra
    perm = torch.randperm(NB, generator=g).to(torch.int32)
    maxB = max(nblk + [1])
    bt = torch.full((len(ctx_lens), maxB), -1, dtype=torch.int32)
    off = 0
    for c, n in enumerate(nblk):
        bt[c, :n] = perm[off:off + n]
        off += n
    kc = torch.randn(NB, KVH, bs, D, generator=g).to(tdt)
    vc = torch.randn(NB, KVH, bs, D, generator=g).to(tdt)
    T = sum(chunk_lens)
    q = torch.randn(T, H, D, generator=g).to(tdt)
    qs = torch.tensor([0] + np.cumsum(chunk_lens).tolist(), dtype=torch.int32)
    ctx = torch.tensor(ctx_lens, dtype=torch.int32)
    return [x.cuda() for x in (q, kc, vc, bt, qs, ctx)]


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("H,KVH,D", [(16, 2, 128), (14, 2, 64), (8, 8, 128), (32, 2, 64)])
@pytest.mark.parametrize("bs", [8, 16, 32, 64])
def test_prompt_and_chunked_prefill_shapes(dtype, H, KVH, D, bs, built_lib):
    # fresh prompts, a chunk after prior context, a one-token chunk (= decode),
    # lengths off the 64-token tiles, an empty chunk
    chunk_lens = [1, 63, 64, 65, 200, 0, 100]
    ctx_lens = [1, 63, 64, 65, 200, 10, 1000]
    q, kc, vc, bt, qs, ctx = _chunks_case(chunk_lens, ctx_lens, H, KVH, D, bs, dtype)
    out = A.paged_prefill_attention(q, kc, vc, bt, qs, ctx, D ** -0.5)
    torch.cuda.synchronize()
    _check(q, kc, vc, bt, qs, ctx, D ** -0.5, dtype, out)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("bs", [4, 24, 128, 192])
def test_block_sizes_off_the_tma_tiling(dtype, bs, built_lib):
    """Block sizes 4 and 24 take the kernel's cp.async loader (a TMA box of a
    block would not tile a 64-token tile); 128 and 192 take TMA copies of a
    64-row part of a block."""
    chunk_lens = [1, 63, 64, 65, 200, 0, 100]
    ctx_lens = [1, 63, 64, 65, 200, 10, 1000]
    q, kc, vc, bt, qs, ctx = _chunks_case(chunk_lens, ctx_lens, 16, 2, 128, bs, dtype, seed=bs)
    out = A.paged_prefill_attention(q, kc, vc, bt, qs, ctx, 128 ** -0.5)
    torch.cuda.synchronize()
    _check(q, kc, vc, bt, qs, ctx, 128 ** -0.5, dtype, out)
    assert _lib.device_status() == 0


def test_stale_nan_slots_past_the_context_never_leak(built_lib):
    """Cache slots past each chunk's context (inside its last block) and the
    whole of an unmapped block hold NaN: the output stays finite and matches
    the oracle, which never reads them."""
    chunk_lens, ctx_lens = [70, 33, 130], [70, 97, 130]
    q, kc, vc, bt, qs, ctx = _chunks_case(chunk_lens, ctx_lens, 16, 2, 128, 16, "bfloat16",
                                          seed=5)
    for c, L in enumerate(ctx_lens):
        last = int(bt[c, (L - 1) // 16])
        kc[last, :, L % 16 or 16:] = float("nan")
        vc[last, :, L % 16 or 16:] = float("nan")
    spare = sorted(set(range(kc.shape[0])) - set(bt[bt >= 0].tolist()))
    kc[spare] = float("nan")
    vc[spare] = float("nan")
    out = A.paged_prefill_attention(q, kc, vc, bt, qs, ctx, 128 ** -0.5)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    _check(q, kc, vc, bt, qs, ctx, 128 ** -0.5, "bfloat16", out)
    assert _lib.device_status() == 0


def test_last_row_of_each_chunk_equals_decode_attention(built_lib):
    chunk_lens, ctx_lens = [300, 17, 1, 900], [300, 517, 4000, 900]
    q, kc, vc, bt, qs, ctx = _chunks_case(chunk_lens, ctx_lens, 16, 2, 128, 16, "bfloat16",
                                          seed=3)
    out = A.paged_prefill_attention(q, kc, vc, bt, qs, ctx, 128 ** -0.5)
    last = (qs[1:] - 1).long()
    dec = A.paged_attention(q[last].contiguous(), kc, vc, bt, ctx, 128 ** -0.5)
    torch.cuda.synchronize()
    np.testing.assert_allclose(O.to_f32(W.to_numpy(out[last]), "bfloat16"),
                               O.to_f32(W.to_numpy(dec), "bfloat16"), atol=4e-3, rtol=2e-2)


def test_negative_blocks_skipped_and_empty_rows_zero(built_lib):
    chunk_lens, ctx_lens = [40, 40], [40, 40]
    q, kc, vc, bt, qs, ctx = _chunks_case(chunk_lens, ctx_lens, 16, 2, 128, 16, "float16")
    bt[0, 0] = -1      # tokens 0..15 of chunk 0 skipped: its rows 0..15 see nothing -> 0
    bt[1, 1] = -1      # a middle block of chunk 1 skipped
    out = A.paged_prefill_attention(q, kc, vc, bt, qs, ctx, 128 ** -0.5)
    torch.cuda.synchronize()
    assert torch.all(out[:16].float() == 0)
    _check(q, kc, vc, bt, qs, ctx, 128 ** -0.5, "float16", out)
    assert _lib.device_status() == 0


def test_long_prompt_many_tiles(built_lib):
    chunk_lens, ctx_lens = [4096, 3000], [4096, 8192]
    q, kc, vc, bt, qs, ctx = _chunks_case(chunk_lens, ctx_lens, 16, 2, 128, 32, "bfloat16",
                                          seed=9)
    out = A.paged_prefill_attention(q, kc, vc, bt, qs, ctx, 128 ** -0.5, max_query_len=4096)
    torch.cuda.synchronize()
    _check(q, kc, vc, bt, qs, ctx, 128 ** -0.5, "bfloat16", out)


def test_prefill_rejects_fp32_and_odd_head_dims():
    q = torch.zeros(4, 2, 80, dtype=torch.float16, device="cuda")
    kc = torch.zeros(4, 1, 16, 80, dtype=torch.float16, device="cuda")
    bt = torch.zeros(1, 1, dtype=torch.int32, device="cuda")
    qs = torch.tensor([0, 4], dtype=torch.int32, device="cuda")
    ctx = torch.tensor([4], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim 64 or 128"):
        A.paged_prefill_attention(q, kc, kc, bt, qs, ctx, 0.1, max_query_len=4)
    q32 = torch.zeros(4, 2, 64, device="cuda")
    kc32 = torch.zeros(4, 1, 16, 64, device="cuda")
    with pytest.raises(RuntimeError, match="float16 and bfloat16"):
        A.paged_prefill_attention(q32, kc32, kc32, bt, qs, ctx, 0.1, max_query_len=4)
