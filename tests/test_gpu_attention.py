"""Paged attention on the GPU (through cscr.attention -> C ABI) against the oracle."""

import glob
import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from cscr import _lib
from cscr import attention as A
from helpers import HALF_TOL, check_attention, oracle_attention_f32, tol_for
from oracle import decode_oracle as O
from paged_decode import workloads as W

pytestmark = pytest.mark.gpu

ATTN_CASES = sorted(glob.glob(str(GOLDEN / "attn_ref_test_*.npz")))


def _long_tail_shard():
    """The long-tail batch's 4-GPU shard that holds its 10295-token sequence
    (31 sequences): each of that sequence's two units is cut into 81 pieces."""
    from paged_decode import partition as Pn

    lens = W.long_tail_lengths(0, 256)
    for shard in Pn.lpt_assign(lens, 4):
        if max(lens[i] for i in shard) == max(lens):
            return [lens[i] for i in shard]
    raise AssertionError("no shard holds the longest sequence")


LONG_TAIL_SHARD = _long_tail_shard()


def _attend(batch, query=None):
    q = batch.query[batch.decode_rows] if query is None else query
    return A.paged_attention(q.contiguous(), batch.key_cache, batch.value_cache,
                             batch.block_tables, batch.seq_lens, batch.scale)


@pytest.fixture(autouse=True)
def _clean_status():
    torch.cuda.set_device(0)
    _lib.device_status(clear=True)
    yield
    torch.cuda.synchronize()


@pytest.mark.parametrize("path", ATTN_CASES, ids=lambda p: p.split("/")[-1][:-4])
def test_reference_test_cases(path, built_lib):
    """The reference test's own case (seed 0, lens [13,1,16], hd 64, bs 8) and its oracle."""
    z = np.load(path)
    dtype = str(z["dtype"])
    tdt = W.TORCH_DTYPES[dtype]
    dev = "cuda"
    out = A.paged_attention(
        query=W.from_numpy(z["query"], tdt, dev), key_cache=W.from_numpy(z["key_cache"], tdt, dev),
        value_cache=W.from_numpy(z["value_cache"], tdt, dev),
        block_tables=torch.from_numpy(z["block_tables"]).to(dev),
        seq_lens=torch.from_numpy(z["seq_lens"]).to(dev), scale=float(z["scale"]))
    got = O.to_f32(W.to_numpy(out), dtype)
    ref = O.to_f32(z["ref"], dtype)
    np.testing.assert_allclose(got, ref, atol=float(z["atol"]), rtol=float(z["rtol"]))
    ref32 = oracle_attention_f32(z["query"], z["key_cache"], z["value_cache"], z["block_tables"],
                                 z["seq_lens"], float(z["scale"]), dtype)
    np.testing.assert_allclose(got, ref32, **tol_for(dtype))


def test_uniform_small_fp32(built_lib):
    batch = W.make_batch(W.uniform_small(0))
    check_attention(batch, _attend(batch))


def test_qwen3b_decode_bf16(built_lib):
    batch = W.make_batch(W.qwen3b_decode(0))
    out = _attend(batch)
    check_attention(batch, out)
    # deterministic: a second call (same workspace, counters back at zero) is bit-identical
    out2 = _attend(batch)
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    assert _lib.device_status() == 0


def test_ragged_batch_decode_fp16(built_lib):
    batch = W.make_batch(W.ragged_batch(0))
    check_attention(batch, _attend(batch))


def test_long_tail_bs32_high_block_ids(built_lib):
    """Heavy-tailed lengths (Pareto 1.2, up to 32k) in a pool whose byte offsets pass 2^31."""
    lens = W.long_tail_lengths(0)
    spec = W.long_tail(0, lens=lens, num_blocks=160_000)  # 160k x 32 KB = 5 GB
    batch = W.make_batch(spec)
    assert batch.block_tables.max().item() * 16 * 1024 > 2 ** 31
    out = _attend(batch)
    check_attention(batch, out)  # every one of the 256 sequences


@pytest.mark.parametrize("heads", ["qwen0.5b", "qwen3b"])
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("context", [512, 8192])
@pytest.mark.parametrize("batch_size", [1, 32, 256])
@pytest.mark.parametrize("block_size", [8, 16, 32])
def test_sweep_point(block_size, batch_size, context, dtype, heads, built_lib):
    spec = W.sweep_point(block_size, batch_size, context, dtype, heads)
    batch = W.make_batch(spec)
    check_attention(batch, _attend(batch))  # every sequence of the point


def _custom_batch(lens, H, KVH, D, bs, dtype, nb_extra=8, seed=0):
    spec = W.DecodeSpec("custom", list(lens), H, KVH, D, bs, dtype,
                        num_blocks=sum(math.ceil(max(L, 0) / bs) for L in lens) + nb_extra,
                        seed=seed)
    return W.make_batch(spec)


@pytest.mark.parametrize("H,KVH,D", [(14, 2, 64), (16, 1, 128), (8, 8, 128), (12, 1, 64),
                                     (4, 2, 64), (32, 2, 128)])
@pytest.mark.parametrize("bs", [8, 16, 32, 64])
def test_head_groupings_and_block_sizes(H, KVH, D, bs, built_lib):
    batch = _custom_batch([1, 2, 15, 16, 17, 100, 333, 1024, 0, 77], H, KVH, D, bs, "bfloat16")
    check_attention(batch, _attend(batch))


@pytest.mark.parametrize("D", [32, 80, 96, 256])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_generic_path_head_dims(D, dtype, built_lib):
    batch = _custom_batch([5, 64, 300, 1], 8, 2, D, 16, dtype)
    check_attention(batch, _attend(batch))


def test_block_size_128_generic(built_lib):
    batch = _custom_batch([5, 130, 700], 16, 2, 128, 128, "float16")
    check_attention(batch, _attend(batch))


def test_negative_blocks_and_empty_sequences(built_lib):
    batch = _custom_batch([0, 40, 40, 1, 64, 0, 200], 16, 2, 128, 16, "bfloat16")
    bt = batch.block_tables.clone()
    bt[1, 1] = -1       # middle block of a sequence skipped
    bt[3, 0] = -1       # the only block of a 1-token sequence: empty softmax -> 0
    bt[4, :] = -1       # all blocks skipped
    batch.block_tables = bt
    out = _attend(batch)
    check_attention(batch, out)
    o = out.float()
    assert torch.all(o[0] == 0) and torch.all(o[3] == 0) and torch.all(o[4] == 0)
    assert torch.all(o[5] == 0)


def test_nan_in_unused_slots_does_not_leak(built_lib):
    """Slots past the context (and unused pool blocks) may hold anything, NaN included."""
    batch = _custom_batch([17, 33, 1, 250, 4000], 16, 2, 128, 16, "bfloat16", nb_extra=32)
    kc, vc = batch.key_cache, batch.value_cache
    bs = 16
    for s, L in enumerate(batch.seq_lens.tolist()):
        last = batch.block_tables[s, (L - 1) // bs].item()
        kc[last, :, (L - 1) % bs + 1:] = float("nan")
        vc[last, :, (L - 1) % bs + 1:] = float("nan")
    used = set(batch.block_tables[batch.block_tables >= 0].tolist())
    unused = [b for b in range(kc.shape[0]) if b not in used]
    kc[unused] = float("nan")
    vc[unused] = float("nan")
    out = _attend(batch)
    assert torch.isfinite(out.float()).all()
    check_attention(batch, out)


def test_seq_len_beyond_table_is_clamped(built_lib):
    batch = _custom_batch([64, 64], 16, 2, 128, 16, "bfloat16")
    batch.seq_lens = torch.tensor([64, 500], dtype=torch.int32, device="cuda")  # 500 > 4*16
    out = _attend(batch)
    assert _lib.device_status() & 0x2
    batch.seq_lens = torch.tensor([64, 64], dtype=torch.int32, device="cuda")
    check_attention(batch, out)


def test_block_id_outside_pool_is_skipped_and_flagged(built_lib):
    batch = _custom_batch([48, 48], 16, 2, 128, 16, "bfloat16")
    bt = batch.block_tables.clone()
    bt[1, 1] = batch.key_cache.shape[0] + 5
    batch.block_tables = bt
    out = _attend(batch)
    assert _lib.device_status() & 0x1
    bt2 = bt.clone()
    bt2[1, 1] = -1
    batch.block_tables = bt2
    check_attention(batch, out)


def test_single_long_sequence_splits(built_lib):
    """One 32k-token sequence is spread over every CTA and merged from partials."""
    batch = _custom_batch([32768], 16, 2, 128, 16, "bfloat16")
    check_attention(batch, _attend(batch))


def test_many_short_sequences(built_lib):
    batch = _custom_batch([1 + (i % 7) for i in range(2000)], 16, 2, 128, 16, "float16")
    check_attention(batch, _attend(batch))


def test_workspace_reuse_across_growing_batches(built_lib):
    """Small batches dirty the scratch that a later, larger batch uses for its
    arrival counters; the op must re-zero that prefix before the larger call."""
    for S in (1, 3, 40, 600, 5, 1200):
        batch = _custom_batch([700 + 37 * i for i in range(S)], 14, 2, 64, 16, "bfloat16")
        check_attention(batch, _attend(batch))


def test_two_streams_use_separate_workspaces(built_lib):
    b1 = W.make_batch(W.qwen3b_decode(1, batch=16))
    b2 = W.make_batch(W.qwen3b_decode(2, batch=16))
    ref1, ref2 = _attend(b1), _attend(b2)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()
    for _ in range(3):
        with torch.cuda.stream(s1):
            o1 = _attend(b1)
        with torch.cuda.stream(s2):
            o2 = _attend(b2)
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int16), ref1.view(torch.int16))
    assert torch.equal(o2.view(torch.int16), ref2.view(torch.int16))


def test_cpu_tensor_raises_reference_message():
    q = torch.zeros(1, 2, 64)
    with pytest.raises(RuntimeError, match="query must be a CUDA tensor"):
        A.paged_attention(q, q.view(1, 2, 1, 64), q.view(1, 2, 1, 64),
                          torch.zeros(1, 1, dtype=torch.int32), torch.ones(1, dtype=torch.int32), 1.0)


@pytest.mark.parametrize("H,KVH,D,bs,lens", [
    (14, 2, 64, 8, [512]),                       # one sequence cut into many pieces
    (16, 2, 128, 16, [512]),
    (14, 2, 64, 16, [1, 2, 15, 16, 17, 100, 333, 1024, 0, 77]),
    (16, 1, 128, 64, [4096, 3, 700]),
    (32, 2, 128, 32, [8192, 9, 2000]),             # two head tiles (group 16)
    (16, 2, 128, 32, LONG_TAIL_SHARD),             # 81 pieces: staged in chunks
    (8, 1, 128, 32, [32768] + [32] * 300),        # 128 pieces: the epilogue warp merges
])
def test_counters_are_zero_after_every_launch(H, KVH, D, bs, lens, built_lib):
    """Split pieces meet on per-(sequence, kv head) arrival counters that every
    launch must leave at zero; a count that never completes would corrupt the
    next launch on the same stream."""
    batch = _custom_batch(lens, H, KVH, D, bs, "bfloat16")
    for _ in range(3):
        out = _attend(batch)
        check_attention(batch, out)
    torch.cuda.synchronize()
    ws = A._workspaces[(torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)]
    assert ws.clean > 0 and int(ws.buf[:ws.clean].count_nonzero()) == 0


@pytest.mark.parametrize("lens,H,KVH,D", [
    ("qwen3b", 16, 2, 128),                 # the 3B decode batch: many two- to five-piece splits
    ([8192, 8192, 300, 5000], 14, 2, 64),   # head dim 64, units cut into 8+ pieces
    ([20000], 16, 2, 128),                  # 32 pieces, two staged chunks
    (LONG_TAIL_SHARD, 16, 2, 128),          # 81 pieces, staged in six chunks
    ([32768] + [32] * 300, 8, 1, 128),      # 128 pieces: more than the consumer warps merge
])
def test_split_merges_give_the_same_bits_every_launch(lens, H, KVH, D, built_lib):
    """Which piece of a split (sequence, kv head) finishes last changes from
    launch to launch, and with it the warps that merge: the epilogue warp or
    the consumer warps of a CTA whose last piece it was. Both use the same
    arithmetic in the same order, so every launch gives the same bits."""
    if lens == "qwen3b":
        batch = W.make_batch(W.qwen3b_decode(5, batch=64))
    else:
        batch = _custom_batch(lens, H, KVH, D, 16, "bfloat16")
    first = _attend(batch)
    for i in range(30):
        out = _attend(batch)
        assert torch.equal(out.view(torch.int16), first.view(torch.int16)), f"launch {i}"
    assert _lib.device_status() == 0
