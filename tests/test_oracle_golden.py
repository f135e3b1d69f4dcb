"""The CPU oracle against fixtures produced by the reference's own code.

The fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py) hold
inputs and outputs of the reference's test oracle (tests/test_paged_attention
.py:42-57), of ``PagedAttentionWithRoPE._write_kv_cache`` and ``__init__``
(src/model_executor/layers/attention.py:53-116) and of
``Worker._prepare_inputs`` (src/worker/worker.py:84-169).
"""

import glob

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import decode_oracle as O
from paged_decode import workloads as W

ATTN_CASES = sorted(glob.glob(str(GOLDEN / "attn_ref_test_*.npz")))
WRITE_CASES = sorted(glob.glob(str(GOLDEN / "write_kv_*.npz")))
COS_CASES = sorted(glob.glob(str(GOLDEN / "cos_sin_*.npz")))


def test_fixture_inventory():
    assert len(ATTN_CASES) == 9
    assert len(WRITE_CASES) == 6
    assert len(COS_CASES) == 9
    assert (GOLDEN / "decode_meta.npz").exists()


@pytest.mark.parametrize("path", ATTN_CASES, ids=lambda p: p.split("/")[-1][:-4])
def test_attention_oracle_matches_reference_test(path):
    z = np.load(path)
    dtype = str(z["dtype"])
    out = O.paged_attention(z["query"], z["key_cache"], z["value_cache"], z["block_tables"],
                            z["seq_lens"], float(z["scale"]), dtype)
    got = O.to_f32(out, dtype)
    ref = O.to_f32(z["ref"], dtype)
    # Both are fp32 math rounded once to dtype: at most one rounding step apart.
    tol = {"float32": 1e-5, "float16": 1e-3, "bfloat16": 8e-3}[dtype]
    np.testing.assert_allclose(got, ref, atol=tol, rtol=tol)
    # and within the reference test's own tolerance (test_paged_attention.py:59-63)
    np.testing.assert_allclose(got, ref, atol=float(z["atol"]), rtol=float(z["rtol"]))


@pytest.mark.parametrize("path", WRITE_CASES, ids=lambda p: p.split("/")[-1][:-4])
def test_write_kv_oracle_bit_exact(path):
    z = np.load(path)
    kc, vc = z["key_cache_in"].copy(), z["value_cache_in"].copy()
    O.write_kv_cache(z["key"], z["value"], z["positions"], kc, vc, z["block_tables"])
    assert np.array_equal(kc.view(np.uint8), z["key_cache_out"].view(np.uint8))
    assert np.array_equal(vc.view(np.uint8), z["value_cache_out"].view(np.uint8))
    # the slot-mapping form of the same write gives the same bits
    bs = kc.shape[2]
    pos = z["positions"].astype(np.int64)
    blk = z["block_tables"][np.arange(len(pos)), pos // bs].astype(np.int64)
    slots = np.where(blk >= 0, blk * bs + pos % bs, -1)
    kc2, vc2 = z["key_cache_in"].copy(), z["value_cache_in"].copy()
    O.reshape_and_cache(z["key"], z["value"], kc2, vc2, slots)
    assert np.array_equal(kc2.view(np.uint8), z["key_cache_out"].view(np.uint8))
    assert np.array_equal(vc2.view(np.uint8), z["value_cache_out"].view(np.uint8))


def test_write_kv_fixture_skips_negative_blocks():
    z = np.load(GOLDEN / "write_kv_float32_bs16.npz")
    bt = z["block_tables"]
    assert (bt < 0).sum() == 2  # the fixture really exercises the skip rule
    changed = (z["key_cache_in"] != z["key_cache_out"]).any(axis=(1, 2, 3))
    assert changed.sum() == len(z["positions"]) - 2


def test_step_metadata_oracle():
    """A prompt + decode step: prompt slots, decode slots and padded positions
    exactly as the reference's _prepare_inputs formed them."""
    z = np.load(GOLDEN / "step_meta.npz")
    pos, slots = O.step_metadata(z["prompt_lens"], z["prompt_tables"], z["context_lens"],
                                 z["decode_tables"], int(z["block_size"]))
    assert np.array_equal(pos, z["positions_padded"])
    assert np.array_equal(slots, z["slots"])
    assert len(pos) == int(z["num_tokens_padded"]) and len(pos) % 8 == 0
    assert np.array_equal(z["context_lens"], z["captured_context_lens"])


def test_decode_metadata_oracle():
    z = np.load(GOLDEN / "decode_meta.npz")
    pos, slots = O.decode_metadata(z["context_lens"], z["block_tables"], int(z["block_size"]))
    assert np.array_equal(pos, z["positions"])
    assert np.array_equal(slots, z["slots"])


@pytest.mark.parametrize("path", COS_CASES, ids=lambda p: p.split("/")[-1][:-4])
def test_cos_sin_table_glue_bit_exact(path):
    """The layer glue and the workload builder rebuild the reference's table bit for bit."""
    from paged_decode.layers import PagedAttentionWithRoPE

    z = np.load(path)
    build = W.TORCH_DTYPES[str(z["build"])]
    rot, base, maxpos = int(z["rot"]), int(z["base"]), int(z["max_position"])
    prev = torch.get_default_dtype()
    torch.set_default_dtype(build)
    try:
        layer = PagedAttentionWithRoPE(4, rot, rot ** -0.5, rot, maxpos, base)
    finally:
        torch.set_default_dtype(prev)
    assert np.array_equal(W.to_numpy(layer.cos_sin_cache), z["table"])
    t2 = W.cos_sin_table(rot, maxpos, base, build, build_dtype=build)
    assert np.array_equal(W.to_numpy(t2), z["table"])


def test_cos_sin_numpy_restatement_close():
    z = np.load(GOLDEN / "cos_sin_float32_rot128_base10000.npz")
    ref = z["table"]
    got = O.cos_sin_cache(128, ref.shape[0], 10000.0)
    np.testing.assert_allclose(got, ref, atol=2e-4, rtol=0)


@pytest.mark.parametrize("dtype", O.DTYPES)
@pytest.mark.parametrize("rot", [64, 32])
def test_rope_oracle_against_torch_restatement(dtype, rot):
    """Independent fp32 torch restatement of pos_encoding_kernel.cu:24-65."""
    g = torch.Generator().manual_seed(1)
    T, H, KVH, hs = 7, 3, 2, 64
    tdt = W.TORCH_DTYPES[dtype]
    q = torch.randn(T, H * hs, generator=g).to(tdt)
    k = torch.randn(T, KVH * hs, generator=g).to(tdt)
    cs = W.cos_sin_table(rot, 100, 10000.0, tdt)
    pos = torch.randint(0, 100, (T,), generator=g)
    out, k_rot = O.rotary_embedding_neox(pos.numpy(), W.to_numpy(q), W.to_numpy(k), hs,
                                         W.to_numpy(cs), dtype)

    def rot_torch(x, nh):
        x = x.float().view(T, nh, hs).clone()
        c = cs.float()[pos][:, None, : rot // 2]
        s = cs.float()[pos][:, None, rot // 2: rot]
        a, b = x[..., : rot // 2].clone(), x[..., rot // 2: rot].clone()
        x[..., : rot // 2] = a * c - b * s
        x[..., rot // 2: rot] = b * c + a * s
        return x.view(T, -1).to(tdt)

    assert np.array_equal(out, W.to_numpy(rot_torch(q, H)))
    assert np.array_equal(k_rot, W.to_numpy(rot_torch(k, KVH)))


def test_oracle_bf16_helpers_round_like_torch():
    x = torch.randn(4096, generator=torch.Generator().manual_seed(3)) * 1000
    bits = O.f32_to_bf16_bits(x.numpy())
    assert np.array_equal(bits, W.to_numpy(x.to(torch.bfloat16)))
    assert np.array_equal(O.bf16_bits_to_f32(bits), x.to(torch.bfloat16).float().numpy())


def test_attention_oracle_semantics_edge_cases():
    """Empty context -> zeros; negative block ids are skipped (attention_kernel.cu:70-72,102)."""
    rng = np.random.default_rng(0)
    S, H, KVH, D, bs, NB = 3, 4, 2, 16, 4, 10
    q = rng.standard_normal((S, H, D)).astype(np.float32)
    kc = rng.standard_normal((NB, KVH, bs, D)).astype(np.float32)
    vc = rng.standard_normal((NB, KVH, bs, D)).astype(np.float32)
    bt = np.array([[0, 1, 2], [3, -1, 4], [5, 6, 7]], np.int32)
    lens = np.array([0, 12, 5], np.int32)
    out = O.paged_attention(q, kc, vc, bt, lens, 0.25, "float32")
    assert np.all(out[0] == 0)
    # seq 1 without its skipped block == seq with only blocks 3 and 4 (8 tokens)
    bt2 = np.array([[3, 4, 0]], np.int32)
    out2 = O.paged_attention(q[1:2], kc, vc, bt2, np.array([8], np.int32), 0.25, "float32")
    np.testing.assert_allclose(out[1], out2[0], rtol=1e-6, atol=1e-6)


def test_prefill_oracle_is_causal_and_ends_in_the_pinned_decode_oracle():
    """The prefill oracle (no reference op exists) against the pinned decode
    oracle: the last row of every chunk is decode attention over the whole
    context, the first row of a fresh prompt sees token 0 only, and changing
    a later token leaves every earlier row unchanged."""
    rng = np.random.default_rng(1)
    H, KVH, D, BS = 8, 2, 64, 8
    lens, ctx = [12, 1, 30], [12, 50, 30]
    T = sum(lens)
    q = rng.standard_normal((T, H, D)).astype(np.float32)
    kc = rng.standard_normal((40, KVH, BS, D)).astype(np.float32)
    vc = rng.standard_normal((40, KVH, BS, D)).astype(np.float32)
    bt = np.full((3, 8), -1, np.int32)
    bt[0, :2] = [3, 9]
    bt[1, :7] = [1, 2, 4, 5, 6, 7, 8]
    bt[2, :4] = [10, 11, 12, 13]
    qs = np.array([0, 12, 13, 43])
    out = O.paged_prefill_attention_f32(q, kc, vc, bt, qs, ctx, 0.125, "float32")
    last = qs[1:] - 1
    dec = O.paged_attention_f32(q[last], kc, vc, bt, np.asarray(ctx), 0.125, "float32")
    np.testing.assert_allclose(out[last], dec, atol=1e-5, rtol=1e-5)
    group = H // KVH
    for h in range(H):
        np.testing.assert_allclose(out[0, h], vc[3, h // group, 0], atol=1e-6)
    kc2 = kc.copy()
    kc2[11, :, 3] += 5.0  # token 8 + 3 = 11 of chunk 2
    out2 = O.paged_prefill_attention_f32(q, kc2, vc, bt, qs, ctx, 0.125, "float32")
    np.testing.assert_array_equal(out2[13:13 + 11], out[13:13 + 11])
    assert not np.allclose(out2[13 + 11:43], out[13 + 11:43])
