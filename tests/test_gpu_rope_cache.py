"""RoPE, the KV-cache writes and their fused form on the GPU against the oracle."""

import glob

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from cscr import _lib
from cscr import cache as C
from cscr import pos_encoding as PE
from helpers import tol_for
from oracle import decode_oracle as O
from paged_decode import workloads as W

pytestmark = pytest.mark.gpu

WRITE_CASES = sorted(glob.glob(str(GOLDEN / "write_kv_*.npz")))


@pytest.fixture(autouse=True)
def _clean_status():
    torch.cuda.set_device(0)
    _lib.device_status(clear=True)
    yield
    torch.cuda.synchronize()


def _rope_case(T, H, KVH, hs, rot, dtype, maxpos=4096, theta=1e6, pos_dtype=torch.int64, seed=0):
    g = torch.Generator().manual_seed(seed)
    tdt = W.TORCH_DTYPES[dtype]
    q = torch.randn(T, H * hs, generator=g).to(tdt).cuda()
    k = torch.randn(T, KVH * hs, generator=g).to(tdt).cuda()
    pos = torch.randint(0, maxpos, (T,), generator=g).to(pos_dtype).cuda()
    cs = W.cos_sin_table(rot, maxpos, theta, tdt).cuda()
    return q, k, pos, cs


def _check_rope(q, k, pos, cs, hs, dtype, out, k_after):
    ref_out, ref_k = O.rotary_embedding_neox(W.to_numpy(pos), W.to_numpy(q), W.to_numpy(k), hs,
                                             W.to_numpy(cs), dtype)
    tol = tol_for(dtype)
    np.testing.assert_allclose(O.to_f32(W.to_numpy(out), dtype), O.to_f32(ref_out, dtype), **tol)
    np.testing.assert_allclose(O.to_f32(W.to_numpy(k_after), dtype), O.to_f32(ref_k, dtype), **tol)
    # The kernel rounds each product and the sum on its own, as the oracle's
    # fp32 numpy expression does, then rounds once to the storage dtype: the
    # same bits, every dtype.
    assert np.array_equal(W.to_numpy(out), ref_out)
    assert np.array_equal(W.to_numpy(k_after), ref_k)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("pos_dtype", [torch.int64, torch.int32])
def test_rope_qwen3b_decode_shape(dtype, pos_dtype, built_lib):
    q, k, pos, cs = _rope_case(64, 16, 2, 128, 128, dtype, pos_dtype=pos_dtype)
    k0 = k.clone()
    out = PE.rotary_embedding_neox(pos, q, k, 128, cs)
    _check_rope(q, k0, pos, cs, 128, dtype, out, k)


@pytest.mark.parametrize("hs,rot", [(128, 64), (64, 64), (72, 72), (80, 32), (64, 16)])
def test_rope_partial_rotary_and_scalar_path(hs, rot, built_lib):
    q, k, pos, cs = _rope_case(33, 3, 1, hs, rot, "bfloat16", maxpos=300, theta=1e4)
    k0 = k.clone()
    out = PE.rotary_embedding_neox(pos, q, k, hs, cs)
    _check_rope(q, k0, pos, cs, hs, "bfloat16", out, k)
    if rot < hs:  # elements beyond rot pass through bit-exact
        qv = q.view(33, 3, hs)[..., rot:]
        assert torch.equal(out.view(33, 3, hs)[..., rot:].view(torch.int16), qv.view(torch.int16))
        kv = k0.view(33, 1, hs)[..., rot:]
        assert torch.equal(k.view(33, 1, hs)[..., rot:].view(torch.int16), kv.view(torch.int16))


def test_rope_ragged_batch_tokens(built_lib):
    spec = W.ragged_batch(0)
    batch = W.make_batch(spec, fill_cache=False)
    T = batch.query.shape[0]
    assert T > 1000
    q = batch.query.reshape(T, -1).contiguous()
    k = batch.key.reshape(T, -1).contiguous()
    k0 = k.clone()
    out = PE.rotary_embedding_neox(batch.positions, q, k, 128, batch.cos_sin_cache)
    _check_rope(q, k0, batch.positions, batch.cos_sin_cache, 128, "float16", out, k)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("slot_dtype", [torch.int64, torch.int32])
def test_reshape_and_cache_bit_exact(dtype, slot_dtype, built_lib):
    spec = W.DecodeSpec("w", [5, 17, 300, 16, 1], 16, 2, 128, 16, dtype, num_blocks=64)
    batch = W.make_batch(spec)
    slots = batch.slot_mapping.clone()
    slots[2] = -1
    slots = slots.to(slot_dtype)
    kc_ref, vc_ref = W.to_numpy(batch.key_cache), W.to_numpy(batch.value_cache)
    O.reshape_and_cache(W.to_numpy(batch.key), W.to_numpy(batch.value), kc_ref, vc_ref,
                        W.to_numpy(slots))
    C.reshape_and_cache(batch.key, batch.value, batch.key_cache, batch.value_cache, slots)
    assert np.array_equal(W.to_numpy(batch.key_cache), kc_ref)
    assert np.array_equal(W.to_numpy(batch.value_cache), vc_ref)


@pytest.mark.parametrize("path", WRITE_CASES, ids=lambda p: p.split("/")[-1][:-4])
def test_write_kv_cache_matches_reference_fixture(path, built_lib):
    """_write_kv_cache semantics (block_tables[row, pos // bs], skip < 0) bit for bit."""
    z = np.load(path)
    tdt = W.TORCH_DTYPES[str(z["dtype"])]
    kc = W.from_numpy(z["key_cache_in"], tdt, "cuda")
    vc = W.from_numpy(z["value_cache_in"], tdt, "cuda")
    C.write_kv_cache(W.from_numpy(z["key"], tdt, "cuda"), W.from_numpy(z["value"], tdt, "cuda"),
                     torch.from_numpy(z["positions"]).cuda(), kc, vc,
                     torch.from_numpy(z["block_tables"]).cuda())
    assert np.array_equal(W.to_numpy(kc), z["key_cache_out"])
    assert np.array_equal(W.to_numpy(vc), z["value_cache_out"])


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("by_table", [False, True])
def test_fused_rope_cache_equals_separate_ops(dtype, by_table, built_lib):
    spec = W.DecodeSpec("f", [5, 17, 300, 16, 1, 4096, 2000, 64], 16, 2, 128, 16, dtype,
                        num_blocks=1024, rope_theta=1e6, max_position=4096)
    a = W.make_batch(spec)
    T = a.query.shape[0]
    q = a.query.reshape(T, -1).contiguous()
    k1 = a.key.reshape(T, -1).contiguous()
    k2 = k1.clone()
    kc1, vc1 = a.key_cache.clone(), a.value_cache.clone()
    kc2, vc2 = a.key_cache.clone(), a.value_cache.clone()
    # separate: rope, then the cache write
    out1 = PE.rotary_embedding_neox(a.positions, q, k1, 128, a.cos_sin_cache)
    C.reshape_and_cache(k1, a.value, kc1, vc1, a.slot_mapping)
    # fused
    if by_table:
        out2 = PE.rotary_embedding_neox_with_cache(a.positions, q, k2, a.value, kc2, vc2, None,
                                                   128, a.cos_sin_cache,
                                                   block_tables=a.token_block_tables)
    else:
        out2 = PE.rotary_embedding_neox_with_cache(a.positions, q, k2, a.value, kc2, vc2,
                                                   a.slot_mapping, 128, a.cos_sin_cache)
    for x, y in ((out1, out2), (k1, k2), (kc1, kc2), (vc1, vc2)):
        assert torch.equal(x.view(torch.int16), y.view(torch.int16))


def test_overlap_previous_waits_for_the_kernel_before_it(built_lib):
    """With overlap_previous the fused launch starts during the attention
    kernel before it. That attention reads the very cache rows the launch
    writes (each sequence's newest token), so an early write would change
    its output; the predecessor-written query must also be read fresh."""
    from cscr import attention as A

    b = W.make_batch(W.qwen3b_decode(3, batch=64))
    S = b.num_decode
    q_attn = b.query[:S].contiguous()
    kc0, vc0 = b.key_cache.clone(), b.value_cache.clone()
    ref_attn = A.paged_attention(q_attn, kc0, vc0, b.block_tables, b.seq_lens, b.scale)
    q2 = b.query.reshape(S, -1).contiguous()
    k0 = b.key.reshape(S, -1).clone()  # the launches rotate their key in place
    k_ref = k0.clone()
    kc_ref, vc_ref = kc0.clone(), vc0.clone()
    rope_ref = PE.rotary_embedding_neox_with_cache(b.positions, q2, k_ref, b.value, kc_ref, vc_ref,
                                                   b.slot_mapping, 128, b.cos_sin_cache)
    torch.cuda.synchronize()
    for _ in range(3):
        kc, vc = kc0.clone(), vc0.clone()
        k = k0.clone()
        q_in = torch.zeros_like(q2)
        torch.cuda.synchronize()
        q_in.copy_(q2)  # a kernel that writes the query just before the launch
        out_attn = A.paged_attention(q_attn, kc, vc, b.block_tables, b.seq_lens, b.scale)
        rope = PE.rotary_embedding_neox_with_cache(b.positions, q_in, k, b.value, kc, vc,
                                                   b.slot_mapping, 128, b.cos_sin_cache,
                                                   overlap_previous=True)
        torch.cuda.synchronize()
        assert torch.equal(out_attn.view(torch.int16), ref_attn.view(torch.int16))
        for x, y in ((rope, rope_ref), (k, k_ref), (kc, kc_ref), (vc, vc_ref)):
            assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    # after a non-kernel predecessor as well
    kc, vc = kc0.clone(), vc0.clone()
    k = k0.clone()
    q_host = q2.cpu().pin_memory()
    q_in = torch.zeros_like(q2)
    torch.cuda.synchronize()
    q_in.copy_(q_host, non_blocking=True)
    rope = PE.rotary_embedding_neox_with_cache(b.positions, q_in, k, b.value, kc, vc,
                                               b.slot_mapping, 128, b.cos_sin_cache,
                                               overlap_previous=True)
    torch.cuda.synchronize()
    assert torch.equal(rope.view(torch.int16), rope_ref.view(torch.int16))
    assert _lib.device_status() == 0


def test_fused_rope_cache_ragged_batch_against_oracle(built_lib):
    spec = W.ragged_batch(1)
    b = W.make_batch(spec)
    T = b.query.shape[0]
    q = b.query.reshape(T, -1).contiguous()
    k = b.key.reshape(T, -1).contiguous()
    q_np, k_np, v_np = W.to_numpy(q), W.to_numpy(k), W.to_numpy(b.value)
    slots = W.to_numpy(b.slot_mapping)
    touched = np.unique(slots // 16)
    kc_before = W.to_numpy(b.key_cache[torch.from_numpy(touched).cuda()])
    vc_before = W.to_numpy(b.value_cache[torch.from_numpy(touched).cuda()])
    out = PE.rotary_embedding_neox_with_cache(b.positions, q, k, b.value, b.key_cache,
                                              b.value_cache, b.slot_mapping, 128, b.cos_sin_cache)
    ref_out, ref_k = O.rotary_embedding_neox(W.to_numpy(b.positions), q_np, k_np, 128,
                                             W.to_numpy(b.cos_sin_cache), "float16")
    assert np.array_equal(W.to_numpy(out), ref_out)
    # the cache must hold exactly the key the kernel left in `key`, and the value
    remap = {int(bk): i for i, bk in enumerate(touched)}
    kc_ref, vc_ref = kc_before.copy(), vc_before.copy()
    local = np.array([remap[int(s) // 16] * 16 + int(s) % 16 for s in slots])
    O.reshape_and_cache(W.to_numpy(k), v_np, kc_ref, vc_ref, local)
    idx = torch.from_numpy(touched).cuda()
    assert np.array_equal(W.to_numpy(b.key_cache[idx]), kc_ref)
    assert np.array_equal(W.to_numpy(b.value_cache[idx]), vc_ref)
    assert np.array_equal(W.to_numpy(k), ref_k)


def test_bad_position_and_slot_are_flagged_not_faulting(built_lib):
    q, k, pos, cs = _rope_case(4, 2, 1, 64, 64, "bfloat16", maxpos=16, theta=1e4)
    pos[1] = 10_000
    PE.rotary_embedding_neox(pos, q, k, 64, cs)
    assert _lib.device_status() & 0x4
    kc = torch.zeros(4, 1, 8, 64, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, 5, 4 * 8 + 3, -1], dtype=torch.int64, device="cuda")
    C.reshape_and_cache(k.view(4, 1, 64), k.view(4, 1, 64), kc, vc, slots)
    assert _lib.device_status() & 0x8
    assert torch.equal(kc[0, 0, 0], k[0]) and torch.equal(kc[0, 0, 5], k[1])


def test_rope_cpu_tensors_raise_reference_message():
    q = torch.zeros(2, 64)
    with pytest.raises(RuntimeError, match="positions must be a CUDA tensor"):
        PE.rotary_embedding_neox(torch.zeros(2, dtype=torch.int64), q, q.clone(), 64,
                                 torch.zeros(8, 64))
