"""Block copies, device-side metadata and the layer glue on the GPU."""

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from cscr import _lib
from cscr import cache as C
from helpers import HALF_TOL, check_attention
from oracle import decode_oracle as O
from paged_decode import metadata as M
from paged_decode import workloads as W
from paged_decode.layers import PagedAttentionWithRoPE

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _dev():
    torch.cuda.set_device(0)
    yield
    torch.cuda.synchronize()


def test_copy_blocks_all_layers_one_launch(built_lib):
    g = torch.Generator(device="cuda").manual_seed(0)
    layers = 5
    kcs = [torch.randn(64, 2, 16, 128, generator=g, device="cuda").to(torch.bfloat16)
           for _ in range(layers)]
    vcs = [torch.randn(64, 2, 16, 128, generator=g, device="cuda").to(torch.bfloat16)
           for _ in range(layers)]
    mapping = {3: [10, 11], 7: [40], 0: [63, 1, 2]}
    ref = [W.to_numpy(c) for c in kcs + vcs]
    O.copy_blocks(ref, mapping)
    C.copy_blocks(kcs, vcs, mapping)
    for got, r in zip(kcs + vcs, ref):
        assert np.array_equal(W.to_numpy(got), r)


@pytest.mark.parametrize("direction", ["d2d", "d2h", "h2d", "h2h"])
def test_swap_blocks(direction, built_lib):
    g = torch.Generator().manual_seed(1)
    src = torch.randn(32, 2, 8, 64, generator=g).to(torch.float16)
    dst = torch.randn(48, 2, 8, 64, generator=g).to(torch.float16)
    mapping = {1: 5, 2: 6, 3: 7, 30: 0, 9: 47}
    ref = W.to_numpy(dst).copy()
    O.swap_blocks(W.to_numpy(src), ref, mapping)
    if direction[0] == "d":
        src = src.cuda()
    if direction[2] == "d":
        dst = dst.cuda()
    C.swap_blocks(src, dst, mapping)
    torch.cuda.synchronize()
    assert np.array_equal(W.to_numpy(dst), ref)


def test_copy_blocks_reference_errors():
    with pytest.raises(RuntimeError, match="same number of layers"):
        C.copy_blocks([torch.zeros(2, 2)], [], {0: [1]})
    with pytest.raises(RuntimeError, match="cache tensors must be CUDA tensors"):
        C.copy_blocks([torch.zeros(2, 2)], [torch.zeros(2, 2)], {0: [1]})


def test_decode_metadata_matches_reference_worker(built_lib):
    z = np.load(GOLDEN / "decode_meta.npz")
    tables = [row[row >= 0].tolist() for row in z["block_tables"]]
    md = M.decode_metadata(tables, z["context_lens"].tolist(), int(z["block_size"]))
    assert np.array_equal(md.positions.cpu().numpy(), z["positions"])
    assert np.array_equal(md.slot_mapping.cpu().numpy(), z["slots"])
    assert np.array_equal(md.context_lens.cpu().numpy(), z["context_lens"])


@pytest.mark.parametrize("build", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("given_positions", [True, False], ids=["positions", "one_launch"])
def test_paged_attention_with_rope_layer(build, given_positions, built_lib):
    """Reference layer forward: RoPE -> _write_kv_cache -> attention, on the fused ops;
    with positions=None (decode positions seq_lens - 1) as one launch."""
    spec = W.DecodeSpec("layer", [1, 17, 64, 300, 2048, 4096, 33, 1000], 16, 2, 128, 16,
                        "bfloat16", num_blocks=2048, rope_theta=1e6, max_position=4096)
    b = W.make_batch(spec)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(build)
    try:
        layer = PagedAttentionWithRoPE(16, 128, 128 ** -0.5, 128, max_position=4096,
                                       base=1_000_000).cuda()
    finally:
        torch.set_default_dtype(prev)
    S = b.num_decode
    cs = layer.cos_sin_cache.to(torch.bfloat16)
    # oracle pipeline on host copies
    q_np = W.to_numpy(b.query.reshape(S, -1))
    k_np = W.to_numpy(b.key.reshape(S, -1))
    q_rot, k_rot = O.rotary_embedding_neox(W.to_numpy(b.positions), q_np, k_np, 128,
                                           W.to_numpy(cs), "bfloat16")
    kc, vc = W.to_numpy(b.key_cache), W.to_numpy(b.value_cache)
    assert torch.equal(b.positions.to(torch.int64), b.seq_lens.to(torch.int64) - 1)
    out = layer(b.positions if given_positions else None, b.query, b.key, b.value,
                b.key_cache, b.value_cache, b.block_tables, b.seq_lens)
    # the layer rotated `key` in place (as the reference does), to the oracle's bits ...
    k_dev = W.to_numpy(b.key.reshape(S, -1))
    assert np.array_equal(k_dev, k_rot)
    # ... and wrote exactly that key and the value where _write_kv_cache would
    O.write_kv_cache(k_dev, W.to_numpy(b.value), W.to_numpy(b.positions), kc, vc,
                     W.to_numpy(b.block_tables))
    assert np.array_equal(W.to_numpy(b.key_cache), kc)
    assert np.array_equal(W.to_numpy(b.value_cache), vc)
    ref = O.paged_attention_f32(q_rot.reshape(S, 16, 128), kc, vc, W.to_numpy(b.block_tables),
                                W.to_numpy(b.seq_lens), b.scale, "bfloat16")
    np.testing.assert_allclose(O.to_f32(W.to_numpy(out), "bfloat16"), ref, **HALF_TOL)


def _device_step(prompt_tables, prompt_lens, decode_tables, context_lens, bs, alignment=8):
    md = M.step_metadata(prompt_tables, prompt_lens, decode_tables, context_lens, bs,
                         alignment=alignment)
    torch.cuda.synchronize()
    return md.positions.cpu().numpy(), md.slot_mapping.cpu().numpy(), md.num_tokens


def test_step_metadata_matches_reference_worker(built_lib):
    """tlb_step_metadata against _prepare_inputs on a mixed prompt + decode step:
    prompt slots, decode slots and the positions padded to a multiple of 8."""
    z = np.load(GOLDEN / "step_meta.npz")
    pt = [row[row >= 0].tolist() for row in z["prompt_tables"]]
    dt = [row[row >= 0].tolist() for row in z["decode_tables"]]
    pos, slots, T = _device_step(pt, z["prompt_lens"].tolist(), dt, z["context_lens"].tolist(),
                                 int(z["block_size"]))
    assert np.array_equal(pos, z["positions_padded"])
    assert T == len(z["slots"])
    assert np.array_equal(slots[:T], z["slots"])
    assert np.all(slots[T:] == -1)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("case", ["decode_only", "prompts_only", "empty_prompt", "negative_block",
                                  "many_prompts", "alignment_1"])
def test_step_metadata_edge_cases(case, built_lib):
    rng = np.random.default_rng(5)
    bs = 16

    def table(L):
        return rng.permutation(100_000)[: -(-L // bs)].tolist()

    plens = {"decode_only": [], "prompts_only": [5, 300, 17], "empty_prompt": [4, 0, 9],
             "negative_block": [40], "many_prompts": rng.integers(0, 50, 3000).tolist(),
             "alignment_1": [3]}[case]
    ctx = [] if case == "prompts_only" else [1, 16, 17, 250]
    ptabs = [table(max(L, 1)) for L in plens]
    dtabs = [table(L) for L in ctx]
    if case == "negative_block":
        ptabs[0][1] = -1
        dtabs[2][1] = -1
    align = 1 if case == "alignment_1" else 8
    pos, slots, T = _device_step(ptabs, plens, dtabs, ctx, bs, alignment=align)
    ref_pos, ref_slots = O.step_metadata(plens, ptabs, ctx, dtabs, bs, alignment=align)
    assert np.array_equal(pos, ref_pos)
    assert np.array_equal(slots[:T], ref_slots)
    assert np.all(slots[T:] == -1) and len(pos) % align == 0
    assert _lib.device_status() == 0


def test_ragged_step_built_on_device_matches_host(built_lib):
    """Config 3 (4 prompts + 252 decode sequences): the device-built positions
    and slot mapping the workload uses equal the host-derived ones."""
    spec = W.ragged_batch(0)
    dev = W.make_batch(spec, fill_cache=False)
    host = W.make_batch(spec, device="cpu", fill_cache=False)
    assert torch.equal(dev.positions.cpu(), host.positions)
    assert torch.equal(dev.slot_mapping.cpu(), host.slot_mapping)
    assert dev.num_prompt_tokens == sum(spec.prefill_lens)
