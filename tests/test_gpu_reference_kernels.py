"""The product kernels against the reference's OWN CUDA kernels, run on the same inputs.

``oracle/build_ref.py`` compiles the reference's pybind extensions
(cscr/attention.cpp + attention_kernel.cu, cscr/pos_encoding.cpp +
pos_encoding_kernel.cu, cscr/cache.cpp + cache_kernel.cu) from its sources,
unchanged, with its own flags (setup.py:4-41: -O3 --use_fast_math) for sm_100a,
into ``oracle/_ref/``. Loaded here by file path under names of their own
(``tlref_*``), they are a second checker beside the numpy oracle:

* RoPE (pos_encoding_kernel.cu:24-65) has no CPU path in the reference, so
  running its kernel is what pins the rotation: ours must agree with it within
  the north-star tolerance (atol 2e-3 / rtol 1e-2 for fp16/bf16, 1e-4 for
  fp32), and both with the fp32 rotation before rounding. The count of
  elements whose bits differ is reported: the reference's ``x * cos - y * sin``
  is compiled with --use_fast_math, which may contract it into a multiply-add,
  while ours rounds each product on its own.
* Paged attention (attention_kernel.cu:24-150) on the config-2 decode batch,
  the config-3 decode sequences, the reference test's own case and head dim
  64 / 128: ours within tolerance of the reference kernel, and both within
  tolerance of the fp32 oracle.
* Block copies (cache_kernel.cu:23-212): bit-identical caches.

Inputs are valid for the reference kernels (every block id inside the pool,
every length within its table): those kernels do not check bounds.
"""

import glob

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from cscr import _lib
from cscr import attention as A
from cscr import cache as C
from cscr import pos_encoding as PE
from helpers import oracle_f32_from_tensors, tol_for
from oracle import build_ref
from oracle import decode_oracle as O
from paged_decode import workloads as W

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not build_ref.built(),
                       reason="reference ops not built (oracle/build_ref.py needs the "
                              "reference sources)"),
]


@pytest.fixture(scope="module")
def ref_rope():
    return build_ref.load_ref_module("tlref_pos_encoding")


@pytest.fixture(scope="module")
def ref_attn():
    return build_ref.load_ref_module("tlref_attention")


@pytest.fixture(scope="module")
def ref_cache():
    return build_ref.load_ref_module("tlref_cache")


@pytest.fixture(autouse=True)
def _device():
    torch.cuda.set_device(0)
    _lib.device_status(clear=True)
    yield
    torch.cuda.synchronize()


def _f32(t: torch.Tensor, dtype: str) -> np.ndarray:
    return O.to_f32(W.to_numpy(t), dtype)


def _rope_f32(pos, x, head_size, cs, dtype):
    """The NeoX rotation in fp32 before the final rounding (cos/sin as stored)."""
    T = x.shape[0]
    rot = cs.shape[1]
    half = rot // 2
    c = _f32(cs, dtype)[W.to_numpy(pos).astype(np.int64)]
    cos, sin = c[:, None, :half], c[:, None, half:rot]
    v = _f32(x, dtype).reshape(T, -1, head_size).copy()
    a, b = v[..., :half].copy(), v[..., half:rot].copy()
    v[..., :half] = a * cos - b * sin
    v[..., half:rot] = b * cos + a * sin
    return v.reshape(T, -1)


def _rope_case(name):
    """(positions, query [T, H*D], key [T, KVH*D], head_size, cos_sin_cache, dtype)."""
    if name == "qwen3b_decode":          # config 2: 64 decode tokens, theta 1e6, bf16
        b = W.make_batch(W.qwen3b_decode(0))
        S = b.num_decode
        return b.positions, b.query.view(S, -1), b.key.view(S, -1), 128, b.cos_sin_cache, "bfloat16"
    if name == "ragged_batch":           # config 3: ~4.9k packed decode + prefill tokens, fp16
        b = W.make_batch(W.ragged_batch(0))
        T = b.query.shape[0]
        return b.positions, b.query.view(T, -1), b.key.view(T, -1), 128, b.cos_sin_cache, "float16"
    # head dim 64 (Qwen2.5-0.5B-like, 14/2 heads), int32 positions, each dtype
    dtype = name.split("_")[-1]
    tdt = W.TORCH_DTYPES[dtype]
    g = torch.Generator().manual_seed(3)
    T = 300
    q = torch.randn(T, 14 * 64, generator=g).to(tdt).cuda()
    k = torch.randn(T, 2 * 64, generator=g).to(tdt).cuda()
    pos = torch.randint(0, 8192, (T,), generator=g).to(torch.int32).cuda()
    cs = W.cos_sin_table(64, 8192, 10000.0, tdt).cuda()
    return pos, q, k, 64, cs, dtype


ROPE_CASES = ["qwen3b_decode", "ragged_batch", "hd64_float32", "hd64_float16", "hd64_bfloat16"]


@pytest.mark.parametrize("case", ROPE_CASES)
def test_rope_matches_reference_kernel(case, ref_rope, record_property):
    pos, q, k, hs, cs, dtype = _rope_case(case)
    k_ref, k_ours = k.clone(), k.clone()
    out_ref = ref_rope.rotary_embedding_neox(postions=pos, query=q, key=k_ref, head_size=hs,
                                             cos_sin_cache=cs)
    out = PE.rotary_embedding_neox(pos, q, k_ours, hs, cs)
    torch.cuda.synchronize()
    tol = tol_for(dtype)
    for ours, ref, raw in ((out, out_ref, q), (k_ours, k_ref, k)):
        np.testing.assert_allclose(_f32(ours, dtype), _f32(ref, dtype), **tol)
        exact = _rope_f32(pos, raw, hs, cs, dtype)
        np.testing.assert_allclose(_f32(ours, dtype), exact, **tol)
        np.testing.assert_allclose(_f32(ref, dtype), exact, **tol)
    differ = int((W.to_numpy(out) != W.to_numpy(out_ref)).sum()
                 + (W.to_numpy(k_ours) != W.to_numpy(k_ref)).sum())
    total = out.numel() + k.numel()
    record_property("bits_differing", differ)
    record_property("elements", total)
    print(f"[rope vs reference kernel] {case}: {differ} of {total} elements differ in their bits")


def _attn_case(name):
    if name == "qwen3b_decode":
        b = W.make_batch(W.qwen3b_decode(0))
        return b.query, b.key_cache, b.value_cache, b.block_tables, b.seq_lens, b.scale, "bfloat16"
    if name == "ragged_batch_decode":
        b = W.make_batch(W.ragged_batch(0))
        return (b.query[b.decode_rows].contiguous(), b.key_cache, b.value_cache,
                b.block_tables, b.seq_lens, b.scale, "float16")
    if name.startswith("hd64"):
        dtype = name.split("_")[-1]
        spec = W.DecodeSpec("hd64", [1, 7, 64, 333, 1024, 2500, 4096, 17], 14, 2, 64, 16, dtype,
                            seed=4)
        b = W.make_batch(spec)
        return b.query, b.key_cache, b.value_cache, b.block_tables, b.seq_lens, b.scale, dtype
    if name == "long_tail_bs32":
        lens = W.long_tail_lengths(0)[:64]
        b = W.make_batch(W.long_tail(0, lens=lens))
        return b.query, b.key_cache, b.value_cache, b.block_tables, b.seq_lens, b.scale, "bfloat16"
    raise KeyError(name)


ATTN_CASES = ["qwen3b_decode", "ragged_batch_decode", "hd64_float16", "hd64_bfloat16",
              "hd64_float32", "long_tail_bs32"]


@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_matches_reference_kernel(case, ref_attn, record_property):
    q, kc, vc, bt, sl, scale, dtype = _attn_case(case)
    out_ref = ref_attn.paged_attention(query=q, key_cache=kc, value_cache=vc, block_tables=bt,
                                       seq_lens=sl, scale=scale)
    out = A.paged_attention(q, kc, vc, bt, sl, scale)
    torch.cuda.synchronize()
    tol = tol_for(dtype)
    got, ref = _f32(out, dtype), _f32(out_ref, dtype)
    np.testing.assert_allclose(got, ref, **tol)
    exact = oracle_f32_from_tensors(q, kc, vc, bt, sl, scale, dtype)
    np.testing.assert_allclose(got, exact, **tol)
    np.testing.assert_allclose(ref, exact, **tol)
    record_property("max_abs_diff_vs_reference", float(np.abs(got - ref).max()))
    assert _lib.device_status() == 0


@pytest.mark.parametrize("path", sorted(glob.glob(str(GOLDEN / "attn_ref_test_*.npz"))),
                         ids=lambda p: p.split("/")[-1][:-4])
def test_reference_test_case_on_both_kernels(path, ref_attn):
    """tests/test_paged_attention.py's own case (seed 0, lens [13, 1, 16], hd 64,
    bs 8) on the reference kernel and ours, with the test's tolerance (:59-63)."""
    z = np.load(path)
    dtype = str(z["dtype"])
    tdt = W.TORCH_DTYPES[dtype]
    args = dict(query=W.from_numpy(z["query"], tdt, "cuda"),
                key_cache=W.from_numpy(z["key_cache"], tdt, "cuda"),
                value_cache=W.from_numpy(z["value_cache"], tdt, "cuda"),
                block_tables=torch.from_numpy(z["block_tables"]).cuda(),
                seq_lens=torch.from_numpy(z["seq_lens"]).cuda(), scale=float(z["scale"]))
    out_ref = ref_attn.paged_attention(**args)
    out = A.paged_attention(**args)
    torch.cuda.synchronize()
    golden = O.to_f32(z["ref"], dtype)
    for o in (out, out_ref):
        np.testing.assert_allclose(_f32(o, dtype), golden, atol=float(z["atol"]),
                                   rtol=float(z["rtol"]))
    np.testing.assert_allclose(_f32(out, dtype), _f32(out_ref, dtype), **tol_for(dtype))


def test_copy_blocks_matches_reference_kernel(ref_cache):
    """copy_blocks over 4 layers with a copy-on-write fan-out: identical caches."""
    g = torch.Generator(device="cuda").manual_seed(7)
    shape = (64, 2, 16, 128)
    layers = [torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
              for _ in range(8)]
    mine = [t.clone() for t in layers]
    mapping = {3: [10, 11, 40], 5: [6], 63: [0, 1]}
    ref_cache.copy_blocks(key_caches=layers[:4], value_caches=layers[4:], block_mapping=mapping)
    C.copy_blocks(mine[:4], mine[4:], mapping)
    torch.cuda.synchronize()
    for a, b in zip(layers, mine):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_swap_blocks_matches_reference_kernel(ref_cache):
    g = torch.Generator(device="cuda").manual_seed(8)
    src = torch.randn(32, 2, 16, 64, generator=g, device="cuda").to(torch.float16)
    mapping = {0: 5, 7: 2, 31: 30, 12: 12}
    for dst_dev in ("cuda", "cpu"):
        d_ref = torch.zeros(32, 2, 16, 64, dtype=torch.float16, device=dst_dev)
        d_ours = d_ref.clone()
        ref_cache.swap_blocks(src=src, dst=d_ref, block_mapping=mapping)
        C.swap_blocks(src, d_ours, mapping)
        torch.cuda.synchronize()
        assert torch.equal(d_ref, d_ours)


def test_reference_modules_do_not_shadow_the_product_package():
    import sys

    import cscr.attention as mine

    mod = build_ref.load_ref_module("tlref_attention")
    assert mod.__name__ == "tlref_attention"
    assert sys.modules["cscr.attention"] is mine
    assert mine.paged_attention is A.paged_attention
    assert mine.__file__.endswith("tinyllama.py_b200/cscr/attention.py")


def test_copy_blocks_speed_beside_the_reference_kernel(ref_cache, record_property):
    """Copy-on-write fan-out over a 36-layer cache (72 caches, 256 block pairs
    each, 151 MB copied, more than the L2): this repository's one-launch copy
    and the reference's copy_blocks (cache_kernel.cu:180-212: a synchronous
    mapping upload, then one launch per cache), timed with CUDA events.
    Reported, with identical results asserted; the rate is not asserted."""
    NB, KVH, bs, D, L = 4096, 2, 16, 128, 36
    g = torch.Generator(device="cuda").manual_seed(11)
    caches = [torch.randn(NB, KVH, bs, D, generator=g, device="cuda").to(torch.bfloat16)
              for _ in range(2 * L)]
    mine = [c.clone() for c in caches]
    perm = torch.randperm(NB, generator=torch.Generator().manual_seed(3)).tolist()
    mapping = {perm[i]: [perm[256 + i]] for i in range(256)}
    block_bytes = KVH * bs * D * 2
    moved = 2 * 256 * 2 * L * block_bytes  # read + write of every copied block

    def timed(fn, reps=5):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    t_ref = timed(lambda: ref_cache.copy_blocks(key_caches=caches[:L], value_caches=caches[L:],
                                                block_mapping=mapping))
    t_ours = timed(lambda: C.copy_blocks(mine[:L], mine[L:], mapping))
    for a, b in zip(caches, mine):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    record_property("us_reference", round(t_ref, 2))
    record_property("us_ours", round(t_ours, 2))
    print(f"[copy_blocks 36 layers, 256 pairs] reference {t_ref:.1f} us "
          f"({moved / t_ref / 1e3:.0f} GB/s), ours {t_ours:.1f} us ({moved / t_ours / 1e3:.0f} GB/s)")
