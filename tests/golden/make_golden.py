"""Generate the golden fixtures of tests/golden/ from the reference's own code.

Run in a container where the reference checkout exists (it is not needed, and
not read, anywhere else):

    python tests/golden/make_golden.py /path/to/tinyllama.py

What each fixture pins, all produced on CPU by the reference's Python:

* ``attn_ref_test_<dtype>_h<H>_kv<KVH>.npz`` — the reference test
  tests/test_paged_attention.py:10-63, executed as written except that its
  tensors live on the CPU; the kernel call is replaced by a stub and the
  test's own oracle output ``ref`` (:42-57) is captured from its final
  ``assert_close``. Inputs and ``ref`` are stored.
* ``cos_sin_<build>_rot<R>_base<B>.npz`` — ``PagedAttentionWithRoPE.__init__``
  (src/model_executor/layers/attention.py:53-80) under a given torch default
  dtype: the cos/sin table buffer it registers.
* ``write_kv_<dtype>_bs<bs>.npz`` — ``PagedAttentionWithRoPE._write_kv_cache``
  (:82-116) on seeded inputs with some negative block ids: caches before and
  after.
* ``decode_meta.npz`` — ``Worker._prepare_inputs`` (src/worker/worker.py:84-169)
  on decode sequence groups; its local ``slot_mappings`` / ``context_lens``
  (computed, then dropped by the reference) are captured with a trace hook.
* ``step_meta.npz`` — the same on a continuous-batching step that mixes prompt
  groups and decode groups of one or two sequences: prompt slots (:111-124),
  decode slots (:144-159) and the positions returned after the pad to a
  multiple of 8 (:163-169).

The reference imports ``cscr`` at module load; the ``cscr`` package of this
repository is put first on ``sys.path`` so that import resolves without the
reference's compiled extensions (none of its ops is called here).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


DT_NAME = {torch.float32: "float32", torch.float16: "float16", torch.bfloat16: "bfloat16"}


def gen_attention(ref_root: Path) -> None:
    src = (ref_root / "tests" / "test_paged_attention.py").read_text()
    src = src.replace('device = "cuda"', 'device = "cpu"')
    src = src.replace("from src.model_executor.layers.attention import paged_attention\n", "")
    captured = {}

    def stub_paged_attention(query, key_cache, value_cache, block_tables, seq_lens, scale):
        captured["inputs"] = dict(query=query.clone(), key_cache=key_cache.clone(),
                                  value_cache=value_cache.clone(),
                                  block_tables=block_tables.clone(), seq_lens=seq_lens.clone(),
                                  scale=scale)
        return torch.zeros_like(query)

    def capture_assert(actual, expected, **kw):
        captured["ref"] = expected.clone()
        captured["tol"] = kw

    ns = {"__name__": "reference_test"}
    exec(compile(src, str(ref_root / "tests" / "test_paged_attention.py"), "exec"), ns)
    ns["paged_attention"] = stub_paged_attention
    test_fn = ns["test_paged_attention_matches_reference"]
    real_assert = torch.testing.assert_close
    torch.testing.assert_close = capture_assert
    try:
        for dtype in (torch.float16, torch.bfloat16, torch.float32):
            for h, kvh in ((4, 4), (4, 2), (8, 1)):
                captured.clear()
                test_fn(dtype, h, kvh)
                inp = captured["inputs"]
                np.savez_compressed(
                    HERE / f"attn_ref_test_{DT_NAME[dtype]}_h{h}_kv{kvh}.npz",
                    query=_np(inp["query"]), key_cache=_np(inp["key_cache"]),
                    value_cache=_np(inp["value_cache"]), block_tables=_np(inp["block_tables"]),
                    seq_lens=_np(inp["seq_lens"]), scale=np.float64(inp["scale"]),
                    ref=_np(captured["ref"]), dtype=DT_NAME[dtype],
                    atol=np.float64(captured["tol"]["atol"]),
                    rtol=np.float64(captured["tol"]["rtol"]))
    finally:
        torch.testing.assert_close = real_assert


def gen_cos_sin(ref_root: Path) -> None:
    from src.model_executor.layers.attention import PagedAttentionWithRoPE

    prev = torch.get_default_dtype()
    try:
        for build in (torch.float32, torch.bfloat16, torch.float16):
            for rot, base, maxpos in ((128, 1000000, 512), (128, 10000, 512), (64, 10000, 512)):
                torch.set_default_dtype(build)
                layer = PagedAttentionWithRoPE(num_heads=4, head_size=rot, scale=rot ** -0.5,
                                               rotary_dim=rot, max_position=maxpos, base=base)
                np.savez_compressed(HERE / f"cos_sin_{DT_NAME[build]}_rot{rot}_base{base}.npz",
                                    table=_np(layer.cos_sin_cache), rot=rot, base=base,
                                    max_position=maxpos, build=DT_NAME[build])
    finally:
        torch.set_default_dtype(prev)


def gen_write_kv(ref_root: Path) -> None:
    from src.model_executor.layers.attention import PagedAttentionWithRoPE

    layer = PagedAttentionWithRoPE(num_heads=4, head_size=32, scale=32 ** -0.5, rotary_dim=32,
                                   max_position=64)
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        for bs in (8, 16):
            g = torch.Generator().manual_seed(7 + bs)
            S, kvh, D, nb, maxb = 12, 2, 32, 48, 4
            key_cache = torch.randn(nb, kvh, bs, D, generator=g).to(dtype)
            value_cache = torch.randn(nb, kvh, bs, D, generator=g).to(dtype)
            perm = torch.randperm(nb, generator=g)[: S * maxb].view(S, maxb).to(torch.int32)
            perm[3, 1] = -1  # tokens of a skipped block
            perm[7, 0] = -1
            positions = torch.randint(0, maxb * bs, (S,), generator=g)
            positions[3] = bs + 2   # lands in the -1 block
            positions[7] = 3        # lands in the -1 block
            key = torch.randn(S, kvh * D, generator=g).to(dtype)
            value = torch.randn(S, kvh, D, generator=g).to(dtype)
            kc0, vc0 = _np(key_cache), _np(value_cache)
            layer._write_kv_cache(key, value, positions, key_cache, value_cache, perm)
            np.savez_compressed(HERE / f"write_kv_{DT_NAME[dtype]}_bs{bs}.npz", key=_np(key),
                                value=_np(value), positions=_np(positions),
                                block_tables=_np(perm), key_cache_in=kc0, value_cache_in=vc0,
                                key_cache_out=_np(key_cache), value_cache_out=_np(value_cache),
                                dtype=DT_NAME[dtype])


def gen_decode_meta(ref_root: Path) -> None:
    from src.sampler_params import SamplerParams
    from src.sequence import SequenceData, SequenceGroupMetadata
    from src.worker.worker import Worker

    rng = np.random.default_rng(3)
    bs = 16
    groups, tables, ctx = [], [], []
    for i in range(20):
        L = int(rng.integers(1, 300))
        nblk = -(-L // bs)
        table = rng.permutation(1000)[:nblk].tolist()
        data = SequenceData(prompt_token_ids=[1] * L)
        groups.append(SequenceGroupMetadata(reqeust_id=str(i), is_prompt=False,
                                            seq_data={i: data},
                                            sampling_params=SamplerParams(),
                                            block_tables={i: table}))
        tables.append(table)
        ctx.append(data.get_len())
    worker = object.__new__(Worker)
    worker.block_size = bs
    captured = {}

    def tracer(frame, event, arg):
        if event == "return" and frame.f_code.co_name == "_prepare_inputs":
            captured.update({k: frame.f_locals[k] for k in
                             ("slot_mappings", "context_lens", "input_postions")})
        return tracer

    sys.settrace(tracer)
    try:
        worker._prepare_inputs(groups)
    finally:
        sys.settrace(None)
    maxb = max(len(t) for t in tables)
    bt = np.full((len(tables), maxb), -1, np.int32)
    for r, t in enumerate(tables):
        bt[r, : len(t)] = t
    n = len(tables)
    np.savez_compressed(HERE / "decode_meta.npz", block_tables=bt,
                        context_lens=np.asarray(captured["context_lens"], np.int32),
                        slots=np.asarray(captured["slot_mappings"], np.int64)[:n],
                        positions=np.asarray(captured["input_postions"], np.int64)[:n],
                        block_size=bs, seq_ctx=np.asarray(ctx, np.int32))


def gen_step_meta(ref_root: Path) -> None:
    """``_prepare_inputs`` on a continuous-batching step: prompt groups (their
    whole prompt, slots from the group's block table, worker.py:95-124) and
    decode groups of one or two sequences (worker.py:126-159), packed prompt
    tokens first, then padded to a multiple of 8 (:163-164)."""
    from src.sampler_params import SamplerParams
    from src.sequence import SequenceData, SequenceGroupMetadata
    from src.worker.worker import Worker

    rng = np.random.default_rng(11)
    bs = 16
    groups = []
    prompt_lens, prompt_tables, dec_tables, dec_ctx = [], [], [], []
    sid = 0
    kinds = ["p", "d", "d", "p", "d", "p", "d", "d", "d", "p", "d"]
    for i, kind in enumerate(kinds):
        if kind == "p":
            L = int(rng.integers(1, 200))
            table = rng.permutation(4000)[: -(-L // bs)].tolist()
            data = SequenceData(prompt_token_ids=rng.integers(1, 1000, L).tolist())
            groups.append(SequenceGroupMetadata(reqeust_id=str(i), is_prompt=True,
                                                seq_data={sid: data},
                                                sampling_params=SamplerParams(),
                                                block_tables={sid: table}))
            prompt_lens.append(L)
            prompt_tables.append(table)
            sid += 1
            continue
        seq_data, tables = {}, {}
        for _ in range(1 + (i % 2)):  # one or two sequences per decode group
            P = int(rng.integers(1, 150))
            data = SequenceData(prompt_token_ids=rng.integers(1, 1000, P).tolist())
            for _ in range(int(rng.integers(0, 60))):
                data.append_token_id(int(rng.integers(1, 1000)), 0.0)
            table = rng.permutation(4000)[: -(-data.get_len() // bs)].tolist()
            seq_data[sid], tables[sid] = data, table
            dec_tables.append(table)
            dec_ctx.append(data.get_len())
            sid += 1
        groups.append(SequenceGroupMetadata(reqeust_id=str(i), is_prompt=False,
                                            seq_data=seq_data, sampling_params=SamplerParams(),
                                            block_tables=tables))
    worker = object.__new__(Worker)
    worker.block_size = bs
    captured = {}

    def tracer(frame, event, arg):
        if event == "return" and frame.f_code.co_name == "_prepare_inputs":
            captured.update({k: list(frame.f_locals[k]) for k in
                             ("slot_mappings", "context_lens", "input_postions")})
        return tracer

    sys.settrace(tracer)
    try:
        tokens, positions = worker._prepare_inputs(groups)
    finally:
        sys.settrace(None)

    def table_array(rows):
        out = np.full((len(rows), max(len(r) for r in rows)), -1, np.int32)
        for r, t in enumerate(rows):
            out[r, : len(t)] = t
        return out

    np.savez_compressed(HERE / "step_meta.npz", block_size=bs,
                        prompt_lens=np.asarray(prompt_lens, np.int32),
                        prompt_tables=table_array(prompt_tables),
                        context_lens=np.asarray(dec_ctx, np.int32),
                        decode_tables=table_array(dec_tables),
                        captured_context_lens=np.asarray(captured["context_lens"], np.int32),
                        slots=np.asarray(captured["slot_mappings"], np.int64),
                        positions_padded=_np(positions), num_tokens_padded=len(tokens))


def main() -> None:
    ref_root = Path(sys.argv[1]).resolve()
    sys.path.insert(0, str(ref_root))
    sys.path.insert(0, str(REPO / "tinyllama.py_b200"))
    torch.manual_seed(0)
    gen_attention(ref_root)
    gen_cos_sin(ref_root)
    gen_write_kv(ref_root)
    gen_decode_meta(ref_root)
    gen_step_meta(ref_root)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
