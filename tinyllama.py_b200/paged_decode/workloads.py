"""Seeded synthetic decode workloads with the shapes of the benchmark configs.

No public dataset is involved: context lengths come from ``numpy.random.
default_rng(seed)`` draws with the stated distributions, q/k/v and the KV pool
are N(0, 1) from a seeded torch generator, and physical blocks are a seeded
random permutation of the pool. Each workload is a decode step: one new token
per sequence at position ``context_len - 1`` whose slot lies in the
sequence's last block, plus, for the continuous-batching shape, prefill
chunks packed before the decode tokens as the reference's worker packs them.

Shapes (H query heads / KVH kv heads / D head dim, bs block size):
  uniform_small   8 seqs, len U[1,512], H16/KVH2/D128, bs16, 512 blocks, fp32
  qwen3b_decode   64 seqs, len U[128,4096], H16/KVH2/D128, bs16, 40k blocks, bf16,
                  RoPE theta 1e6
  ragged_batch    252 decode seqs, len clip(lognormal(ln 1024, 1.0), 16, 8192)
                  + 4 prefill chunks U[256,2048], fp16, H16/KVH2/D128, bs16
  long_tail       256 seqs, len clip(32 * (1 + pareto(1.2)), 32, 32768), bs32, bf16
  sweep point     bs x batch x uniform context x dtype x head shape
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

TORCH_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


@dataclass
class DecodeSpec:
    name: str
    seq_lens: list[int]
    num_heads: int = 16
    num_kv_heads: int = 2
    head_dim: int = 128
    block_size: int = 16
    dtype: str = "bfloat16"
    num_blocks: int | None = None      # pool size; None = just enough (+ slack)
    rope_theta: float = 10000.0
    max_position: int | None = None    # cos/sin rows; None = max(seq_lens) rounded up
    prefill_lens: list[int] = field(default_factory=list)  # RoPE + cache write only
    seed: int = 0

    @property
    def group(self) -> int:
        return self.num_heads // self.num_kv_heads

    def blocks_needed(self) -> int:
        bs = self.block_size
        return sum(math.ceil(max(L, 0) / bs) for L in self.seq_lens) + sum(
            math.ceil(L / bs) for L in self.prefill_lens)

    @property
    def max_blocks_per_seq(self) -> int:
        bs = self.block_size
        return max(1, max(math.ceil(max(L, 0) / bs) for L in self.seq_lens))


def uniform_small(seed: int = 0) -> DecodeSpec:
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 513, size=8).tolist()
    return DecodeSpec("uniform_small", lens, 16, 2, 128, 16, "float32", num_blocks=512, seed=seed)


def qwen3b_decode(seed: int = 0, batch: int = 64) -> DecodeSpec:
    rng = np.random.default_rng(seed)
    lens = rng.integers(128, 4097, size=batch).tolist()
    return DecodeSpec("qwen3b_decode", lens, 16, 2, 128, 16, "bfloat16",
                      num_blocks=40000, rope_theta=1e6, max_position=4096, seed=seed)


def ragged_batch(seed: int = 0, sigma: float = 1.0) -> DecodeSpec:
    rng = np.random.default_rng(seed)
    dec = np.clip(np.round(rng.lognormal(math.log(1024), sigma, size=252)), 16, 8192)
    pre = rng.integers(256, 2049, size=4)
    return DecodeSpec("ragged_batch", dec.astype(int).tolist(), 16, 2, 128, 16, "float16",
                      max_position=8192, prefill_lens=pre.tolist(), seed=seed)


def long_tail_lengths(seed: int = 0, batch: int = 256) -> list[int]:
    rng = np.random.default_rng(seed)
    lens = np.clip(np.floor(32 * (1 + rng.pareto(1.2, size=batch))), 32, 32768)
    return lens.astype(int).tolist()


def long_tail(seed: int = 0, lens: list[int] | None = None, num_blocks: int | None = None) -> DecodeSpec:
    lens = lens if lens is not None else long_tail_lengths(seed)
    return DecodeSpec("long_tail", lens, 16, 2, 128, 32, "bfloat16", num_blocks=num_blocks,
                      max_position=32768, seed=seed)


SWEEP_HEADS = {"qwen0.5b": (14, 2, 64), "qwen3b": (16, 2, 128)}


def sweep_point(block_size: int, batch: int, context: int, dtype: str, heads: str,
                seed: int = 0) -> DecodeSpec:
    h, kvh, d = SWEEP_HEADS[heads]
    return DecodeSpec(f"sweep_bs{block_size}_b{batch}_ctx{context}_{dtype}_{heads}",
                      [context] * batch, h, kvh, d, block_size, dtype, max_position=context,
                      seed=seed)


def sweep_points():
    for bs in (8, 16, 32):
        for batch in (1, 32, 256):
            for ctx in (512, 8192):
                for dtype in ("float16", "bfloat16"):
                    for heads in SWEEP_HEADS:
                        yield sweep_point(bs, batch, ctx, dtype, heads)


def cos_sin_table(rotary_dim: int, max_position: int, base: float, dtype: torch.dtype,
                  build_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """cos/sin table built exactly as src/model_executor/layers/attention.py:71-79.

    ``build_dtype`` is the torch default dtype in force while the reference
    builds it (the model dtype once the loader has called set_default_dtype).
    """
    prev = torch.get_default_dtype()
    torch.set_default_dtype(build_dtype)
    try:
        inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2) / rotary_dim))
        t = torch.arange(max_position).float()
        freqs = torch.einsum("i,j -> ij", t, inv_freq.float())
        cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1)
        cache = cache.to(torch.get_default_dtype())
    finally:
        torch.set_default_dtype(prev)
    return cache.to(dtype)


@dataclass
class DecodeBatch:
    """Device (or host) tensors of one decode step."""
    spec: DecodeSpec
    query: torch.Tensor          # [T, H, D]   new tokens (prefill tokens, then decode)
    key: torch.Tensor            # [T, KVH, D]
    value: torch.Tensor          # [T, KVH, D]
    positions: torch.Tensor      # [T] int64
    slot_mapping: torch.Tensor   # [T] int64
    token_block_tables: torch.Tensor  # [T, maxB_all] int32 (row of each token's sequence)
    block_tables: torch.Tensor   # [S, maxB] int32 (decode sequences)
    seq_lens: torch.Tensor       # [S] int32
    key_cache: torch.Tensor      # [NB, KVH, bs, D]
    value_cache: torch.Tensor
    cos_sin_cache: torch.Tensor  # [max_position, D]
    scale: float
    num_prompt_tokens: int = 0   # prefill tokens packed before the decode tokens

    @property
    def num_decode(self) -> int:
        return self.block_tables.shape[0]

    @property
    def decode_rows(self) -> slice:
        """Rows of query / key / value holding the decode tokens."""
        return slice(self.num_prompt_tokens, self.num_prompt_tokens + self.num_decode)


def make_batch(spec: DecodeSpec, device="cuda", fill_cache: bool = True,
               build_dtype: torch.dtype | None = None,
               caches: tuple[torch.Tensor, torch.Tensor] | None = None) -> DecodeBatch:
    """Materialise a decode step for `spec` on `device`.

    ``caches``: an existing (key_cache, value_cache) pool of ``spec.num_blocks``
    blocks to place the batch in (a large per-GPU pool shared by several
    steps); only the blocks the batch uses are filled, with N(0, 1) values.
    """
    dev = torch.device(device)
    dtype = TORCH_DTYPES[spec.dtype]
    bs, H, KVH, D = spec.block_size, spec.num_heads, spec.num_kv_heads, spec.head_dim
    rng = np.random.default_rng(spec.seed + 1)
    dec_lens = [max(int(L), 0) for L in spec.seq_lens]
    S = len(dec_lens)
    nb_dec = [math.ceil(L / bs) for L in dec_lens]
    nb_pre = [math.ceil(L / bs) for L in spec.prefill_lens]
    need = sum(nb_dec) + sum(nb_pre)
    NB = spec.num_blocks if spec.num_blocks is not None else max(need + 16, 64)
    if NB < need:
        raise ValueError(f"pool of {NB} blocks cannot hold the {need} blocks the batch needs")
    perm = rng.permutation(NB)[:need].astype(np.int64)

    maxB = max([1] + nb_dec)
    tables = np.zeros((S, maxB), np.int32)
    off = 0
    for s, n in enumerate(nb_dec):
        tables[s, :n] = perm[off:off + n]
        off += n
    pre_tables = []
    for n in nb_pre:
        pre_tables.append(perm[off:off + n])
        off += n

    # new tokens packed as the reference's worker packs them
    # (src/worker/worker.py:95-159): every prefill chunk's tokens, then one
    # per decode sequence
    pos, slots, tok_rows = [], [], []
    maxB_all = max([maxB] + nb_pre)
    for c, L in enumerate(spec.prefill_lens):
        row = np.zeros(maxB_all, np.int32)
        row[:len(pre_tables[c])] = pre_tables[c]
        for p in range(L):
            pos.append(p)
            slots.append(int(pre_tables[c][p // bs]) * bs + p % bs)
            tok_rows.append(row)
    for s, L in enumerate(dec_lens):
        p = L - 1
        pos.append(p)
        slots.append(int(tables[s, p // bs]) * bs + p % bs if p >= 0 else -1)
        row = np.zeros(maxB_all, np.int32)
        row[:maxB] = tables[s]
        tok_rows.append(row)
    T = len(pos)
    n_prompt = T - S

    g = torch.Generator(device="cpu").manual_seed(spec.seed)
    gen_dev = torch.Generator(device=dev).manual_seed(spec.seed) if dev.type == "cuda" else g

    def randn(*shape, generator):
        return torch.randn(*shape, generator=generator, device=generator.device,
                           dtype=torch.float32).to(dtype).to(dev)

    query = randn(T, H, D, generator=g)
    key = randn(T, KVH, D, generator=g)
    value = randn(T, KVH, D, generator=g)
    if caches is not None:
        kc, vc = caches
        if tuple(kc.shape) != (NB, KVH, bs, D) or kc.shape != vc.shape or kc.dtype != dtype:
            raise ValueError("caches must be two [num_blocks, kv_heads, block_size, head_dim] "
                             "tensors of the batch dtype")
        if fill_cache and need:
            idx = torch.from_numpy(perm).to(kc.device)
            for c in (kc, vc):
                c.index_copy_(0, idx, torch.randn(need, KVH, bs, D, generator=gen_dev,
                                                  device=gen_dev.device,
                                                  dtype=torch.float32).to(dtype).to(dev))
    elif fill_cache:
        kc = torch.randn(NB, KVH, bs, D, generator=gen_dev, device=gen_dev.device,
                         dtype=dtype if dev.type == "cuda" else torch.float32).to(dtype).to(dev)
        vc = torch.randn(NB, KVH, bs, D, generator=gen_dev, device=gen_dev.device,
                         dtype=dtype if dev.type == "cuda" else torch.float32).to(dtype).to(dev)
    else:
        kc = torch.empty(NB, KVH, bs, D, dtype=dtype, device=dev)
        vc = torch.empty(NB, KVH, bs, D, dtype=dtype, device=dev)
    max_pos = spec.max_position or max([1] + dec_lens + list(spec.prefill_lens))
    cs = cos_sin_table(D, max_pos, spec.rope_theta, dtype,
                       build_dtype if build_dtype is not None else torch.float32).to(dev)
    positions = torch.tensor(pos, dtype=torch.int64, device=dev)
    slot_mapping = torch.tensor(slots, dtype=torch.int64, device=dev)
    if spec.prefill_lens and dev.type == "cuda":
        # A step with prompts: positions and slots come from the device-side
        # builder, from the block tables and lengths the block manager holds.
        from paged_decode import metadata as M

        md = M.step_metadata([t.tolist() for t in pre_tables], list(spec.prefill_lens),
                             [tables[s, :nb_dec[s]].tolist() for s in range(S)], dec_lens, bs,
                             device=dev)
        positions, slot_mapping = md.positions[:T], md.slot_mapping[:T]
    return DecodeBatch(
        spec=spec, query=query, key=key, value=value,
        positions=positions, slot_mapping=slot_mapping,
        token_block_tables=torch.from_numpy(np.stack(tok_rows)).to(dev),
        block_tables=torch.from_numpy(tables).to(dev),
        seq_lens=torch.tensor(dec_lens, dtype=torch.int32, device=dev),
        key_cache=kc, value_cache=vc, cos_sin_cache=cs, scale=D ** -0.5,
        num_prompt_tokens=n_prompt)


def to_numpy(t: torch.Tensor) -> np.ndarray:
    """Host numpy copy; bfloat16 comes back as uint16 bit patterns."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def from_numpy(a: np.ndarray, dtype: torch.dtype, device="cpu") -> torch.Tensor:
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def compact_for_oracle(batch: DecodeBatch):
    """Host copies of the attention inputs with the pool cut to the used blocks.

    The oracle only reads blocks named by the block tables, so gathering just
    those (and renumbering the tables) gives the same result from a much
    smaller host copy of a large pool.
    """
    tables = batch.block_tables.cpu().numpy()
    lens = batch.seq_lens.cpu().numpy()
    bs = batch.spec.block_size
    used_mask = np.zeros(tables.shape, bool)
    for s, L in enumerate(lens):
        n = min(math.ceil(max(int(L), 0) / bs), tables.shape[1])
        used_mask[s, :n] = True
    used = np.unique(tables[used_mask & (tables >= 0)])
    remap = {int(b): i for i, b in enumerate(used)}
    new_tables = np.full(tables.shape, -1, np.int32)
    for s in range(tables.shape[0]):
        for j in range(tables.shape[1]):
            b = int(tables[s, j])
            if used_mask[s, j] and b >= 0:
                new_tables[s, j] = remap[b]
    idx = torch.from_numpy(used.astype(np.int64)).to(batch.key_cache.device)
    kc = to_numpy(batch.key_cache.index_select(0, idx)) if len(used) else to_numpy(batch.key_cache[:1])
    vc = to_numpy(batch.value_cache.index_select(0, idx)) if len(used) else to_numpy(batch.value_cache[:1])
    return kc, vc, new_tables, lens
