"""tlb_paged_attention_no_alloc against tlb_paged_attention.

The allocation-free entry point serves callers that cannot allocate device
memory per call (an engine that gave all free memory to its KV pool, a host
binding only the C header): its scratch is a fixed device array inside the
library. Called through the C ABI twice in a row, it must give what the
workspace entry point gives, within the tolerance of the other attention
tests. This file is collected last on purpose; it passes alone or after the
rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

from cscr import _lib
from cscr import attention as A
from helpers import tol_for
from oracle import decode_oracle as O
from paged_decode import workloads as W

pytestmark = pytest.mark.gpu


def _no_alloc(lib, q, kc, vc, bt, sl, scale, stream):
    out = torch.empty_like(q)
    S, H, D = q.shape
    NB, KVH, BS, _ = kc.shape
    rc = lib.tlb_paged_attention_no_alloc(
        out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), sl.data_ptr(),
        S, H, KVH, D, NB, BS, bt.shape[1], float(scale), _lib.DTYPE_CODE[q.dtype], 0, stream)
    assert rc == 0, _lib.last_error()
    return out


@pytest.mark.parametrize("spec", [
    W.qwen3b_decode(5, batch=64),
    W.DecodeSpec("small_fp16_g7", [1, 17, 300, 2048, 0, 33], 14, 2, 64, 16, "float16",
                 num_blocks=512),
], ids=lambda s: s.name)
def test_no_alloc_matches_workspace_entry_point(spec, built_lib):
    torch.cuda.set_device(0)
    lib = _lib.load()
    b = W.make_batch(spec)
    S = b.num_decode
    q = b.query[:S].contiguous()
    ref = A.paged_attention(q, b.key_cache, b.value_cache, b.block_tables, b.seq_lens, b.scale)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row share (and must re-clean) the static scratch
        out = _no_alloc(lib, q, b.key_cache, b.value_cache, b.block_tables, b.seq_lens, b.scale,
                        stream)
        torch.cuda.synchronize()
        np.testing.assert_allclose(O.to_f32(W.to_numpy(out), spec.dtype),
                                   O.to_f32(W.to_numpy(ref), spec.dtype), **tol_for(spec.dtype))
    assert _lib.device_status() == 0


def test_no_alloc_rejects_batches_beyond_its_scratch(built_lib):
    torch.cuda.set_device(0)
    lib = _lib.load()
    # 3M sequences x 2 kv heads of arrival counters alone exceed the fixed array;
    # the size check fails before any pointer is used or kernel launched.
    rc = lib.tlb_paged_attention_no_alloc(8, 8, 8, 8, 8, 8, 3_000_000, 16, 2, 128, 10, 16, 4,
                                          0.1, _lib.DTYPE_CODE[torch.bfloat16], 0,
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == 4
    assert "static buffer" in _lib.last_error()
