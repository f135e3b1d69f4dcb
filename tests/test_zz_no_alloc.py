"""tlb_paged_attention_no_alloc against tlb_paged_attention, through the C ABI.

The allocation-free entry point is for callers that cannot allocate device
memory per call: an engine that handed every free byte to its KV pool after
profiling (as the reference's worker sizes its cache) has nothing left for
attention scratch, and a host that binds only the C header may have no CUDA
allocator at all. Its scratch is a fixed device array inside the library,
shared by every call on a device.

Both entry points run the same kernel with the same partition and merge
order, so their outputs must be bit-identical; each is also checked against
the fp32 oracle at the north-star tolerance. The batches go large -> small ->
large, so a small call's partial results sit where the large call's arrival
counters live and the large call must clear them first.

This file is collected last on purpose; it passes alone in a fresh process or
after the rest of the suite.
"""

import ctypes

import pytest
import torch

from cscr import _lib
from helpers import check_attention
from paged_decode import workloads as W

pytestmark = pytest.mark.gpu

NO_ALLOC_BYTES = 16 << 20  # TLB_NO_ALLOC_SCRATCH_BYTES


@pytest.fixture(autouse=True)
def _device():
    torch.cuda.set_device(0)
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    _lib.device_status(clear=True)
    yield
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    torch.cuda.synchronize()


def _args(b):
    q = b.query[: b.num_decode].contiguous()
    NB, KVH, BS, _ = b.key_cache.shape
    S, H, D = q.shape
    return q, (q.data_ptr(), b.key_cache.data_ptr(), b.value_cache.data_ptr(),
               b.block_tables.data_ptr(), b.seq_lens.data_ptr(), S, H, KVH, D, NB, BS,
               b.block_tables.shape[1], float(b.scale), _lib.DTYPE_CODE[q.dtype])


def _no_alloc(lib, b):
    q, a = _args(b)
    out = torch.empty_like(q)
    rc = lib.tlb_paged_attention_no_alloc(out.data_ptr(), *a, 0,
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    return out


def _with_fresh_workspace(lib, b):
    """The workspace entry point with a freshly zeroed workspace of its own."""
    q, a = _args(b)
    S, H, KVH, D = a[5], a[6], a[7], a[8]
    need = ctypes.c_size_t(0)
    assert lib.tlb_paged_attention_workspace_size(S, H, KVH, D, a[13], ctypes.byref(need)) == 0
    ws = torch.zeros(max(need.value, 256), dtype=torch.uint8, device="cuda")
    out = torch.empty_like(q)
    rc = lib.tlb_paged_attention(out.data_ptr(), *a, ws.data_ptr(), ws.numel(), 0,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    return out


def _bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def _batch(kind, n):
    if kind == "qwen3b_bf16":
        return W.make_batch(W.qwen3b_decode(5 + n, batch=n))
    lens = [1, 17, 300, 2048, 0, 33, 4096, 900][:n] if n < 8 else \
        [(97 * i) % 4000 + 1 for i in range(n)]
    dtype = {"hd64_fp16": "float16", "fp32_generic": "float32"}[kind]
    H, KVH, D = (14, 2, 64) if kind == "hd64_fp16" else (16, 2, 128)
    spec = W.DecodeSpec(kind, lens, H, KVH, D, 16, dtype,
                        num_blocks=sum(-(-L // 16) for L in lens) + 8, seed=n)
    return W.make_batch(spec)


@pytest.mark.parametrize("kind", ["qwen3b_bf16", "hd64_fp16", "fp32_generic"])
def test_no_alloc_matches_workspace_entry_point(kind, built_lib):
    lib = _lib.load()
    for n in (64, 5, 64):  # large -> small -> large, calls back to back
        b = _batch(kind, n)
        out = _no_alloc(lib, b)
        ref = _with_fresh_workspace(lib, b)
        torch.cuda.synchronize()
        assert torch.equal(_bits(out), _bits(ref)), f"batch of {n}"
        check_attention(b, out)
    assert _lib.device_status() == 0


def test_no_alloc_rejects_batches_beyond_its_scratch(built_lib):
    """4M sequences x 2 kv heads need more scratch than the fixed array: the call
    is refused with a clear error before any memset or launch. (The pointers
    are real, 256-byte aligned device memory, so the bf16 / head-dim-128 call
    takes the path that needs scratch; its size is checked first.)"""
    lib = _lib.load()
    S = 4_000_000
    need = ctypes.c_size_t(0)
    assert lib.tlb_paged_attention_workspace_size(S, 16, 2, 128, _lib.DTYPE_CODE[torch.bfloat16],
                                                  ctypes.byref(need)) == 0
    assert need.value > NO_ALLOC_BYTES
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    assert p % 256 == 0
    rc = lib.tlb_paged_attention_no_alloc(p, p, p, p, p, p, S, 16, 2, 128, 10, 16, 4, 0.1,
                                          _lib.DTYPE_CODE[torch.bfloat16], 0,
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == 4
    assert "static buffer" in _lib.last_error()
    torch.cuda.synchronize()
    assert int(buf.count_nonzero()) == 0


def test_no_alloc_recovers_after_a_wait_gave_up(built_lib):
    """A launch whose waits gave up may leave counters set in the static array;
    reading the status word marks it for clearing before the next call."""
    lib = _lib.load()
    b = _batch("qwen3b_bf16", 64)
    ref = _with_fresh_workspace(lib, b)
    _lib.set_wait_limit(0)  # gives up at once: deterministic status
    _no_alloc(lib, b)
    _lib.set_wait_limit(16)  # lets part of the work through: counters left set
    for _ in range(3):
        _no_alloc(lib, b)
    torch.cuda.synchronize()
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    assert _lib.device_status() & _lib.STATUS_WAIT_TIMEOUT
    for _ in range(2):
        out = _no_alloc(lib, b)
        torch.cuda.synchronize()
        assert torch.equal(_bits(out), _bits(ref))
    assert _lib.device_status() == 0
