"""Bounded waits of the tensor-core attention kernel: a wait that gives up is
reported, and the next call on the same workspace is correct again.

Every pipeline wait of the kernel (a stage's data, a free stage, a hand-off to
the epilogue warp, a phase of the consumer warps' merge) probes its mbarrier
at most ``tlb_attention_set_wait_limit`` times, then sets
TLB_STATUS_WAIT_TIMEOUT, lets the copies it already issued land (those drains
keep the default bound: an issued copy always lands) and returns. These tests
lower the bound so that waits run out on purpose. Nothing here faults, traps
or spins: every input is valid and in bounds, and every wait still ends.

A kernel that gave up may leave split pieces' arrival counters set in its
workspace. Reading the status word (``_lib.device_status``) marks this
device's workspaces for re-zeroing, so the next call is exact again.
"""

import numpy as np
import pytest
import torch

from cscr import _lib
from cscr import attention as A
from helpers import check_attention
from paged_decode import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _default_limit():
    torch.cuda.set_device(0)
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    _lib.device_status(clear=True)
    yield
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    torch.cuda.synchronize()
    _lib.device_status(clear=True)


def _attend(b):
    return A.paged_attention(b.query, b.key_cache, b.value_cache, b.block_tables, b.seq_lens,
                             b.scale)


def _workspace():
    return A._workspaces[(torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)]


def test_zero_limit_gives_up_and_next_call_is_exact(built_lib):
    b = W.make_batch(W.qwen3b_decode(5, batch=64))
    good = _attend(b)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0

    _lib.set_wait_limit(0)  # every pipeline wait gives up at once
    _attend(b)
    torch.cuda.synchronize()
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    status = _lib.device_status()  # reading it marks the workspaces for re-zeroing
    assert status & _lib.STATUS_WAIT_TIMEOUT
    assert _workspace().clean == 0

    again = _attend(b)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(again.view(torch.int16), good.view(torch.int16))


@pytest.mark.parametrize("limit", [1, 4, 32, 512])
def test_small_limits_end_and_recover(limit, built_lib):
    """Limits that let part of the work through: some pieces publish partials
    and take tickets, others give up. Every launch ends; after the status is
    read, the next call with the default bound gives the exact bits again and
    leaves every counter at zero."""
    lens = [8192, 8192, 300, 5000, 20000, 64, 1, 4096]
    spec = W.DecodeSpec("splits", lens, 16, 2, 128, 16, "bfloat16",
                        num_blocks=sum(-(-L // 16) for L in lens) + 8, seed=2)
    b = W.make_batch(spec)
    good = _attend(b)
    torch.cuda.synchronize()
    _lib.set_wait_limit(limit)
    for _ in range(3):
        _attend(b)
    torch.cuda.synchronize()
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    status = _lib.device_status()
    assert status & ~_lib.STATUS_WAIT_TIMEOUT == 0  # nothing but timeouts
    again = _attend(b)
    torch.cuda.synchronize()
    assert torch.equal(again.view(torch.int16), good.view(torch.int16))
    ws = _workspace()
    assert int(ws.buf[:ws.clean].count_nonzero()) == 0
    check_attention(b, again)


def test_timeout_raises_under_debug_checks(built_lib, monkeypatch):
    """With TLB_DEBUG-style checking on, the op itself raises with the reason."""
    b = W.make_batch(W.qwen3b_decode(1, batch=16))
    monkeypatch.setattr(_lib, "DEBUG", True)
    _lib.set_wait_limit(0)
    with pytest.raises(RuntimeError, match="bounded pipeline wait timed out"):
        _attend(b)
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    out = _attend(b)  # checked too: must raise nothing
    check_attention(b, out)


def test_fused_step_times_out_and_recovers(built_lib):
    """The one-launch decode step (RoPE + cache write + attention) under a zero
    limit gives up and says so. What it left in the key and the caches is not
    promised, so after recovery the step runs on fresh copies of the inputs
    and must match the two-launch form bit for bit."""
    spec = W.qwen3b_decode(3, batch=32)
    S = 32
    b = W.make_batch(spec)
    _lib.set_wait_limit(0)
    A.paged_attention_with_rope(b.query, b.key.view(S, -1), b.value, b.key_cache,
                                b.value_cache, b.block_tables, b.seq_lens, b.cos_sin_cache,
                                b.scale)
    torch.cuda.synchronize()
    _lib.set_wait_limit(_lib.WAIT_LIMIT_DEFAULT)
    assert _lib.device_status() & _lib.STATUS_WAIT_TIMEOUT
    b2 = W.make_batch(spec)
    q_raw = b2.query.clone()
    out = A.paged_attention_with_rope(b2.query, b2.key.view(S, -1), b2.value, b2.key_cache,
                                      b2.value_cache, b2.block_tables, b2.seq_lens,
                                      b2.cos_sin_cache, b2.scale)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    # the same step as two launches on a third copy: identical bits
    b3 = W.make_batch(spec)
    from cscr import pos_encoding as PE

    q_rot = PE.rotary_embedding_neox_with_cache(b3.positions, b3.query.view(S, -1),
                                                b3.key.view(S, -1), b3.value, b3.key_cache,
                                                b3.value_cache, b3.slot_mapping, 128,
                                                b3.cos_sin_cache)
    ref = A.paged_attention(q_rot.view(S, 16, 128), b3.key_cache, b3.value_cache,
                            b3.block_tables, b3.seq_lens, b3.scale)
    torch.cuda.synchronize()
    assert torch.equal(q_raw.view(torch.int16), b2.query.view(torch.int16))
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert np.array_equal(W.to_numpy(b2.key_cache), W.to_numpy(b3.key_cache))
