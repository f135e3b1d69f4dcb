"""Loader and ctypes binding of libtinyllama_b200.so (the sm_100a C ABI).

The op modules of this package call the library through the prototypes
declared here; no compute runs in Python and there is no CPU path: if the
library is missing or a tensor is not on a CUDA device the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_NAME = "libtinyllama_b200.so"
LIB_PATH = Path(__file__).resolve().with_name(LIB_NAME)

TLB_OK = 0
TLB_ERR_UNSUPPORTED = 2
DTYPE_CODE = {
    torch.float32: 0,
    torch.float16: 1,
    torch.bfloat16: 2,
    torch.int32: 3,
    torch.int64: 4,
}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> argtypes (all return int status unless listed in _RESTYPES)
_PROTOS = {
    "tlb_last_error": [],
    "tlb_version": [],
    "tlb_get_device_status": [ctypes.POINTER(ctypes.c_uint32), _i32, _vp],
    "tlb_attention_set_wait_limit": [ctypes.c_uint32],
    "tlb_paged_attention_workspace_size": [_i64, _i64, _i64, _i64, _i32, ctypes.POINTER(_sz)],
    "tlb_paged_attention_workspace_zeroed_bytes": [_i64, _i64, ctypes.POINTER(_sz)],
    "tlb_paged_attention": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                            _i64, _f32, _i32, _vp, _sz, ctypes.c_uint, _vp],
    "tlb_paged_attention_no_alloc": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                     _i64, _i64, _f32, _i32, ctypes.c_uint, _vp],
    "tlb_paged_attention_with_rope": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                      _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32,
                                      _vp, _sz, ctypes.c_uint, _vp],
    "tlb_paged_prefill_attention": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                    _i64, _i64, _i64, _i64, _f32, _i32, _vp],
    "tlb_rotary_embedding_neox": [_vp, _vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64,
                                  _i64, _i64, _i64, _i64, _i32, _vp],
    "tlb_reshape_and_cache": [_vp, _vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64,
                              _i64, _i32, _vp],
    "tlb_write_kv_cache": [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                           _i64, _i64, _i32, _vp],
    "tlb_rotary_embedding_neox_with_cache": [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i32,
                                             _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64,
                                             _i64, _i64, _i64, _i64, _i64, _i64, _i32,
                                             ctypes.c_uint, _vp],
    "tlb_copy_blocks": [ctypes.POINTER(_vp), _i64, ctypes.POINTER(_i64), _i64, _i64, _vp],
    "tlb_swap_blocks": [_vp, _i32, _vp, _i32, ctypes.POINTER(_i64), _i64, _i64, _vp],
    "tlb_decode_metadata": [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp],
    "tlb_step_metadata": [_vp, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp,
                          _vp],
}
_RESTYPES = {"tlb_last_error": ctypes.c_char_p, "tlb_version": ctypes.c_char_p}

# Exported names, in the order include/tinyllama_b200.h declares them.
EXPORTS = tuple(_PROTOS)

_lib = None
_lock = threading.Lock()


def load():
    """Load (once) and return the ctypes handle of the library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = Path(os.environ.get("TLB_LIBRARY", LIB_PATH))
            if not path.exists():
                raise RuntimeError(
                    f"{LIB_NAME} is not built ({path}); run `python tinyllama.py_b200/build.py`")
            lib = ctypes.CDLL(str(path))
            for name, args in _PROTOS.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().tlb_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    """Raise RuntimeError with the library's message for a non-zero status."""
    if rc != TLB_OK:
        raise RuntimeError(last_error() or f"tinyllama_b200 call failed with status {rc}")
    if DEBUG:
        device_status(clear=True, raise_on_error=True)


def torch_check(cond: bool, msg: str) -> None:
    """TORCH_CHECK equivalent: RuntimeError with the reference's message."""
    if not cond:
        raise RuntimeError(msg)


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class device_guard:
    """Make `device` current for the duration of a call (OptionalCUDAGuard)."""

    __slots__ = ("index", "prev")

    def __init__(self, device: torch.device):
        self.index = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


STATUS_WAIT_TIMEOUT = 0x10
STATUS_BITS = {
    0x1: "block id outside the KV pool",
    0x2: "seq_len larger than max_blocks_per_seq * block_size",
    0x4: "position outside the cos/sin table",
    0x8: "slot or logical block outside the cache",
    0x10: "a bounded pipeline wait timed out",
}

def set_wait_limit(tries: int) -> None:
    """Probes before a pipeline wait of the attention kernels gives up
    (failure injection for tests; TLB_WAIT_LIMIT_DEFAULT restores)."""
    check(load().tlb_attention_set_wait_limit(int(tries)))


WAIT_LIMIT_DEFAULT = 1 << 22

# With TLB_DEBUG=1 every op synchronises and raises on a non-zero device
# status word (bounds problems the kernels skipped instead of faulting).
DEBUG = os.environ.get("TLB_DEBUG", "0") not in ("", "0")


def device_status(clear: bool = True, raise_on_error: bool = False) -> int:
    """Read (and clear) the current device's status word; see STATUS_BITS."""
    v = ctypes.c_uint32(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    rc = load().tlb_get_device_status(ctypes.byref(v), 1 if clear else 0, stream_of(dev))
    if rc != TLB_OK:
        raise RuntimeError(last_error())
    if v.value & STATUS_WAIT_TIMEOUT:
        # A kernel that gave up a wait may have left arrival counters set in
        # the attention workspaces of this device: zero them before reuse.
        from . import attention

        attention.invalidate_workspaces(dev.index)
    if raise_on_error and v.value:
        names = [m for b, m in STATUS_BITS.items() if v.value & b]
        raise RuntimeError("tinyllama_b200 device status: " + "; ".join(names))
    return v.value
