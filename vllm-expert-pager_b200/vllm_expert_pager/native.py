"""Load ``libxpager.so`` (the CUDA kernels and the host server) through ctypes.

The reference compiles its C server at first use (native.py of
monochromegane/vllm-expert-pager); here the library is built ahead of time
(``make -C vllm-expert-pager_b200/csrc``, or ``__graft_entry__.build()``) and
ships in the package directory.  There is no fallback: if the library is
missing or a call fails, an exception says why.
"""

from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libxpager.so")

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_long = ctypes.c_long

# name -> (restype, argtypes); the order follows include/xpager.h.
_SIGNATURES = {
    "xp_version": (_i32, []),
    "xp_status_string": (ctypes.c_char_p, [_i32]),
    "xp_acquire_pair": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _p, _i64, _p, _p, _p,
                              _p, _p, _p, _p, _i64, _p, _p, _p]),
    "xp_acquire": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _p, _i64, _p, _p, _p, _p]),
    "xp_need_mask": (_i32, [_p, _i32, _i64, _i64, _p, _p]),
    "xp_seed": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _p, _i64, _p, _i64, _p, _p, _p, _p]),
    "xp_plan_chunks": (_i32, [_i64, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p,
                              _p]),
    "xp_plan_working": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _p, _i64, _p, _p, _i64,
                               _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "xp_gather_rows": (_i32, [_p, _i64, _p, _p, _p, _i64,
                              _p, _p, _p, _p, _i64, _i64,
                              _p, _p, _p, _p, _i64, _i64,
                              _p, _p, _i64, _p, _p, _i64,
                              _p, _i32, _i64, _i32,
                              _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "xp_fetch_publish": (_i32, [_p, _i64, _p, _i64, _i64, _p, _p, _p, _i64, _i64, _p]),
    "xp_fetch_wait": (_i32, [_p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "xp_fetch": (_i32, [_p, _i64, _p, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "xp_decode_step": (_i32, [_p, _i32, _i64, _i64,
                              _p, _p, _p, _p, _i64, _p, _p, _p, _p,
                              _p, _p, _p, _p, _i64, _p, _p,
                              _p, _i64,
                              _p, _p, _p, _i64, _i64,
                              _p, _p, _p, _i64, _i64,
                              _p, _p, _i64, _p, _p, _i64,
                              _i32, _i64, _i32, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p,
                              _p, _p]),
    "xp_set_step_wait_ns": (_i32, [_i64, _i64]),
    "xp_decode_step_noalloc": (_i32, [_p, _i32, _i64, _i64,
                                      _p, _p, _p, _p, _i64, _p, _p, _p,
                                      _p, _p, _p, _p, _i64, _p, _p,
                                      _p, _i64,
                                      _p, _p, _i64, _i64,
                                      _p, _p, _i64, _i64,
                                      _p, _p, _i64, _p, _p, _i64,
                                      _i32, _p, _i64, _i32, _i64, _p, _p, _p, _i64, _i64, _i64,
                                      _i64, _p, _p]),
    "xp_decode_rows": (_i32, [_p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _p,
                              _i64, _p]),
    "xp_encode_row": (_i32, [_p, _i64, _i64, _i64, _p, _p, ctypes.POINTER(_i64)]),
    "xp_encode_scratch_bytes": (_i64, [_i64, _i64, _i64]),
    "xp_encode_rows": (_i32, [_p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _p]),
    "xp_pinned_alloc": (_i32, [_i64, _i32, ctypes.POINTER(_p), ctypes.POINTER(_p)]),
    "xp_pinned_free": (_i32, [_p, _i64]),
    "xp_device_pointer": (_i32, [_p, ctypes.POINTER(_p)]),
    "ssd_start": (_p, [_i32, _p, _p] + [_long] * 6 + [_i32, _p, _p, _i32]),
    "ssd_stop": (None, [_p]),
    "ssd_stats": (None, [_p, ctypes.POINTER(_long), ctypes.POINTER(_long),
                         ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_long)]),
    "ssd_error": (ctypes.c_char_p, [_p]),
    "ssd_test_delay": (None, [_p, ctypes.c_double]),
    "ssd_numa_node": (_i32, [_p]),
    "ssd_set_read_chunk": (None, [_p, _long]),
    "ssd_set_used_bytes": (None, [_p, _p]),
    "ssd_bytes_read": (_long, [_p]),
}

XP_OK = 0
XP_EINVAL = -22
XP_ERANGE = -34
XP_EPITCH = -75

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library.  Raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"vllm-expert-pager: {LIB_PATH} is missing; build it with "
                "`make -C vllm-expert-pager_b200/csrc` (there is no fallback path)"
            )
        so = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(so, name)
            fn.restype = res
            fn.argtypes = args
        _lib = so
    return _lib


def check(rc: int, what: str) -> None:
    """Raise for a non-zero status of a libxpager call."""
    if rc != XP_OK:
        msg = lib().xp_status_string(rc).decode(errors="replace")
        exc = ValueError if rc < 0 else RuntimeError
        raise exc(f"vllm-expert-pager: {what} failed ({rc}: {msg})")


def ptr(t: torch.Tensor | None) -> int | None:
    """Device (or host) address of a tensor, None for None."""
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    """Handle of the current CUDA stream of ``device`` (captured streams included)."""
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise ValueError(
                f"vllm-expert-pager: expected a CUDA tensor, got one on {t.device}"
            )
