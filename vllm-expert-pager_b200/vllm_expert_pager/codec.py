"""Lossless compression of fp8 e4m3 expert rows (RAM and SSD tiers).

Mirrors src/vllm_expert_pager/codec.py of monochromegane/vllm-expert-pager and
keeps its record format byte for byte (codec.py:22-26): a header of G+1 int32
group starts, the sign+mantissa nibbles as 32-bit words in (group, word,
lane) order, then the Huffman words of each group in refill order.  Exponent
codes are canonical, bit-reversed and at most LIMIT bits; the 512-byte LUT of a
row lives in a VRAM table, not in the record.

``encode`` runs at load time in the native library (encode.cpp, a loop over the
row on the host); ``decode_rows`` expands staging rows on the GPU
(decode.cu).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from vllm_expert_pager import native

# Maximum code length; the LUT has 2**LIMIT entries.
LIMIT = 9
LUT_BYTES = 1 << LIMIT
# Values handled by one lane, and lanes per group (one warp).
CHUNK = 512
LANES = 32
# A row's value count must be a multiple of this.
GROUP = CHUNK * LANES


def pitch_of(n_values: int, ratio: float, align: int) -> int:
    """Fixed record length: ratio times the raw size, rounded up to align (codec.py:117-119)."""
    return -(-int(n_values * ratio) // align) * align


def groups(n_bytes: int, chunk: int = CHUNK) -> int:
    """Number of groups in one row."""
    return n_bytes // (chunk * LANES)


def encode(raw: torch.Tensor, pitch: int, chunk: int = CHUNK) -> tuple[torch.Tensor, torch.Tensor]:
    """Compress a uint8 row (N,). Returns ``(record of pitch bytes, 512 B LUT)`` on raw's device.

    Raises ValueError if the row does not fit in the record (codec.py:125-193).
    """
    N = raw.numel()
    if N % (chunk * LANES):
        raise ValueError(f"row of {N} values is not a multiple of {chunk * LANES}")
    host = np.ascontiguousarray(raw.reshape(-1).detach().cpu().numpy().view(np.uint8))
    record = np.empty(pitch, dtype=np.uint8)
    lut = np.empty(LUT_BYTES, dtype=np.uint8)
    used = ctypes.c_int64(0)
    rc = native.lib().xp_encode_row(host.ctypes.data, N, pitch, chunk, record.ctypes.data,
                                    lut.ctypes.data, ctypes.byref(used))
    if rc == native.XP_EPITCH:
        nbytes = used.value
        raise ValueError(
            f"compressed row is {nbytes} B, pitch is {pitch} B; "
            f"VLLM_EXPERT_PAGER_PITCH must be at least {nbytes / N:.4f}"
        )
    native.check(rc, "encode")
    return (torch.from_numpy(record).to(raw.device), torch.from_numpy(lut).to(raw.device))


def decode_rows(
    todo: torch.Tensor,
    dst_row: torch.Tensor,
    cache_row: torch.Tensor,
    staging: list[torch.Tensor],
    dst: list[torch.Tensor],
    lut: torch.Tensor,
    skip: torch.Tensor | None = None,
    chunk: int = CHUNK,
) -> None:
    """Expand ``staging[name][j]`` (the j-th compressed row of todo) into ``dst[name][dst_row[e]]``.

    Same contract as codec.py:297-327: two-element lists in name order,
    ``staging`` ``(*, pitch)`` uint8, ``dst`` ``(*, N)`` uint8, ``lut`` this
    layer's ``(E, 2, 512)`` uint8.  Experts with ``cache_row[e] >= 0`` and, with
    ``skip``, those listed in it are not expanded.
    """
    native.require_cuda(todo, dst_row, cache_row, lut, *staging, *dst, skip)
    K = todo.shape[0]
    P0, P1 = staging[0].shape[1], staging[1].shape[1]
    N0, N1 = dst[0].shape[1], dst[1].shape[1]
    native.check(
        native.lib().xp_decode_rows(
            todo.data_ptr(), K, dst_row.data_ptr(), cache_row.data_ptr(), lut.data_ptr(),
            staging[0].data_ptr(), P0, dst[0].data_ptr(), N0,
            staging[1].data_ptr(), P1, dst[1].data_ptr(), N1,
            native.ptr(skip), chunk, native.stream_of(todo.device),
        ),
        "decode_rows",
    )  # fmt: skip
