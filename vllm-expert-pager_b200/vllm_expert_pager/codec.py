"""Lossless compression of fp8 e4m3 expert rows (RAM and SSD tiers).

Mirrors src/vllm_expert_pager/codec.py of monochromegane/vllm-expert-pager and
keeps its record format byte for byte (codec.py:22-26): a header of G+1 int32
group starts, the sign+mantissa nibbles as 32-bit words in (group, word,
lane) order, then the Huffman words of each group in refill order.  Exponent
codes are canonical, bit-reversed and at most LIMIT bits; the 512-byte LUT of a
row lives in a VRAM table, not in the record.

``encode`` runs at load time: rows on a GPU are encoded there in batches
(``encode_rows``, encode_gpu.cu), as the reference encodes with torch ops on the
GPU; rows on the host go to the native host encoder (encode.cpp).
``decode_rows`` expands staging rows on the GPU (decode.cu).
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


def _pitch_error(nbytes: int, pitch: int, N: int) -> ValueError:
    return ValueError(
        f"compressed row is {nbytes} B, pitch is {pitch} B; "
        f"VLLM_EXPERT_PAGER_PITCH must be at least {nbytes / N:.4f}"
    )


# Rows per launch of the GPU encoder (its grid's y extent).
_ENCODE_BATCH = 65535


def encode_rows(raw: torch.Tensor, pitch: int, chunk: int = CHUNK) -> tuple[torch.Tensor, torch.Tensor]:
    """Compress uint8 rows ``(R, N)`` on their GPU (encode_gpu.cu).

    Returns ``(records (R, pitch), LUTs (R, 512))`` on raw's device, each row
    byte-identical to codec.encode of the reference (codec.py:125-193).  Raises
    ValueError, as the reference does for its row, if a row does not fit in the
    record; this reads the record sizes back (one synchronisation per call).
    """
    native.require_cuda(raw)
    raw = raw.detach().contiguous().view(torch.uint8)
    raw = raw.reshape(raw.shape[0], -1) if raw.dim() > 1 else raw.reshape(1, -1)
    if raw.data_ptr() % 16:
        raw = raw.clone()
    R, N = raw.shape
    if N % (chunk * LANES):
        raise ValueError(f"row of {N} values is not a multiple of {chunk * LANES}")
    dev = raw.device
    records = torch.empty((R, pitch), dtype=torch.uint8, device=dev)
    luts = torch.empty((R, LUT_BYTES), dtype=torch.uint8, device=dev)
    used = torch.empty((R,), dtype=torch.int64, device=dev)
    lib = native.lib()
    for r0 in range(0, R, _ENCODE_BATCH):
        r1 = min(R, r0 + _ENCODE_BATCH)
        nb = lib.xp_encode_scratch_bytes(r1 - r0, N, chunk)
        if nb < 0:
            raise ValueError(f"cannot encode rows of {N} values with chunk {chunk}")
        scratch = torch.empty((max(nb, 1),), dtype=torch.uint8, device=dev)
        native.check(
            lib.xp_encode_rows(raw[r0].data_ptr(), r1 - r0, N, pitch, chunk,
                               records[r0].data_ptr(), luts[r0].data_ptr(),
                               used[r0:].data_ptr(), scratch.data_ptr(), nb,
                               native.stream_of(dev)),
            "encode_rows",
        )
    over = (used > pitch).nonzero()
    if over.numel():
        raise _pitch_error(int(used[int(over[0])]), pitch, N)
    return records, luts


def encode(raw: torch.Tensor, pitch: int, chunk: int = CHUNK) -> tuple[torch.Tensor, torch.Tensor]:
    """Compress a uint8 row (N,). Returns ``(record of pitch bytes, 512 B LUT)`` on raw's device.

    A row on a GPU is encoded there (``encode_rows``); a row on the host by the
    native host encoder.  Raises ValueError if the row does not fit in the
    record (codec.py:125-193).
    """
    N = raw.numel()
    if N % (chunk * LANES):
        raise ValueError(f"row of {N} values is not a multiple of {chunk * LANES}")
    if raw.is_cuda:
        records, luts = encode_rows(raw.reshape(1, -1), pitch, chunk)
        return records[0], luts[0]
    host = np.ascontiguousarray(raw.reshape(-1).detach().cpu().numpy().view(np.uint8))
    record = np.empty(pitch, dtype=np.uint8)
    lut = np.empty(LUT_BYTES, dtype=np.uint8)
    used = ctypes.c_int64(0)
    rc = native.lib().xp_encode_row(host.ctypes.data, N, pitch, chunk, record.ctypes.data,
                                    lut.ctypes.data, ctypes.byref(used))
    if rc == native.XP_EPITCH:
        raise _pitch_error(used.value, pitch, N)
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
