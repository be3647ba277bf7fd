"""ctypes loader for ``oracle/liboracle.so``.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may use it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def build() -> str:
    """Compile liboracle.so with make (gcc only, seconds)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "liboracle.so")


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        so = ctypes.CDLL(path)
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        so.oracle_decode_row.argtypes = [p, i64, p, i64, i64, p]
        so.oracle_decode_row.restype = i32
        so.oracle_decode_rows.argtypes = [p, i64, p, i64, i64, i64, p, i32]
        so.oracle_decode_rows.restype = i32
        so.oracle_copy_rows.argtypes = [p, i64, p, p, i64, p, i64, i64, i32]
        so.oracle_copy_rows.restype = i32
        _LIB = so
    return _LIB


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def decode(rec: np.ndarray, lut: np.ndarray, n: int, chunk: int = 512) -> np.ndarray:
    """Decode one record (uint8) with its 512-B LUT into n raw bytes."""
    rec = np.ascontiguousarray(rec, dtype=np.uint8)
    lut = np.ascontiguousarray(lut, dtype=np.uint8)
    out = np.zeros(n, dtype=np.uint8)
    rc = lib().oracle_decode_row(_ptr(rec), rec.size, _ptr(lut), n, chunk, _ptr(out))
    if rc:
        raise ValueError(f"oracle decode failed ({rc})")
    return out


def decode_rows(recs: np.ndarray, luts: np.ndarray, n: int, chunk: int = 512,
                threads: int = 1) -> np.ndarray:
    """Decode records ``recs[rows, pitch]`` with ``luts[rows, 512]`` on ``threads`` threads."""
    recs = np.ascontiguousarray(recs, dtype=np.uint8)
    luts = np.ascontiguousarray(luts, dtype=np.uint8)
    rows, pitch = recs.shape
    out = np.zeros((rows, n), dtype=np.uint8)
    rc = lib().oracle_decode_rows(_ptr(recs), pitch, _ptr(luts), rows, n, chunk, _ptr(out),
                                  threads)
    if rc:
        raise ValueError(f"oracle decode failed ({rc})")
    return out


def copy_rows(src_ptr: int, src_pitch: int, src_rows: np.ndarray, dst_ptr: int,
              dst_pitch: int, dst_rows: np.ndarray, row_bytes: int, threads: int) -> None:
    """memcpy rows ``src_rows[i] -> dst_rows[i]`` between two host buffers."""
    s = np.ascontiguousarray(src_rows, dtype=np.int64)
    d = np.ascontiguousarray(dst_rows, dtype=np.int64)
    lib().oracle_copy_rows(src_ptr, src_pitch, _ptr(s), dst_ptr, dst_pitch, _ptr(d), s.size,
                           row_bytes, threads)
