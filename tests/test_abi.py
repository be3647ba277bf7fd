"""The C-ABI library loads and exports every entry point include/xpager.h declares.

No GPU needed: only symbol lookup and host-side argument checks.
"""

import ctypes
import os
import re

from vllm_expert_pager import native

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "xpager.h")


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    return [m.group(1) for m in
            re.finditer(r"^(?:const\s+)?[a-z_0-9]+\s*\*?\s*([a-z_0-9]+)\s*\(", text, flags=re.M)]


def test_header_declares_entry_points():
    names = declared()
    assert "xp_gather_rows" in names and "ssd_start" in names and len(names) >= 20


def test_library_exports_every_declared_symbol():
    so = ctypes.CDLL(native.LIB_PATH)
    for name in declared():
        assert hasattr(so, name), name


def test_bindings_cover_the_header():
    assert sorted(declared()) == sorted(native._SIGNATURES)


def test_status_strings_and_version():
    lib = native.lib()
    assert lib.xp_version() >= 1
    assert b"invalid" in lib.xp_status_string(native.XP_EINVAL)
    assert b"pitch" in lib.xp_status_string(native.XP_EPITCH)


def test_device_calls_reject_bad_arguments_before_launching():
    # Argument checks run on the host and return before any CUDA call.
    lib = native.lib()
    assert lib.xp_acquire(None, 3, 1, 16, None, None, None, None, 4, None, None, None,
                          None) == native.XP_EINVAL
    assert lib.xp_decode_rows(None, 1, None, None, None, None, 0, None, 0, None, 0, None, 0,
                              None, 7, None) == native.XP_EINVAL
    assert lib.xp_fetch_wait(None, 1, None, None, None, 256, 4, 1, 1, None) == native.XP_EINVAL


def test_fetch_wait_limits_are_checked_before_launching():
    # A wait interval above one hour or more than 2**20 re-publishes is refused, so the
    # device-side time limit (giveup + 2) * retry_ns cannot overflow.
    lib = native.lib()
    buf = (ctypes.c_int64 * 64)()
    p = ctypes.addressof(buf)
    one_hour = 3600 * 10**9
    assert lib.xp_fetch_wait(p, 1, p, p, p, 8, 4, one_hour + 1, 1, None) == native.XP_EINVAL
    assert lib.xp_fetch_wait(p, 1, p, p, p, 8, 4, 1, (1 << 20) + 1, None) == native.XP_EINVAL
    assert lib.xp_fetch(p, 1, p, 0, 0, p, p, p, 8, 4, one_hour + 1, 1, None) == native.XP_EINVAL
    assert lib.xp_fetch(p, 1, p, 0, 0, p, p, p, 8, 4, 1, -1, None) == native.XP_EINVAL


def test_encode_scratch_size_and_argument_checks():
    lib = native.lib()
    # 2 MiB rows, chunk 512: G = 128 groups -> 256-byte-rounded per-row scratch.
    per_row = lib.xp_encode_scratch_bytes(1, 2 * 1024 * 1024, 512)
    assert per_row > 0 and per_row % 256 == 0 and per_row >= 4 * (2 * 128 + 1)
    assert lib.xp_encode_scratch_bytes(8, 2 * 1024 * 1024, 512) == 8 * per_row
    assert lib.xp_encode_scratch_bytes(1, 1000, 512) == -1  # not a multiple of 32 * chunk
    assert lib.xp_encode_scratch_bytes(1, 4096, 12) == -1   # chunk not a multiple of 8
    assert lib.xp_encode_rows(None, 1, 4096, 8192, 64, None, None, None, None, 0,
                              None) == native.XP_EINVAL
    assert lib.xp_encode_rows(None, 0, 4096, 8192, 64, None, None, None, None, 0,
                              None) == native.XP_OK


def test_step_wait_limits_are_checked():
    lib = native.lib()
    one_hour = 3600 * 10**9
    assert lib.xp_set_step_wait_ns(one_hour + 1, -1) == native.XP_EINVAL
    assert lib.xp_set_step_wait_ns(-1, one_hour + 1) == native.XP_EINVAL
    assert lib.xp_set_step_wait_ns(-1, -1) == native.XP_OK


def test_noalloc_sizes_are_bounded_before_multiplying():
    # K above the step's list limit, or a pitch beyond the array, is XP_ERANGE before
    # K x (P0 + P1) x 4 is formed: 8 x 2**60 words would wrap to a small size.
    lib = native.lib()
    table_a = [None] * 4 + [8] + [None] * 3
    table_b = [None] * 4 + [16] + [None] * 2

    def call(K, P0, P1):
        return lib.xp_decode_step_noalloc(
            None, 4, K, 32, *table_a, *table_b, None, 0,
            None, None, 16, P0, None, None, 16, P1,
            None, None, 4, None, None, 4,
            1, None, 512, 16, 0, None, None, None, 256, 4, 1, 1, None, None)

    assert call(8, 1 << 60, 16) == native.XP_ERANGE
    assert call(8, 16, 1 << 60) == native.XP_ERANGE
    assert call(2049, 16, 16) == native.XP_ERANGE
    assert call(4, 1 << 22, 1 << 22) == native.XP_ERANGE  # 4 x 32 MiB: beyond the array
