"""CPU oracle for the fp8-exponent Huffman codec.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU baseline
legs) may import this module.  The product encoder lives in the package's
native library; this file is the independent checker.

Restates monochromegane/vllm-expert-pager ``src/vllm_expert_pager/codec.py``:

* ``huffman_lengths`` / ``code_lengths``: codec.py:61-87 (same heap order, so
  the same code lengths on ties);
* ``Code``: codec.py:90-114 (canonical, bit-reversed, 512-entry LUT of
  ``sym << 4 | len``);
* ``pitch_of``: codec.py:117-119;
* ``encode``: codec.py:125-193 (record layout codec.py:22-26, refill order
  codec.py:150-181), here in numpy;
* ``decode_py``: the sequential decoder of the reference's
  tests/test_codec.py:49-79, for small rows.  ``decode`` uses the C
  restatement in ``oracle/decode.c`` (same loop) through ``oracle/_lib.py``.

Parity pin: tests/test_oracle_codec.py compares ``encode`` byte for byte with
records and LUTs that the reference's own ``codec.encode`` produced
(tests/golden/make_golden.py), and decodes them back to the raw bytes.
"""

from __future__ import annotations

import heapq

import numpy as np

LIMIT = 9
LUT_BYTES = 1 << LIMIT
CHUNK = 512
LANES = 32
GROUP = CHUNK * LANES


def huffman_lengths(counts: list[float]) -> list[int]:
    """Plain Huffman code lengths; heap entries are (count, tiebreak, members)."""
    heap = [(c, i, (i,)) for i, c in enumerate(counts)]
    heapq.heapify(heap)
    lengths = [0] * len(counts)
    nxt = len(counts)
    while len(heap) > 1:
        c1, _, m1 = heapq.heappop(heap)
        c2, _, m2 = heapq.heappop(heap)
        for s in m1 + m2:
            lengths[s] += 1
        heapq.heappush(heap, (c1 + c2, nxt, m1 + m2))
        nxt += 1
    return lengths


def code_lengths(hist, limit: int = LIMIT) -> list[int]:
    """Length-limited code lengths: raise rare counts until the tree fits."""
    counts = [float(max(int(c), 1)) for c in hist]
    k = 0
    while True:
        lengths = huffman_lengths(counts)
        if max(lengths) <= limit:
            return lengths
        k += 1
        floor = sum(counts) / 2 ** (limit - k)
        counts = [max(c, floor) for c in counts]


class Code:
    """Canonical code for the 16 exponent symbols with its decode LUT."""

    def __init__(self, hist) -> None:
        self.lengths = code_lengths(hist)
        order = sorted(range(16), key=lambda s: (self.lengths[s], s))
        canon = [0] * 16
        code = 0
        for i, s in enumerate(order):
            if i:
                code = (code + 1) << (self.lengths[s] - self.lengths[order[i - 1]])
            canon[s] = code
        self.codes = [
            int(format(canon[s], f"0{self.lengths[s]}b")[::-1], 2) for s in range(16)
        ]
        lut = np.full(LUT_BYTES, -1, dtype=np.int64)
        for s in range(16):
            n = self.lengths[s]
            x = self.codes[s] | (np.arange(1 << (LIMIT - n), dtype=np.int64) << n)
            if (lut[x] >= 0).any():
                raise AssertionError("codes are not prefix-free")
            lut[x] = (s << 4) | n
        if (lut < 0).any():
            raise AssertionError("codes do not fill the LUT (Kraft sum < 1)")
        self.lut = lut.astype(np.uint8)


def pitch_of(n_values: int, ratio: float, align: int) -> int:
    return -(-int(n_values * ratio) // align) * align


def encode(raw, pitch: int, chunk: int = CHUNK):
    """Compress a uint8 row. Returns ``(record uint8[pitch], lut uint8[512], used_bytes)``."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    N = raw.size
    if N % (chunk * LANES):
        raise ValueError(f"row of {N} values is not a multiple of {chunk * LANES}")
    C, G = N // chunk, N // (chunk * LANES)
    exp = ((raw >> 3) & 15).astype(np.int64)
    sm = ((raw >> 7) << 3) | (raw & 7)
    fixed = (sm[0::2] | (sm[1::2] << 4)).astype(np.uint8)
    fixed = fixed.reshape(G, LANES, chunk // 8, 4).transpose(0, 2, 1, 3).reshape(-1)

    code = Code(np.bincount(exp, minlength=16).tolist())
    lengths = np.asarray(code.lengths, dtype=np.int64)
    codes = np.asarray(code.codes, dtype=np.int64)
    n = lengths[exp].reshape(C, chunk)
    before = np.cumsum(n, axis=1) - n
    # The k-th refill of a chunk happens at its first symbol i with
    # before[i] >= 32k - (LIMIT - 1); nw is the chunk's word count.
    nw = (before[:, -1] + (LIMIT - 1)) // 32 + 1
    total_words = int(nw.sum())
    head = 4 * (G + 1) + N // 2
    nbytes = head + 4 * total_words
    if nbytes > pitch:
        raise ValueError(
            f"compressed row is {nbytes} B, pitch is {pitch} B; "
            f"VLLM_EXPERT_PAGER_PITCH must be at least {nbytes / N:.4f}"
        )
    # Per-chunk bit streams, concatenated.
    wbase = np.cumsum(nw) - nw
    start = (wbase * 32)[:, None] + before
    v = codes[exp].reshape(C, chunk)
    w, sh = start >> 5, start & 31
    # The bit ranges of the codes do not overlap, so a sum equals an OR; every
    # partial sum stays below 2**32 and is exact in float64.
    lo = np.bincount(w.reshape(-1), ((v << sh) & 0xFFFFFFFF).reshape(-1).astype(np.float64),
                     minlength=total_words + 1)
    hi = np.bincount((w + 1).reshape(-1), (v >> (32 - sh)).reshape(-1).astype(np.float64),
                     minlength=total_words + 2)
    words = lo[: total_words + 1].astype(np.int64) + hi[: total_words + 1].astype(np.int64)
    # Order words by (group, refilling symbol index, lane).
    kmax = int(nw.max())
    thr = 32 * np.arange(kmax, dtype=np.int64) - (LIMIT - 1)
    # One searchsorted over all chunks: offset chunk c by c * OFF (OFF exceeds
    # every bit position and threshold of a chunk).
    OFF = 1 << 24
    shift = np.arange(C, dtype=np.int64)[:, None] * OFF
    flat = np.searchsorted((before + shift).reshape(-1), (thr[None, :] + shift).reshape(-1),
                           side="left")
    at = flat.reshape(C, kmax) - np.arange(C, dtype=np.int64)[:, None] * chunk
    valid = at < chunk
    c_idx = np.broadcast_to(np.arange(C, dtype=np.int64)[:, None], (C, kmax))
    key = ((c_idx // LANES) * chunk + at) * LANES + (c_idx % LANES)
    src = (wbase[:, None] + np.arange(kmax, dtype=np.int64)[None, :])[valid]
    interleaved = words[src[np.argsort(key[valid], kind="stable")]]
    per_group = nw.reshape(G, LANES).sum(axis=1)
    gstart = np.concatenate([np.cumsum(per_group) - per_group, [per_group.sum()]])

    out = np.zeros(pitch, dtype=np.uint8)
    out[: 4 * (G + 1)] = gstart.astype(np.uint32).view(np.uint8)
    out[4 * (G + 1) : head] = fixed
    out[head:nbytes] = interleaved.astype(np.uint32).view(np.uint8)
    return out, code.lut.copy(), nbytes


def decode_py(rec, lut, n: int, chunk: int = CHUNK) -> np.ndarray:
    """Sequential reference decoder (tests/test_codec.py:49-79); small rows only."""
    rec = np.ascontiguousarray(rec, dtype=np.uint8)
    lut = np.ascontiguousarray(lut, dtype=np.uint8)
    G = n // (chunk * LANES)
    i32 = rec[: (len(rec) // 4) * 4].view(np.uint32)
    nib_w = (4 * (G + 1)) // 4  # nibble words start right after the header
    huff_w = (4 * (G + 1) + n // 2) // 4
    out = np.zeros(n, dtype=np.uint8)
    for g in range(G):
        rp = int(i32[g])
        buf, level = [0] * LANES, [0] * LANES
        for i in range(chunk):
            m, k = divmod(i, 8)
            for lane in range(LANES):
                if level[lane] < LIMIT:
                    buf[lane] |= int(i32[huff_w + rp]) << level[lane]
                    level[lane] += 32
                    rp += 1
                ent = int(lut[buf[lane] & (LUT_BYTES - 1)])
                buf[lane] >>= ent & 15
                level[lane] -= ent & 15
                nib = int(i32[nib_w + (g * (chunk // 8) + m) * LANES + lane])
                s = (nib >> (4 * k)) & 15
                out[(g * LANES + lane) * chunk + i] = ((s & 8) << 4) | ((ent >> 4) << 3) | (s & 7)
        if rp > int(i32[g + 1]):
            raise ValueError(f"group {g} reads past its words")
    return out
