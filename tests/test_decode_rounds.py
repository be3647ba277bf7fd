"""The refill schedule of the GPU decoder (decode.cu), modelled on the CPU.

The record format (monochromegane/vllm-expert-pager src/vllm_expert_pager/codec.py:
22-26, 204-245) refills a lane's bit buffer with one 32-bit word before every
symbol at which it holds fewer than 9 bits, the lanes refilling at the same
symbol taking consecutive words in lane order.  decode_ring_kernel does not
follow that schedule literally: it decodes 8 symbols in rounds of 3, 3 and 2
symbols (step_triple, step_pair) and, per round,

* finds the one symbol of the round at which each lane refills, if any, from
  its current buffer alone (a lane refills at most once in three consecutive
  symbols, and before a symbol it does not refill at it holds >= 9 valid bits,
  enough to look up that symbol's length);
* gives the round's refilling lanes their words in the format's order (the
  first symbol's refilling lanes in lane order, then the second's, ...);
* inserts each word right above the lane's valid bits before the round's
  first symbol, at most 26 bits up, so a 64-bit buffer holds it.

This test runs that schedule on the CPU (one lane at a time, no GPU) and checks
that it decodes the reference's golden records and records of other exponent
distributions byte for byte like the sequential decoder of the CPU oracle, and
that the insert position bound holds.  It pins the algorithm; the GPU tests pin
the kernel.
"""

import numpy as np
import pytest

from oracle import codec as oc

GOLDEN = np.load(__file__.rsplit("/", 1)[0] + "/golden/codec.npz")
ROUNDS = (3, 3, 2)  # symbols per ballot round within each 8 symbols
LANES, LIMIT = 32, 9


def decode_rounds(rec: np.ndarray, lut: np.ndarray, n: int, chunk: int) -> np.ndarray:
    G = n // (chunk * LANES)
    i32 = rec[: (len(rec) // 4) * 4].view(np.uint32)
    nib_w, huff_w = G + 1, (4 * (G + 1) + n // 2) // 4
    ent_of = [int(x) for x in lut]
    out = np.zeros(n, np.uint8)
    for g in range(G):
        off = int(i32[g])
        buf, lvl = [0] * LANES, [0] * LANES
        i, r = 0, 0
        while i < chunk:
            D = ROUNDS[r % len(ROUNDS)]
            r += 1
            # the round's refill symbol of each lane, from its current bits only
            at = [None] * LANES
            for lane in range(LANES):
                level, b = lvl[lane], buf[lane]
                for k in range(D):
                    if level < LIMIT:
                        at[lane] = k
                        break
                    ln = ent_of[b & 511] & 15
                    level, b = level - ln, b >> ln
            count = [at.count(k) for k in range(D)]
            taken = [0] * D
            for lane in range(LANES):
                k = at[lane]
                if k is None:
                    continue
                rank = sum(count[:k]) + taken[k]
                taken[k] += 1
                assert lvl[lane] <= 26, "insert position above 26 bits"
                buf[lane] |= int(i32[huff_w + off + rank]) << lvl[lane]
                lvl[lane] += 32
                assert lvl[lane] <= 64
            off += sum(count)
            for k in range(D):
                for lane in range(LANES):
                    e = ent_of[buf[lane] & 511]
                    buf[lane] >>= e & 15
                    lvl[lane] -= e & 15
                    v = i + k
                    nib = int(i32[nib_w + (g * (chunk // 8) + v // 8) * LANES + lane])
                    s = (nib >> (4 * (v % 8))) & 15
                    out[(g * LANES + lane) * chunk + v] = ((s & 8) << 4) | ((e >> 4) << 3) | (s & 7)
            i += D
        assert off <= int(i32[g + 1]), "read past the group's words"
    return out


@pytest.mark.parametrize("name", ["c512_0", "c512_1", "c512_2", "c512_3", "c64_0", "c64_3"])
def test_rounds_decode_the_reference_records(name):
    raw, rec, lut = GOLDEN[name + "_raw"], GOLDEN[name + "_rec"], GOLDEN[name + "_lut"]
    chunk = 512 if name.startswith("c512") else 64
    assert np.array_equal(decode_rounds(rec, lut, raw.size, chunk), raw)


@pytest.mark.parametrize("dist", ["uniform", "peaked", "two_symbols"])
def test_rounds_match_the_sequential_decoder(dist):
    """Flat histograms give long codes and frequent refills; a two-symbol row gives
    1-bit codes and rare refills: the schedule must not depend on the shape."""
    rng = np.random.default_rng(7)
    n = 512 * 32
    if dist == "uniform":
        exp = rng.integers(0, 16, n)
    elif dist == "peaked":
        p = np.array([1, 1, 1, 1, 2, 4, 8, 16, 32, 64, 125, 228, 315, 188, 15, 1], float)
        exp = rng.choice(16, n, p=p / p.sum())
    else:
        exp = rng.choice([9, 10], n)
    raw = ((rng.integers(0, 256, n) & 0x87) | (exp << 3)).astype(np.uint8)
    rec, lut, _ = oc.encode(raw, oc.pitch_of(n, 1.1, 4096))  # flat rows do not compress
    want = oc.decode_py(rec, lut, n)
    assert np.array_equal(want, raw)
    assert np.array_equal(decode_rounds(rec, lut, n, 512), want)
