"""The GPU decoder's round schedule and bit arithmetic (decode.cu), modelled on the CPU.

The record format (monochromegane/vllm-expert-pager src/vllm_expert_pager/codec.py:
22-26, 204-245) refills a lane's bit buffer with one 32-bit word before every
symbol at which it holds fewer than 9 bits, the lanes refilling at the same
symbol taking consecutive words in lane order.  decode_ring_kernel does not
follow that schedule literally: it decodes 8 symbols in rounds of 3, 3 and 2
symbols (round3, round2) and, per round,

* finds the one symbol of the round at which each lane refills, if any, from
  table entries looked up in its current buffer (a lane refills at most once in
  three consecutive symbols, and before a symbol it does not refill at it holds
  >= 9 valid bits, so that symbol's entry is exact);
* gives the round's refilling lanes their words in the format's order (the
  first symbol's refilling lanes in lane order, then the second's, ...), from
  three cumulative ballots and one popcount per lane;
* inserts each word right above the lane's valid bits before the round's
  first symbol (at most bit 27: the buffer keeps stream bit j at bit j + 1);
* looks windows up with as many bits as the row's longest code;
* decodes the round's symbols from the new buffer with wrapping funnel shifts
  whose amount is the 16-bit table entry len | sym << 12 itself, re-looking up
  the first two symbols only in lanes whose refill came at or before them;
* keeps the level as (26 - level) << 25, updated by entry x 2^25 multiply-adds;
* packs the exponent fields of 4 symbols with multiplies (e >> 9, e >> 1,
  e << 7, e << 15) and merges the sign/mantissa nibbles by a byte permute.

This test runs that arithmetic on the CPU, 32-bit op for op (numpy, one array
element per lane, no GPU), and checks that it decodes the reference's golden
records and records of other exponent distributions byte for byte like the
sequential decoder of the CPU oracle, and that the insert position and level
counter stay in the ranges the kernel relies on.  It pins the algorithm; the GPU
tests pin the kernel.
"""

import numpy as np
import pytest

from oracle import codec as oc

GOLDEN = np.load(__file__.rsplit("/", 1)[0] + "/golden/codec.npz")
LANES = 32
M32 = 0xFFFFFFFF
LT = np.array([(1 << lane) - 1 for lane in range(LANES)], np.uint64)
NV_START, NV_REFILL = 26 << 25, 18 << 25


def _s32(x):
    x = np.asarray(x, np.int64) & M32
    return np.where(x >= 1 << 31, x - (1 << 32), x)


def _shf_r_wrap(lo, hi, c):
    """PTX shf.r.wrap.b32: low word of (hi:lo) >> (c & 31)."""
    v = (hi.astype(np.uint64) << 32) | lo.astype(np.uint64)
    return ((v >> (c.astype(np.uint64) & 31)) & M32).astype(np.uint64)


def _ballot(pred):
    return int(sum(1 << i for i in np.nonzero(pred)[0]))


def _popc(x):
    return np.array([bin(int(v)).count("1") for v in x], np.uint64)


def _table(lut):
    lut = lut.astype(np.uint64)
    return (lut & 15) | ((lut >> 4) << 12)


def decode_rounds(rec: np.ndarray, lut: np.ndarray, n: int, chunk: int) -> np.ndarray:
    G = n // (chunk * LANES)
    i32 = rec[: (len(rec) // 4) * 4].view(np.uint32).astype(np.uint64)
    nib_w, huff_w = G + 1, (4 * (G + 1) + n // 2) // 4
    T = _table(lut)
    # windows are looked up with as many bits as the row's longest code
    msk = ((1 << int((lut & 15).max())) - 1) << 1
    look = lambda x: T[(x & msk) >> 1]  # noqa: E731  (the table byte address is x & msk)
    out = np.zeros(n, np.uint8)
    zero = np.zeros(LANES, np.uint64)
    for g in range(G):
        off = int(i32[g])
        lo, hi = zero.copy(), zero.copy()
        nv = np.full(LANES, NV_START, np.int64)
        for m in range(chunk // 8):
            ents = []
            for size in (3, 3, 2):
                e0 = look(lo)
                t1 = _s32(nv + (e0.astype(np.int64) << 25))
                p0, q = nv >= NV_REFILL, t1 >= NV_REFILL
                if size == 3:
                    e1 = look(_shf_r_wrap(lo, hi, e0))
                    ev = _s32(t1 + (e1.astype(np.int64) << 25)) >= NV_REFILL
                    b0, b1, b2 = _ballot(p0), _ballot(q), _ballot(ev)
                    bs = np.where(p0, b0, np.where(q, b1, b2)).astype(np.uint64)
                    mb = np.where(p0, 0, np.where(q, b0, b1)).astype(np.uint64)
                else:
                    ev = q
                    b0, b2 = _ballot(p0), _ballot(ev)
                    bs = np.where(p0, b0, b2).astype(np.uint64)
                    mb = np.where(p0, 0, b0).astype(np.uint64)
                rank = _popc((bs & LT) | (mb & ~LT & M32))
                word = i32[huff_w + off + rank.astype(np.int64)]
                off += bin(b2).count("1")
                s = (nv.astype(np.uint64) & M32) >> 25
                assert np.all(s[ev] <= 26), "insert above bit 27"
                mul = np.where(s < 32, (1 << 27) >> np.minimum(s, 31), 0).astype(np.uint64)
                old = (hi << 32) | lo
                assert np.all(old[ev] < mul[ev]), "bits at or above the insert position"
                buf = old + np.where(ev, word * mul, 0)
                lo, hi = buf & M32, buf >> 32
                nv = np.where(ev, nv - (32 << 25), nv)
                # decode from the new buffer; the first entries again only where stale
                d0 = np.where(p0, look(lo), e0)
                x = _shf_r_wrap(lo, hi, d0)
                if size == 3:
                    d1 = np.where(q, look(x), e1)
                    x = _shf_r_wrap(x, zero, d1)
                    d = [d0, d1, look(x)]
                else:
                    d = [d0, look(x)]
                sh = sum(d) & M32
                lo, hi = _shf_r_wrap(lo, hi, sh), _shf_r_wrap(hi, zero, sh)
                nv = _s32(nv + (sh.astype(np.int64) << 25))
                assert np.all((nv >= -32 << 25) & (nv <= NV_START)), "level out of range"
                ents += d
            mulhi = lambda a, b: (a * b) >> 32  # noqa: E731
            words = []
            for h in range(2):
                e = ents[4 * h: 4 * h + 4]
                acc = (mulhi(e[0], 1 << 23) + mulhi(e[1], 1 << 31) + (e[2] << 7) + (e[3] << 15)) & M32
                words.append(acc)
            nw = i32[nib_w + (g * (chunk // 8) + m) * LANES + np.arange(LANES)]
            ev_ = ((nw & 0x0F0F0F0F) * 17) & M32
            od_ = ((((nw * (1 << 28)) >> 32) & 0x0F0F0F0F) * 17) & M32
            for h, sel in enumerate(((0, 4, 1, 5), (2, 6, 3, 7))):
                src = (od_ << 32) | ev_
                t = sum(((src >> (8 * b)) & 0xFF) << (8 * i) for i, b in enumerate(sel))
                w = (words[h] & 0x78787878) | (t & ~np.uint64(0x78787878) & M32)
                for k in range(4):
                    pos = (g * LANES + np.arange(LANES)) * chunk + 8 * m + 4 * h + k
                    out[pos] = (w >> (8 * k)) & 0xFF
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
