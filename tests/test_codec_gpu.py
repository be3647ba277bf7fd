"""GPU decoder (decode.cu, via the C ABI) against the reference's records and the CPU oracle.

Bit-exact: the expanded slot bytes equal the raw fp8 rows.
"""

import os

import numpy as np
import pytest
import torch

from oracle import _lib as oracle_lib
from oracle import codec as oc
from rowgen import rows

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = torch.device("cuda")


def decode_one(rec: np.ndarray, lut: np.ndarray, n: int, chunk: int, rec1=None, lut1=None,
               n1=None) -> list[np.ndarray]:
    """Decode one expert (names 0 and 1) through decode_rows; name 1 defaults to name 0."""
    from vllm_expert_pager import codec

    rec1 = rec if rec1 is None else rec1
    lut1 = lut if lut1 is None else lut1
    n1 = n if n1 is None else n1
    stg = [torch.from_numpy(r.copy()).to(DEV).view(1, -1) for r in (rec, rec1)]
    dst = [torch.zeros((1, m), dtype=torch.uint8, device=DEV) for m in (n, n1)]
    luts = torch.from_numpy(np.stack([lut, lut1])[None]).to(DEV)
    todo = torch.zeros((1,), dtype=torch.int64, device=DEV)
    dst_row = torch.zeros((1,), dtype=torch.int64, device=DEV)
    cache_row = torch.full((1,), -1, dtype=torch.int64, device=DEV)
    codec.decode_rows(todo, dst_row, cache_row, stg, dst, luts, chunk=chunk)
    torch.cuda.synchronize()
    return [d[0].cpu().numpy() for d in dst]


@pytest.mark.parametrize("chunk", [64, 512])
@pytest.mark.parametrize("i", range(4), ids=["realistic", "uniform", "geometric", "constant"])
def test_decodes_reference_records(chunk, i):
    g = np.load(os.path.join(GOLDEN, "codec.npz"))
    raw, rec, lut = g[f"c{chunk}_{i}_raw"], g[f"c{chunk}_{i}_rec"], g[f"c{chunk}_{i}_lut"]
    a, b = decode_one(rec, lut, raw.size, chunk)
    assert np.array_equal(a, raw) and np.array_equal(b, raw)


def test_decodes_config1_experts():
    """Config 1: 8 full-size experts (w13 2 MiB + w2 1 MiB) round-trip byte for byte."""
    from vllm_expert_pager import codec, synthetic

    for ex in synthetic.fp8_experts(8, seed=0):
        raws = [synthetic.row_bytes(ex[name][0]).numpy() for name in synthetic.SHAPES]
        encs = [codec.encode(torch.from_numpy(r), codec.pitch_of(r.size, 0.89, 4096)) for r in raws]
        got = decode_one(encs[0][0].numpy(), encs[0][1].numpy(), raws[0].size, 512,
                         encs[1][0].numpy(), encs[1][1].numpy(), raws[1].size)
        assert np.array_equal(got[0], raws[0]) and np.array_equal(got[1], raws[1])


@pytest.mark.parametrize("seed", range(6))
def test_random_distributions_match_oracle(seed):
    """Skewed, flat and degenerate exponent histograms at several chunk sizes."""
    rng = np.random.default_rng(seed)
    chunk = [8, 16, 64, 512, 128, 32][seed]
    n = 32 * chunk * int(rng.integers(1, 5))
    p = rng.dirichlet(np.full(16, [0.05, 0.3, 1.0, 5.0, 0.1, 2.0][seed]))
    raw = rows(100 + seed, n, p.tolist()).numpy()
    rec, lut, _ = oc.encode(raw, oc.pitch_of(n, 1.5, 4096) + 4096, chunk)
    a, _ = decode_one(rec, lut, n, chunk)
    assert np.array_equal(a, oracle_lib.decode(rec, lut, n, chunk))
    assert np.array_equal(a, raw)


@pytest.mark.parametrize("chunk,offset", [(512, 16), (48, 0), (80, 16), (512, 0)])
def test_store_widths_decode_alike(chunk, offset):
    """The kernel stores 32 bytes per lane per 32 symbols when every lane chunk starts on a
    32-byte boundary and holds whole 32-value blocks, else 16 bytes per 16 symbols: rows
    that start 16 bytes into an allocation and chunks of 48 or 80 values take the 16-byte
    stores, and both store paths leave the bytes around the rows untouched."""
    from vllm_expert_pager import codec

    rng = np.random.default_rng(chunk + offset)
    n = 32 * chunk * 3
    p = rng.dirichlet(np.full(16, 0.5))
    raws = [rows(300 + chunk + k, n, p.tolist()).numpy() for k in range(2)]
    encs = [oc.encode(r, oc.pitch_of(n, 1.5, 4096) + 4096, chunk) for r in raws]
    stg = [torch.from_numpy(e[0].copy()).to(DEV).view(1, -1) for e in encs]
    luts = torch.from_numpy(np.stack([encs[0][1], encs[1][1]])[None]).to(DEV)
    backing = [torch.full((n + 64,), 0xA5, dtype=torch.uint8, device=DEV) for _ in range(2)]
    dst = [b[offset: offset + n].view(1, n) for b in backing]
    assert all(d.data_ptr() % 16 == 0 for d in dst)
    todo = torch.zeros((1,), dtype=torch.int64, device=DEV)
    dst_row = torch.zeros((1,), dtype=torch.int64, device=DEV)
    cache_row = torch.full((1,), -1, dtype=torch.int64, device=DEV)
    codec.decode_rows(todo, dst_row, cache_row, stg, dst, luts, chunk=chunk)
    torch.cuda.synchronize()
    for k in range(2):
        b = backing[k].cpu().numpy()
        assert np.array_equal(b[offset: offset + n], raws[k]), k
        assert np.all(b[:offset] == 0xA5) and np.all(b[offset + n:] == 0xA5), k


def _canonical(lut: np.ndarray) -> bool:
    """The decoder's fast-path rule: each window's code length is 1 + the number of
    thresholds lim[L] (windows with codes of at most L bits) that the window, read
    most-significant bit first, reaches."""
    lens = lut.astype(np.int64) & 15
    lim = [(lens <= L).sum() for L in range(1, 9)]
    r = np.array([int(format(x, "09b")[::-1], 2) for x in range(512)])
    return bool(((lens >= 1) & (lens == 1 + sum((r >= t).astype(np.int64) for t in lim))).all())


def _complemented(rec: np.ndarray, lut: np.ndarray, n: int, chunk: int):
    """The same row under the bit-complemented code: every Huffman word inverted,
    lut'[x] = lut[x ^ 511].  Prefix-free, complete and with the same lengths (so
    the same refills), but longer codes come first: not canonical."""
    G = n // (chunk * 32)
    head = 4 * (G + 1) + n // 2
    end = head + 4 * int(rec[: 4 * (G + 1)].view(np.uint32)[-1])
    out = rec.copy()
    out[head:end] ^= 0xFF
    return out, lut[np.arange(512) ^ 511].copy()


@pytest.mark.parametrize("chunk", [64, 512])
def test_non_canonical_lut_decodes_through_the_table(chunk):
    """A valid but non-canonical code takes the LUT-chain step and still matches."""
    n = 32 * chunk * 3
    p = np.random.default_rng(11).dirichlet(np.full(16, 0.3))
    raw = rows(11, n, p.tolist()).numpy()
    rec, lut, _ = oc.encode(raw, oc.pitch_of(n, 1.5, 4096) + 4096, chunk)
    rec2, lut2 = _complemented(rec, lut, n, chunk)
    assert _canonical(lut) and not _canonical(lut2)
    a, _ = decode_one(rec2, lut2, n, chunk)
    assert np.array_equal(a, oracle_lib.decode(rec2, lut2, n, chunk))
    assert np.array_equal(a, raw)


def test_relabelled_symbols_come_from_the_lut():
    """Permuting the LUT's symbols keeps the code canonical; the bytes follow the LUT."""
    n = 32 * 512 * 2
    raw = rows(12, n).numpy()
    rec, lut, _ = oc.encode(raw, oc.pitch_of(n, 1.5, 4096) + 4096, 512)
    perm = np.random.default_rng(12).permutation(16)
    lut2 = ((perm[lut >> 4] << 4) | (lut & 15)).astype(np.uint8)
    assert _canonical(lut2)
    a, _ = decode_one(rec, lut2, n, 512)
    want = (raw & 0x87) | (perm[(raw >> 3) & 15] << 3).astype(np.uint8)
    assert np.array_equal(a, oracle_lib.decode(rec, lut2, n, 512))
    assert np.array_equal(a, want)


def test_decode_rows_follows_todo_and_skips():
    """The reference test_codec.py::test_decode_rows_follows_todo_and_skips, at CHUNK=64."""
    from vllm_expert_pager import codec

    CHUNK, E = 64, 8
    N = 2 * CHUNK * 32
    ns = (N, N // 2)
    pitches = [codec.pitch_of(n, 1.25, 4096) for n in ns]
    raws = {e: [rows(10 * e + k, n) for k, n in enumerate(ns)] for e in (3, 5, 6)}
    staging = [torch.zeros((3, p), dtype=torch.uint8, device=DEV) for p in pitches]
    lut = torch.zeros((E, 2, codec.LUT_BYTES), dtype=torch.uint8, device=DEV)
    for j, e in enumerate((3, 5, 6)):
        for k in range(2):
            staging[k][j], lut[e, k] = codec.encode(raws[e][k].to(DEV), pitches[k], CHUNK)
    dst = [torch.zeros((2, n), dtype=torch.uint8, device=DEV) for n in ns]
    todo = torch.tensor([3, 5, 6], dtype=torch.int64, device=DEV)
    dst_row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    dst_row[3], dst_row[5], dst_row[6] = 1, 0, 0
    cache_row = torch.full((E,), -1, dtype=torch.int64, device=DEV)
    cache_row[5] = 2
    skip = torch.tensor([6, -1, -1], dtype=torch.int64, device=DEV)
    codec.decode_rows(todo, dst_row, cache_row, staging, dst, lut, skip=skip, chunk=CHUNK)
    torch.cuda.synchronize()
    for k in range(2):
        assert torch.equal(dst[k][1].cpu(), raws[3][k])
        assert not dst[k][0].any()
    codec.decode_rows(todo, dst_row, cache_row, staging, dst, lut, chunk=CHUNK)
    torch.cuda.synchronize()
    for k in range(2):
        assert torch.equal(dst[k][0].cpu(), raws[6][k])


def test_decode_rejects_bad_shapes():
    from vllm_expert_pager import codec

    t = torch.zeros((1,), dtype=torch.int64, device=DEV)
    stg = [torch.zeros((1, 4096), dtype=torch.uint8, device=DEV)] * 2
    dst = [torch.zeros((1, 1000), dtype=torch.uint8, device=DEV)] * 2  # not a multiple of 32*chunk
    lut = torch.zeros((1, 2, 512), dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError):
        codec.decode_rows(t, t, t, stg, dst, lut, chunk=64)


@pytest.mark.parametrize("chunk", [512, 40], ids=["ring", "window"])
def test_corrupt_records_stay_inside_their_rows(chunk):
    """A corrupt record decodes to wrong bytes and nothing else: its group offsets are
    clamped to the record, its ring and table addresses are masked, and every store goes
    to its own destination row.  Staging rows of random bytes whose headers hold random,
    decreasing, zero and past-the-record offsets leave the canary rows around their
    destinations untouched, and a valid decode right after is exact.  LUTs stay valid
    (codes of at most 9 bits); the ring path (chunk 512) also takes a random LUT."""
    from vllm_expert_pager import codec

    rng = np.random.default_rng(chunk)
    E, groups = 4, 4
    N = groups * 32 * chunk
    ns = (N, N // 2) if chunk == 512 else (N, N)
    pitches = [codec.pitch_of(n, 1.25, 4096) for n in ns]
    raws = {e: [rows(40 + 2 * e + k, n) for k, n in enumerate(ns)] for e in range(E)}
    good = [torch.zeros((E, p), dtype=torch.uint8, device=DEV) for p in pitches]
    lut = torch.zeros((E, 2, codec.LUT_BYTES), dtype=torch.uint8, device=DEV)
    for e in range(E):
        for k in range(2):
            good[k][e], lut[e, k] = codec.encode(raws[e][k].to(DEV), pitches[k], chunk)
    bad = []
    for k, (n, p) in enumerate(zip(ns, pitches)):
        b = rng.integers(0, 256, (E, p), dtype=np.uint8)
        G = n // (32 * chunk)
        hdr = b[:, : 4 * (G + 1)].view(np.int32)
        hdr[0] = rng.integers(-(2**31), 2**31 - 1, G + 1)  # anything
        hdr[1] = np.linspace(2**31 - 1, -(2**20), G + 1).astype(np.int32)  # decreasing
        hdr[2] = 0  # every group empty: the ring is never filled
        hdr[3] = np.arange(G + 1, dtype=np.int32) * (p // 4) + p  # past the record
        bad.append(torch.from_numpy(b).to(DEV))
    todo = torch.arange(E, dtype=torch.int64, device=DEV)
    dst_row = torch.arange(1, E + 1, dtype=torch.int64, device=DEV)  # rows 0 and E+1: canaries
    cache_row = torch.full((E,), -1, dtype=torch.int64, device=DEV)
    dst = [torch.full((E + 2, n), 0xA5, dtype=torch.uint8, device=DEV) for n in ns]

    def canaries_intact():
        return all(bool((d[0] == 0xA5).all()) and bool((d[E + 1] == 0xA5).all()) for d in dst)

    passes = [lut]
    if chunk == 512:
        passes.append(torch.from_numpy(rng.integers(0, 256, tuple(lut.shape), dtype=np.uint8)).to(DEV))
    for table in passes:
        codec.decode_rows(todo, dst_row, cache_row, bad, dst, table, chunk=chunk)
        torch.cuda.synchronize()
        assert canaries_intact()
        codec.decode_rows(todo, dst_row, cache_row, good, dst, lut, chunk=chunk)
        torch.cuda.synchronize()
        assert canaries_intact()
        for e in range(E):
            for k in range(2):
                assert torch.equal(dst[k][e + 1].cpu(), raws[e][k])
