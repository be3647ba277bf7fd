"""The host SSD server and its request-ring protocol, without a GPU.

A Python thread plays the GPU side of the ring (the reference's
``_fetch_publish``/``_fetch_wait``, gather.py:197-277): it fills a request slot,
stores ``seq`` last, and waits for ``done``.  The server under test is this
repository's C++ server (``libxpager.so``); when ``oracle/_ref/libssd_ref.so``
was built from the reference's own C server (oracle/build_ref.py), every
scenario also runs against it and the outcomes must agree: RAM-tier rows,
``done``, statistics and error text.  (x86 keeps the order of the two plain
stores, so the Python publisher needs no fence.)
"""

import ctypes
import os
import time

import numpy as np
import pytest

from vllm_expert_pager import native

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libssd_ref.so")
RING = 4
PITCH = (8192, 4096)


def load_server(path):
    if path is None:
        return native.lib()
    so = ctypes.CDLL(path)
    so.ssd_start.restype = ctypes.c_void_p
    so.ssd_start.argtypes = ([ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_long] * 6
                             + [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int])
    so.ssd_stop.argtypes = [ctypes.c_void_p]
    so.ssd_stats.argtypes = [ctypes.c_void_p] + [ctypes.POINTER(ctypes.c_long)] * 2 + [
        ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_long)]
    so.ssd_error.restype = ctypes.c_char_p
    so.ssd_error.argtypes = [ctypes.c_void_p]
    so.ssd_test_delay.argtypes = [ctypes.c_void_p, ctypes.c_double]
    return so


SERVERS = [None] + ([REF] if os.path.exists(REF) else [])
IDS = ["xpager"] + (["reference"] if os.path.exists(REF) else [])


def aligned(nbytes: int) -> np.ndarray:
    raw = np.zeros(nbytes + 4096, dtype=np.uint8)
    off = (-raw.ctypes.data) % 4096
    return raw[off : off + nbytes]


class Ring:
    """The pinned ring, RAM-tier rows and paging file of one server instance."""

    def __init__(self, so, tmp_path, L, E, R, working=2, workers=7, pitch=PITCH):
        self.so, self.L, self.E, self.R = so, L, E, R
        self.pitch = tuple(pitch)
        self.block = 1 << (E - 1).bit_length()
        self.slot_words = 2 + 2 * self.block
        self.req = np.zeros(2 + RING * self.slot_words, dtype=np.int64)
        self.done = np.zeros(1, dtype=np.int64)
        self.rows = L * R + working
        self.record = sum(self.pitch)
        self.pinned = [aligned(self.rows * p) for p in self.pitch]
        rng = np.random.default_rng(L * 1000 + E)
        self.file = rng.integers(0, 256, L * E * self.record, dtype=np.uint8)
        path = str(tmp_path / f"pager-{id(self)}.bin")
        self.file.tofile(path)
        try:
            self.fd = os.open(path, os.O_RDONLY | os.O_DIRECT)
        except OSError:
            self.fd = os.open(path, os.O_RDONLY)
        ptrs = (ctypes.c_void_p * 2)(*(p.ctypes.data for p in self.pinned))
        pitch = (ctypes.c_long * 2)(*self.pitch)
        self.h = so.ssd_start(self.fd, ctypes.c_void_p(self.req.ctypes.data),
                              ctypes.c_void_p(self.done.ctypes.data), RING, self.block, L, E,
                              self.rows, self.record, 2, ptrs, pitch, workers)
        assert self.h
        self.seq = 0

    def publish(self, layer, experts, rows, seq=None):
        self.seq = self.seq + 1 if seq is None else seq
        s = 2 + (self.seq % RING) * self.slot_words
        self.req[s + 2 : s + 2 + 2 * self.block] = -1
        self.req[s + 2 : s + 2 + len(experts)] = experts
        self.req[s + 2 + self.block : s + 2 + self.block + len(rows)] = rows
        self.req[s + 1] = layer
        self.req[s] = self.seq  # last
        return self.seq

    def wait(self, seq, timeout=10.0):
        t0 = time.time()
        while self.done[0] < seq:
            if time.time() - t0 > timeout:
                raise TimeoutError(f"done={self.done[0]} < {seq}")
            time.sleep(0.0005)

    def stats(self):
        f, r, m = ctypes.c_long(), ctypes.c_long(), ctypes.c_long()
        io = ctypes.c_double()
        self.so.ssd_stats(ctypes.c_void_p(self.h), ctypes.byref(f), ctypes.byref(r),
                          ctypes.byref(io), ctypes.byref(m))
        return f.value, r.value, m.value

    def error(self):
        e = self.so.ssd_error(ctypes.c_void_p(self.h))
        return None if e is None else e.decode()

    def row(self, k, row):
        p = self.pitch[k]
        return self.pinned[k][row * p : (row + 1) * p]

    def expected(self, k, layer, e):
        off = (layer * self.E + e) * self.record + sum(self.pitch[:k])
        return self.file[off : off + self.pitch[k]]

    def close(self):
        self.so.ssd_stop(ctypes.c_void_p(self.h))
        os.close(self.fd)


@pytest.fixture(params=SERVERS, ids=IDS)
def server(request, tmp_path):
    so = load_server(request.param)
    made = []

    def make(*a, **k):
        r = Ring(so, tmp_path, *a, **k)
        made.append(r)
        return r

    yield make
    for r in made:
        r.close()


def test_serves_requests_in_order(server):
    r = server(2, 8, 4)
    for i in range(20):
        a, b = 4 + i % 4, 4 + (i + 1) % 4
        rows = [1 * 4 + i % 4, 1 * 4 + (i + 1) % 4]
        r.wait(r.publish(1, [a, b], rows))
        for k in range(2):
            assert np.array_equal(r.row(k, rows[0]), r.expected(k, 1, a))
            assert np.array_equal(r.row(k, rows[1]), r.expected(k, 1, b))
    assert r.stats() == (20, 40, 0) and r.error() is None


def test_many_experts_in_one_request(server):
    r = server(1, 32, 16, workers=7)
    r.wait(r.publish(0, list(range(16, 32)), list(range(16))))
    for s in range(16):
        for k in range(2):
            assert np.array_equal(r.row(k, s), r.expected(k, 0, 16 + s))
    assert r.stats() == (1, 16, 0)


def test_failed_read_still_writes_done(server):
    r = server(2, 8, 4)
    r.wait(r.publish(1, [4, 5], [10**6, 0]))
    assert r.error() is not None and "outside the RAM tier" in r.error()
    assert np.array_equal(r.row(0, 0), r.expected(0, 1, 5))


def test_out_of_range_expert_is_an_error(server):
    r = server(2, 8, 4)
    r.wait(r.publish(1, [9], [0]))
    assert "out of range" in r.error()


def test_gap_in_seq_counts_missed(server):
    # The server watches slot (last+1) % RING.  Requests 2..5 never reached it
    # (given up by the "GPU"); request 6 lands in the same slot as 2.
    r = server(2, 8, 4)
    r.wait(r.publish(0, [5], [0]))
    r.wait(r.publish(0, [6], [1], seq=2 + RING))
    assert r.stats()[2] == RING
    assert np.array_equal(r.row(0, 1), r.expected(0, 0, 6))


def test_rewrites_done_when_republish_counter_moves(server):
    r = server(2, 8, 4)
    seq = r.publish(1, [4], [4])
    r.wait(seq)
    r.done[0] = 0
    r.req[0] += 1
    r.wait(seq, timeout=5)


def test_test_delay_holds_the_request(server):
    r = server(2, 8, 4)
    r.so.ssd_test_delay(ctypes.c_void_p(r.h), 0.3)
    t0 = time.time()
    r.wait(r.publish(1, [4], [4]))
    assert time.time() - t0 >= 0.25
    r.so.ssd_test_delay(ctypes.c_void_p(r.h), 0.0)


def test_ring_wraps_with_outstanding_requests(server):
    """Up to RING requests may be outstanding; done advances in order."""
    r = server(2, 16, 8)
    seqs = [r.publish(i % 2, [8 + i], [(i % 2) * 8 + i]) for i in range(RING - 1)]
    r.wait(seqs[-1])
    for i in range(RING - 1):
        for k in range(2):
            assert np.array_equal(r.row(k, (i % 2) * 8 + i), r.expected(k, i % 2, 8 + i))


@pytest.mark.skipif(not os.path.exists(REF), reason="reference server not built")
def test_random_sequence_matches_reference_server(tmp_path):
    """The same 60 random requests through both servers leave identical RAM tiers and stats."""
    rng = np.random.default_rng(5)
    rings = [Ring(load_server(p), tmp_path, 3, 24, 8) for p in (None, REF)]
    try:
        for _ in range(60):
            layer = int(rng.integers(0, 3))
            n = int(rng.integers(1, 9))
            experts = rng.choice(24, n, replace=False).tolist()
            rows = rng.choice(3 * 8 + 2, n, replace=False).tolist()
            for ring in rings:
                ring.wait(ring.publish(layer, experts, rows))
        a, b = rings
        for k in range(2):
            assert np.array_equal(a.pinned[k], b.pinned[k])
        assert a.stats() == b.stats() and a.error() == b.error() is None
    finally:
        for ring in rings:
            ring.close()


@pytest.mark.skipif(not os.path.exists(REF), reason="reference server not built")
def test_chunked_reads_match_the_reference_server(tmp_path):
    """This server splitting every record into page-sized jobs, against the reference's
    server reading whole records: 40 random requests leave identical RAM tiers and stats."""
    rng = np.random.default_rng(11)
    rings = [Ring(load_server(p), tmp_path, 3, 24, 8) for p in (None, REF)]
    try:
        rings[0].so.ssd_set_read_chunk(ctypes.c_void_p(rings[0].h), 4096)
        for _ in range(40):
            layer = int(rng.integers(0, 3))
            n = int(rng.integers(1, 9))
            experts = rng.choice(24, n, replace=False).tolist()
            rows = rng.choice(3 * 8 + 2, n, replace=False).tolist()
            for ring in rings:
                ring.wait(ring.publish(layer, experts, rows))
        a, b = rings
        for k in range(2):
            assert np.array_equal(a.pinned[k], b.pinned[k])
        assert a.stats() == b.stats() and a.error() == b.error() is None
    finally:
        for ring in rings:
            ring.close()


def test_threads_bound_to_the_ram_tier_node(tmp_path):
    """The server runs on the CPUs of the NUMA node holding the RAM tier (or stays
    unbound when the kernel reports no node), and still serves requests."""
    so = native.lib()
    r = Ring(so, tmp_path, L=1, E=8, R=4)
    try:
        node = so.ssd_numa_node(ctypes.c_void_p(r.h))
        nodes = sorted(int(d[4:]) for d in os.listdir("/sys/devices/system/node")
                       if d.startswith("node") and d[4:].isdigit()) \
            if os.path.isdir("/sys/devices/system/node") else []
        assert node == -1 or node in nodes
        if node >= 0:
            with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
                want = f.read().strip()
            lists = []
            for tid in os.listdir("/proc/self/task"):
                try:
                    with open(f"/proc/self/task/{tid}/status") as f:
                        lists += [ln.split(":", 1)[1].strip() for ln in f
                                  if ln.startswith("Cpus_allowed_list")]
                except OSError:
                    pass
            assert want in lists  # at least the server and worker threads
        seq = r.publish(0, [3], [1])
        r.wait(seq)
        assert np.array_equal(r.row(0, 1), r.expected(0, 0, 3))
    finally:
        r.close()
    assert so.ssd_numa_node(None) == -1


@pytest.mark.parametrize("chunk", [0, 4096, 5000, 8192, 12288, 20480, 1 << 20])
def test_chunked_reads_fill_the_same_rows(tmp_path, chunk):
    """ssd_set_read_chunk splits each record read into page-aligned jobs (a chunk of
    8192 B spans the two names' pieces of a 20480-B record; 5000 B rounds down to
    one page; 0 and sizes of a record or more read whole records): the RAM-tier rows,
    done and the statistics (reads count records) are those of whole-record reads."""
    so = native.lib()
    r = Ring(so, tmp_path, L=2, E=16, R=8, pitch=(12288, 8192))
    try:
        so.ssd_set_read_chunk(ctypes.c_void_p(r.h), chunk)
        rng = np.random.default_rng(chunk)
        for _ in range(12):
            layer = int(rng.integers(0, 2))
            n = int(rng.integers(1, 6))
            experts = rng.choice(16, n, replace=False).tolist()
            rows = rng.choice(2 * 8 + 2, n, replace=False).tolist()
            r.wait(r.publish(layer, experts, rows))
            for e, row in zip(experts, rows):
                for k in range(2):
                    assert np.array_equal(r.row(k, row), r.expected(k, layer, e))
        assert r.stats()[0] == 12 and r.error() is None
    finally:
        r.close()


def test_chunked_read_failure_still_writes_done(tmp_path):
    """A chunked request whose row is outside the RAM tier reports the error once and
    still completes (done = seq); the request's other expert is read."""
    so = native.lib()
    r = Ring(so, tmp_path, L=2, E=8, R=4, pitch=(12288, 8192))
    try:
        so.ssd_set_read_chunk(ctypes.c_void_p(r.h), 4096)
        r.wait(r.publish(1, [4, 5], [10**6, 0]))
        assert r.error() is not None and "outside the RAM tier" in r.error()
        for k in range(2):
            assert np.array_equal(r.row(k, 0), r.expected(k, 1, 5))
    finally:
        r.close()


def test_pipelined_requests_finish_in_order(tmp_path):
    """Two requests published back to back (chunk k+1's before chunk k's wait, as the
    working path does): this server reads them with up to two in flight, and done
    still only moves in seq order, each value after all of that request's rows landed.
    A watcher thread records every done value it sees and checks, at that moment,
    that the rows of every request up to it hold their records.  Requests alternate
    between two faces of rows, and request q+2 (which overwrites request q's face) is
    published only after the watcher has checked request q, as the working path reuses
    a face only after its MoE has read it."""
    import threading

    r = Ring(native.lib(), tmp_path, L=2, E=64, R=8, working=128, workers=7,
             pitch=(65536, 32768))
    native.lib().ssd_set_read_chunk(ctypes.c_void_p(r.h), 16384)
    try:
        seen, bad = [], []
        reqs = {}
        checked = {q: threading.Event() for q in range(1, 7)}

        def watch():
            last = 0
            t0 = time.time()
            while last < 6 and time.time() - t0 < 20:
                d = int(r.done[0])
                if d != last:
                    seen.append(d)
                    for q in range(last + 1, d + 1):
                        layer, experts, rows = reqs[q]
                        for e, row in zip(experts, rows):
                            for k in (0, 1):
                                if not np.array_equal(r.row(k, row), r.expected(k, layer, e)):
                                    bad.append((q, e, k))
                        checked[q].set()
                    last = d
                time.sleep(0.0001)

        plan = []
        for q in range(1, 7):
            layer = q % 2
            experts = list(range((q * 7) % 40, (q * 7) % 40 + 24))
            rows = [2 * 8 + (q % 2) * 64 + i for i in range(24)]  # alternating faces
            plan.append((layer, experts, rows))
        th = threading.Thread(target=watch)
        for q, (layer, experts, rows) in enumerate(plan, 1):
            reqs[q] = (layer, experts, rows)
        th.start()
        # publish k+1 before waiting for k (two in flight), as the working path does
        r.publish(*plan[0])
        for q in range(2, 7):
            if q >= 3:
                assert checked[q - 2].wait(20), f"request {q - 2} never checked"
            r.publish(*plan[q - 1])
            r.wait(q - 1)
        r.wait(6)
        th.join()
        assert seen == sorted(seen) and seen[-1] == 6
        assert not bad, bad[:5]
        assert r.error() is None and r.stats()[:2] == (6, 6 * 24)
    finally:
        r.close()


@pytest.mark.parametrize("chunk", [0, 4096, 8192])
def test_used_bytes_reads_only_the_data_pages(tmp_path, chunk):
    """ssd_set_used_bytes: each record piece is read only up to the page holding its
    last used byte (0 or a length of the whole pitch or more reads the whole piece);
    the rest of the RAM-tier row keeps its old bytes, and ssd_bytes_read counts the
    bytes read."""
    so = native.lib()
    L, E, R = 2, 8, 4
    pitch = (12288, 8192)
    r = Ring(so, tmp_path, L=L, E=E, R=R, pitch=pitch)
    try:
        so.ssd_set_read_chunk(ctypes.c_void_p(r.h), chunk)
        rng = np.random.default_rng(chunk + 1)
        used = np.zeros(L * E * 2, dtype=np.int64)
        for i in range(L * E):
            used[2 * i] = [0, 1, 4096, 4097, 9000, 12288, 20000][i % 7]
            used[2 * i + 1] = [100, 8192, 0, 4096, 5000][i % 5]
        so.ssd_set_used_bytes(ctypes.c_void_p(r.h), ctypes.c_void_p(used.ctypes.data))
        for k in range(2):
            r.pinned[k][:] = 0xEE
        want_bytes = 0
        for step in range(6):
            layer = int(rng.integers(0, L))
            experts = rng.choice(E, 3, replace=False).tolist()
            rows = [3 * step % (L * R), 3 * step % (L * R) + 1, 3 * step % (L * R) + 2]
            for k in range(2):
                for row in rows:
                    r.row(k, row)[:] = 0xEE
            r.wait(r.publish(layer, experts, rows))
            for e, row in zip(experts, rows):
                for k in range(2):
                    u = int(used[2 * (layer * E + e) + k])
                    n = pitch[k] if u <= 0 or u >= pitch[k] else -(-u // 4096) * 4096
                    got, want = r.row(k, row), r.expected(k, layer, e)
                    assert np.array_equal(got[:n], want[:n]), (e, k, n)
                    assert np.all(got[n:] == 0xEE), (e, k, n)
                    want_bytes += n
        assert r.error() is None
        assert so.ssd_bytes_read(ctypes.c_void_p(r.h)) == want_bytes
    finally:
        r.close()


def test_used_bytes_null_reads_whole_records(tmp_path):
    """ssd_set_used_bytes(NULL) restores whole-record reads."""
    so = native.lib()
    r = Ring(so, tmp_path, L=1, E=4, R=2, pitch=(8192, 4096))
    try:
        used = np.full(8, 1, dtype=np.int64)
        so.ssd_set_used_bytes(ctypes.c_void_p(r.h), ctypes.c_void_p(used.ctypes.data))
        so.ssd_set_used_bytes(ctypes.c_void_p(r.h), None)
        r.wait(r.publish(0, [1, 2], [0, 1]))
        for e, row in ((1, 0), (2, 1)):
            for k in range(2):
                assert np.array_equal(r.row(k, row), r.expected(k, 0, e))
        assert so.ssd_bytes_read(ctypes.c_void_p(r.h)) == 2 * (8192 + 4096)
    finally:
        r.close()
