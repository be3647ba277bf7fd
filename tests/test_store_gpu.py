"""Store + request ring + host server, driven by the GPU (port of the reference's tests/test_store.py).

The GPU publishes requests into pinned memory, the C++ host server preadv's
records from a paging file in tmp_path into RAM-tier rows and writes done; the
fetch kernel sees it and ends.  Every GPU wait here is bounded: the store's
retry interval is set to tens of milliseconds, so even a host that never
answers releases the GPU within a second.
"""

import os
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

L, E, R = 2, 8, 4
GROUP = 512 * 32
ROW_BYTES = {"w13_weight": 2 * GROUP, "w2_weight": GROUP}
PITCH = 1.0
WORKING_ROWS = 2
DEV = torch.device("cuda")


def pattern(layer: int, expert: int, name: str) -> torch.Tensor:
    return torch.full((ROW_BYTES[name] // 4,), layer * 1000 + expert * 10 + len(name),
                      dtype=torch.int32)


def encoded(store, layer: int, expert: int, name: str) -> torch.Tensor:
    from vllm_expert_pager import codec

    row = pattern(layer, expert, name)
    if not store.compress:
        return row
    return codec.encode(row.view(torch.uint8), store.pitch[name])[0].view(torch.int32)


def read_back(store, row: torch.Tensor, layer: int, expert: int, name: str) -> bool:
    """A RAM-tier row the host server filled from the paging file holds the record.

    A compressed record is read only up to the page holding its last used word
    (header, nibbles, Huffman words: all the decoder reads), so only that prefix
    is compared; the rest of the row keeps older bytes.
    """
    want = encoded(store, layer, expert, name)
    if not store.compress:
        return torch.equal(row, want)
    G = ROW_BYTES[name] // GROUP
    used = 4 * (G + 1 + ROW_BYTES[name] // 8 + int(want[G]))
    n = min(-(-used // 4096) * 4096, store.pitch[name]) // 4
    return torch.equal(row[:n], want[:n])


def make_store(tmp_path, num_layers, num_experts, ram_slots, compress=True):
    from vllm_expert_pager.store import Store

    s = Store(num_layers, num_experts, ram_slots, WORKING_ROWS, ROW_BYTES, compress, PITCH,
              str(tmp_path / "expert_pager.bin"), DEV)
    s.retry_ns = 50_000_000  # 50 ms between re-publishes, 8 tries: < 0.5 s worst case
    for layer in range(num_layers):
        for e in range(num_experts):
            for name in ROW_BYTES:
                s.write(layer, e, name, pattern(layer, e, name))
    return s


@pytest.fixture
def make(tmp_path):
    made = []

    def _make(*args, **kwargs):
        s = make_store(tmp_path, *args, **kwargs)
        made.append(s)
        return s

    yield _make
    for s in made:
        s.release()


@pytest.fixture(params=[True, False], ids=["compressed", "raw"])
def store(make, request):
    return make(L, E, R, compress=request.param)


def capture_fetch(store, todo, row, layer):
    from vllm_expert_pager.gather import fetch_rows

    base = layer * store.ram_slots
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        fetch_rows(todo, row, base, layer, store)  # warm-up (empty request)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fetch_rows(todo, row, base, layer, store)
    torch.cuda.synchronize()
    return g


def test_warm_start_rows(store):
    for layer in range(L):
        for e in range(R):
            for name in ROW_BYTES:
                assert torch.equal(store.pinned[name][layer * R + e], encoded(store, layer, e, name))


def test_fetch_reads_missing_experts_in_graph(store):
    todo = torch.full((R,), -1, dtype=torch.int64, device=DEV)
    row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    layer = 1
    g = capture_fetch(store, todo, row, layer)
    for i in range(20):
        a, b = 4 + i % 4, 4 + (i + 1) % 4
        sa, sb = i % R, (i + 1) % R
        todo.copy_(torch.tensor([a, b, -1, -1]))
        row[a], row[b] = sa, sb
        g.replay()
        torch.cuda.synchronize()
        assert store.failed is None, store.failed
        for name in ROW_BYTES:
            assert read_back(store, store.pinned[name][layer * R + sa], layer, a, name)
            assert read_back(store, store.pinned[name][layer * R + sb], layer, b, name)
    assert store.fetches == 20 and store.reads == 40
    seq_before = int(store.seq)
    todo.fill_(-1)
    g.replay()
    torch.cuda.synchronize()
    assert int(store.seq) == seq_before and store.fetches == 20


def test_fetch_gathers_ram_hits_while_reading_ssd(store):
    """The decode shape: gather+fetch, decode, gather of the SSD experts, decode; in a graph."""
    from vllm_expert_pager import codec
    from vllm_expert_pager.gather import gather_rows

    layer, S = 1, 3
    base = layer * R
    W = [n // 4 for n in ROW_BYTES.values()]
    src = [store.view[name] for name in ROW_BYTES]
    cache = [torch.zeros((S, w), dtype=torch.int32, device=DEV) for w in W]
    dst = [torch.zeros((S, n), dtype=torch.uint8, device=DEV) for n in ROW_BYTES.values()]
    dst_rows = [d.view(torch.int32) for d in dst]
    staging = [torch.zeros((S, store.pitch[name]), dtype=torch.uint8, device=DEV)
               for name in ROW_BYTES]
    stg = [t.view(torch.int32) for t in staging]
    scale = [torch.arange(E * 8, dtype=torch.int32, device=DEV).view(E, 8) * (i + 1)
             for i in range(2)]
    scale_dst = [torch.zeros((S, 8), dtype=torch.int32, device=DEV) for _ in range(2)]
    todo = torch.full((S,), -1, dtype=torch.int64, device=DEV)
    ssd = torch.full((S,), -1, dtype=torch.int64, device=DEV)
    dst_row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    cache_row = torch.full((E,), -1, dtype=torch.int64, device=DEV)
    src_row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    lut = store.layer_lut(layer)

    def step():
        stg_or_none = stg if store.compress else None
        gather_rows(todo, dst_row, cache_row, src_row, base, src, cache, dst_rows, stg_or_none,
                    scale, scale_dst, fetch=(ssd, layer, store))
        if store.compress:
            codec.decode_rows(todo, dst_row, cache_row, staging, dst, lut, skip=ssd)
        gather_rows(ssd, dst_row, cache_row, src_row, base, src, cache, dst_rows, stg_or_none,
                    scale, scale_dst)
        if store.compress:
            codec.decode_rows(ssd, dst_row, cache_row, staging, dst, lut)

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        step()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
    torch.cuda.synchronize()
    for i in range(6):
        a, b, c = i % 2, 2, R + i % (E - R)
        todo.copy_(torch.tensor([a, c, b]))
        ssd.copy_(torch.tensor([c, -1, -1]))
        src_row[a], src_row[b], src_row[c] = a, b, R - 1
        dst_row[a], dst_row[c], dst_row[b] = 0, 1, 2
        dst[0].zero_(), dst[1].zero_()
        g.replay()
        torch.cuda.synchronize()
        assert store.failed is None, store.failed
        for k, name in enumerate(ROW_BYTES):
            raw = [pattern(layer, x, name).view(torch.uint8).to(DEV) for x in (a, c, b)]
            for r in range(3):
                assert torch.equal(dst[k][r], raw[r])
            assert torch.equal(scale_dst[k][0], scale[k][a])
            assert torch.equal(scale_dst[k][1], scale[k][c])
            assert torch.equal(scale_dst[k][2], scale[k][b])
    assert store.fetches == 6 and store.reads == 6


def test_fetch_reads_many_experts_at_once(make):
    from vllm_expert_pager.store import _READ_WORKERS

    E2, R2 = 4 * _READ_WORKERS, 2 * _READ_WORKERS
    store = make(1, E2, R2)
    todo = torch.full((R2,), -1, dtype=torch.int64, device=DEV)
    row = torch.zeros((E2,), dtype=torch.int64, device=DEV)
    g = capture_fetch(store, todo, row, 0)
    missing = list(range(R2, E2))
    todo.copy_(torch.tensor(missing))
    row[R2:] = torch.arange(R2, device=DEV)
    g.replay()
    torch.cuda.synchronize()
    assert store.failed is None, store.failed
    assert store.fetches == 1 and store.reads == R2
    for s, e in enumerate(missing):
        for name in ROW_BYTES:
            assert read_back(store, store.pinned[name][s], 0, e, name)


def test_failed_read_releases_gpu(store):
    todo = torch.full((R,), -1, dtype=torch.int64, device=DEV)
    row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    layer = 1
    g = capture_fetch(store, todo, row, layer)
    todo.copy_(torch.tensor([4, 5, -1, -1]))
    row[4], row[5] = 10**6, 0
    g.replay()
    torch.cuda.synchronize()
    assert store.failed is not None and "outside the RAM tier" in store.failed, store.failed
    for name in ROW_BYTES:
        assert read_back(store, store.pinned[name][layer * R + 0], layer, 5, name)


def test_slow_host_makes_the_fetch_republish_the_request(store):
    todo = torch.full((R,), -1, dtype=torch.int64, device=DEV)
    row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    layer = 1
    g = capture_fetch(store, todo, row, layer)
    store.test_delay(0.2)  # longer than the 50 ms re-publish interval, shorter than 8 of them
    todo.copy_(torch.tensor([4, -1, -1, -1]))
    row[4] = 0
    g.replay()
    torch.cuda.synchronize()
    store.test_delay(0.0)
    assert store.failed is None, store.failed
    assert int(store.req[store.retry_at]) >= 1
    assert int(store.req[store.giveup_at]) == 0
    assert store.fetches == 1 and store.reads == 1
    for name in ROW_BYTES:
        assert read_back(store, store.pinned[name][layer * R], layer, 4, name)


def test_fetch_gives_up_when_the_host_never_answers(store):
    todo = torch.full((R,), -1, dtype=torch.int64, device=DEV)
    row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    g = capture_fetch(store, todo, row, 1)
    store.test_delay(60.0)
    todo.copy_(torch.tensor([4, -1, -1, -1]))
    row[4] = 0
    t0 = time.perf_counter()
    g.replay()
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    store.test_delay(0.0)
    assert waited < 5, f"the fetch waited {waited:.1f} s"
    assert int(store.req[store.giveup_at]) == 1
    assert int(store.req[store.retry_at]) >= 1
    for _ in range(300):
        if store.fetches == 1:
            break
        time.sleep(0.01)
    assert store.fetches == 1 and store.missed == 0


def test_serve_resends_done_when_the_fetch_is_still_spinning(store):
    todo = torch.full((R,), -1, dtype=torch.int64, device=DEV)
    row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    g = capture_fetch(store, todo, row, 1)
    todo.copy_(torch.tensor([4, -1, -1, -1]))
    row[4] = 0
    g.replay()
    torch.cuda.synchronize()
    served = int(store.done[0])
    assert served > 0
    store.done[0] = 0
    store.req[store.retry_at] += 1
    for _ in range(200):
        if int(store.done[0]) == served:
            break
        time.sleep(0.01)
    assert int(store.done[0]) == served


def test_pinned_tier_is_not_rounded_to_pow2(make):
    """The RAM tier takes rows x pitch bytes (page rounded), not the next power of two."""
    s = make(1, 3, 2)  # 2 + 2 rows x (32 KiB + 16 KiB)
    for name, p in s.pitch.items():
        assert s.pinned[name].numel() * 4 == s.rows * p
    assert sum(b.nbytes for b in s._buffers[:2]) == s.rows * s.record_bytes


def test_rejects_foreign_file(tmp_path):
    from vllm_expert_pager.store import Store

    path = tmp_path / "expert_pager.bin"
    path.write_bytes(b"not a paging file")
    with pytest.raises(FileExistsError):
        Store(L, E, R, WORKING_ROWS, ROW_BYTES, True, PITCH, str(path), DEV)


def test_rejects_rows_over_pitch(tmp_path):
    from vllm_expert_pager.store import Store

    s = Store(1, 2, 1, WORKING_ROWS, ROW_BYTES, True, 0.5, str(tmp_path / "expert_pager.bin"), DEV)
    try:
        row = torch.randint(-(2**31), 2**31 - 1, (ROW_BYTES["w2_weight"] // 4,), dtype=torch.int32)
        with pytest.raises(ValueError, match="VLLM_EXPERT_PAGER_PITCH must be at least"):
            s.write(0, 0, "w2_weight", row)
    finally:
        s.release()


def test_o_direct_paging_file_layout(make, tmp_path):
    """Records sit at (layer * E + e) * record_bytes, w13 then w2 (store.py:459-475,595-599)."""
    s = make(L, E, R, compress=False)
    with open(tmp_path / "expert_pager.bin", "rb") as f:
        data = f.read()
    assert len(data) == L * E * s.record_bytes
    for layer in range(L):
        for e in range(E):
            off = (layer * E + e) * s.record_bytes
            for name in ROW_BYTES:
                o = off + s.offset[name]
                got = torch.frombuffer(bytearray(data[o : o + s.pitch[name]]), dtype=torch.int32)
                assert torch.equal(got, pattern(layer, e, name))
    assert os.path.getsize(tmp_path / "expert_pager.bin") == L * E * s.record_bytes


def test_server_reads_used_pages_of_compressed_records(store):
    """The host server reads each compressed record piece only up to the page of its
    last used word (Store.write records the used length): bytes_read counts exactly
    those pages, fewer than whole records."""
    todo = torch.full((R,), -1, dtype=torch.int64, device=DEV)
    row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    layer = 1
    g = capture_fetch(store, todo, row, layer)
    before = store.bytes_read
    todo.copy_(torch.tensor([4, 6, -1, -1]))
    row[4], row[6] = 0, 1
    g.replay()
    torch.cuda.synchronize()
    assert store.failed is None, store.failed
    if not store.compress:  # raw rows: whole records
        assert store.bytes_read - before == 2 * store.record_bytes
        return
    want = 0
    for e in (4, 6):
        for name in ROW_BYTES:
            rec = encoded(store, layer, e, name)
            G = ROW_BYTES[name] // GROUP
            used = 4 * (G + 1 + ROW_BYTES[name] // 8 + int(rec[G]))
            want += min(-(-used // 4096) * 4096, store.pitch[name])
    assert store.bytes_read - before == want
    assert want < 2 * store.record_bytes
