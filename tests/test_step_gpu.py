"""The fused decode step (xp_decode_step) against the reference's launch sequence.

Two identical pagers (each with its own Store and paging file) take the same
routing: one through ``LayerPager.decode(fused=True)`` (one launch + one decode
launch), the other through the reference's sequence (acquire, gather with the
fused fetch CTA, decode with skip, gather of the SSD misses, decode).  Tables,
expert_map, slab bytes and SSD statistics must agree after every step, and
every needed expert's slot must hold its raw rows byte for byte.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
E, S, W = 32, 8, 8


def build(tmp_path, tag, compress, R, experts):
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS, LayerPager, WorkingSlab
    from vllm_expert_pager.store import Store

    row_bytes = {n: r * c for n, (r, c) in synthetic.SHAPES.items()}
    path = str(tmp_path / f"pager-{tag}.bin") if R < E else None
    store = Store(1, E, R, 2 * W, row_bytes, compress, 0.89, path, DEV)
    store.retry_ns = 200_000_000
    for n in PARAMS:
        q = experts[n][0].cpu()
        for e in range(E):
            store.write(0, e, n, q[e])
    scales = {f"{n[:-7]}_weight_scale": experts[n][1] for n in PARAMS}
    shapes = {n: (synthetic.SHAPES[n], torch.float8_e4m3fn) for n in PARAMS}
    all_shapes = dict(shapes)
    all_shapes.update({k: (tuple(v.shape[1:]), v.dtype) for k, v in scales.items()})
    return store, LayerPager(store, 0, S, scales, shapes, WorkingSlab(W, all_shapes, store, DEV))


@pytest.mark.parametrize("compress,R", [(True, 16), (False, 16), (False, 32), (True, 32)],
                         ids=["compressed-ssd", "raw-ssd", "raw-ram", "compressed-ram"])
def test_fused_step_matches_reference_sequence(tmp_path, compress, R):
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS

    experts = synthetic.fp8_experts_device(E, DEV, seed=4)
    sa, fused = build(tmp_path, "a", compress, R, experts)
    sb, ref = build(tmp_path, "b", compress, R, experts)
    try:
        g = torch.Generator(device=DEV).manual_seed(9)
        for step in range(40):
            k = S if step % 5 else 3
            ids = torch.randperm(E, generator=g, device=DEV)[:k].to(torch.int32).view(1, -1)
            ra = fused.decode(ids, fused=True)
            rb = ref.decode(ids, fused=False)
            torch.cuda.synchronize()
            assert torch.equal(ra.expert_map, rb.expert_map), step
            for t in ("vram", "ram"):
                for attr in ("slot_of", "expert_in", "last_used", "counters"):
                    assert torch.equal(getattr(getattr(fused, t), attr),
                                       getattr(getattr(ref, t), attr)), (step, t, attr)
            emap = ra.expert_map.cpu()
            for e in ids.view(-1).tolist():
                s = int(emap[e])
                for n in PARAMS:
                    assert torch.equal(ra.slabs[n][s].view(torch.uint8),
                                       experts[n][0][e].view(torch.uint8)), (step, e, n)
                    sn = f"{n[:-7]}_weight_scale"
                    assert torch.equal(ra.slabs[sn][s], experts[n][1][e])
        assert fused.step_errors() == 0
        assert sa.failed is None and sb.failed is None
        assert (sa.fetches, sa.reads) == (sb.fetches, sb.reads)
        if R < E:
            assert sa.reads > 0
    finally:
        sa.release()
        sb.release()


def test_fused_step_replays_in_a_cuda_graph(tmp_path):
    """Captured once (compressed + SSD tier), replayed with new routing each time."""
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS

    experts = synthetic.fp8_experts_device(E, DEV, seed=5)
    store, pager = build(tmp_path, "g", True, 16, experts)
    try:
        ids = torch.zeros((1, S), dtype=torch.int32, device=DEV)
        ids.copy_(torch.arange(S, dtype=torch.int32).view(1, -1))
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            pager.decode(ids)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                res = pager.decode(ids)
        torch.cuda.synchronize()
        g = torch.Generator(device=DEV).manual_seed(1)
        for _ in range(25):
            ids.copy_(torch.randperm(E, generator=g, device=DEV)[:S].to(torch.int32).view(1, -1))
            graph.replay()
            torch.cuda.synchronize()
            emap = res.expert_map.cpu()
            for e in ids.view(-1).tolist():
                for n in PARAMS:
                    assert torch.equal(res.slabs[n][int(emap[e])].view(torch.uint8),
                                       experts[n][0][e].view(torch.uint8))
        assert pager.step_errors() == 0 and store.failed is None and store.reads > 0
        del graph
    finally:
        store.release()


@pytest.mark.parametrize("compress,R", [(False, 32), (True, 16)], ids=["raw-ram", "compressed-ssd"])
def test_host_ids_and_host_map_match_device_ids(tmp_path, compress, R):
    """Pinned host ids (read by the kernel) and the kernel's host copy of expert_map
    give the same step as device ids."""
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS

    experts = synthetic.fp8_experts_device(E, DEV, seed=5)
    sa, host = build(tmp_path, "h", compress, R, experts)
    sb, dev = build(tmp_path, "d", compress, R, experts)
    try:
        g = torch.Generator().manual_seed(11)
        for step in range(30):
            k = S if step % 4 else 5
            ids_h = torch.randperm(E, generator=g)[:k].to(torch.int32).pin_memory()
            map_h = torch.full((E,), -7, dtype=torch.int32).pin_memory()
            ra = host.decode(ids_h, map_out=map_h)
            rb = dev.decode(ids_h.to(DEV))
            torch.cuda.synchronize()
            assert torch.equal(ra.expert_map, rb.expert_map), step
            assert torch.equal(map_h, rb.expert_map.cpu()), step
            for t in ("vram", "ram"):
                for attr in ("slot_of", "expert_in", "last_used", "counters"):
                    assert torch.equal(getattr(getattr(host, t), attr),
                                       getattr(getattr(dev, t), attr)), (step, t, attr)
            for e in ids_h.tolist():
                s = int(map_h[e])
                for n in PARAMS:
                    assert torch.equal(ra.slabs[n][s].view(torch.uint8),
                                       experts[n][0][e].view(torch.uint8)), (step, e, n)
        with pytest.raises(ValueError, match="pinned"):
            host.decode(torch.zeros((1, S), dtype=torch.int32))
        with pytest.raises(ValueError, match="map_out"):
            host.decode(torch.zeros((1, S), dtype=torch.int32, device=DEV),
                        map_out=torch.zeros(E, dtype=torch.int32))
    finally:
        sa.release()
        sb.release()


def test_step_refuses_more_ctas_than_fit_at_once(tmp_path):
    """The copy CTAs wait for the table and fetch CTAs, so a grid that cannot be
    resident all at once is refused (XP_ERANGE) instead of timing out."""
    from vllm_expert_pager import gather, synthetic

    experts = synthetic.fp8_experts_device(E, DEV, seed=6)
    store, pager = build(tmp_path, "c", False, 16, experts)
    ids = torch.arange(S, dtype=torch.int32, device=DEV).view(1, -1)
    saved = gather.GATHER_CTAS
    try:
        gather.GATHER_CTAS = 1024  # 1027 CTAs of 256 threads with the tables' shared memory
        with pytest.raises(ValueError, match="-34"):
            pager.decode(ids)
        gather.GATHER_CTAS = 32
        pager.decode(ids)
        torch.cuda.synchronize()
        assert pager.step_errors() == 0
    finally:
        gather.GATHER_CTAS = saved
        store.release()


def test_step_give_ups_reach_the_host_copy_and_the_hook_check(tmp_path):
    """A step whose SSD-flag wait runs out (1 ms limit, host server delayed) counts
    the give-ups in the pinned host copy that step_errors() reads without a sync."""
    from vllm_expert_pager import native, synthetic

    experts = synthetic.fp8_experts_device(E, DEV, seed=7)
    store, pager = build(tmp_path, "e", True, 16, experts)
    lib = native.lib()
    try:
        store.retry_ns = 2_000_000_000  # the fetch CTA itself neither re-publishes nor gives up
        store.test_delay(0.3)
        assert lib.xp_set_step_wait_ns(-1, 1_000_000) == native.XP_OK
        ids = torch.arange(16, 16 + S, dtype=torch.int32, device=DEV).view(1, -1)  # RAM misses
        pager.decode(ids)
        torch.cuda.synchronize()
        n = pager.step_errors()
        # Concurrent give-ups may store their counts out of order: the host copy
        # can lag the device counter, but it moved.
        assert 0 < n <= int(pager.step_scratch[3])
        assert store.failed is None
    finally:
        lib.xp_set_step_wait_ns(-1, -1)
        store.test_delay(0.0)
        store.release()


def test_compressed_step_copies_only_the_used_record_words(tmp_path):
    """With compressed rows the fused step reads each record's used length from its
    header and copies only those words over the host link: staging bytes past them keep
    what was there, bytes within equal the record, and the decoded slots equal the raw
    rows."""
    from vllm_expert_pager import codec, synthetic
    from vllm_expert_pager.pager import PARAMS

    experts = synthetic.fp8_experts_device(E, DEV, seed=8)
    store, pager = build(tmp_path, "t", True, 32, experts)  # every expert in RAM
    try:
        for t in pager.decode_staging:
            t.fill_(0xAB)
        ids = torch.arange(S, dtype=torch.int32, device=DEV).view(1, -1) + 3
        res = pager.decode(ids)
        torch.cuda.synchronize()
        todo = pager.acquire._vram_todo[:S].cpu().tolist()
        ram_slot = pager.acquire.ram_slot.cpu()
        trimmed = 0
        for k, n in enumerate(PARAMS):
            N = store.row_bytes[n]
            G = N // codec.GROUP
            for j, e in enumerate(todo):
                if e < 0:
                    continue
                rec = store.pinned[n][int(ram_slot[e])]
                used = 4 * (G + 1 + N // 8 + int(rec[G]))
                stg = pager.decode_staging[k][j].cpu()
                assert torch.equal(stg[:used], rec.view(torch.uint8)[:used]), (n, e)
                assert bool((stg[used:] == 0xAB).all()), (n, e)
                trimmed += store.pitch[n] - used
                assert torch.equal(res.slabs[n][int(res.expert_map[e])].view(torch.uint8),
                                   experts[n][0][e].view(torch.uint8)), (n, e)
        assert trimmed > 0
    finally:
        store.release()


def test_corrupt_used_lengths_stay_inside_the_record(tmp_path):
    """The used length the fused step copies comes from the record's last header word;
    a corrupt one cannot move the copy outside the record: a huge value copies the whole
    pitch, a negative one only the header and nibble words, and the staging bytes past
    the copy keep theirs.  (The decode then clamps the same word to the record.)"""
    from vllm_expert_pager import codec, synthetic
    from vllm_expert_pager.pager import PARAMS

    experts = synthetic.fp8_experts_device(E, DEV, seed=9)
    store, pager = build(tmp_path, "c", True, 32, experts)  # expert e in RAM row e
    try:
        huge, neg = 4, 5
        for n in PARAMS:
            G = store.row_bytes[n] // codec.GROUP
            store.pinned[n][huge][G] = 2**31 - 1
            store.pinned[n][neg][G] = -5
        for t in pager.decode_staging:
            t.fill_(0xAB)
        ids = torch.arange(S, dtype=torch.int32, device=DEV).view(1, -1) + 3  # experts 3..10
        pager.decode(ids)
        torch.cuda.synchronize()
        todo = pager.acquire._vram_todo[:S].cpu().tolist()
        seen = set()
        for k, n in enumerate(PARAMS):
            N, P = store.row_bytes[n], store.pitch[n]
            G = N // codec.GROUP
            for j, e in enumerate(todo):
                if e not in (huge, neg):
                    continue
                seen.add(e)
                rec = store.pinned[n][e].view(torch.uint8)
                used = P if e == huge else 4 * (G + 1 + N // 8)
                stg = pager.decode_staging[k][j].cpu()
                assert torch.equal(stg[:used], rec[:used]), (n, e)
                assert bool((stg[used:] == 0xAB).all()), (n, e)
        assert seen == {huge, neg}
        assert pager.step_errors() == 0
    finally:
        store.release()
