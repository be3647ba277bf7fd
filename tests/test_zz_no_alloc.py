"""xp_decode_step_noalloc (the entry point for callers that cannot allocate) vs the allocating path.

Callers such as a serving engine that has reserved all free device memory for
its own pools, or a host driving the C ABI alone, cannot hand the library
scratch buffers.  ``xp_decode_step_noalloc`` takes its scratch (the step's
flags and the compressed staging rows) from an array compiled into the
library.  Its results must equal, byte for byte, those of the existing entry
points with caller-provided scratch (``xp_decode_step`` + ``xp_decode_rows``,
via ``LayerPager.decode``) on two calls in a row; the second call finds the
first call's leftovers in the shared array.  Kept in its own file, collected
last, and independent of the other tests' state.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
E, S, R, W = 32, 8, 16, 8


def build(tmp_path, tag, experts):
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS, LayerPager, WorkingSlab
    from vllm_expert_pager.store import Store

    row_bytes = {n: r * c for n, (r, c) in synthetic.SHAPES.items()}
    store = Store(1, E, R, 2 * W, row_bytes, True, 0.89, str(tmp_path / f"p-{tag}.bin"), DEV)
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


def noalloc_step(pager, ids):
    """One decode step of ``pager`` through xp_decode_step_noalloc (C ABI)."""
    from vllm_expert_pager import codec, native

    store, pair, a, b = pager.store, pager.acquire, pager.vram, pager.ram
    cw, sw = pager.cache_rows[:2], pager.cache_rows[2:]
    rv = pager.ram_view
    rc = native.lib().xp_decode_step_noalloc(
        ids.data_ptr(), ids.element_size(), ids.numel(), E,
        *a._table_args(), pair.expert_map.data_ptr(), pair.vram_slot.data_ptr(),
        pair._vram_todo.data_ptr(),
        *b._table_args(), pair.ram_slot.data_ptr(), pair._ram_todo.data_ptr(),
        a.no_cache.data_ptr(), 0,
        rv[0].data_ptr(), cw[0].data_ptr(), cw[0].shape[1], rv[0].shape[1],
        rv[1].data_ptr(), cw[1].data_ptr(), cw[1].shape[1], rv[1].shape[1],
        pager.scale_rows[0].data_ptr(), sw[0].data_ptr(), sw[0].shape[1],
        pager.scale_rows[1].data_ptr(), sw[1].data_ptr(), sw[1].shape[1],
        1, store.layer_lut(0).data_ptr(), codec.CHUNK, 16, 0,
        store.seq.data_ptr(), store.req_dev, store.done_dev, store.block, store.ring,
        store.retry_ns, store.giveup, torch.cuda.current_stream().cuda_stream)
    native.check(rc, "decode_step_noalloc")


def test_noalloc_step_matches_the_allocating_path(tmp_path):
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS

    experts = synthetic.fp8_experts_device(E, DEV, seed=21)
    sa, ref = build(tmp_path, "ref", experts)
    sb, dut = build(tmp_path, "dut", experts)
    try:
        g = torch.Generator(device=DEV).manual_seed(2)
        for call in range(2):  # two calls in a row share the library's scratch array
            # Experts >= R miss in RAM, so the SSD request and the staging are both used.
            ids = torch.cat([torch.randperm(R, generator=g, device=DEV)[:4],
                             R + torch.randperm(E - R, generator=g, device=DEV)[:4]])
            ids = ids.to(torch.int32).view(1, -1)
            ra = ref.decode(ids)
            noalloc_step(dut, ids)
            torch.cuda.synchronize()
            assert torch.equal(ra.expert_map, dut.expert_map), call
            for t in ("vram", "ram"):
                for attr in ("slot_of", "expert_in", "last_used", "counters"):
                    assert torch.equal(getattr(getattr(ref, t), attr),
                                       getattr(getattr(dut, t), attr)), (call, t, attr)
            for n in list(PARAMS) + [f"{p[:-7]}_weight_scale" for p in PARAMS]:
                assert torch.equal(ref.cache_slab[n].view(torch.uint8),
                                   dut.cache_slab[n].view(torch.uint8)), (call, n)
            emap = dut.expert_map.cpu()
            for e in ids.view(-1).tolist():
                for n in PARAMS:
                    assert torch.equal(dut.cache_slab[n][int(emap[e])].view(torch.uint8),
                                       experts[n][0][e].view(torch.uint8)), (call, e, n)
        assert sb.failed is None and sb.reads == sa.reads > 0
    finally:
        sa.release()
        sb.release()


def test_noalloc_step_rejects_staging_beyond_its_array():
    """K x (P0 + P1) x 4 + 256 bytes above the array: XP_ERANGE, nothing launched."""
    from vllm_expert_pager import native

    big = 1 << 22  # words per record: 16 MiB each, 8 rows x 2 names -> 256 MiB
    table_a = [None] * 4 + [S] + [None] * 3  # slot_of..counters, slots, map, slot, todo
    table_b = [None] * 4 + [R] + [None] * 2
    rc = native.lib().xp_decode_step_noalloc(
        None, 4, 8, E, *table_a, *table_b, None, 0,
        None, None, big, big, None, None, big, big,
        None, None, 4, None, None, 4,
        1, None, 512, 16, 0, None, None, None, 256, 4, 1, 1, None)
    assert rc == native.XP_ERANGE
