"""xp_decode_step_noalloc (the entry point for callers that cannot allocate) vs the allocating path.

Callers such as a serving engine that has reserved all free device memory for
its own pools, or a host driving the C ABI alone, cannot hand the library
scratch buffers.  ``xp_decode_step_noalloc`` takes its scratch (the step's
flags and the compressed staging rows) from an array compiled into the
library.  Its results must equal, byte for byte, those of the existing entry
points with caller-provided scratch (``xp_decode_step`` + ``xp_decode_rows``,
via ``LayerPager.decode``) on two calls in a row; the second call finds the
first call's leftovers in the shared array.  Layer 0 and layer 1 of a two-layer
store are both checked, so the layer's RAM-tier base and decode tables count.
A step whose wait gives up must be visible to the caller through
``errors_out``.  Kept in its own file, collected last, and independent of the
other tests' state.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
E, S, R, W, L = 32, 8, 16, 8, 2


def build(tmp_path, tag, experts):
    """A two-layer compressed store (layer l holds experts[l]) and a pager per layer."""
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS, LayerPager, WorkingSlab
    from vllm_expert_pager.store import Store

    row_bytes = {n: r * c for n, (r, c) in synthetic.SHAPES.items()}
    store = Store(L, E, R, 2 * W, row_bytes, True, 0.89, str(tmp_path / f"p-{tag}.bin"), DEV)
    store.retry_ns = 200_000_000
    for layer in range(L):
        for n in PARAMS:
            q = experts[layer][n][0].cpu()
            for e in range(E):
                store.write(layer, e, n, q[e])
    shapes = {n: (synthetic.SHAPES[n], torch.float8_e4m3fn) for n in PARAMS}
    pagers, working = [], None
    for layer in range(L):
        scales = {f"{n[:-7]}_weight_scale": experts[layer][n][1] for n in PARAMS}
        if working is None:
            all_shapes = dict(shapes)
            all_shapes.update({k: (tuple(v.shape[1:]), v.dtype) for k, v in scales.items()})
            working = WorkingSlab(W, all_shapes, store, DEV)
        pagers.append(LayerPager(store, layer, S, scales, shapes, working))
    return store, pagers


def noalloc_step(pager, ids, errors_out=None):
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
        a.no_cache.data_ptr(), pager.layer * store.ram_slots,
        rv[0].data_ptr(), cw[0].data_ptr(), cw[0].shape[1], rv[0].shape[1],
        rv[1].data_ptr(), cw[1].data_ptr(), cw[1].shape[1], rv[1].shape[1],
        pager.scale_rows[0].data_ptr(), sw[0].data_ptr(), sw[0].shape[1],
        pager.scale_rows[1].data_ptr(), sw[1].data_ptr(), sw[1].shape[1],
        1, store.layer_lut(pager.layer).data_ptr(), codec.CHUNK, 16, pager.layer,
        store.seq.data_ptr(), store.req_dev, store.done_dev, store.block, store.ring,
        store.retry_ns, store.giveup, native.ptr(errors_out),
        torch.cuda.current_stream().cuda_stream)
    native.check(rc, "decode_step_noalloc")


def routing(g):
    # Experts >= R miss in RAM, so the SSD request and the staging are both used.
    ids = torch.cat([torch.randperm(R, generator=g, device=DEV)[:4],
                     R + torch.randperm(E - R, generator=g, device=DEV)[:4]])
    return ids.to(torch.int32).view(1, -1)


def test_noalloc_step_matches_the_allocating_path(tmp_path):
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS

    experts = [synthetic.fp8_experts_device(E, DEV, seed=21 + layer) for layer in range(L)]
    sa, refs = build(tmp_path, "ref", experts)
    sb, duts = build(tmp_path, "dut", experts)
    errors = torch.zeros((1,), dtype=torch.int32, pin_memory=True)
    try:
        g = torch.Generator(device=DEV).manual_seed(2)
        # Two calls in a row on layer 0 share the library's scratch array; then one
        # on layer 1, whose RAM rows start at 1 x R and whose decode tables differ.
        for call, layer in enumerate((0, 0, 1)):
            ref, dut = refs[layer], duts[layer]
            ids = routing(g)
            ra = ref.decode(ids)
            noalloc_step(dut, ids, errors)
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
                                       experts[layer][n][0][e].view(torch.uint8)), (call, e, n)
        assert int(errors[0]) == 0
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
    for P0, P1 in ((big, big), (1 << 60, 16), (16, 1 << 60)):
        rc = native.lib().xp_decode_step_noalloc(
            None, 4, 8, E, *table_a, *table_b, None, 0,
            None, None, big, P0, None, None, big, P1,
            None, None, 4, None, None, 4,
            1, None, 512, 16, 0, None, None, None, 256, 4, 1, 1, None, None)
        assert rc == native.XP_ERANGE, (P0, P1)


def test_noalloc_step_reports_a_wait_that_gave_up(tmp_path):
    """The array's own give-up counter is out of the host's reach; errors_out is how a
    caller learns that a step's SSD wait ran out (1 ms limit, host server delayed)."""
    from vllm_expert_pager import native, synthetic

    experts = [synthetic.fp8_experts_device(E, DEV, seed=31 + layer) for layer in range(L)]
    store, pagers = build(tmp_path, "gu", experts)
    lib = native.lib()
    errors = torch.zeros((1,), dtype=torch.int32, pin_memory=True)
    try:
        store.retry_ns = 2_000_000_000  # the fetch CTA neither re-publishes nor gives up
        store.test_delay(0.3)
        assert lib.xp_set_step_wait_ns(-1, 1_000_000) == native.XP_OK
        ids = torch.arange(R, R + S, dtype=torch.int32, device=DEV).view(1, -1)  # all in SSD
        noalloc_step(pagers[0], ids, errors)
        torch.cuda.synchronize()
        assert int(errors[0]) > 0
        assert store.failed is None
    finally:
        lib.xp_set_step_wait_ns(-1, -1)
        store.test_delay(0.0)
        store.release()
