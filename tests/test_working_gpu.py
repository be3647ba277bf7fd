"""Chunked working-slab path: the MoE output is bit-identical to an unpaged run.

The reference claims (README.md:40-57, experts.py:479-488) that running a
prefill's experts through the W-row working slab in chunks, collecting the
per-expert contributions and taking the top-k sum once, matches a single run
bit for bit; no reference test checks it.  Here the same vLLM Triton FP8 MoE
runs (a) once over all experts resident in HBM, (b) through
``LayerPager.working_chunks`` (seed/acquire + plan_chunks + gathers from pinned
RAM, SSD reads for experts outside the RAM tier, GPU decode of compressed
rows, chunk k+1's copies overlapped with chunk k's MoE), and the outputs must
be ``torch.equal``.  Both runs use one kernel config so that only the paging
differs.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
E, S, W, T, TOPK = 64, 8, 16, 256, 8


def build(tmp_path, compress: bool, ram_slots: int):
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS, LayerPager, WorkingSlab
    from vllm_expert_pager.store import Store

    experts = synthetic.fp8_experts_device(E, DEV, seed=1)
    row_bytes = {n: r * c for n, (r, c) in synthetic.SHAPES.items()}
    path = str(tmp_path / "pager.bin") if ram_slots < E else None
    store = Store(1, E, ram_slots, 2 * W, row_bytes, compress, 0.89, path, DEV)
    store.retry_ns = 200_000_000
    for n in PARAMS:
        q = experts[n][0].cpu()
        for e in range(E):
            store.write(0, e, n, q[e])
    scales = {f"{n[:-7]}_weight_scale": experts[n][1] for n in PARAMS}
    shapes = {n: (synthetic.SHAPES[n], torch.float8_e4m3fn) for n in PARAMS}
    all_shapes = dict(shapes)
    all_shapes.update({k: (tuple(v.shape[1:]), v.dtype) for k, v in scales.items()})
    working = WorkingSlab(W, all_shapes, store, DEV)
    pager = LayerPager(store, 0, S, scales, shapes, working)
    return store, pager, experts, scales


@pytest.mark.parametrize("compress,ram_slots", [(True, 32), (False, 32), (False, 64), (True, 64)],
                         ids=["compressed-ssd", "raw-ssd", "raw-ram", "compressed-ram"])
@pytest.mark.parametrize("overlap", [True, False], ids=["overlap", "serial"])
def test_chunked_prefill_is_bit_identical(tmp_path, compress, ram_slots, overlap):
    from vllm_expert_pager import moe

    store, pager, experts, scales = build(tmp_path, compress, ram_slots)
    try:
        g = torch.Generator(device=DEV).manual_seed(7)
        # A few decode steps first so some experts are VRAM hits (copied from the cache slab).
        for _ in range(6):
            ids = torch.randperm(E, generator=g, device=DEV)[:TOPK].to(torch.int32)
            pager.decode(ids.view(1, -1))
        x = (torch.randn((T, 2048), generator=g, device=DEV) * 0.5).to(torch.bfloat16)
        topk_ids = torch.rand((T, E), generator=g, device=DEV).topk(TOPK).indices.to(torch.int32)
        topk_w = torch.softmax(torch.randn((T, TOPK), generator=g, device=DEV), -1)
        w13, w2 = experts["w13_weight"][0], experts["w2_weight"][0]
        s13, s2 = experts["w13_weight"][1], experts["w2_weight"][1]
        config = moe.moe_config(w13.shape, w2.shape, TOPK, T)
        ref3 = moe.contributions(x, w13, w2, s13, s2, topk_w, topk_ids, None, E, config)
        ref = torch.empty_like(x)
        moe.moe_sum(ref3, ref)

        out = torch.empty_like(x)
        acc = {}

        def run_chunk(k, n, slabs, expert_map):
            c3 = moe.contributions(x, slabs["w13_weight"], slabs["w2_weight"],
                                   slabs["w13_weight_scale"], slabs["w2_weight_scale"], topk_w,
                                   topk_ids, expert_map, E, config)
            acc["c"] = c3 if "c" not in acc else acc["c"].add_(c3)
            if k == n - 1:
                moe.moe_sum(acc["c"], out)
            return out

        pager.working_chunks(topk_ids, run_chunk, overlap=overlap)
        torch.cuda.synchronize()
        assert store.failed is None, store.failed
        assert int(store.req[store.giveup_at]) == 0
        assert torch.equal(acc["c"], ref3)
        assert torch.equal(out, ref)
        if ram_slots < E:
            assert store.reads > 0  # the SSD tier was exercised
    finally:
        store.release()


def test_decode_step_after_prefill_reads_the_right_rows(tmp_path):
    """Decode steps after a working step page in byte-identical rows (tables stayed consistent)."""
    from vllm_expert_pager.pager import PARAMS

    store, pager, experts, scales = build(tmp_path, True, 32)
    try:
        g = torch.Generator(device=DEV).manual_seed(3)
        topk_ids = torch.rand((64, E), generator=g, device=DEV).topk(TOPK).indices.to(torch.int32)
        pager.working_chunks(topk_ids, lambda k, n, slabs, m: None)
        for _ in range(20):
            ids = torch.randperm(E, generator=g, device=DEV)[:TOPK].to(torch.int32).view(1, -1)
            res = pager.decode(ids)
            torch.cuda.synchronize()
            emap = res.expert_map.cpu()
            for e in ids.view(-1).tolist():
                s = int(emap[e])
                for n in PARAMS:
                    assert torch.equal(res.slabs[n][s].view(torch.uint8).cpu(),
                                       experts[n][0][e].view(torch.uint8).cpu()), (e, n)
                    sn = f"{n[:-7]}_weight_scale"
                    assert torch.equal(res.slabs[sn][s], scales[sn][e])
        assert store.failed is None
    finally:
        store.release()


def test_config5_prefill_is_bit_identical(tmp_path):
    """Config 5's shape: a 2048-token prefill with uniform top-8 routing over 256
    experts (nearly all of them needed), S=32, W=64 (5 chunks), RAM tier of 128
    compressed rows + the SSD paging file, chunk copies overlapped with the MoE.
    The chunked output equals vLLM's MoE over all experts resident, bit for bit."""
    from vllm_expert_pager import moe, synthetic
    from vllm_expert_pager.pager import PARAMS, LayerPager, WorkingSlab
    from vllm_expert_pager.store import Store

    E5, S5, W5, R5, T5 = 256, 32, 64, 128, 2048
    experts = synthetic.fp8_experts_device(E5, DEV, seed=17)
    row_bytes = {n: r * c for n, (r, c) in synthetic.SHAPES.items()}
    store = Store(1, E5, R5, 2 * W5, row_bytes, True, 0.89, str(tmp_path / "p5.bin"), DEV)
    try:
        for n in PARAMS:
            q = experts[n][0]
            for e in range(E5):
                store.write(0, e, n, q[e])
        scales = {f"{n[:-7]}_weight_scale": experts[n][1] for n in PARAMS}
        shapes = {n: (synthetic.SHAPES[n], torch.float8_e4m3fn) for n in PARAMS}
        all_shapes = dict(shapes)
        all_shapes.update({k: (tuple(v.shape[1:]), v.dtype) for k, v in scales.items()})
        pager = LayerPager(store, 0, S5, scales, shapes,
                           WorkingSlab(W5, all_shapes, store, DEV))
        g = torch.Generator(device=DEV).manual_seed(8)
        for _ in range(4):  # some VRAM hits, as after decode steps
            ids = torch.randperm(E5, generator=g, device=DEV)[:TOPK].to(torch.int32)
            pager.decode(ids.view(1, -1))
        x = (torch.randn((T5, 2048), generator=g, device=DEV) * 0.5).to(torch.bfloat16)
        topk_ids = synthetic.uniform_routing(T5, E5, TOPK, seed=5).to(DEV)
        topk_w = torch.softmax(torch.randn((T5, TOPK), generator=g, device=DEV), -1)
        w13, w2 = experts["w13_weight"][0], experts["w2_weight"][0]
        s13, s2 = experts["w13_weight"][1], experts["w2_weight"][1]
        config = moe.moe_config(w13.shape, w2.shape, TOPK, T5)
        ref = torch.empty_like(x)
        moe.moe_sum(moe.contributions(x, w13, w2, s13, s2, topk_w, topk_ids, None, E5, config),
                    ref)
        out = torch.empty_like(x)
        acc = {}

        def run_chunk(k, n, slabs, expert_map):
            c3 = moe.contributions(x, slabs["w13_weight"], slabs["w2_weight"],
                                   slabs["w13_weight_scale"], slabs["w2_weight_scale"], topk_w,
                                   topk_ids, expert_map, E5, config)
            acc["c"] = c3 if "c" not in acc else acc["c"].add_(c3)
            acc["n"] = n
            if k == n - 1:
                moe.moe_sum(acc["c"], out)

        pager.working_chunks(topk_ids, run_chunk, overlap=True)
        torch.cuda.synchronize()
        assert acc["n"] == E5 // W5 + 1
        assert store.failed is None, store.failed
        assert int(store.req[store.giveup_at]) == 0
        assert store.reads > 0  # the SSD tier served experts outside the RAM tier
        assert torch.equal(out, ref)
    finally:
        store.release()
