"""Slot-table kernels (table.cu, via the C ABI) against the reference's golden digests and the oracle.

Bit-exact: every table array, counter and output after every step.
"""

import os
import random

import numpy as np
import pytest
import torch

from digest import digest
from oracle.table import OracleTable

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = torch.device("cuda")


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def split(vals, off):
    return [vals[off[i] : off[i + 1]] for i in range(len(off) - 1)]


def tstate(t) -> bytes:
    E, S = t.num_experts, t.num_slots
    c = t.counters
    return digest(t.slot_of[:E], t.expert_in[:S], t.last_used[:S], c[0:1], c[1:2], c[2:3])


def make_tables(E, S, R, warm):
    from vllm_expert_pager.table import ExpertTable

    vram, ram = ExpertTable(E, S, DEV), ExpertTable(E, R, DEV)
    if warm:
        ram.slot_of[:R] = ram.experts[:R]
        ram.expert_in[:R] = ram.experts[:R]
    return vram, ram


def set_state(t, g, prefix):
    E, S = t.num_experts, t.num_slots
    t.slot_of[:E] = torch.from_numpy(g[f"{prefix}_slot_of"].astype(np.int64)).to(DEV)
    t.expert_in[:S] = torch.from_numpy(g[f"{prefix}_expert_in"].astype(np.int64)).to(DEV)
    t.last_used[:S] = torch.from_numpy(g[f"{prefix}_last_used"].astype(np.int64)).to(DEV)
    t.counters.copy_(torch.from_numpy(g[f"{prefix}_counters"].astype(np.int64)).to(DEV))


def oracle_of(t) -> OracleTable:
    o = OracleTable(t.num_experts, t.num_slots)
    o.slot_of = t.slot_of[: t.num_experts].cpu().numpy().copy()
    o.expert_in = t.expert_in[: t.num_slots].cpu().numpy().copy()
    o.last_used = t.last_used[: t.num_slots].cpu().numpy().copy()
    o.step, o.hits, o.misses = (int(x) for x in t.counters.cpu())
    return o


@pytest.mark.parametrize("ci", range(5))
@pytest.mark.parametrize("ids_dtype", [torch.int32, torch.int64])
def test_acquire_pair_matches_reference(ci, ids_dtype):
    from vllm_expert_pager.acquire import AcquirePair

    g = load("acquire.npz")
    E, S, R, warm = (int(x) for x in g["configs"][ci])
    vram, ram = make_tables(E, S, R, bool(warm))
    pair = AcquirePair(vram, ram)
    for step, ids in enumerate(split(g[f"c{ci}_ids"], g[f"c{ci}_off"])):
        t = torch.tensor(ids.reshape(1, -1), dtype=ids_dtype, device=DEV)
        todo, ssd = pair(t)
        got = [tstate(vram), digest(pair.expert_map, pair.vram_slot, todo), tstate(ram),
               digest(pair.ram_slot, ssd)]
        assert got == list(g[f"c{ci}_digests"][step]), f"config {ci} step {step}"


@pytest.mark.parametrize("ci", range(5))
def test_single_acquire_matches_reference(ci):
    g = load("acquire.npz")
    E, S, R, warm = (int(x) for x in g["configs"][ci])
    vram, ram = make_tables(E, S, R, bool(warm))
    for step, ids in enumerate(split(g[f"c{ci}_ids"], g[f"c{ci}_off"])):
        t = torch.tensor(ids, dtype=torch.int64, device=DEV)
        emap, slot, todo = vram.acquire(t)
        _, src, ssd = ram.acquire(t)
        got = [tstate(vram), digest(emap, slot, todo), tstate(ram), digest(src, ssd)]
        assert got == list(g[f"c{ci}_digests"][step]), f"config {ci} step {step}"


def test_zipf_trace_matches_reference():
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.acquire import AcquirePair

    g = load("zipf.npz")
    trace = synthetic.zipf_trace(4096, layer=0)
    assert digest(trace) == g["trace_digest"][0]
    vram, ram = make_tables(256, 32, 256, True)
    pair = AcquirePair(vram, ram)
    dtrace = trace.to(DEV)
    for i in range(trace.shape[0]):
        todo, ssd = pair(dtrace[i])
        got = [tstate(vram), digest(pair.expert_map, pair.vram_slot, todo), tstate(ram),
               digest(pair.ram_slot, ssd)]
        assert got == list(g["digests"][i]), f"step {i}"


def test_acquire_pair_replays_in_a_cuda_graph():
    """Captured once, replayed with new ids in the same buffer: matches the oracle."""
    from vllm_expert_pager.acquire import AcquirePair

    E, S, R = 256, 32, 128
    vram, ram = make_tables(E, S, R, True)
    ovram, oram = oracle_of(vram), oracle_of(ram)
    pair = AcquirePair(vram, ram)
    ids = torch.zeros((1, 8), dtype=torch.int32, device=DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        pair(ids)  # warm-up (also a real step, mirrored below)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            todo, ssd = pair(ids)
    torch.cuda.synchronize()
    ovram.acquire([0] * 8)
    oram.acquire([0] * 8)
    rng = random.Random(5)
    for _ in range(100):
        new = [rng.randrange(E) for _ in range(8)]
        ids.copy_(torch.tensor([new], dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize()
        emap, _, otodo = ovram.acquire(new)
        _, _, ossd = oram.acquire(new)
        assert np.array_equal(pair.expert_map.cpu().numpy(), emap)
        assert np.array_equal(todo.cpu().numpy(), otodo)
        assert np.array_equal(ssd.cpu().numpy(), ossd)
        assert [digest(x) for x in oracle_of(vram).state()] == [digest(x) for x in ovram.state()]


def test_acquire_edge_cases_match_oracle():
    """Empty steps, ids outside [0, E), K == S, one slot, big tables."""
    rng = random.Random(11)
    for E, S in ((16, 1), (16, 16), (256, 512), (300, 7), (1024, 1024)):
        from vllm_expert_pager.table import ExpertTable

        t = ExpertTable(E, S, DEV)
        o = OracleTable(E, S)
        for _ in range(60):
            k = rng.choice([0, 1, S, rng.randint(0, S)])
            ids = [rng.randrange(-3, E + 3) for _ in range(k)]
            emap, slot, todo = t.acquire(torch.tensor(ids, dtype=torch.int64, device=DEV))
            oe, os_, ot = o.acquire(ids)
            assert np.array_equal(emap.cpu().numpy(), oe)
            assert np.array_equal(slot.cpu().numpy(), os_)
            assert np.array_equal(todo.cpu().numpy(), ot)
            assert [digest(x) for x in oracle_of(t).state()] == [digest(x) for x in o.state()]


PLAN_KEYS = ("dst_row", "src_row", "maps", "todo", "ssd", "late")


def _working_step(ram, vram, ids, W, ram_base, working_base, top, impl="separate"):
    """One working-step planning: the reference's separate calls, or one fused launch."""
    if impl == "fused":
        from vllm_expert_pager.table import WorkingPlan

        plan = WorkingPlan(ram.num_experts, W, ram.num_slots, vram.num_slots, DEV)
        need, _, out = plan(ram, vram, ids, ram_base, working_base, top)
        return need, out
    E = ram.num_experts
    need = ram.need_mask(ids)
    cached_row = vram.slot_of[:E].clone()
    before = ram.slot_of[:E].clone()
    if ids.numel() <= ram.num_slots:
        ram.acquire(ids)
    else:
        ram.seed(vram, ids, need, top=top)
    return need, ram.plan_chunks(before, need, cached_row, W, ram_base, working_base)


@pytest.mark.parametrize("impl", ["separate", "fused"])
@pytest.mark.parametrize(
    "case", ["prefill_r128", "prefill_r256", "batch8_r128", "sc_seed", "sc_acquire",
             "sc_alternate", "sc_negative"]
)
def test_working_cases_match_reference(case, impl):
    from vllm_expert_pager.table import ExpertTable

    g = load("working.npz")
    E, S, R, W, L, layer = (int(x) for x in g[f"{case}_cfg"])
    vram, ram = ExpertTable(E, S, DEV), ExpertTable(E, R, DEV)
    set_state(vram, g, f"{case}_pre_vram")
    set_state(ram, g, f"{case}_pre_ram")
    top = g[f"{case}_top"]
    ids = torch.from_numpy(g[f"{case}_ids"].astype(np.int64)).to(DEV)
    need, plan = _working_step(ram, vram, ids, W, layer * R, L * R,
                               torch.from_numpy(top).to(DEV) if top.size else None, impl)
    for key, got in zip(PLAN_KEYS, plan):
        assert np.array_equal(got.cpu().numpy(), g[f"{case}_{key}"]), key
    for key in ("slot_of", "expert_in", "last_used"):
        n = E if key == "slot_of" else R
        assert np.array_equal(getattr(ram, key)[:n].cpu().numpy(), g[f"{case}_post_ram_{key}"])
    assert ram.counters.cpu().tolist() == g[f"{case}_post_ram_counters"].tolist()


@pytest.mark.parametrize("impl", ["separate", "fused"])
@pytest.mark.parametrize("case", ["prefill_r128", "prefill_r256"])
def test_seed_tie_rule_matches_oracle(case, impl):
    """Without a replayed choice, the kernel's lowest-id tie rule equals the oracle's."""
    from oracle.table import working_step
    from vllm_expert_pager.table import ExpertTable

    g = load("working.npz")
    E, S, R, W, L, layer = (int(x) for x in g[f"{case}_cfg"])
    vram, ram = ExpertTable(E, S, DEV), ExpertTable(E, R, DEV)
    set_state(vram, g, f"{case}_pre_vram")
    set_state(ram, g, f"{case}_pre_ram")
    ovram, oram = oracle_of(vram), oracle_of(ram)
    ids_np = g[f"{case}_ids"].astype(np.int64)
    _, plan = _working_step(ram, vram, torch.from_numpy(ids_np).to(DEV), W, layer * R, L * R,
                            None, impl)
    _, _, _, oplan = working_step(oram, ovram, ids_np, W, layer * R, L * R)
    for key, a, b in zip(PLAN_KEYS, plan, oplan):
        assert np.array_equal(a.cpu().numpy(), b), key
    assert [digest(x) for x in oracle_of(ram).state()] == [digest(x) for x in oram.state()]


@pytest.mark.parametrize("impl", ["separate", "fused"])
@pytest.mark.parametrize("W", [1, 3, 4])
def test_mixed_working_steps_match_reference(W, impl):
    from vllm_expert_pager.table import ExpertTable

    g = load("working.npz")
    E, R, S, L, layer = 16, 6, 3, 2, 1
    ram, vram = ExpertTable(E, R, DEV), ExpertTable(E, S, DEV)
    ids_l = split(g[f"mix{W}_ids"], g[f"mix{W}_off"])
    tops = split(g[f"mix{W}_top"], g[f"mix{W}_top_off"])
    for step, ids_np in enumerate(ids_l):
        ids = torch.from_numpy(ids_np.reshape(1, -1)).to(DEV)
        want = list(g[f"mix{W}_digests"][step])
        if g[f"mix{W}_kinds"][step] == 0:
            _, _, todo = ram.acquire(ids)
            emap, slot, vtodo = vram.acquire(ids)
            got = [tstate(ram), tstate(vram), digest(todo, emap, slot, vtodo)]
        else:
            top = torch.from_numpy(tops[step]).to(DEV) if len(tops[step]) else None
            need, plan = _working_step(ram, vram, ids, W, layer * R, L * R, top, impl)
            got = [tstate(ram), tstate(vram), digest(need, *plan)]
        assert got == want, f"W={W} step {step}"


def test_need_mask_matches_oracle():
    from vllm_expert_pager.table import ExpertTable

    rng = random.Random(3)
    t = ExpertTable(256, 32, DEV)
    o = OracleTable(256, 32)
    for k in (0, 1, 8, 300, 16384):
        ids = [rng.randrange(-2, 260) for _ in range(k)]
        got = t.need_mask(torch.tensor(ids, dtype=torch.int32, device=DEV))
        assert np.array_equal(got.cpu().numpy(), o.need_mask(ids))
