"""Pin the CPU table oracle (oracle/table.py) to the reference's own outputs.

The golden digests come from the reference ``ExpertTable`` run on CPU tensors
(tests/golden/make_golden.py).  These tests need no GPU.
"""

import os
import random

import numpy as np
import pytest

from digest import digest
from oracle.table import OracleTable, working_step

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def tstate(t: OracleTable) -> bytes:
    return digest(*t.state())


def split(vals, off):
    return [vals[off[i] : off[i + 1]] for i in range(len(off) - 1)]


def make_tables(E, S, R, warm):
    vram, ram = OracleTable(E, S), OracleTable(E, R)
    if warm:
        ram.warm(R)
    return vram, ram


@pytest.mark.parametrize("ci", range(5))
def test_acquire_matches_reference_digests(ci):
    g = load("acquire.npz")
    E, S, R, warm = (int(x) for x in g["configs"][ci])
    vram, ram = make_tables(E, S, R, bool(warm))
    for step, ids in enumerate(split(g[f"c{ci}_ids"], g[f"c{ci}_off"])):
        emap, slot, todo = vram.acquire(ids)
        _, src, ssd = ram.acquire(ids)
        want = g[f"c{ci}_digests"][step]
        got = [tstate(vram), digest(emap, slot, todo), tstate(ram), digest(src, ssd)]
        assert got == list(want), f"config {ci} step {step}"


def test_zipf_trace_matches_reference():
    from vllm_expert_pager import synthetic

    g = load("zipf.npz")
    trace = synthetic.zipf_trace(4096, layer=0)
    assert digest(trace.numpy()) == g["trace_digest"][0]
    vram, ram = make_tables(256, 32, 256, True)
    for i in range(trace.shape[0]):
        ids = trace[i].numpy()
        emap, slot, todo = vram.acquire(ids)
        _, src, ssd = ram.acquire(ids)
        assert np.array_equal(todo, g["vram_todo"][i]), f"step {i}"
        got = [tstate(vram), digest(emap, slot, todo), tstate(ram), digest(src, ssd)]
        assert got == list(g["digests"][i]), f"step {i}"
    assert [vram.hits, vram.misses] == g["final_vram_hits"].tolist()
    assert [ram.hits, ram.misses] == g["final_ram_hits"].tolist()


@pytest.mark.parametrize("W", [1, 3, 4])
def test_mixed_working_steps_match_reference(W):
    g = load("working.npz")
    E, R, S, L, layer = 16, 6, 3, 2, 1
    ram_base, working_base = layer * R, L * R
    ram, vram = OracleTable(E, R), OracleTable(E, S)
    ids_l = split(g[f"mix{W}_ids"], g[f"mix{W}_off"])
    tops = split(g[f"mix{W}_top"], g[f"mix{W}_top_off"])
    for step, ids in enumerate(ids_l):
        want = list(g[f"mix{W}_digests"][step])
        if g[f"mix{W}_kinds"][step] == 0:
            _, _, todo = ram.acquire(ids)
            emap, slot, vtodo = vram.acquire(ids)
            got = [tstate(ram), tstate(vram), digest(todo, emap, slot, vtodo)]
        else:
            top = tops[step] if len(tops[step]) else None
            need, _, _, plan = working_step(ram, vram, ids, W, ram_base, working_base, top=top)
            got = [tstate(ram), tstate(vram), digest(need, *plan)]
        assert got == want, f"W={W} step {step}"


def _restore(t: OracleTable, g, prefix):
    t.slot_of = g[f"{prefix}_slot_of"].astype(np.int64).copy()
    t.expert_in = g[f"{prefix}_expert_in"].astype(np.int64).copy()
    t.last_used = g[f"{prefix}_last_used"].astype(np.int64).copy()
    t.step, t.hits, t.misses = (int(x) for x in g[f"{prefix}_counters"])


PLAN_KEYS = ("dst_row", "src_row", "maps", "todo", "ssd", "late")


@pytest.mark.parametrize(
    "case", ["prefill_r128", "prefill_r256", "batch8_r128", "sc_seed", "sc_acquire",
             "sc_alternate", "sc_negative"]
)
def test_working_cases_match_reference(case):
    g = load("working.npz")
    E, S, R, W, L, layer = (int(x) for x in g[f"{case}_cfg"])
    vram, ram = OracleTable(E, S), OracleTable(E, R)
    _restore(vram, g, f"{case}_pre_vram")
    _restore(ram, g, f"{case}_pre_ram")
    top = g[f"{case}_top"]
    need, _, _, plan = working_step(ram, vram, g[f"{case}_ids"], W, layer * R, L * R,
                                    top=top if top.size else None)
    for key, got in zip(PLAN_KEYS, plan):
        assert np.array_equal(got, g[f"{case}_{key}"]), key
    for key in ("slot_of", "expert_in", "last_used"):
        assert np.array_equal(getattr(ram, key), g[f"{case}_post_ram_{key}"]), key
    assert [ram.step, ram.hits, ram.misses] == g[f"{case}_post_ram_counters"].tolist()


def test_prefill_topk_choice_is_a_valid_topk():
    """The reference's logged topk and the oracle's lowest-id rule pick sets with
    the same counts (they may differ only among equal counts)."""
    from oracle.table import top_experts

    g = load("working.npz")
    for case in ("prefill_r128", "prefill_r256"):
        ids = g[f"{case}_ids"].reshape(-1).astype(np.int64)
        counts = np.bincount(ids[ids >= 0], minlength=256)
        ref_top = g[f"{case}_top"]
        mine = top_experts(counts, ref_top.size)
        assert sorted(counts[ref_top]) == sorted(counts[mine])


def test_oracle_matches_plain_python_lru():
    """Same cross-check as the reference test_table.py::ReferenceLRU (S in 1,4,8)."""
    for S in (1, 4, 8):
        rng = random.Random(0)
        t = OracleTable(16, S)
        slot_of, stamp, step = {}, [0] * S, 1
        for _ in range(300):
            ids = [rng.randrange(16) for _ in range(rng.randint(1, S))]
            t.acquire(ids)
            exps = set(ids)
            hits = {e for e in exps if e in slot_of}
            protected = {slot_of[e] for e in hits}
            for e in sorted(exps - hits):
                victim = min((s for s in range(S) if s not in protected),
                             key=lambda s: (stamp[s], s))
                for old, s in list(slot_of.items()):
                    if s == victim:
                        del slot_of[old]
                slot_of[e] = victim
                protected.add(victim)
            for e in exps:
                stamp[slot_of[e]] = step
            step += 1
            assert {e for e in range(16) if t.slot_of[e] >= 0} == set(slot_of)
