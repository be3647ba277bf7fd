"""Record golden vectors from the reference implementation (monochromegane/vllm-expert-pager).

Run from the repository root with the reference's ``src`` directory first on
the import path, so that ``vllm_expert_pager`` resolves to the REFERENCE:

    PYTHONPATH=<reference checkout>/src python tests/golden/make_golden.py

It imports only the reference's CPU-capable modules: ``table.py`` (torch ops on
CPU tensors) and ``codec.py`` (``encode`` is torch ops; importing it needs
triton, which only defines the GPU decoder).  The seeded inputs come from this
repository's ``synthetic.py``, loaded by file path.  Outputs go to
``tests/golden/*.npz``; the CPU tests check the oracle against them and the GPU
tests check the CUDA kernels against them.

Recorded:
* acquire.npz  -- the reference test_acquire.py scenarios (4 table configs x 200
  random steps, plus one with vLLM's -1 ids), per-step digests of both tables'
  state and outputs of ``ExpertTable.acquire``;
* zipf.npz     -- the config-2 trace (4096 Zipf(1.1) steps, E=256, S=32,
  R=256) through both tables, per-step digests and VRAM miss lists;
* working.npz  -- ``need_mask`` / ``acquire`` / ``seed`` / ``plan_chunks`` over the
  random mixed steps of test_table.py, the three scenario tests, and three
  E=256 working steps (prefill 2048x8 with R=128 and R=256, batch-8 decode);
  every ``torch.topk`` choice made inside ``seed`` is logged so the oracle can
  replay it (its tie order is implementation-defined);
* codec.npz    -- ``code_lengths`` of assorted histograms, records and LUTs of
  the test_codec.py distributions (CHUNK 64 and 512), and digests + LUTs of the
  config-1 experts (8 x (w13, w2), pitch 0.89).
"""

from __future__ import annotations

import importlib.util
import os
import random
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
from digest import digest  # noqa: E402

from vllm_expert_pager import codec as ref_codec  # noqa: E402  (the reference)
from vllm_expert_pager import table as ref_table  # noqa: E402

if os.path.abspath(ref_table.__file__).startswith(REPO):
    raise SystemExit("vllm_expert_pager must resolve to the reference, not this repository")

_spec = importlib.util.spec_from_file_location(
    "xp_synthetic", os.path.join(REPO, "vllm-expert-pager_b200", "vllm_expert_pager", "synthetic.py")
)
synthetic = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(synthetic)

ExpertTable = ref_table.ExpertTable
CPU = torch.device("cpu")

# ---- topk logging: record the indices every torch.topk call returns ----
_topk_log: list[np.ndarray] = []
_orig_topk = torch.Tensor.topk


def _logged_topk(self, *args, **kwargs):
    r = _orig_topk(self, *args, **kwargs)
    _topk_log.append(r.indices.clone().numpy())
    return r


def tstate(t: ExpertTable) -> bytes:
    E, S = t.num_experts, t.num_slots
    return digest(t.slot_of[:E], t.expert_in[:S], t.last_used[:S], t.step.view(1),
                  t.hits.view(1), t.misses.view(1))


def full_state(t: ExpertTable) -> dict[str, np.ndarray]:
    E, S = t.num_experts, t.num_slots
    return {
        "slot_of": t.slot_of[:E].numpy().copy(),
        "expert_in": t.expert_in[:S].numpy().copy(),
        "last_used": t.last_used[:S].numpy().copy(),
        "counters": np.array([int(t.step), int(t.hits), int(t.misses)], dtype=np.int64),
    }


def make_tables(E, S, R, warm):
    vram, ram = ExpertTable(E, S, CPU), ExpertTable(E, R, CPU)
    if warm:
        ram.slot_of[:R] = ram.experts[:R]
        ram.expert_in[:R] = ram.experts[:R]
    return vram, ram


def flat(lists):
    off = np.cumsum([0] + [len(x) for x in lists]).astype(np.int64)
    vals = np.concatenate([np.asarray(x, dtype=np.int64).reshape(-1) for x in lists]) \
        if lists else np.zeros(0, np.int64)
    return vals, off


# ---------------------------------------------------------------------------
# acquire.npz
# ---------------------------------------------------------------------------

ACQUIRE_CONFIGS = [(16, 4, 8, False, 0.0), (16, 4, 4, True, 0.0), (256, 102, 256, True, 0.0),
                   (256, 32, 128, True, 0.0), (16, 4, 8, True, 0.25)]


def make_acquire():
    out = {"configs": np.array([c[:4] for c in ACQUIRE_CONFIGS], dtype=np.int64),
           "invalid_p": np.array([c[4] for c in ACQUIRE_CONFIGS])}
    for ci, (E, S, R, warm, p_invalid) in enumerate(ACQUIRE_CONFIGS):
        rng = random.Random(0)
        vram, ram = make_tables(E, S, R, warm)
        ids_l, dig = [], []
        for _ in range(200):
            k = rng.randint(1, S)
            ids = [rng.randrange(E) for _ in range(k)]
            if p_invalid:
                ids = [-1 if rng.random() < p_invalid else x for x in ids]
            t = torch.tensor([ids], dtype=torch.int32)
            emap, slot, todo = vram.acquire(t)
            _, src, ssd = ram.acquire(t)
            ids_l.append(ids)
            dig.append([tstate(vram), digest(emap, slot, todo), tstate(ram), digest(src, ssd)])
        v, o = flat(ids_l)
        out[f"c{ci}_ids"], out[f"c{ci}_off"] = v, o
        out[f"c{ci}_digests"] = np.array(dig, dtype="S24")
    np.savez_compressed(os.path.join(HERE, "acquire.npz"), **out)


# ---------------------------------------------------------------------------
# zipf.npz (config 2)
# ---------------------------------------------------------------------------


def make_zipf():
    E, S, R = 256, 32, 256
    trace = synthetic.zipf_trace(4096, E, 8, 1.1, layer=0)
    vram, ram = make_tables(E, S, R, True)
    dig, vtodo, rtodo = [], [], []
    for i in range(trace.shape[0]):
        t = trace[i : i + 1]
        emap, slot, todo = vram.acquire(t)
        _, src, ssd = ram.acquire(t)
        dig.append([tstate(vram), digest(emap, slot, todo), tstate(ram), digest(src, ssd)])
        vtodo.append(todo.numpy().astype(np.int16))
        rtodo.append(ssd.numpy().astype(np.int16))
    np.savez_compressed(
        os.path.join(HERE, "zipf.npz"),
        trace_digest=np.frombuffer(digest(trace), dtype="S24"),
        trace_head=trace[:16].numpy(),
        digests=np.array(dig, dtype="S24"),
        vram_todo=np.stack(vtodo),
        ram_todo=np.stack(rtodo),
        final_vram_hits=np.array([int(vram.hits), int(vram.misses)]),
        final_ram_hits=np.array([int(ram.hits), int(ram.misses)]),
    )


# ---------------------------------------------------------------------------
# working.npz
# ---------------------------------------------------------------------------


def working_step(ram, vram, ids, W, ram_base, working_base):
    """experts.py:501-510 on CPU tensors; returns the logged topk (or None) and the plan."""
    E = ram.num_experts
    need = ram.need_mask(ids)
    cached_row = vram.slot_of[:E].clone()
    before = ram.slot_of[:E].clone()
    _topk_log.clear()
    torch.Tensor.topk = _logged_topk
    try:
        if ids.numel() <= ram.num_slots:
            ram.acquire(ids)
        else:
            ram.seed(vram, ids, need)
    finally:
        torch.Tensor.topk = _orig_topk
    top = _topk_log[0] if _topk_log else None
    plan = ram.plan_chunks(before, need, cached_row, W, ram_base, working_base)
    return top, need, plan


def make_working():
    out = {}
    # (a) the random mixed steps of test_table.py::test_plan_chunks_random_steps
    for W in (1, 3, 4):
        rng = random.Random(W)
        E, R, S, L, layer = 16, 6, 3, 2, 1
        ram_base, working_base = layer * R, L * R
        ram, vram = ExpertTable(E, R, CPU), ExpertTable(E, S, CPU)
        ids_l, kinds, dig, tops = [], [], [], []
        for _ in range(200):
            k = rng.randint(1, 2 * E)
            ids_py = [rng.randrange(E) for _ in range(k)]
            ids = torch.tensor([ids_py])
            if k <= S:
                _, _, todo = ram.acquire(ids)
                emap, slot, vtodo = vram.acquire(ids)
                kinds.append(0)
                dig.append([tstate(ram), tstate(vram), digest(todo, emap, slot, vtodo)])
                tops.append([])
            else:
                top, need, plan = working_step(ram, vram, ids, W, ram_base, working_base)
                kinds.append(1)
                dig.append([tstate(ram), tstate(vram), digest(need, *plan)])
                tops.append([] if top is None else top.tolist())
            ids_l.append(ids_py)
        v, o = flat(ids_l)
        tv, to = flat(tops)
        out[f"mix{W}_ids"], out[f"mix{W}_off"] = v, o
        out[f"mix{W}_kinds"] = np.array(kinds, dtype=np.int8)
        out[f"mix{W}_digests"] = np.array(dig, dtype="S24")
        out[f"mix{W}_top"], out[f"mix{W}_top_off"] = tv, to

    # (b) E=256 working steps: prefill (seed) with R=128 and R=256, batch-8 decode (acquire)
    cases = [
        ("prefill_r128", 32, 128, 3, synthetic.uniform_routing(2048, seed=3)),
        ("prefill_r256", 32, 256, 3, synthetic.uniform_routing(2048, seed=3)),
        ("batch8_r128", 32, 128, 5, synthetic.zipf_trace(72, layer=5)[64:72].reshape(1, -1)),
    ]
    E, W, L = 256, 64, 40
    for name, S, R, layer, ids in cases:
        vram, ram = make_tables(E, S, R, True)
        warmup = synthetic.zipf_trace(64, layer=layer)
        for i in range(64):
            vram.acquire(warmup[i : i + 1])
            ram.acquire(warmup[i : i + 1])
        for tname, t in (("vram", vram), ("ram", ram)):
            for key, val in full_state(t).items():
                out[f"{name}_pre_{tname}_{key}"] = val
        ram_base, working_base = layer * R, L * R
        top, need, plan = working_step(ram, vram, ids, W, ram_base, working_base)
        out[f"{name}_ids"] = ids.numpy().astype(np.int16)
        out[f"{name}_cfg"] = np.array([E, S, R, W, L, layer], dtype=np.int64)
        out[f"{name}_top"] = np.zeros(0, np.int64) if top is None else top.astype(np.int64)
        out[f"{name}_need"] = need.numpy()
        for key, val in zip(("dst_row", "src_row", "maps", "todo", "ssd", "late"), plan):
            out[f"{name}_{key}"] = val.numpy().astype(np.int32)
        for key, val in full_state(ram).items():
            out[f"{name}_post_ram_{key}"] = val

    # (c) the three scenario tests of test_table.py (E=16)
    def scenario(R, S, L, W, layer, ram_ids, vram_ids, ids, key):
        ram, vram = ExpertTable(16, R, CPU), ExpertTable(16, S, CPU)
        ram.acquire(torch.tensor(ram_ids)) if ram_ids is not None else None
        vram.acquire(torch.tensor(vram_ids)) if vram_ids is not None else None
        pre = {**{f"pre_ram_{k}": v for k, v in full_state(ram).items()},
               **{f"pre_vram_{k}": v for k, v in full_state(vram).items()}}
        top, need, plan = working_step(ram, vram, torch.tensor(ids), W, layer * R, L * R)
        out[f"{key}_cfg"] = np.array([16, S, R, W, L, layer], dtype=np.int64)
        out[f"{key}_ids"] = np.array(ids, dtype=np.int64)
        out[f"{key}_top"] = np.zeros(0, np.int64) if top is None else top.astype(np.int64)
        for k, v in pre.items():
            out[f"{key}_{k}"] = v
        for k, v in zip(("dst_row", "src_row", "maps", "todo", "ssd", "late"), plan):
            out[f"{key}_{k}"] = v.numpy().astype(np.int64)
        for k, v in full_state(ram).items():
            out[f"{key}_post_ram_{k}"] = v

    scenario(4, 2, 3, 2, 1, [[0, 1, 2, 3]], [[0, 9]], [[5, 6], [5, 6], [5, 0], [7, 1]], "sc_seed")
    scenario(4, 2, 2, 4, 0, [[0, 1, 2, 3]], [[2, 3]], [[2, 5], [3, 3]], "sc_acquire")
    scenario(4, 2, 1, 3, 0, None, None, np.arange(12).reshape(3, 4).tolist(), "sc_alternate")
    scenario(4, 2, 1, 3, 0, None, None, [[3, -1], [3, -1], [5, -1]], "sc_negative")
    np.savez_compressed(os.path.join(HERE, "working.npz"), **out)


# ---------------------------------------------------------------------------
# codec.npz
# ---------------------------------------------------------------------------

_EXP_P = [0.0] * 4 + [0.001, 0.002, 0.004, 0.008, 0.016, 0.032, 0.064, 0.125, 0.228, 0.315,
                      0.188, 0.015]


def rows(seed: int, n: int, p=_EXP_P) -> torch.Tensor:
    """The reference test_codec.py row generator (exponents drawn from p)."""
    g = torch.Generator().manual_seed(seed)
    exp = torch.multinomial(torch.tensor(p, dtype=torch.float64), n, replacement=True,
                            generator=g)
    sm = torch.randint(0, 256, (n,), dtype=torch.uint8, generator=g) & 0x87
    return sm | (exp.to(torch.uint8) << 3)


def used_bytes(rec: torch.Tensor, n: int, chunk: int) -> int:
    G = n // (chunk * 32)
    total = int(rec[4 * G : 4 * G + 4].view(torch.int32)[0])
    return 4 * (G + 1) + n // 2 + 4 * total


def make_codec():
    out = {}
    rng = random.Random(7)
    hists = [[2**k for k in range(16)], [1] * 16, [0] * 15 + [100], [5] * 8 + [0] * 8]
    hists += [[rng.randrange(0, 1 << rng.randrange(1, 20)) for _ in range(16)] for _ in range(40)]
    out["hists"] = np.array(hists, dtype=np.int64)
    out["lengths"] = np.array([ref_codec.code_lengths(h) for h in hists], dtype=np.int64)

    # test_codec.py distributions at CHUNK=64 (N = 2 groups) and at the production CHUNK=512
    for chunk in (64, 512):
        N = 2 * chunk * 32
        pitch = ref_codec.pitch_of(N, 1.25, 4096)
        raws = [rows(0, N), rows(1, N, [1.0] * 16), rows(2, N, [2.0**k for k in range(16)]),
                torch.full((N,), 13 << 3, dtype=torch.uint8)]
        for i, raw in enumerate(raws):
            rec, lut = ref_codec.encode(raw, pitch, chunk)
            out[f"c{chunk}_{i}_raw"] = raw.numpy()
            out[f"c{chunk}_{i}_rec"] = rec.numpy()
            out[f"c{chunk}_{i}_lut"] = lut.numpy()
            out[f"c{chunk}_{i}_used"] = np.array(used_bytes(rec, N, chunk))
    try:
        ref_codec.encode(rows(3, 4096), 4096 // 4, 64)
    except ValueError as e:
        out["over_pitch_msg"] = np.array(str(e))

    # config 1: 8 experts, pitch 0.89
    experts = synthetic.fp8_experts(8, seed=0)
    dig, luts, used, pitches = [], [], [], []
    for ex in experts:
        d_e, l_e, u_e = [], [], []
        for name in synthetic.SHAPES:
            q, scale = ex[name]
            raw = synthetic.row_bytes(q)
            pitch = ref_codec.pitch_of(raw.numel(), 0.89, 4096)
            rec, lut = ref_codec.encode(raw, pitch)
            d_e.append([digest(raw), digest(scale.view(torch.int32)), digest(rec)])
            l_e.append(lut.numpy())
            u_e.append(used_bytes(rec, raw.numel(), 512))
            if len(pitches) < 2:
                pitches.append(pitch)
        dig.append(d_e)
        luts.append(l_e)
        used.append(u_e)
    out["cfg1_digests"] = np.array(dig, dtype="S24")
    out["cfg1_luts"] = np.array(luts, dtype=np.uint8)
    out["cfg1_used"] = np.array(used, dtype=np.int64)
    out["cfg1_pitch"] = np.array(pitches, dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "codec.npz"), **out)


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for fn in (make_acquire, make_zipf, make_working, make_codec):
        fn()
        print(fn.__name__, "done", flush=True)
