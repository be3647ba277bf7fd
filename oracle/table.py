"""CPU oracle for the expert slot table.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline``
leg and its ``--impl reference`` arm) may import this module, and only as the
checker or as the timed CPU baseline.  The product path never calls it.

This is a numpy restatement of ``ExpertTable`` from monochromegane/vllm-expert-pager
(``src/vllm_expert_pager/table.py``).  Each method cites the lines it follows.
Differences from the reference, all deliberate and stated here:

* The arrays carry no trailing sink element; the reference's sink (index E or
  S) only absorbs masked scatters and is never read (table.py:22-26).
* Expert ids ``>= num_experts`` are ignored like negative ids.  The reference's
  torch version raises on ids ``> E`` and its Triton version ignores them.
* ``seed`` picks its top-(R-S) experts by count with ties broken by the lower
  expert id.  The reference calls ``torch.topk`` (table.py:161), whose tie order
  is implementation-defined (it differs between CPU and CUDA).  ``seed`` takes
  an optional ``top`` override so a test can replay the reference's own choice.

Parity pin: tests/test_oracle_table.py checks every method against digests of
the reference's own outputs, recorded by tests/golden/make_golden.py.
"""

from __future__ import annotations

import numpy as np

# Added to the victim key of slots whose expert is used this step
# (table.py:14-16).
PROTECT = 1 << 40

I64 = np.int64


def _ids(ids, num_experts: int) -> np.ndarray:
    """Flattened int64 ids; invalid ids (negative or >= E) become -1 (table.py:58-61)."""
    a = np.asarray(ids, dtype=I64).reshape(-1)
    return np.where((a >= 0) & (a < num_experts), a, -1)


def top_experts(counts: np.ndarray, k: int) -> np.ndarray:
    """The k experts with the highest counts, ties broken by the lower id."""
    order = np.argsort(-counts, kind="stable")
    return order[:k].astype(I64)


class OracleTable:
    """Expert -> slot LRU table for one layer (table.py:19-54)."""

    def __init__(self, num_experts: int, num_slots: int) -> None:
        if num_slots < 1:
            raise ValueError(f"num_slots must be >= 1, got {num_slots}")
        self.num_experts, self.num_slots = num_experts, num_slots
        self.slot_of = np.full(num_experts, -1, dtype=I64)
        self.expert_in = np.full(num_slots, -1, dtype=I64)
        self.last_used = np.zeros(num_slots, dtype=I64)
        self.step = 1
        self.hits = 0
        self.misses = 0

    def warm(self, count: int) -> None:
        """Expert e < count sits in slot e (the RAM warm start, experts.py:256-259)."""
        r = np.arange(count, dtype=I64)
        self.slot_of[:count] = r
        self.expert_in[:count] = r

    def state(self) -> list[np.ndarray]:
        """``[slot_of, expert_in, last_used, step, hits, misses]`` as int64 arrays."""
        return [
            self.slot_of.copy(),
            self.expert_in.copy(),
            self.last_used.copy(),
            np.array([self.step], dtype=I64),
            np.array([self.hits], dtype=I64),
            np.array([self.misses], dtype=I64),
        ]

    def copy(self) -> "OracleTable":
        t = OracleTable(self.num_experts, self.num_slots)
        t.slot_of, t.expert_in = self.slot_of.copy(), self.expert_in.copy()
        t.last_used = self.last_used.copy()
        t.step, t.hits, t.misses = self.step, self.hits, self.misses
        return t

    # ---- shared (table.py:63-71) ----

    def need_mask(self, ids) -> np.ndarray:
        need = np.zeros(self.num_experts, dtype=bool)
        a = _ids(ids, self.num_experts)
        need[a[a >= 0]] = True
        return need

    # ---- cache path (table.py:75-128) ----

    def acquire(self, ids):
        """Returns ``(expert_map, slot, todo)`` like table.py:75-128.

        ``slot[e]`` is the table's slot of expert e after the update (-1 if not
        cached): the reference evaluates ``torch.where(miss, victim, current)``
        with ``current`` a view of ``slot_of`` taken before the scatters, so it
        reads the updated values (table.py:95,118).
        """
        E, S = self.num_experts, self.num_slots
        K = int(np.asarray(ids).size)
        need = self.need_mask(ids)
        current = self.slot_of.copy()
        hit = need & (current >= 0)
        miss = need & (current < 0)

        occupant = self.expert_in
        slot_used = (occupant >= 0) & hit[np.clip(occupant, 0, None)]
        key = self.last_used + slot_used.astype(I64) * PROTECT
        order = np.argsort(key, kind="stable")
        rank = np.cumsum(miss.astype(I64)) - 1
        victim = order[np.clip(rank, 0, S - 1)].astype(I64)

        evicted = self.expert_in[victim]
        clear = miss & (evicted >= 0)
        self.slot_of[evicted[clear]] = -1
        experts = np.nonzero(miss)[0].astype(I64)
        self.slot_of[experts] = victim[miss]
        self.expert_in[victim[miss]] = experts

        slot = self.slot_of.copy()
        self.last_used[slot[need]] = self.step
        self.step += 1
        self.hits += int(hit.sum())
        self.misses += int(miss.sum())

        expert_map = np.where(need, slot, -1).astype(I64)
        todo = np.full(K, -1, dtype=I64)
        todo[rank[miss]] = experts
        return expert_map, slot, todo

    # ---- working-buffer path (table.py:132-247) ----

    def pack(self, mask: np.ndarray) -> np.ndarray:
        """Ids set in ``mask`` packed from the front, -1 padded to E (table.py:132-138)."""
        out = np.full(self.num_experts, -1, dtype=I64)
        idx = np.nonzero(mask)[0]
        out[: idx.size] = idx
        return out

    def seed(self, vram: "OracleTable", ids, need: np.ndarray, top=None) -> np.ndarray:
        """Seed the RAM tier from a prefill's routing (table.py:140-171).

        Returns the top list used.  ``top`` overrides the choice of the
        R - S most referenced experts (to replay the reference's topk order).
        """
        E, R, S = self.num_experts, self.num_slots, vram.num_slots
        hits, misses = self.hits, self.misses
        a = _ids(ids, E)
        counts = np.bincount(a[a >= 0], minlength=E).astype(I64)
        if top is None:
            top = top_experts(counts, max(R - S, 1))
        top = np.asarray(top, dtype=I64)
        top = np.where(counts[top] > 0, top, top[0])
        if R > S:
            self.acquire(top)
        v = vram.expert_in[:S]
        vc = np.clip(v, 0, None)
        ok = (v >= 0) & ((self.slot_of[vc] >= 0) | need[vc])
        self.acquire(np.where(ok, v, top[0]))
        self.hits, self.misses = hits, misses
        return top

    def plan_chunks(self, before, need, cached_row, rows: int, ram_base: int,
                    working_base: int):
        """Chunk layout of a working-buffer step (table.py:173-247).

        Returns ``(dst_row, src_row, maps, todo, ssd, late)``; numpy's floor
        division and modulo match torch's on negative values.
        """
        E, W = self.num_experts, rows
        N = -(-E // W) + 1
        before = np.asarray(before, dtype=I64)
        cached_row = np.asarray(cached_row, dtype=I64)
        after = self.slot_of
        old_ok = (before >= 0) & ((after < 0) | (after == before))
        ssd = ~old_ok & (need | (before >= 0))
        first = need & ~ssd
        a = np.cumsum(first.astype(I64))
        b = np.cumsum(ssd.astype(I64))
        boundary = (a[-1] + W - 1) // W * W
        pos = np.where(first, a - 1, boundary + b - 1)
        dst_row = pos % W
        shared = working_base + (pos // W % 2) * W + dst_row
        src_row = np.where(
            old_ok, before + ram_base, np.where(after >= 0, after + ram_base, shared)
        )
        chunk = np.where(need, pos // W, -1)
        maps = np.where(chunk[None, :] == np.arange(N)[:, None], dst_row[None, :], -1)

        def listing(mask):
            out = np.full(N * W, -1, dtype=I64)
            out[pos[mask]] = np.nonzero(mask)[0]
            return out

        return (
            dst_row.astype(I64),
            src_row.astype(I64),
            maps.astype(I64),
            listing(need & (~ssd | (cached_row >= 0))),
            listing(ssd),
            listing(need & ssd & (cached_row < 0)),
        )


def working_step(ram: OracleTable, vram: OracleTable, ids, rows: int, ram_base: int,
                 working_base: int, top=None):
    """The planning part of one working-buffer step (experts.py:501-510).

    Returns ``(need, before, cached_row, plan)`` where ``plan`` is the tuple of
    ``plan_chunks``.
    """
    E = ram.num_experts
    need = ram.need_mask(ids)
    cached_row = vram.slot_of[:E].copy()
    before = ram.slot_of.copy()
    if int(np.asarray(ids).size) <= ram.num_slots:
        ram.acquire(ids)
    else:
        ram.seed(vram, ids, need, top=top)
    plan = ram.plan_chunks(before, need, cached_row, rows, ram_base, working_base)
    return need, before, cached_row, plan
