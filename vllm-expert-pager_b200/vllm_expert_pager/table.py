"""Expert-to-slot table kept in device memory, updated by CUDA kernels.

Mirrors ``ExpertTable`` of monochromegane/vllm-expert-pager
(src/vllm_expert_pager/table.py): the same attributes (``slot_of``,
``expert_in``, ``last_used``, ``step``, ``hits``, ``misses``, ``experts``,
``no_cache``), the same trailing sink element on each array, and the same
methods with the same results.  Every method is a single kernel launch from
``libxpager.so`` (table.cu) that reads and writes device memory only, so all of
them run under CUDA graphs and the host never reads a value.

Differences: the tables live on a CUDA device only (the reference's torch ops
also ran on CPU tensors; the CPU restatement used by the tests is in oracle/),
and ``seed`` breaks ties among equally referenced experts by the lower id (the
reference's ``torch.topk`` tie order is implementation-defined).  ``step``,
``hits`` and ``misses`` are 0-dim views of one ``counters`` int64[3] tensor.
"""

from __future__ import annotations

import torch

from vllm_expert_pager import native

# Added to the victim key of slots used in this step (table.py:14-16).
_PROTECT = 1 << 40


def _ids(topk_ids: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Flat contiguous int32/int64 ids and their element size."""
    ids = topk_ids.reshape(-1)
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int64)
    if not ids.is_contiguous():
        ids = ids.contiguous()
    return ids, ids.element_size()


class ExpertTable:
    """Expert -> slot table for one layer. Replacement is LRU (table.py:19-54)."""

    def __init__(self, num_experts: int, num_slots: int, device: torch.device) -> None:
        if num_slots < 1:
            raise ValueError(f"num_slots must be >= 1, got {num_slots}")
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("vllm-expert-pager: ExpertTable lives on a CUDA device")
        self.num_experts = num_experts
        self.num_slots = num_slots
        self.device = device
        i64 = {"dtype": torch.int64, "device": device}
        self.slot_of = torch.full((num_experts + 1,), -1, **i64)
        self.expert_in = torch.full((num_slots + 1,), -1, **i64)
        self.last_used = torch.zeros((num_slots + 1,), **i64)
        self.counters = torch.zeros((3,), **i64)
        self.counters[0] = 1
        self.step, self.hits, self.misses = self.counters[0], self.counters[1], self.counters[2]
        self.experts = torch.arange(num_experts, **i64)
        self.no_cache = torch.full((num_experts,), -1, **i64)

    def _table_args(self) -> list:
        return [self.slot_of.data_ptr(), self.expert_in.data_ptr(), self.last_used.data_ptr(),
                self.counters.data_ptr(), self.num_slots]

    # ---- shared ----

    def need_mask(self, topk_ids: torch.Tensor) -> torch.Tensor:
        """The experts needed in this step as a bool mask (table.py:63-71)."""
        native.require_cuda(topk_ids)
        ids, nb = _ids(topk_ids)
        need = torch.empty((self.num_experts,), dtype=torch.uint8, device=self.device)
        native.check(
            native.lib().xp_need_mask(ids.data_ptr(), nb, ids.numel(), self.num_experts,
                                      need.data_ptr(), native.stream_of(self.device)),
            "need_mask",
        )
        return need.view(torch.bool)

    # ---- cache path ----

    def acquire(self, topk_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Assign a slot to every needed expert and update the table (table.py:75-128).

        Requires ``topk_ids.numel() <= num_slots``.  Returns ``(expert_map,
        slot, todo)``: int64 ``[E]`` slot of each needed expert (-1 otherwise),
        int64 ``[E]`` every expert's slot after the update, and int64 ``[K]``
        the missed experts in ascending order, -1 padded.
        """
        native.require_cuda(topk_ids)
        ids, nb = _ids(topk_ids)
        K, E = ids.numel(), self.num_experts
        i64 = {"dtype": torch.int64, "device": self.device}
        expert_map = torch.empty((E,), **i64)
        slot = torch.empty((E,), **i64)
        todo = torch.empty((K,), **i64)
        native.check(
            native.lib().xp_acquire(ids.data_ptr(), nb, K, E, *self._table_args(),
                                    expert_map.data_ptr(), slot.data_ptr(),
                                    todo.data_ptr() if K else None,
                                    native.stream_of(self.device)),
            "acquire",
        )
        return expert_map, slot, todo

    # ---- working-buffer path ----

    def pack(self, mask: torch.Tensor) -> torch.Tensor:
        """The experts set in ``mask``, packed from the front and -1 padded to E (table.py:132-138)."""
        E = self.num_experts
        rank = torch.cumsum(mask.to(torch.int64), 0) - 1
        out = torch.full((E + 1,), -1, dtype=torch.int64, device=self.device)
        out.index_put_((torch.where(mask, rank, E),), self.experts)
        return out[:E]

    def seed(self, vram: "ExpertTable", topk_ids: torch.Tensor, need: torch.Tensor,
             top: torch.Tensor | None = None) -> torch.Tensor:
        """Update this (RAM-tier) table from a prefill's routing (table.py:140-171).

        Acquires the R - S most referenced experts of ``topk_ids`` (ties: lower
        id first), then the VRAM tier's experts that are in this table or in
        ``need``; hits and misses are not counted.  ``top`` (int64
        ``[max(R-S,1)]``) replays a given choice instead.  Returns the list used.
        """
        native.require_cuda(topk_ids, need)
        ids, nb = _ids(topk_ids)
        R, S = self.num_slots, vram.num_slots
        ntop = max(R - S, 1)
        top_out = torch.empty((ntop,), dtype=torch.int64, device=self.device)
        need_u8 = need.to(torch.uint8) if need.dtype != torch.uint8 else need
        if not need_u8.is_contiguous():
            need_u8 = need_u8.contiguous()
        if top is not None:
            top = top.to(device=self.device, dtype=torch.int64).contiguous()
            if top.numel() != ntop:
                raise ValueError(f"top must have {ntop} entries, got {top.numel()}")
        native.check(
            native.lib().xp_seed(ids.data_ptr(), nb, ids.numel(), self.num_experts,
                                 *self._table_args(), vram.expert_in.data_ptr(), S,
                                 need_u8.data_ptr(), native.ptr(top), top_out.data_ptr(),
                                 native.stream_of(self.device)),
            "seed",
        )
        return top_out

    def plan_chunks(self, before: torch.Tensor, need: torch.Tensor, cached_row: torch.Tensor,
                    rows: int, ram_base: int, working_base: int) -> tuple[torch.Tensor, ...]:
        """Chunk layout of a working-buffer step after the table update (table.py:173-247).

        Returns ``(dst_row, src_row, maps, todo, ssd, late)`` with N =
        ceil(E / rows) + 1 chunks: ``maps`` is int64 ``[N, E]``, the lists int64
        ``[N * rows]``.
        """
        native.require_cuda(before, need, cached_row)
        E, W = self.num_experts, rows
        N = -(-E // W) + 1
        i64 = {"dtype": torch.int64, "device": self.device}
        before = before[:E].contiguous()
        cached_row = cached_row[:E].contiguous()
        need_u8 = (need.to(torch.uint8) if need.dtype != torch.uint8 else need).contiguous()
        dst_row, src_row = torch.empty((E,), **i64), torch.empty((E,), **i64)
        maps = torch.empty((N, E), **i64)
        todo, ssd, late = (torch.empty((N * W,), **i64) for _ in range(3))
        native.check(
            native.lib().xp_plan_chunks(E, self.slot_of.data_ptr(), before.data_ptr(),
                                        need_u8.data_ptr(), cached_row.data_ptr(), W, ram_base,
                                        working_base, dst_row.data_ptr(), src_row.data_ptr(),
                                        maps.data_ptr(), todo.data_ptr(), ssd.data_ptr(),
                                        late.data_ptr(), native.stream_of(self.device)),
            "plan_chunks",
        )
        return dst_row, src_row, maps, todo, ssd, late


class WorkingPlan:
    """The planning of a working-path step in one launch (xp_plan_working).

    Replaces the sequence ``need_mask`` -> ``slot_of[:E].clone()`` -> ``acquire``
    (K <= R) or ``seed`` -> ``plan_chunks`` that _expert_pager_forward_working
    issues as separate operations (experts.py:500-511); the results are the
    same.  The outputs live in buffers allocated here once, at fixed addresses
    (graph-safe); each call overwrites them.
    """

    def __init__(self, num_experts: int, rows: int, ram_slots: int, vram_slots: int,
                 device: torch.device) -> None:
        E, W = num_experts, rows
        self.num_experts, self.rows, self.device = E, W, torch.device(device)
        N = -(-E // W) + 1
        i64 = {"dtype": torch.int64, "device": self.device}
        self.need = torch.zeros((E,), dtype=torch.uint8, device=self.device)
        self.before = torch.empty((E,), **i64)
        self.dst_row, self.src_row = torch.empty((E,), **i64), torch.empty((E,), **i64)
        self.maps = torch.empty((N, E), **i64)
        self.todo, self.ssd, self.late = (torch.empty((N * W,), **i64) for _ in range(3))
        self.top = torch.empty((max(ram_slots - vram_slots, 1),), **i64)

    def __call__(self, ram: ExpertTable, vram: ExpertTable, topk_ids: torch.Tensor,
                 ram_base: int, working_base: int, top: torch.Tensor | None = None):
        """Plan one step on the RAM table ``ram``; returns ``(need, cached_row, plan)`` with
        ``plan = (dst_row, src_row, maps, todo, ssd, late)`` as ``plan_chunks`` returns it."""
        native.require_cuda(topk_ids)
        E = self.num_experts
        if ram.num_experts != E or vram.num_experts != E:
            raise ValueError("tables and plan must have the same number of experts")
        ids, nb = _ids(topk_ids)
        ntop = max(ram.num_slots - vram.num_slots, 1)
        if top is not None:
            top = top.to(device=self.device, dtype=torch.int64).contiguous()
            if top.numel() != ntop:
                raise ValueError(f"top must have {ntop} entries, got {top.numel()}")
        cached_row = vram.slot_of[:E]
        native.check(
            native.lib().xp_plan_working(
                ids.data_ptr(), nb, ids.numel(), E, *ram._table_args(),
                vram.expert_in.data_ptr(), cached_row.data_ptr(), vram.num_slots, self.rows,
                ram_base, working_base, native.ptr(top), self.top.data_ptr(),
                self.need.data_ptr(), self.before.data_ptr(), self.dst_row.data_ptr(),
                self.src_row.data_ptr(), self.maps.data_ptr(), self.todo.data_ptr(),
                self.ssd.data_ptr(), self.late.data_ptr(), native.stream_of(self.device)),
            "plan_working",
        )
        plan = (self.dst_row, self.src_row, self.maps, self.todo, self.ssd, self.late)
        return self.need.view(torch.bool), cached_row, plan
