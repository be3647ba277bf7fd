"""Update the VRAM and RAM slot tables in one launch (the decode path).

Mirrors ``AcquirePair`` of monochromegane/vllm-expert-pager
(src/vllm_expert_pager/acquire.py:144-185): fixed-address outputs
``expert_map`` (int32 ``[E]``), ``vram_slot``/``ram_slot`` (int64 ``[E]``) and
the miss lists, written by one launch of ``xp_acquire_pair`` (table.cu: one CTA
per table) instead of a Triton kernel.
"""

from __future__ import annotations

import torch

from vllm_expert_pager import native
from vllm_expert_pager.table import ExpertTable, _ids

# Largest table the kernel accepts (include/xpager.h XP_MAX_SLOTS).
MAX_SLOTS = 2048


class AcquirePair:
    """Update the VRAM and RAM tables in one launch; outputs at fixed addresses."""

    def __init__(self, vram: ExpertTable, ram: ExpertTable) -> None:
        if vram.num_experts != ram.num_experts:
            raise ValueError("both tables must have the same number of experts")
        if max(vram.num_slots, ram.num_slots) > MAX_SLOTS:
            raise ValueError(f"at most {MAX_SLOTS} slots per table")
        E, device = vram.num_experts, vram.device
        self.vram, self.ram = vram, ram
        i64 = {"dtype": torch.int64, "device": device}
        # Values of unneeded experts are never read.
        self.expert_map = torch.full((E,), -1, dtype=torch.int32, device=device)
        self.vram_slot = torch.zeros((E,), **i64)
        self.ram_slot = torch.zeros((E,), **i64)
        self._vram_todo = torch.full((vram.num_slots,), -1, **i64)
        self._ram_todo = torch.full((ram.num_slots,), -1, **i64)

    def __call__(self, topk_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Update both tables and return ``(vram_todo, ram_todo)`` of length K.

        ``expert_map``, ``vram_slot`` and ``ram_slot`` are written to the
        attribute buffers.  Requires ``topk_ids.numel() <= vram.num_slots``.
        """
        native.require_cuda(topk_ids)
        ids, nb = _ids(topk_ids)
        K = ids.numel()
        a, b = self.vram, self.ram
        native.check(
            native.lib().xp_acquire_pair(
                ids.data_ptr(), nb, K, a.num_experts,
                *a._table_args(), self.expert_map.data_ptr(), self.vram_slot.data_ptr(),
                self._vram_todo.data_ptr(),
                *b._table_args(), self.ram_slot.data_ptr(), self._ram_todo.data_ptr(),
                native.stream_of(a.device),
            ),
            "acquire_pair",
        )  # fmt: skip
        return self._vram_todo[:K], self._ram_todo[:K]
