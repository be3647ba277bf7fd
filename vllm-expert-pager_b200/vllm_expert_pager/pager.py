"""Per-layer expert paging: the decode path and the chunked working-slab path.

This is the paging half of ``ExpertPagerRoutedExperts`` in
monochromegane/vllm-expert-pager (src/vllm_expert_pager/experts.py), without
vLLM: ``experts.py`` of this package owns a ``LayerPager`` per MoE layer and
only adds the vLLM hooks around it, and the benchmark drives it directly.

* Decode (``topk_ids.numel() <= cache_slots``, experts.py:380-453): one
  ``xp_decode_step`` launch updates the VRAM and RAM tables, copies the
  RAM-resident misses (pinned host memory -> slab, or -> staging when
  compressed) while a CTA asks the host for the SSD misses and waits, then
  copies the rows the host read; one decode launch expands the staged rows when
  compressed.  (``fused=False`` runs the reference's sequence instead: acquire,
  gather + fetch, decode, gather, decode.)  The MoE then runs on the cache slab
  with ``expert_map``.
* Working (``numel() > cache_slots``, experts.py:455-577): the RAM table
  acquires or is seeded, ``plan_chunks`` lays the needed experts out in N
  chunks of W rows, and each chunk is copied into a working slab and run
  through the MoE, whose per-expert contributions are summed once at the end.
  Chunk k+1's copies run on a side stream into the other half of a 2W-row
  working slab while chunk k's MoE runs (the reference runs them one after
  another on one stream); events order each half's copy before its MoE and
  the MoE before the half is overwritten.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from vllm_expert_pager import codec
from vllm_expert_pager.acquire import AcquirePair
from vllm_expert_pager.gather import (
    as_rows,
    fetch_publish_rows,
    fetch_wait_rows,
    gather_rows,
)
from vllm_expert_pager.store import Store
from vllm_expert_pager.table import ExpertTable, WorkingPlan

# Expert weights paged through the slabs, in the gather's name order.
PARAMS = ("w13_weight", "w2_weight")


class WorkingSlab:
    """The working rows shared by every layer (experts.py:79-83,290-318).

    ``halves`` halves of W rows each (2 for the overlapped chunk loop): chunk k
    uses half k % halves.  Holds weights and scales in slot order, plus the
    staging for compressed prefill rows (W rows x pitch per half).
    """

    def __init__(self, rows: int, shapes: dict[str, tuple[tuple[int, ...], torch.dtype]],
                 store: Store, device: torch.device, halves: int = 2) -> None:
        self.rows, self.halves = rows, halves
        self.slab = {
            name: torch.empty((halves * rows, *shape), dtype=dtype, device=device)
            for name, (shape, dtype) in shapes.items()
        }
        self.staging = None
        if store.compress:
            self.staging = [
                torch.empty((halves * rows, store.pitch[n]), dtype=torch.uint8, device=device)
                for n in PARAMS
            ]

    def half(self, h: int) -> dict[str, torch.Tensor]:
        W = self.rows
        return {n: t[h * W : (h + 1) * W] for n, t in self.slab.items()}


@dataclass
class DecodeResult:
    slabs: dict[str, torch.Tensor]
    expert_map: torch.Tensor


class LayerPager:
    """Tables, slabs and paging launches of one MoE layer."""

    def __init__(self, store: Store, layer: int, cache_slots: int,
                 scales: dict[str, torch.Tensor], weight_shapes: dict[str, tuple],
                 working: WorkingSlab) -> None:
        self.store, self.layer = store, layer
        E, R, S = store.num_experts, store.ram_slots, cache_slots
        device = store.device
        self.num_experts, self.cache_slots = E, S
        self.vram = ExpertTable(E, S, device)
        self.ram = ExpertTable(E, R, device)
        # Warm start: expert e < R was written to RAM-tier slot e (experts.py:256-259).
        self.ram.slot_of[:R] = self.ram.experts[:R]
        self.ram.expert_in[:R] = self.ram.experts[:R]
        self.acquire = AcquirePair(self.vram, self.ram)
        self.expert_map = self.acquire.expert_map
        self.planner = WorkingPlan(E, working.rows, R, S, device)
        self.scale_names = list(scales)
        self.cache_slab = {
            name: torch.empty((S, *shape), dtype=dtype, device=device)
            for name, (shape, dtype) in weight_shapes.items()
        }
        for name, s in scales.items():
            self.cache_slab[name] = torch.empty((S, *s.shape[1:]), dtype=s.dtype, device=device)
        self.working = working
        order = list(PARAMS) + self.scale_names
        self.cache_rows = [as_rows(self.cache_slab[n]) for n in order]
        self.scale_rows = [as_rows(scales[n]) for n in self.scale_names]
        self.cache_bytes = [self.cache_slab[n].view(torch.uint8).reshape(S, -1) for n in PARAMS]
        self.working_rows = [[as_rows(working.half(h)[n]) for n in order]
                             for h in range(working.halves)]
        self.working_bytes = [[working.half(h)[n].view(torch.uint8).reshape(working.rows, -1)
                               for n in PARAMS] for h in range(working.halves)]
        # In decode the working slab is idle, so its head stages compressed rows
        # (S rows x pitch; experts.py:338-353).
        self.decode_staging = None
        if store.compress:
            flat = {n: working.slab[n].view(torch.uint8).reshape(-1) for n in PARAMS}
            need = {n: S * store.pitch[n] for n in PARAMS}
            if any(need[n] > flat[n].numel() for n in PARAMS):
                raise ValueError(
                    "VLLM_EXPERT_PAGER_WORKING_ROWS cannot hold the decode staging of "
                    f"{S} compressed rows"
                )
            self.decode_staging = [flat[n][: need[n]].view(S, store.pitch[n]) for n in PARAMS]
        self.ram_view = [store.view[n] for n in PARAMS]
        self.side = torch.cuda.Stream(device=device)
        # The working path's decodes: beside the copies, so that chunk k's decode
        # does not hold back chunk k+1's copy over the host link.
        self.expand_side = torch.cuda.Stream(device=device)
        # Flags of the fused decode step (zero between launches; word 3 counts
        # waits that gave up).
        self.step_scratch = torch.zeros((4,), dtype=torch.int32, device=device)
        # Pinned host copy of that count, stored by the kernel when a wait gives
        # up; the host reads it without synchronising (graph replays included).
        self.step_errors_host = torch.zeros((1,), dtype=torch.int32, pin_memory=True)
        self._step_errors_np = self.step_errors_host.numpy()

    # ---- decode (experts.py:380-453) ----

    def decode(self, topk_ids: torch.Tensor, gather_events: list | None = None,
               fused: bool = True, map_out: torch.Tensor | None = None,
               decode_events: list | None = None) -> DecodeResult:
        """Page in this step's experts; returns the cache slab and expert_map.

        ``fused`` (default): one ``xp_decode_step`` launch does the table
        updates, the RAM copies, the SSD request and wait and the copies of the
        rows read (plus one decode launch when compressed).  ``fused=False``
        runs the reference's launch sequence (acquire, gather+fetch, decode,
        gather, decode).  ``gather_events``: if a list, a (start, end) pair of
        timing events around the copying launch is appended; ``decode_events``
        likewise around the decode launch of a compressed fused step, as
        (start, end, rows) with rows a device scalar: the rows it expands.

        Host-driven callers (fused path): ``topk_ids`` may be a pinned host
        tensor (int32 or int64, contiguous), which the kernel reads through the
        host link, and ``map_out`` a pinned host int32 ``[E]`` tensor that the
        kernel fills with this step's expert_map -- no copy-engine transfer per
        step.  Neither buffer may be rewritten by the host before the step has
        run on the GPU.
        """
        if fused:
            return self._decode_fused(topk_ids, gather_events, map_out, decode_events)
        if map_out is not None:
            raise ValueError("map_out needs the fused decode step")
        store, layer = self.store, self.layer
        todo, ssd_todo = self.acquire(topk_ids)
        dst_row, src_row = self.acquire.vram_slot, self.acquire.ram_slot
        cached_row = self.vram.no_cache
        base = layer * store.ram_slots
        lut = store.layer_lut(layer)
        staging = self.decode_staging
        rows = (
            self.ram_view, self.cache_rows[:2], self.cache_rows[:2],
            [t.view(torch.int32) for t in staging] if staging is not None else None,
            self.scale_rows, self.cache_rows[2:],
        )  # fmt: skip
        if gather_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        gather_rows(todo, dst_row, cached_row, src_row, base, *rows,
                    fetch=(ssd_todo, layer, store))
        if gather_events is not None:
            ev[1].record()
            gather_events.append(ev)
        if store.compress:
            codec.decode_rows(todo, dst_row, cached_row, staging, self.cache_bytes, lut,
                              skip=ssd_todo)
        gather_rows(ssd_todo, dst_row, cached_row, src_row, base, *rows)
        if store.compress:
            codec.decode_rows(ssd_todo, dst_row, cached_row, staging, self.cache_bytes, lut)
        return DecodeResult(self.cache_slab, self.expert_map)

    def _decode_fused(self, topk_ids, gather_events=None, map_out=None,
                      decode_events=None) -> DecodeResult:
        from vllm_expert_pager import gather as gather_mod
        from vllm_expert_pager import native
        from vllm_expert_pager.table import _ids

        store, layer = self.store, self.layer
        if topk_ids.device.type == "cpu":
            # Pinned host ids are read by the kernel through the host link (UVA).
            ids = topk_ids.reshape(-1)
            if not (ids.is_pinned() and ids.is_contiguous()
                    and ids.dtype in (torch.int32, torch.int64)):
                raise ValueError("host topk_ids must be pinned, contiguous int32/int64")
            nb = ids.element_size()
        else:
            native.require_cuda(topk_ids)
            ids, nb = _ids(topk_ids)
        if map_out is not None and not (
                map_out.device.type == "cpu" and map_out.is_pinned() and map_out.is_contiguous()
                and map_out.dtype == torch.int32 and map_out.numel() == self.num_experts):
            raise ValueError(f"map_out must be a pinned host int32 tensor of {self.num_experts}")
        K = ids.numel()
        pair, a, b = self.acquire, self.vram, self.ram
        staging = self.decode_staging
        st = [t.view(torch.int32) for t in staging] if staging is not None else [None, None]
        cw, sw = self.cache_rows[:2], self.cache_rows[2:]
        fetch = store.path is not None
        if gather_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        native.check(
            native.lib().xp_decode_step(
                ids.data_ptr(), nb, K, self.num_experts,
                *a._table_args(), pair.expert_map.data_ptr(), native.ptr(map_out),
                pair.vram_slot.data_ptr(),
                pair._vram_todo.data_ptr(),
                *b._table_args(), pair.ram_slot.data_ptr(), pair._ram_todo.data_ptr(),
                a.no_cache.data_ptr(), layer * store.ram_slots,
                self.ram_view[0].data_ptr(), cw[0].data_ptr(), native.ptr(st[0]),
                cw[0].shape[1], self.ram_view[0].shape[1],
                self.ram_view[1].data_ptr(), cw[1].data_ptr(), native.ptr(st[1]),
                cw[1].shape[1], self.ram_view[1].shape[1],
                self.scale_rows[0].data_ptr(), sw[0].data_ptr(), sw[0].shape[1],
                self.scale_rows[1].data_ptr(), sw[1].data_ptr(), sw[1].shape[1],
                int(store.compress), codec.CHUNK if store.compress else 0,
                gather_mod.GATHER_CTAS, layer,
                store.seq.data_ptr() if fetch else None, store.req_dev if fetch else None,
                store.done_dev if fetch else None, store.block, store.ring, store.retry_ns,
                store.giveup, self.step_scratch.data_ptr(), self.step_errors_host.data_ptr(),
                native.stream_of(store.device),
            ),
            "decode_step",
        )  # fmt: skip
        if gather_events is not None:
            ev[1].record()
            gather_events.append(ev)
        if store.compress:
            if decode_events is not None:
                rows = (pair._vram_todo[:K] >= 0).sum()  # every VRAM miss is expanded
                dv = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                dv[0].record()
            codec.decode_rows(pair._vram_todo[:K], pair.vram_slot, a.no_cache, staging,
                              self.cache_bytes, store.layer_lut(layer))
            if decode_events is not None:
                dv[1].record()
                decode_events.append((*dv, rows))
        return DecodeResult(self.cache_slab, self.expert_map)

    def step_errors(self) -> int:
        """Waits of the fused decode step that gave up so far (a step with one holds
        stale rows).  Reads the pinned host copy the kernel keeps: no device
        synchronisation, so it is safe between graph replays and during capture,
        and it may miss a give-up of a step still running on the GPU."""
        return int(self._step_errors_np[0])

    # ---- working path (experts.py:455-577) ----

    def plan(self, topk_ids: torch.Tensor):
        """Update the RAM table and lay the step's experts out in chunks (experts.py:501-510):
        need_mask, the slot_of copy, acquire or seed, and plan_chunks in one launch."""
        store = self.store
        _, cached_row, plan = self.planner(self.ram, self.vram, topk_ids,
                                           self.layer * store.ram_slots, store.working_base)
        return cached_row, plan

    def working_chunks(self, topk_ids: torch.Tensor, run_chunk, overlap: bool = True,
                       decode_events: list | None = None, copy_events: list | None = None):
        """Run the working path; ``run_chunk(k, n, slabs, expert_map)`` runs chunk k's MoE.

        With ``overlap`` chunk k+1's copies go to the other half of the working
        slab on a side stream while chunk k's MoE runs on the current stream.
        ``decode_events`` / ``copy_events``: if lists, (start, end, rows)
        timing events around every decode / gather launch (on the copy stream)
        are appended, rows a device scalar: the rows expanded (decode) or read
        from the RAM tier (gather).  Returns the last ``run_chunk`` result.
        """
        store, layer = self.store, self.layer
        W = self.working.rows
        cached_row, (dst_row, src_row, maps, todo, ssd, late) = self.plan(topk_ids)
        N = maps.shape[0]
        lut = store.layer_lut(layer)
        tickets = store.ticket_chunk
        halves = self.working.halves if overlap else 1
        staging = self.working.staging
        main = torch.cuda.current_stream(store.device)
        side = self.side if overlap else main
        dec = self.expand_side if overlap else main

        def rows(h):
            wr = self.working_rows[h]
            stg = None
            if staging is not None:
                stg = [t[h * W : (h + 1) * W].view(torch.int32) for t in staging]
            return (self.ram_view, self.cache_rows[:2], wr[:2], stg, self.scale_rows, wr[2:])

        def timing(events):
            if events is None:
                return None
            return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def rows_read(part):
            if decode_events is None and copy_events is None:
                return None
            # Entries not in the cache slab: read from the RAM tier, and expanded.
            return ((part >= 0) & (cached_row[part.clamp(min=0)] < 0)).sum()

        def copy(part, h):
            ev = timing(copy_events)
            if ev:
                ev[0].record()
            gather_rows(part, dst_row, cached_row, src_row, 0, *rows(h),
                        chunk=codec.CHUNK if store.compress else 0)
            if ev:
                ev[1].record()
                copy_events.append((*ev, rows_read(part)))

        def expand(part, h):
            stg = [t[h * W : (h + 1) * W] for t in staging]
            ev = timing(decode_events)
            if ev:
                ev[0].record()
            codec.decode_rows(part, dst_row, cached_row, stg, self.working_bytes[h], lut)
            if ev:
                ev[1].record()
                decode_events.append((*ev, rows_read(part)))

        def chunk(t, k):
            return t[k * W : (k + 1) * W]

        def ticket(k):
            return tickets[k % 2 : k % 2 + 1]

        copied = [torch.cuda.Event() for _ in range(N)]
        consumed = [torch.cuda.Event() for _ in range(N)]
        # Compressed rows: chunk k's RAM rows are expanded on the decode stream while
        # the copy stream goes on with the SSD wait, the SSD rows and chunk k+1's
        # copies (into the other staging half).  A half's staging and slab rows are
        # reused two chunks later, after the MoE that read them (consumed), which
        # itself waited for their decode (copied).
        early = [torch.cuda.Event() for _ in range(N)]
        gathered = [torch.cuda.Event() for _ in range(N)]
        out = None
        side.wait_stream(main)  # the plan is on the main stream
        with torch.cuda.stream(side):
            fetch_publish_rows(chunk(ssd, 0), src_row, 0, layer, store, ticket(0))
        for k in range(N):
            h = k % halves
            with torch.cuda.stream(side):
                if k >= halves:
                    side.wait_event(consumed[k - halves])  # the half's previous MoE is done
                copy(chunk(todo, k), h)
                early[k].record(side)
                if k + 1 < N:
                    fetch_publish_rows(chunk(ssd, k + 1), src_row, 0, layer, store, ticket(k + 1))
                fetch_wait_rows(chunk(ssd, k), store, ticket(k))
                copy(chunk(late, k), h)
                gathered[k].record(side)
            if store.compress:
                with torch.cuda.stream(dec):
                    dec.wait_event(early[k])
                    expand(chunk(todo, k), h)
                    dec.wait_event(gathered[k])
                    expand(chunk(late, k), h)
                    copied[k].record(dec)
            else:
                copied[k] = gathered[k]
            main.wait_event(copied[k])
            self.expert_map.copy_(maps[k])
            out = run_chunk(k, N, self.working.half(h), self.expert_map)
            consumed[k].record(main)
        return out
