"""Copy missed expert rows into VRAM slots, and request reads from the host.

Mirrors src/vllm_expert_pager/gather.py of monochromegane/vllm-expert-pager:
``as_rows``, ``gather_rows``, ``fetch_rows``, ``fetch_publish_rows`` and
``fetch_wait_rows`` keep their arguments and semantics; each is one launch of
``libxpager.so`` (gather.cu).  The source rows are the RAM tier (pinned host
memory the SMs read over the host link with 16-byte loads) or the cache slab;
which experts to copy comes from device index arrays, so the launches replay
under CUDA graphs.

Waiting for the host is bounded by time rather than by a spin count: every
``store.retry_ns`` nanoseconds the request is published again, and after
``store.giveup`` re-publishes the wait ends and the give-up counter moves
(the reference: 2**18 spins, about 0.5-1.2 s, and 8 tries).
"""

from __future__ import annotations

import torch

from vllm_expert_pager import native

# Copying CTAs of the gather.  Each keeps 16 KiB of loads in flight, so this
# sets the bytes in flight on the host link (tuned on B200; the reference's
# 4 x 16 KiB suited a PCIe 4.0 RTX 4090).
GATHER_CTAS = 16


def as_rows(t: torch.Tensor) -> torch.Tensor:
    """View a tensor whose leading axis is the expert axis as ``(E, W)`` int32 (gather.py:314-325)."""
    if not t.is_contiguous():
        raise ValueError("expert weights must be contiguous")
    row_bytes = t[0].numel() * t.element_size()
    if row_bytes % 4:
        raise ValueError(f"row size {row_bytes} B is not a multiple of 4")
    return t.view(torch.int32).reshape(t.shape[0], -1)


def _device_of(*ts: torch.Tensor) -> torch.device:
    for t in ts:
        if t is not None and t.device.type == "cuda":
            return t.device
    return torch.device("cuda", torch.cuda.current_device())


def gather_rows(
    todo: torch.Tensor,
    dst_row: torch.Tensor,
    cache_row: torch.Tensor,
    src_row: torch.Tensor,
    base: int,
    src: list[torch.Tensor],
    cache: list[torch.Tensor],
    dst: list[torch.Tensor],
    stg: list[torch.Tensor] | None,
    scale: list[torch.Tensor],
    scale_dst: list[torch.Tensor],
    fetch: tuple[torch.Tensor, int, object] | None = None,
    ctas: int | None = None,
    chunk: int = 0,
) -> None:
    """Copy the rows and scales of the experts in ``todo`` (gather.py:328-393).

    Each list has two elements in name order (w13, w2), int32 row views.
    Experts with ``cache_row[e] >= 0`` are copied from the cache slab to row
    ``dst_row[e]`` of ``dst``; the others from RAM-tier row ``src_row[e] +
    base`` of ``src``: into row j (their index in todo) of ``stg`` when
    compressed, else into row ``dst_row[e]`` of ``dst``.  Scales always go from
    ``scale[e]`` to ``scale_dst[dst_row[e]]``.  ``src`` may be pinned CPU
    tensors (read through their device mapping) or device views of them.

    With ``fetch=(ssd_todo, layer, store)`` one more CTA of the same launch asks
    the host to read ``ssd_todo`` from SSD and waits, while the copy skips those
    experts; a later ``gather_rows(ssd_todo, ...)`` copies them.

    ``chunk`` (not in the reference): with compressed rows, the records' values
    per lane; when > 0, only each record's used words (header, nibbles, Huffman
    words) are copied from the RAM tier, the rest of its staging row is left as
    it was (the decoder never reads it).  0 copies whole records.
    """
    W0, W1 = dst[0].shape[1], dst[1].shape[1]
    P0, P1 = src[0].shape[1], src[1].shape[1]
    compress = stg is not None
    if compress:
        if (P0, P1) != (stg[0].shape[1], stg[1].shape[1]):
            raise ValueError("staging rows must have the RAM tier's pitch")
    else:
        if (P0, P1) != (W0, W1):
            raise ValueError("uncompressed RAM rows must have the slab's row size")
    K = todo.shape[0]
    device = _device_of(todo)
    native.require_cuda(todo, dst_row, cache_row, src_row, *dst, *scale, *scale_dst)
    if fetch is None:
        ssd, layer, store = None, 0, None
        seq = req = done = None
        block = ring = retry = giveup = 0
    else:
        ssd, layer, store = fetch
        if ssd.shape[0] != K:
            raise ValueError(f"ssd_todo has {ssd.shape[0]} entries, todo has {K}")
        seq, req, done = store.seq.data_ptr(), store.req_dev, store.done_dev
        block, ring, retry, giveup = store.block, store.ring, store.retry_ns, store.giveup
    st = stg if compress else [None, None]
    native.check(
        native.lib().xp_gather_rows(
            todo.data_ptr(), K, dst_row.data_ptr(), cache_row.data_ptr(), src_row.data_ptr(), base,
            _src_ptr(src[0]), cache[0].data_ptr(), dst[0].data_ptr(), native.ptr(st[0]), W0, P0,
            _src_ptr(src[1]), cache[1].data_ptr(), dst[1].data_ptr(), native.ptr(st[1]), W1, P1,
            scale[0].data_ptr(), scale_dst[0].data_ptr(), scale[0].shape[1],
            scale[1].data_ptr(), scale_dst[1].data_ptr(), scale[1].shape[1],
            native.ptr(ssd), int(compress), int(chunk) if compress else 0, ctas or GATHER_CTAS,
            layer, seq, req, done, block, ring, retry, giveup,
            native.stream_of(device),
        ),
        "gather_rows",
    )  # fmt: skip


def _src_ptr(t: torch.Tensor) -> int:
    """Device address of a RAM-tier view: pinned CPU tensors go through their mapping."""
    if t.device.type == "cpu":
        dev = native.ctypes.c_void_p()
        native.check(native.lib().xp_device_pointer(t.data_ptr(), native.ctypes.byref(dev)),
                     "device_pointer")
        return dev.value
    return t.data_ptr()


def fetch_rows(todo: torch.Tensor, row: torch.Tensor, base: int, layer: int, store) -> None:
    """Ask the host to read the experts in ``todo`` from SSD and wait (gather.py:396-407).

    Expert ``e`` lands in RAM-tier row ``row[e] + base``.  Does nothing if
    ``todo`` is empty.
    """
    native.require_cuda(todo, row)
    native.check(
        native.lib().xp_fetch(todo.data_ptr(), todo.shape[0], row.data_ptr(), base, layer,
                              store.seq.data_ptr(), store.req_dev, store.done_dev, store.block,
                              store.ring, store.retry_ns, store.giveup,
                              native.stream_of(todo.device)),
        "fetch_rows",
    )


def fetch_publish_rows(todo: torch.Tensor, row: torch.Tensor, base: int, layer: int, store,
                       ticket: torch.Tensor) -> None:
    """Publish the request of ``fetch_rows`` without waiting (gather.py:410-431).

    ``ticket`` (one int64 on the device) receives the published seq.  If
    ``todo`` is empty nothing is published and ``ticket`` is left as it is.  At
    most ``store.ring`` requests may be outstanding.
    """
    native.require_cuda(todo, row, ticket)
    native.check(
        native.lib().xp_fetch_publish(todo.data_ptr(), todo.shape[0], row.data_ptr(), base, layer,
                                      store.seq.data_ptr(), ticket.data_ptr(), store.req_dev,
                                      store.block, store.ring, native.stream_of(todo.device)),
        "fetch_publish_rows",
    )


def fetch_wait_rows(todo: torch.Tensor, store, ticket: torch.Tensor) -> None:
    """Wait for done to reach the seq in ``ticket``; nothing if ``todo`` is empty (gather.py:434-439)."""
    native.require_cuda(todo, ticket)
    native.check(
        native.lib().xp_fetch_wait(todo.data_ptr(), todo.shape[0], ticket.data_ptr(),
                                   store.req_dev, store.done_dev, store.block, store.ring,
                                   store.retry_ns, store.giveup, native.stream_of(todo.device)),
        "fetch_wait_rows",
    )
