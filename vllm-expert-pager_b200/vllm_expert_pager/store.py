"""RAM and SSD tiers for expert weights.

Mirrors ``Store`` of monochromegane/vllm-expert-pager (src/vllm_expert_pager/store.py):
the same constructor, validation messages, row numbering, paging-file layout,
request ring and statistics.  What changed:

* The RAM tier is page-aligned pinned memory from ``xp_pinned_alloc``: mmap,
  placed on the GPU's NUMA node, then registered with the driver.  Nothing is
  rounded up to a power of two, and each of 1..8 replicas keeps its tier next
  to its own GPU.  ``pinned[name]`` is a CPU tensor over it; ``view[name]`` is a
  CUDA tensor over the same bytes (the reference used vLLM's
  ``get_accelerator_view_from_cpu_tensor``).
* The host server is the C++ one in ``libxpager.so`` (same C ABI as the
  reference's C server: ssd_start/ssd_stop/ssd_stats/ssd_error/ssd_test_delay),
  which also splits each record read into page-aligned jobs read by all its
  threads at once (``VLLM_EXPERT_PAGER_READ_CHUNK``, 512 KiB; 0 reads whole
  records as the reference does), and reads a compressed record only up to the
  last page of each name's used words (``VLLM_EXPERT_PAGER_READ_USED``, on; the
  decoder never reads past them), ~8 % fewer disk bytes per record.
* The GPU's wait for the host is bounded by time: ``retry_ns`` between
  re-publishes and ``giveup`` re-publishes (settable per store).

Layout: rows ``[0, L*R)`` are the RAM tier (slot s of layer l is row l*R + s),
followed by the shared working rows.  The paging file holds fixed-length
records ``[layer][expert]`` of the w13 row then the w2 row, each at its pitch.
"""

from __future__ import annotations

import ctypes
import faulthandler
import logging
import os
import signal
import threading

import numpy as np
import torch

from vllm_expert_pager import codec, native

logger = logging.getLogger(f"vllm.{__name__}")

# Page size.  O_DIRECT reads need page-aligned offsets, lengths and buffers, so
# the pinned tier's base, every row pitch and every record are whole pages.
_ALIGN = 4096
# Threads that read the experts of one layer concurrently (the server itself
# and the workers): 8 as in the reference (store.py:59-64), which measured an
# NVMe saturating at 8 outstanding reads.  VLLM_EXPERT_PAGER_READ_WORKERS sets
# it for devices that want a deeper queue.
_READ_WORKERS = max(1, int(os.environ.get("VLLM_EXPERT_PAGER_READ_WORKERS", "8")))
# Bytes per read job of the SSD server (whole 4 KiB pages): each record read is
# split into jobs of this size that the read threads take concurrently, so a
# request of one or two experts keeps all of them busy.  0 reads whole records,
# one per thread, as the reference does.  VLLM_EXPERT_PAGER_READ_CHUNK sets it.
_READ_CHUNK = max(0, int(os.environ.get("VLLM_EXPERT_PAGER_READ_CHUNK", str(512 << 10))))
# Compressed records are read only up to the last page of each name's used
# words (header, nibbles, Huffman words); 0 reads whole records.
_READ_USED = os.environ.get("VLLM_EXPERT_PAGER_READ_USED", "1") != "0"
# Slots in the request ring (store.py:65-67).
RING = 4
# GPU wait for the host: re-publish every RETRY_NS, give up after GIVEUP
# re-publishes.  The reference spins 2**18 times (0.5-1.2 s) per try, 8 tries.
RETRY_NS = 500_000_000
GIVEUP = 8


class _CudaView:
    """__cuda_array_interface__ over a device (UVA) address, for torch.as_tensor."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str) -> None:
        self.__cuda_array_interface__ = {
            "data": (ptr, False),
            "shape": shape,
            "typestr": typestr,
            "version": 3,
            "strides": None,
            "stream": None,
        }


def numa_node_of(device: torch.device) -> int:
    """NUMA node of a GPU from sysfs, -1 if unknown."""
    try:
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            return int(f.read().strip())
    except (OSError, ValueError, AttributeError, RuntimeError):
        return -1


class PinnedBuffer:
    """Pinned, device-mapped host memory with a CPU tensor and a CUDA tensor over it."""

    def __init__(self, nbytes: int, device: torch.device, numa_node: int = -1) -> None:
        self.nbytes = -(-nbytes // _ALIGN) * _ALIGN
        host, dev = ctypes.c_void_p(), ctypes.c_void_p()
        native.check(
            native.lib().xp_pinned_alloc(self.nbytes, numa_node, ctypes.byref(host),
                                         ctypes.byref(dev)),
            f"pinned allocation of {self.nbytes} B",
        )
        self.host_ptr, self.dev_ptr = host.value, dev.value
        buf = (ctypes.c_uint8 * self.nbytes).from_address(self.host_ptr)
        self.cpu = torch.frombuffer(buf, dtype=torch.uint8)
        with torch.cuda.device(device):
            self.cuda = torch.as_tensor(_CudaView(self.dev_ptr, (self.nbytes,), "|u1"),
                                        device=device)

    def free(self) -> None:
        if self.host_ptr:
            native.lib().xp_pinned_free(self.host_ptr, self.nbytes)
            self.host_ptr = None


class Store:
    """One per model: the RAM tier's pinned rows, the paging file and the host server."""

    def __init__(
        self,
        num_layers: int,
        num_experts: int,
        ram_slots: int,
        working_rows: int,
        row_bytes: dict[str, int],
        compress: bool,
        pitch_ratio: float,
        path: str | None,
        device: torch.device,
        numa_node: int | None = None,
    ) -> None:
        L, E, R = num_layers, num_experts, ram_slots
        if not 1 <= R <= E:
            raise ValueError(f"VLLM_EXPERT_PAGER_RAM_SLOTS must be in [1, {E}], got {R}")
        if working_rows < 1:
            raise ValueError(f"working_rows must be >= 1, got {working_rows}")
        if R < E and path is None:
            raise ValueError(
                "VLLM_EXPERT_PAGER_SSD_PATH is required when "
                "VLLM_EXPERT_PAGER_RAM_SLOTS < num_experts"
            )
        for name, nbytes in row_bytes.items():
            unit = codec.GROUP if compress else _ALIGN
            if nbytes % unit:
                raise ValueError(f"{name}: row of {nbytes} B is not a multiple of {unit}")
        self._handle = None
        self._buffers: list[PinnedBuffer] = []
        self.num_layers, self.num_experts, self.ram_slots = L, E, R
        self.layers = 0
        self.device = torch.device(device)
        self.compress = compress
        self.names = list(row_bytes)
        self.row_bytes = dict(row_bytes)
        self.pitch = {
            name: codec.pitch_of(nbytes, pitch_ratio, _ALIGN) if compress else nbytes
            for name, nbytes in row_bytes.items()
        }
        self.record_bytes = sum(self.pitch.values())
        self.offset = {}
        pos = 0
        for name in self.names:
            self.offset[name] = pos
            pos += self.pitch[name]
        self.working_base = L * R
        self.rows = L * R + working_rows
        self.numa_node = numa_node_of(self.device) if numa_node is None else numa_node
        logger.info(
            "vllm-expert-pager: RAM tier %d rows x %d B (%s) = %.2f GiB pinned (NUMA node %d)",
            self.rows, self.record_bytes,
            f"compressed from {sum(row_bytes.values())} B" if compress else "raw",
            self.rows * self.record_bytes / 2**30, self.numa_node,
        )  # fmt: skip
        self.pinned: dict[str, torch.Tensor] = {}
        self.view: dict[str, torch.Tensor] = {}
        for name, nbytes in self.pitch.items():
            b = self._alloc(self.rows * nbytes)
            self.pinned[name] = b.cpu[: self.rows * nbytes].view(torch.int32).view(self.rows, -1)
            self.view[name] = b.cuda[: self.rows * nbytes].view(torch.int32).view(self.rows, -1)
        # Decode tables, 512 bytes per (layer, expert, name); with raw rows
        # only a single layer's worth exists, so the kernels still get a pointer.
        self.lut = torch.zeros(
            (L if compress else 1, E, len(self.names), codec.LUT_BYTES),
            dtype=torch.uint8, device=self.device,
        )  # fmt: skip

        # The request ring, in pinned host memory (store.py:434-451): two
        # counters (re-publishes, give-ups), then RING request slots, each
        # holding seq and layer followed by B expert ids and B RAM rows, where B
        # is E rounded up to a power of two; done[0] follows the ring.
        self.block = 1 << (E - 1).bit_length()
        self.ring = RING
        self.retry_at, self.giveup_at = 0, 1
        self.slot_words = 2 + 2 * self.block
        ring = self._alloc(8 * (2 + RING * self.slot_words) + 8)
        n = 2 + RING * self.slot_words
        self.req = ring.cpu[: 8 * n].view(torch.int64)
        self.done = ring.cpu[8 * n : 8 * n + 8].view(torch.int64)
        self.req_dev, self.done_dev = ring.dev_ptr, ring.dev_ptr + 8 * n
        self.req_view = ring.cuda[: 8 * n].view(torch.int64)
        self.done_view = ring.cuda[8 * n : 8 * n + 8].view(torch.int64)
        self.seq = torch.zeros((1,), dtype=torch.int64, device=self.device)
        self.ticket_chunk = torch.zeros((2,), dtype=torch.int64, device=self.device)
        self.retry_ns, self.giveup = RETRY_NS, GIVEUP

        self.path = path if R < E else None
        self.fd_w = self.fd_r = None
        if self.path is not None:
            size = L * E * self.record_bytes
            if os.path.exists(path) and os.path.getsize(path) != size:
                raise FileExistsError(
                    f"{path} exists and is not a paging file of {size} B; remove it first"
                )
            self.fd_w = os.open(path, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
            self.fd_r = os.open(path, os.O_RDONLY | getattr(os, "O_DIRECT", 0))
            logger.info("vllm-expert-pager: paging file %s (%.1f GiB)", path, size / 2**30)
            self._start_server()
        if threading.current_thread() is threading.main_thread():
            faulthandler.register(signal.SIGUSR2, all_threads=True)

    def _alloc(self, nbytes: int) -> PinnedBuffer:
        b = PinnedBuffer(nbytes, self.device, self.numa_node)
        self._buffers.append(b)
        return b

    def _start_server(self) -> None:
        n = len(self.names)
        pinned = (ctypes.c_void_p * n)(*(self.pinned[k].data_ptr() for k in self.names))
        pitch = (ctypes.c_long * n)(*(self.pitch[k] for k in self.names))
        self._so = native.lib()
        self._handle = self._so.ssd_start(
            self.fd_r, ctypes.c_void_p(self.req.data_ptr()), ctypes.c_void_p(self.done.data_ptr()),
            self.ring, self.block, self.num_layers, self.num_experts, self.rows,
            self.record_bytes, n, pinned, pitch, _READ_WORKERS - 1,
        )  # fmt: skip
        if not self._handle:
            raise RuntimeError("vllm-expert-pager: cannot start the SSD server")
        self._so.ssd_set_read_chunk(ctypes.c_void_p(self._handle), _READ_CHUNK)
        # Used bytes of each record piece, filled by write(); 0 = the whole piece.
        self._used = np.zeros(self.num_layers * self.num_experts * n, dtype=np.int64)
        if self.compress and _READ_USED:
            self._so.ssd_set_used_bytes(ctypes.c_void_p(self._handle),
                                        ctypes.c_void_p(self._used.ctypes.data))

    def close(self) -> None:
        """Stop the host server and release the pinned memory and files."""
        if getattr(self, "_handle", None):
            self._so.ssd_stop(ctypes.c_void_p(self._handle))
            self._handle = None
        for fd in ("fd_w", "fd_r"):
            if getattr(self, fd, None) is not None:
                os.close(getattr(self, fd))
                setattr(self, fd, None)

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def release(self) -> None:
        """close() and free the pinned buffers (no tensor over them may be used after)."""
        self.close()
        torch.cuda.synchronize(self.device)
        for b in self._buffers:
            b.free()
        self._buffers = []

    def test_delay(self, seconds: float) -> None:
        """For tests: delay the host between seeing a request and serving it."""
        self._so.ssd_test_delay(ctypes.c_void_p(self._handle), seconds)

    def mark_used(self, layer: int, expert: int, name: str, record) -> None:
        """Note how many bytes of a compressed record written to the paging file hold
        data (header G + 1 words, nibbles N / 8 words, then header[G] Huffman words),
        so that the host server reads it only up to that page.  ``write`` calls it;
        a caller that writes records to the paging file itself calls it per record
        (``record``: the record's int32 words on the host)."""
        if getattr(self, "_used", None) is None:
            return
        G = self.row_bytes[name] // codec.GROUP
        used = 4 * (G + 1 + self.row_bytes[name] // 8 + max(int(record[G]), 0))
        k = (layer * self.num_experts + expert) * len(self.names) + self.names.index(name)
        self._used[k] = min(used, self.pitch[name])

    # ---- statistics (written by the host server) ----

    def _stats(self) -> tuple[int, int, float, int]:
        if not self._handle:
            return 0, 0, 0.0, 0
        fetches, reads, missed = (ctypes.c_long() for _ in range(3))
        io_seconds = ctypes.c_double()
        self._so.ssd_stats(ctypes.c_void_p(self._handle), ctypes.byref(fetches),
                           ctypes.byref(reads), ctypes.byref(io_seconds), ctypes.byref(missed))
        return fetches.value, reads.value, io_seconds.value, missed.value

    @property
    def fetches(self) -> int:
        """Requests served."""
        return self._stats()[0]

    @property
    def reads(self) -> int:
        """Experts read."""
        return self._stats()[1]

    @property
    def io_seconds(self) -> float:
        """Total time from seeing a request to writing done."""
        return self._stats()[2]

    @property
    def bytes_read(self) -> int:
        """Bytes the host server has read from the paging file."""
        return int(self._so.ssd_bytes_read(ctypes.c_void_p(self._handle))) if self._handle else 0

    @property
    def missed(self) -> int:
        """Requests the GPU gave up on before they arrived."""
        return self._stats()[3]

    @property
    def failed(self) -> str | None:
        """Description of a failed read, if any (forward checks it and raises)."""
        if not self._handle:
            return None
        err = self._so.ssd_error(ctypes.c_void_p(self._handle))
        return None if err is None else err.decode(errors="replace")

    def layer_lut(self, layer: int) -> torch.Tensor:
        """The LUTs ``(E, names, 512)`` of a layer (unused without compression)."""
        return self.lut[layer if self.compress else 0]

    def add_layer(self) -> int:
        """Hand out a layer number; layers register in construction order."""
        if self.layers >= self.num_layers:
            raise RuntimeError(f"more MoE layers than num_hidden_layers={self.num_layers}")
        self.layers += 1
        return self.layers - 1

    # ---- load time ----

    def write(self, layer: int, expert: int, name: str, row: torch.Tensor) -> None:
        """Put one expert's row (compressed if compress) in the paging file and the RAM tier.

        The RAM tier gets it only when expert < R (slot e), as in store.py:576-599.
        """
        raw = row.contiguous().view(torch.uint8).reshape(-1)
        if raw.numel() != self.row_bytes[name]:
            raise ValueError(
                f"{name}: expert {expert} of layer {layer} has {raw.numel()} B, "
                f"expected {self.row_bytes[name]}"
            )
        if self.compress:
            # Encoded on the GPU when the store has one (encode_gpu.cu), as the
            # reference encodes with torch ops on the device (store.py:588).
            src = raw.to(self.device) if self.device.type == "cuda" else raw.cpu()
            record, lut = codec.encode(src, self.pitch[name])
            self.lut[layer, expert, self.names.index(name)] = lut.to(self.device)
            words = record.view(torch.int32)
        else:
            words = raw.view(torch.int32)
        if expert < self.ram_slots:
            self.pinned[name][layer * self.ram_slots + expert].copy_(words)
        if self.fd_w is not None:
            offset = (layer * self.num_experts + expert) * self.record_bytes + self.offset[name]
            host = np.ascontiguousarray(words.cpu().numpy())
            os.pwrite(self.fd_w, memoryview(host), offset)
            if self.compress:
                self.mark_used(layer, expert, name, host)
