"""Benchmark of the expert-paging hot path on B200 (one JSON line on rank 0).

Headline (``value``, BASELINE.json config 2, "single MoE layer decode paging"):
256 FP8 experts of 3 MiB (w13 [1024, 2048] + w2 [2048, 512], N(0, 0.02)
quantised with 128x128 block scales), CACHE_SLOTS=32, RAM_SLOTS=256
uncompressed in pinned host memory, batch-1 top-8 routing drawn Zipf(1.1) over
a seeded permutation (4096-step trace).  One bench step = one window of
``--window`` consecutive decode steps of the trace (512 by default), each one
fused launch: both LRU table updates, the gather of the missed rows from pinned
RAM over the host link (+ the SSD-fetch CTA, idle here).

  value    = bytes paged in (misses x 3 MiB) / device time of the timed steps,
             summed over ranks (independent replicas, weak scaling)
  e2e      = the same through the public API, host-driven: every decode step
             reads its routing ids from pinned host memory and writes its
             expert_map back to pinned host memory (by the step kernel itself)
  roofline = the step kernel's achieved host-link GB/s (algorithmic bytes /
             CUDA-event duration of its launches) against the pinned-H2D copy
             bandwidth measured here with the copy engine
  links    = per rank: that copy bandwidth with the link idle and with every
             rank copying, the RAM tier's NUMA node, the GPU's PCI address
  configs  = (one GPU) config 4, where gather and decode run together: the
             40-layer paged MoE with the compressed RAM tier (R=128) and the
             O_DIRECT paging file at batch 1 and 8 under CUDA graphs, each with
             the in-run host-link roofline of its copy kernel, the in-run HBM
             roofline of the decode kernel and the SSD rate vs the disk's peak;
             and config 5, the chunked 2048-token prefill (8 layers) on the SSD
             tier and on a RAM-resident compressed tier, overlapped and serial
  kernels  = decode / acquire / encode kernels alone, and the reference's own
             Triton kernels on the same inputs (a subprocess)
  cpu_baseline = the reference's own CPU code (its ExpertTable on CPU tensors +
             a threaded memcpy; a subprocess), the numpy port beside it, and
             config 1's codec on the host cores

``--impl reference`` times the reference's own CPU code (see run_reference).
"""

from __future__ import annotations

import argparse
import json
import os
import select
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vllm-expert-pager_b200"))
sys.path.insert(0, ROOT)

METRIC = "paged expert GB/s per B200 (gather+decode) vs host-link/HBM roofline; tok/s"
E, S, R, TOPK = 256, 32, 256, 8
EXPERT_BYTES = 1024 * 2048 + 2048 * 512  # w13 [1024, 2048] + w2 [2048, 512] fp8 bytes
TRACE_STEPS = 4096


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--window", type=int, default=512)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--ctas", type=int, default=0, help="gather CTAs (0 = library default)")
    p.add_argument("--workload", choices=["paging", "decode", "model", "compressed", "prefill",
                                          "reference-triton", "links"],
                   default="paging",
                   help="paging: config 2 (the headline line); decode: the decode kernel alone; "
                        "model/compressed/prefill: configs 3/4/5 on a paged 40-layer MoE; "
                        "reference-triton: the reference's own Triton kernels from baseline/_ref "
                        "on the inputs of paging/decode (one GPU); links: every rank's "
                        "pinned->device copy bandwidth alone and with all ranks copying")
    p.add_argument("--layers", type=int, default=40, help="MoE layers of configs 3-5")
    p.add_argument("--tokens", type=int, default=512, help="decode tokens of configs 3-4")
    p.add_argument("--c4-tokens", type=int, default=256,
                   help="batch-1 decode tokens of the default line's config-4 entries "
                        "(batch 8 runs a quarter as many steps)")
    p.add_argument("--c5-layers", type=int, default=8,
                   help="layers of the default line's config-5 prefill entry")
    p.add_argument("--skip", default="",
                   help="comma-separated parts of the default line to leave out: "
                        "compressed, prefill, reference_triton, cpu, kernels")
    return p.parse_args()


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _reduce(x: float, world: int, op: str) -> float:
    """max/sum of a per-rank scalar over all ranks (NCCL: a CUDA tensor; gloo: CPU)."""
    if world == 1:
        return x
    import torch.distributed as dist

    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, "max")


def sum_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, "sum")


def aggregate(moved: float, ms: float, world: int) -> tuple[float, float, float]:
    """Whole-job throughput of independent replicas: (GB/s, bytes of all ranks, slowest ms).

    Every rank pages its own experts; the job moves the sum of the ranks' bytes
    in the time of the slowest rank.
    """
    ms_max = max_over_ranks(ms, world)
    total = sum_over_ranks(moved, world)
    return total / (ms_max * 1e-3) / 1e9, total, ms_max


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index, self.proc = index, None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        # nvidia-smi takes a moment to start: wait for its first (idle, discarded)
        # sample so that a short timed region still gets sampled.
        ready, _, _ = select.select([self.proc.stdout], [], [], 10.0)
        if ready:
            self.proc.stdout.readline()
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self):
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def build_workload(device: torch.device):
    """Pinned RAM tier with 256 experts, the layer's pager, and the Zipf trace."""
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.pager import PARAMS, LayerPager, WorkingSlab
    from vllm_expert_pager.store import Store

    row_bytes = {n: r * c for n, (r, c) in synthetic.SHAPES.items()}
    store = Store(1, E, R, 2 * 64, row_bytes, False, 0.89, None, device)
    gen = torch.Generator(device=device).manual_seed(0)
    scales = {}
    for name, (r, c) in synthetic.SHAPES.items():
        sc = torch.empty((E, r // 128, c // 128), dtype=torch.float32, device=device)
        for e0 in range(0, E, 32):  # 32 experts at a time on the device
            w = (torch.randn((32, r, c), generator=gen, device=device) * 0.02).to(torch.bfloat16)
            blocks = w.float().view(32, r // 128, 128, c // 128, 128)
            amax = blocks.abs().amax(dim=(2, 4)) / 448.0
            q = (blocks / amax[:, :, None, :, None]).to(torch.float8_e4m3fn).view(32, r, c)
            store.pinned[name][e0 : e0 + 32].copy_(q.view(torch.int32).reshape(32, -1))
            sc[e0 : e0 + 32] = amax
            del w, blocks, q
        scales[f"{name[:-7]}_weight_scale"] = sc
    shapes = {n: (synthetic.SHAPES[n], torch.float8_e4m3fn) for n in PARAMS}
    shapes.update({k: (v.shape[1:], v.dtype) for k, v in scales.items()})
    working = WorkingSlab(64, {n: (tuple(s), d) for n, (s, d) in shapes.items()}, store, device)
    pager = LayerPager(store, 0, S, scales, {n: (synthetic.SHAPES[n], torch.float8_e4m3fn)
                                             for n in PARAMS}, working)
    trace = synthetic.zipf_trace(TRACE_STEPS, E, TOPK, 1.1, layer=0)
    return store, pager, trace


def measure_h2d_peak(device, world: int = 1, reps: int = 6) -> float:
    """Copy-engine pinned->device bandwidth (GB/s), 1 GiB, best of ``reps``, from pinned
    memory placed on the GPU's NUMA node as the RAM tier is (xp_pinned_alloc).

    With several ranks every rank copies at the same time (a barrier before each
    copy), so the figure is one replica's share of the host links and host memory
    while all replicas page, which is the bench's own load.
    """
    from vllm_expert_pager import store as store_mod

    n = 1 << 30
    pinned = store_mod.PinnedBuffer(n, device, store_mod.numa_node_of(device))
    src = pinned.cpu
    dst = torch.empty(n, dtype=torch.uint8, device=device)
    best = 0.0
    for _ in range(reps):
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, n / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    pinned.free()
    return best


def check_slab(store, pager) -> None:
    """The slots hold the rows of the experts the VRAM table says they hold."""
    from vllm_expert_pager.pager import PARAMS

    expert_in = pager.vram.expert_in[:S].cpu().tolist()
    for s, e in enumerate(expert_in[:8]):
        if e < 0:
            continue
        for k, n in enumerate(PARAMS):
            got = pager.cache_rows[k][s].cpu()
            want = store.pinned[n][e]
            if not torch.equal(got, want):
                raise SystemExit(f"slab row {s} does not hold expert {e} ({n})")


def hbm_peak() -> tuple[float, str]:
    """HBM copy bandwidth from MEASURED_PEAKS.json (driver-written), else the pool fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (measured)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def bench_decode(device, rows_per_launch: int, launches: int = 48, distinct: int = 64,
                 reps: int = 5) -> dict:
    """Decode kernel alone: compressed config-1 experts staged in HBM -> raw slab rows.

    ``distinct`` experts (encoded at pitch 0.89 with the native encoder) sit in a
    staging buffer and a destination slab of as many rows, both larger than L2;
    each launch expands ``rows_per_launch`` of them, rotating through the set.
    Algorithmic bytes per row = used record bytes + raw bytes written + the
    512-byte LUT, per name.
    """
    from vllm_expert_pager import codec, synthetic

    names = list(synthetic.SHAPES)
    gen = torch.Generator().manual_seed(0)
    recs = {n: [] for n in names}
    luts = torch.zeros((distinct, 2, 512), dtype=torch.uint8)
    used = 0
    for e in range(distinct):
        ex = synthetic.fp8_expert(gen) if e < 8 else None
        for k, n in enumerate(names):
            if ex is None:  # reuse the 8 generated experts' bytes, shifted, to save host time
                raw = recs[n][e % 8][1]
            else:
                raw = synthetic.row_bytes(ex[n][0])
            pitch = codec.pitch_of(raw.numel(), 0.89, 4096)
            rec, lut = codec.encode(raw, pitch)
            G = raw.numel() // codec.GROUP
            used += 4 * (G + 1) + raw.numel() // 2 + 4 * int(rec[4 * G : 4 * G + 4].view(torch.int32))
            recs[n].append((rec, raw))
            luts[e, k] = lut
    stg = [torch.stack([r for r, _ in recs[n]]).to(device) for n in names]
    dst = [torch.empty((distinct, recs[n][0][1].numel()), dtype=torch.uint8, device=device)
           for n in names]
    lut_d = luts.to(device)
    raw_bytes = sum(recs[n][0][1].numel() for n in names)
    per_row = used / distinct + raw_bytes + 2 * 512
    K = rows_per_launch
    starts = list(range(0, distinct - K + 1, K))
    todos = [torch.arange(s0, s0 + K, dtype=torch.int64, device=device) for s0 in starts]
    ident = torch.arange(distinct, dtype=torch.int64, device=device)
    no_cache = torch.full((distinct,), -1, dtype=torch.int64, device=device)

    views = [[x[s0 : s0 + K] for x in stg] for s0 in starts]

    def launch(i):
        # launch i expands experts [s0, s0+K): staging row j holds expert s0+j, whose
        # raw row goes to dst row s0+j (dst_row = identity)
        j = i % len(starts)
        codec.decode_rows(todos[j], ident, no_cache, views[j], dst, lut_d)

    for i in range(4):
        launch(i)
    torch.cuda.synchronize()
    # The launches are captured in a CUDA graph and timed by replaying it between
    # two events on its stream: per-launch events around a Python call would also
    # count the host's launch time whenever that exceeds the kernel's (small K).
    s = torch.cuda.Stream(device=device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for i in range(launches):
                launch(i)
    torch.cuda.synchronize()
    best = None
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            a.record()
            graph.replay()
            b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / launches
        best = us if best is None else min(best, us)
    del graph
    for n, d, k in zip(names, dst, range(2)):  # parity spot check: expanded rows == raw rows
        for e in range(0, distinct, 17):
            if not torch.equal(d[e].cpu(), recs[n][e][1]):
                raise SystemExit(f"decode mismatch: expert {e} {n}")
    peak, src = hbm_peak()
    achieved = K * per_row / (best * 1e-6) / 1e9
    return {"rows_per_launch": K, "us_per_launch": round(best, 2),
            "algorithmic_bytes_per_launch": int(K * per_row), "achieved": round(achieved, 1),
            "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4), "bound": "hbm",
            "peak_source": src,
            "how": f"{launches} launches captured in a CUDA graph, replay timed with CUDA events "
                   f"on its stream, best of {reps}"}


class PagedMoE:
    """A Qwen3-style MoE stack (hidden 2048, moe_inter 512, 256 experts, top-8, FP8
    128x128 block scales, random-init weights and routers) whose expert weights
    are paged: one LayerPager per layer, one Store, one shared working slab.

    The 256 x layers experts are drawn from a pool of ``pool`` distinct seeded
    experts (layer l, expert e -> pool[perm_l[e]]), so that loading the RAM
    tier and writing the paging file of 40 layers takes seconds; every (layer,
    expert) row is still a separate record read over the host link or from
    the SSD.
    """

    def __init__(self, device, layers=40, S=32, R=256, compress=False, path=None, W=64,
                 overlap=True, pool=64, seed=0):
        from concurrent.futures import ThreadPoolExecutor

        from vllm_expert_pager import codec, moe, synthetic
        from vllm_expert_pager.pager import PARAMS, LayerPager, WorkingSlab
        from vllm_expert_pager.store import Store

        self.device, self.L, self.S, self.overlap = device, layers, S, overlap
        row_bytes = {n: r * c for n, (r, c) in synthetic.SHAPES.items()}
        self.store = store = Store(layers, E, R, 2 * W, row_bytes, compress, 0.89, path, device)
        pw = synthetic.fp8_experts_device(pool, device, seed=seed)
        g = torch.Generator().manual_seed(seed + 1)
        self.assign = [torch.randperm(E, generator=g) % pool for _ in range(layers)]
        recs, luts = {}, torch.zeros((pool, 2, 512), dtype=torch.uint8, device=device)
        if compress:
            host = {n: pw[n][0].cpu() for n in PARAMS}
            jobs = [(p, k, n) for p in range(pool) for k, n in enumerate(PARAMS)]

            def enc(job):
                p, k, n = job
                raw = host[n][p].view(torch.uint8).reshape(-1)
                return job, codec.encode(raw, store.pitch[n])

            with ThreadPoolExecutor(os.cpu_count() or 4) as ex:
                for (p, k, n), (rec, lut) in ex.map(enc, jobs):
                    recs[p, n] = rec.view(torch.int32)
                    luts[p, k] = lut.to(device)
        for layer in range(layers):
            a = self.assign[layer]
            for k, n in enumerate(PARAMS):
                if compress:
                    rows = torch.stack([recs[int(p), n] for p in a[:R]])
                    store.lut[layer, :, k] = luts[a.to(device), k]
                else:
                    rows = pw[n][0][a[:R].to(device)].view(torch.int32).reshape(R, -1).cpu()
                store.pinned[n][layer * R : (layer + 1) * R].copy_(rows)
            if store.fd_w is not None:  # the paging file: all E records of the layer
                blob = torch.empty((E, store.record_bytes), dtype=torch.uint8)
                for k, n in enumerate(PARAMS):
                    off = store.offset[n]
                    for e in range(E):
                        src = recs[int(a[e]), n] if compress else \
                            pw[n][0][int(a[e])].view(torch.int32).reshape(-1).cpu()
                        blob[e, off : off + store.pitch[n]] = src.view(torch.uint8)
                        if compress:
                            store.mark_used(layer, e, n, src)
                os.pwrite(store.fd_w, memoryview(blob.numpy()), layer * E * store.record_bytes)
        if store.fd_w is not None:
            os.fsync(store.fd_w)
        self.pool_weights = pw
        # Mean used bytes of an expert's records (header + nibbles + Huffman words).
        self.used_mean = float(sum(store.row_bytes.values()))
        if compress:
            used = 0
            for (p, n), rec in recs.items():
                N = store.row_bytes[n]
                G = N // codec.GROUP
                used += 4 * (G + 1) + N // 2 + 4 * int(rec[G])
            self.used_mean = used / pool
        shapes = {n: (synthetic.SHAPES[n], torch.float8_e4m3fn) for n in PARAMS}
        all_shapes = dict(shapes)
        all_shapes.update({f"{n[:-7]}_weight_scale": (tuple(pw[n][1].shape[1:]), torch.float32)
                           for n in PARAMS})
        self.working = WorkingSlab(W, all_shapes, store, device, halves=2 if overlap else 1)
        self.pagers = []
        for layer in range(layers):
            a = self.assign[layer].to(device)
            scales = {f"{n[:-7]}_weight_scale": pw[n][1][a].contiguous() for n in PARAMS}
            self.pagers.append(LayerPager(store, layer, S, scales, shapes, self.working))
        gr = torch.Generator(device=device).manual_seed(seed + 2)
        self.router = [(torch.randn((2048, E), generator=gr, device=device) * 0.02).to(torch.bfloat16)
                       for _ in range(layers)]
        self.moe = moe
        self.configs = {}

    def config(self, T):
        if T not in self.configs:
            self.configs[T] = self.moe.moe_config((E, 1024, 2048), (E, 2048, 512), TOPK, T)
        return self.configs[T]

    def layer(self, l, h, events=None):
        """One MoE layer with paged experts: route, page, run vLLM's fused MoE, add residual.

        ``events``: None, or a dict of lists that receive timing events of the
        paging launches (``step``: the fused decode step; ``decode``: decode
        launches; ``copy``: working-path gathers), as LayerPager records them."""
        moe, pager = self.moe, self.pagers[l]
        T = h.shape[0]
        logits = (h @ self.router[l]).float()
        w, ids = torch.softmax(logits, -1).topk(TOPK)
        w = (w / w.sum(-1, keepdim=True)).float()
        ids = ids.to(torch.int32)
        cfg = self.config(T)
        out = torch.empty_like(h)
        ev = events or {}
        if ids.numel() <= self.S:
            res = pager.decode(ids, gather_events=ev.get("step"), decode_events=ev.get("decode"))
            s = res.slabs
            c3 = moe.contributions(h, s["w13_weight"], s["w2_weight"], s["w13_weight_scale"],
                                   s["w2_weight_scale"], w, ids, res.expert_map, E, cfg)
            moe.moe_sum(c3, out)
        else:
            acc = {}

            def run_chunk(k, n, s, expert_map):
                c3 = moe.contributions(h, s["w13_weight"], s["w2_weight"],
                                       s["w13_weight_scale"], s["w2_weight_scale"], w, ids,
                                       expert_map, E, cfg)
                acc["c"] = c3 if "c" not in acc else acc["c"].add_(c3)
                if k == n - 1:
                    moe.moe_sum(acc["c"], out)

            pager.working_chunks(ids, run_chunk, overlap=self.overlap,
                                 decode_events=ev.get("decode"), copy_events=ev.get("copy"))
        return h + out

    def forward(self, h, events=None):
        for l in range(self.L):
            h = self.layer(l, h, events)
        return h

    def misses(self) -> int:
        return sum(int(p.vram.counters[2]) for p in self.pagers)

    def check(self, layers=4):
        """Slots of the first layers hold the rows of the experts their tables name."""
        from vllm_expert_pager.pager import PARAMS

        for l in range(min(layers, self.L)):
            p = self.pagers[l]
            ein = p.vram.expert_in[: self.S].cpu().tolist()
            for s, e in enumerate(ein[:4]):
                if e < 0:
                    continue
                src = int(self.assign[l][e])
                for n in PARAMS:
                    if not torch.equal(p.cache_slab[n][s].view(torch.uint8),
                                       self.pool_weights[n][0][src].view(torch.uint8)):
                        raise SystemExit(f"layer {l} slot {s}: wrong rows for expert {e} ({n})")

    def release(self):
        self.store.release()


def timed(fn, reps=1):
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / reps


def decode_row_bytes(m) -> float:
    """Algorithmic bytes of expanding one expert of ``m``: the used record bytes read
    (mean over the pool's records), the raw bytes written and the two 512-byte LUTs."""
    raw = sum(m.store.row_bytes.values())
    return m.used_mean + raw + 2 * 512


def _sum_events(evs) -> tuple[float, int, int]:
    """(total ms, rows, launches) of a list of (start, end, rows) timing triples."""
    ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    rows = sum(int(e[2]) for e in evs)
    return ms, rows, len(evs)


def model_decode(m, device, batch: int, tokens: int, h2d_peak: float | None = None,
                 probe: int = 8, seed: int = 11) -> dict:
    """Configs 3 and 4: ``tokens`` decode steps of batch ``batch`` through the paged
    MoE ``m``, replayed from one CUDA graph and timed with CUDA events; then ``probe``
    more steps run eagerly with CUDA events around every paging launch, which give
    the in-run rooflines of the copy and decode kernels (same model and tables, right
    after the timed replays; the probe's layer steps are synchronised one by one so
    that each fused step can be told apart by whether the host read the SSD for it)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    emb = (torch.randn((16, batch, 2048), generator=gen, device=device) * 0.5).to(torch.bfloat16)
    x = torch.empty((batch, 2048), dtype=torch.bfloat16, device=device)
    x.copy_(emb[0])
    for t in range(3):  # eager warm-up (Triton JIT, tables)
        x.copy_(emb[t])
        m.forward(x)
    torch.cuda.synchronize()
    s = torch.cuda.Stream(device=device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        m.forward(x)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            y = m.forward(x)
    torch.cuda.synchronize()
    for t in range(3, 8):
        x.copy_(emb[t])
        graph.replay()
    torch.cuda.synchronize()
    store = m.store
    miss0, reads0, bytes0 = m.misses(), store.reads, store.bytes_read
    gu0 = int(store.req[store.giveup_at])

    def run():
        for t in range(tokens):
            x.copy_(emb[8 + t % 8])
            graph.replay()

    with Clocks(torch.cuda.current_device()) as clocks:
        ms = timed(run)
    misses = m.misses() - miss0
    reads = store.reads - reads0
    disk_bytes = store.bytes_read - bytes0
    finite = bool(torch.isfinite(y).all())
    del graph
    m.check()
    # The fused step and the working path's gather copy a compressed record's used
    # words only (its header says how many).
    step_bytes = m.used_mean if store.compress else EXPERT_BYTES
    res = {"layers": m.L, "batch": batch, "tokens": tokens, "ms": round(ms, 2),
           "tok_per_s": round(tokens * batch / (ms * 1e-3), 2),
           "tpot_ms": round(ms / tokens, 3),
           "path": "decode (fused step)" if batch * TOPK <= m.S else "working slab (chunks)",
           "ssd_reads": reads,
           "ssd_gb_per_s": round(disk_bytes / (ms * 1e-3) / 1e9, 3),
           "ssd_bytes_per_read": round(disk_bytes / reads) if reads else None,
           "ssd_failed": store.failed,
           "giveups": int(store.req[store.giveup_at]) - gu0,
           "step_errors": sum(p.step_errors() for p in m.pagers),
           "clocks": clocks.summary(), "finite": finite}
    if batch * TOPK <= m.S:
        res["paged_gb_per_s"] = round(misses * step_bytes / (ms * 1e-3) / 1e9, 3)
        res["paged_bytes_per_miss"] = int(step_bytes)
        res["vram_misses_per_layer_step"] = round(misses / (tokens * m.L), 3)

    # Probe: the same steps eagerly, with events around every paging launch.
    ev = {"step": [], "decode": [], "copy": []}
    steps = []  # per fused step: (misses, did the host read the SSD for it)
    torch.cuda.synchronize()
    for t in range(probe):
        h = emb[t % 8].clone()
        for layer in range(m.L):
            pager = m.pagers[layer]
            r0, n0 = store.reads, len(ev["step"])
            c0 = int(pager.vram.counters[2])
            h = m.layer(layer, h, ev)
            torch.cuda.synchronize()
            if len(ev["step"]) > n0:
                steps.append((int(pager.vram.counters[2]) - c0, store.reads > r0))
    hbm, hsrc = hbm_peak()
    probe_res = {"tokens": probe * batch, "how": "eager steps after the timed replays; CUDA "
                 "events around each paging launch on its stream; kernel times summed"}
    if ev["decode"]:
        d_ms, d_rows, d_n = _sum_events(ev["decode"])
        per_row = decode_row_bytes(m)
        ach = d_rows * per_row / (d_ms * 1e-3) / 1e9 if d_ms > 0 else 0.0
        probe_res["decode"] = {
            "kernel": "decode_ring_kernel", "bound": "hbm", "launches": d_n,
            "rows_per_launch": round(d_rows / max(d_n, 1), 2),
            "us_per_launch": round(1e3 * d_ms / max(d_n, 1), 2),
            "algorithmic_bytes_per_row": int(per_row),
            "bytes_how": "mean used record bytes of the pool's records + raw bytes + 2 LUTs",
            "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(ach / hbm, 4), "peak_source": hsrc}
    if ev["step"]:
        t_all = [a.elapsed_time(b) for a, b in ev["step"]]
        ram = [(ms_, n) for ms_, (n, ssd) in zip(t_all, steps) if not ssd and n > 0]
        link = {"kernel": "step_kernel (both table updates + the copies of the misses; on "
                          "steps that read the SSD it also waits for the host)",
                "bound": "host_link", "launches": len(t_all),
                "launches_with_ssd": sum(1 for _, ssd in steps if ssd), "unit": "GB/s"}
        if ram:
            b_ = sum(n for _, n in ram) * step_bytes
            ach = b_ / (sum(ms_ for ms_, _ in ram) * 1e-3) / 1e9
            link.update({"achieved": round(ach, 3),
                         "how": "steps served from the RAM tier alone: bytes copied for "
                                "their misses (compressed: the records' used bytes, mean over "
                                "the pool) / their step-kernel time"})
            if h2d_peak:
                link.update({"peak": round(h2d_peak, 3), "frac": round(ach / h2d_peak, 4)})
        probe_res["host_link"] = link
    if ev["copy"]:
        c_ms, c_rows, c_n = _sum_events(ev["copy"])
        ach = c_rows * step_bytes / (c_ms * 1e-3) / 1e9 if c_ms > 0 else 0.0
        link = {"kernel": "gather_kernel (working path: RAM tier -> staging)",
                "bound": "host_link", "launches": c_n, "rows": c_rows, "unit": "GB/s",
                "achieved": round(ach, 3),
                "how": "rows copied from the RAM tier x bytes per row (compressed: the "
                       "records' used bytes, mean over the pool) / gather_kernel time"}
        if h2d_peak:
            link.update({"peak": round(h2d_peak, 3), "frac": round(ach / h2d_peak, 4)})
        probe_res["host_link"] = link
        res["paged_gb_per_s"] = round(c_rows * step_bytes / (probe * batch) * res["tok_per_s"]
                                      / 1e9, 3)
        res["paged_gb_per_s_how"] = "record bytes per token of the probe steps x timed tok/s"
    res["probe"] = probe_res
    return res


def run_model_decode(args, device, compress: bool, R: int, batch: int, tokens: int,
                     path=None) -> dict:
    """Configs 3 and 4 as separate lines (``--workload model|compressed``)."""
    m = PagedMoE(device, layers=args.layers, S=S, R=R, compress=compress, path=path)
    m.store.retry_ns = 500_000_000
    try:
        return model_decode(m, device, batch, tokens)
    finally:
        m.release()


def run_prefill(args, device, path) -> dict:
    """Config 5: a 2048-token prefill with uniform top-8 routing through every layer,
    copies overlapped with the MoE and serial, on two compressed tiers: ``ssd`` (R=128
    + the paging file: the disk bounds the layer) and ``ram`` (R=E=256, every record in
    pinned RAM, no SSD: the host link bounds the copies, so the overlap shows)."""
    from vllm_expert_pager import synthetic

    out = {}
    for tier, R_, p_ in (("ssd", 128, path), ("ram", E, None)):
        res = {}
        # One model per tier: its working slab has two halves; the serial run uses one.
        m = PagedMoE(device, layers=args.layers, S=S, R=R_, compress=True, path=p_,
                     overlap=True)
        gen = torch.Generator(device=device).manual_seed(13)
        T = 2048
        h = (torch.randn((T, 2048), generator=gen, device=device) * 0.5).to(torch.bfloat16)
        ids = synthetic.uniform_routing(T, seed=5).to(device)
        w = torch.softmax(torch.randn((T, TOPK), generator=gen, device=device), -1)
        cfg = m.config(T)
        moe = m.moe
        for overlap in (True, False):

            def layer_paged(l):
                acc = {}
                o = torch.empty_like(h)

                def run_chunk(k, n, s, expert_map):
                    c3 = moe.contributions(h, s["w13_weight"], s["w2_weight"],
                                           s["w13_weight_scale"], s["w2_weight_scale"], w, ids,
                                           expert_map, E, cfg)
                    acc["c"] = c3 if "c" not in acc else acc["c"].add_(c3)
                    if k == n - 1:
                        moe.moe_sum(acc["c"], o)

                m.pagers[l].working_chunks(ids, run_chunk, overlap=overlap)
                return o

            layer_paged(0)  # warm-up (JIT)
            torch.cuda.synchronize()
            reads0, bytes0 = m.store.reads, m.store.bytes_read
            with Clocks(torch.cuda.current_device()) as clocks:
                ms = timed(lambda: [layer_paged(l) for l in range(args.layers)])
            reads = m.store.reads - reads0
            disk_bytes = m.store.bytes_read - bytes0
            # MoE alone on resident weights (the pool), for the overlap fraction.
            pw = m.pool_weights
            pool_ids = (ids % pw["w13_weight"][0].shape[0]).to(torch.int32)
            moe_ms = timed(lambda: [moe.moe_sum(moe.contributions(
                h, pw["w13_weight"][0], pw["w2_weight"][0], pw["w13_weight"][1],
                pw["w2_weight"][1], w, pool_ids, None, pw["w13_weight"][0].shape[0], cfg),
                torch.empty_like(h)) for _ in range(args.layers)])
            res["overlap" if overlap else "serial"] = {
                "ms_per_layer": round(ms / args.layers, 3), "ssd_reads": reads,
                "ssd_gb_per_s": round(disk_bytes / (ms * 1e-3) / 1e9, 3),
                "ssd_bytes_per_read": round(disk_bytes / reads) if reads else None,
                "moe_only_ms_per_layer": round(moe_ms / args.layers, 3),
                "clocks": clocks.summary()}
        res["giveups"] = int(m.store.req[m.store.giveup_at])
        res["ssd_failed"] = m.store.failed
        m.release()
        o, s_ = res["overlap"]["ms_per_layer"], res["serial"]["ms_per_layer"]
        moe_ms = res["serial"]["moe_only_ms_per_layer"]
        res["hidden_fraction_of_moe"] = round(max(0.0, min(1.0, (s_ - o) / max(moe_ms, 1e-9))), 3)
        res["tier"] = (f"R={R_} compressed" + (" + O_DIRECT paging file" if p_ else
                                                ", every record in pinned RAM, no SSD"))
        out[tier] = res
    return out


def disk_peak(path: str, record_bytes: int, seconds: float = 3.0) -> dict:
    """Raw read bandwidth of the paging file: random O_DIRECT preadv's into
    page-aligned buffers, of whole records and of the server's read-job size
    (512 KiB chunks at record offsets), from 8 and from 32 threads for ``seconds``
    each; the best of the four."""
    import mmap
    import random
    import threading

    from vllm_expert_pager import store as store_mod

    size = os.path.getsize(path)
    n = size // record_bytes
    chunk = store_mod._READ_CHUNK if 0 < store_mod._READ_CHUNK < record_bytes else record_bytes
    best = None
    for nbytes in sorted({record_bytes, chunk // 4096 * 4096}):
        for threads in (8, 32):
            try:
                fd = os.open(path, os.O_RDONLY | os.O_DIRECT)
            except OSError:
                return {"unavailable": "O_DIRECT open failed"}
            total = [0] * threads
            stop = time.perf_counter() + seconds

            def reader(i):
                buf = mmap.mmap(-1, nbytes)
                rng = random.Random(i)
                pieces = record_bytes // nbytes
                while time.perf_counter() < stop:
                    off = rng.randrange(n) * record_bytes + rng.randrange(pieces) * nbytes
                    total[i] += os.preadv(fd, [buf], off)
                buf.close()

            t0 = time.perf_counter()
            ts = [threading.Thread(target=reader, args=(i,)) for i in range(threads)]
            for t in ts:
                t.start()
            for t in ts:
                t.join()
            dt = time.perf_counter() - t0
            os.close(fd)
            gbs = sum(total) / dt / 1e9
            if best is None or gbs > best["gb_per_s"]:
                best = {"gb_per_s": round(gbs, 3), "threads": threads, "read_bytes": nbytes}
    best["how"] = ("random O_DIRECT preadv on the paging file, whole records or the server's "
                   "read-job size, 8 or 32 threads; the best")
    return best


def compressed_configs(args, device, h2d_peak: float) -> dict:
    """Config 4 in the default line: the 40-layer paged MoE with the compressed RAM tier
    (R=128, pitch 0.89) and the O_DIRECT paging file, batch 1 (decode path: one fused
    step + one decode launch per layer) and batch 8 (K=64 > S: every step on the
    working slab), each replayed from a CUDA graph, with the in-run rooflines of the
    copy and decode kernels and the SSD rate against the disk's own peak."""
    base = os.environ.get("XP_BENCH_DIR", "/tmp")
    path = os.path.join(base, f"xpager_bench_c4_{os.getpid()}.bin")
    out = {}
    m = None
    try:
        m = PagedMoE(device, layers=args.layers, S=S, R=128, compress=True, path=path)
        m.store.retry_ns = 500_000_000
        b1 = args.c4_tokens
        out["compressed_b1"] = model_decode(m, device, 1, b1, h2d_peak)
        out["compressed_b8"] = model_decode(m, device, 8, max(b1 // 4, 8), h2d_peak, probe=2)
        peak = disk_peak(path, m.store.record_bytes)
        for v in out.values():
            if "gb_per_s" in peak:
                v["ssd_frac_of_disk_peak"] = round(v["ssd_gb_per_s"] / peak["gb_per_s"], 3)
        out["disk_peak"] = peak
        out["model"] = (f"{args.layers} layers, hidden 2048, moe_inter 512, E=256, top-8, fp8 "
                        "128x128 block scales, random-init routers; the 256 x layers experts are "
                        "drawn from a pool of 64 seeded experts (every (layer, expert) is its own "
                        "record in the RAM tier and the paging file); CACHE_SLOTS=32, "
                        "RAM_SLOTS=128 compressed at pitch 0.89, O_DIRECT paging file")
    finally:
        if m is not None:
            m.release()
        if os.path.exists(path):
            os.unlink(path)
    return out


def prefill_configs(args, device) -> dict:
    """Config 5 in the default line: the 2048-token prefill through ``--c5-layers`` layers
    on the compressed SSD tier (R=128 + paging file) and on a RAM-resident compressed tier
    (R=E), each with chunk k+1's copies overlapped with chunk k's MoE and serial, with the
    SSD rate against the disk's own peak."""
    import copy as _copy

    base = os.environ.get("XP_BENCH_DIR", "/tmp")
    path = os.path.join(base, f"xpager_bench_c5_{os.getpid()}.bin")
    a = _copy.copy(args)
    a.layers = args.c5_layers
    try:
        out = run_prefill(a, device, path)
        if os.path.exists(path):
            from vllm_expert_pager.codec import pitch_of
            from vllm_expert_pager import synthetic

            record = sum(pitch_of(r * c, 0.89, 4096) for r, c in synthetic.SHAPES.values())
            peak = disk_peak(path, record)
            out["disk_peak"] = peak
            if "gb_per_s" in peak:
                for mode in ("overlap", "serial"):
                    v = out["ssd"][mode]
                    v["ssd_frac_of_disk_peak"] = round(v["ssd_gb_per_s"] / peak["gb_per_s"], 3)
    finally:
        if os.path.exists(path):
            os.unlink(path)
    out["layers"] = a.layers
    out["workload"] = ("2048-token prefill, uniform top-8 over E=256, CACHE_SLOTS=32, "
                       "WORKING_ROWS=64 (5 chunks per layer), the 40-layer model's layers")
    return out


def link_info(device, store, world: int, rank: int, concurrent: float) -> list[dict] | dict:
    """This rank's host link: the pinned->device copy bandwidth with the link idle (the
    ranks measure one after another), the figure with all ranks copying at once, the
    NUMA node of its RAM tier and its GPU's PCI address.  Gathered to rank 0."""
    idle = None
    for r in range(world):
        barrier(world)
        if r == rank:
            idle = measure_h2d_peak(device, 1, reps=3)
    barrier(world)
    p = torch.cuda.get_device_properties(device)
    info = {"rank": rank, "pci_bus_id": f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:"
                                       f"{p.pci_device_id:02x}.0",
            "ram_tier_numa_node": store.numa_node, "h2d_idle_gb_s": round(idle, 3),
            "h2d_concurrent_gb_s": round(concurrent, 3)}
    if world == 1:
        return [info]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, info)
    return out


def run_links(args) -> None:
    """--workload links: the host side of the replicas.  Every rank allocates a pinned
    buffer on its GPU's NUMA node and measures the copy-engine pinned->device bandwidth
    (1 GiB, best of 6) alone (ranks one after another) and with every rank copying at
    once; rank 0 prints the per-rank figures and their sums, so that GPU subsets chosen
    with CUDA_VISIBLE_DEVICES (two behind one PCIe switch, two behind different ones)
    show which shared resource caps the aggregate: a switch uplink or host memory."""
    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    from vllm_expert_pager import store as store_mod

    class _Tier:  # what link_info reads from a Store
        numa_node = store_mod.numa_node_of(device)

    concurrent = measure_h2d_peak(device, world)
    links = link_info(device, _Tier, world, rank, concurrent)
    if rank == 0:
        print(json.dumps({"workload": "links", "n_gpus": world, "links": links,
                          "sum_idle_gb_s": round(sum(x["h2d_idle_gb_s"] for x in links), 3),
                          "sum_concurrent_gb_s": round(sum(x["h2d_concurrent_gb_s"]
                                                           for x in links), 3),
                          "visible": os.environ.get("CUDA_VISIBLE_DEVICES")}), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_json_subprocess(argv: list[str], timeout: float) -> dict:
    """Run ``bench.py`` with ``argv`` in a fresh process (no torchrun variables) and
    return the last JSON line it printed, or {"unavailable": why}."""
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT")}
    try:
        p = subprocess.run([sys.executable, os.path.abspath(__file__), *argv], env=env,
                           capture_output=True, text=True, timeout=timeout)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"timed out after {timeout:.0f} s"}
    for ln in reversed(p.stdout.strip().splitlines()):
        if ln.startswith("{"):
            return json.loads(ln)
    return {"unavailable": f"rc {p.returncode}: {p.stderr.strip()[-300:]}"}


def run_model_workload(args):
    """--workload model|compressed|prefill: configs 3, 4 and 5 (one JSON line each)."""
    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    base = os.environ.get("XP_BENCH_DIR", "/tmp")
    path = os.path.join(base, f"xpager_bench_{rank}.bin")
    try:
        if args.workload == "model":
            res = {"config3": run_model_decode(args, device, False, 256, 1, args.tokens)}
        elif args.workload == "compressed":
            res = {"config4_batch1": run_model_decode(args, device, True, 128, 1, args.tokens,
                                                      path),
                   "config4_batch8": run_model_decode(args, device, True, 128, 8,
                                                      max(args.tokens // 4, 8), path)}
        else:
            res = {"config5": run_prefill(args, device, path)}
            res["config5"]["layers"] = args.layers
        if os.path.exists(path):
            from vllm_expert_pager import synthetic
            from vllm_expert_pager.codec import pitch_of

            record = sum(pitch_of(r * c, 0.89, 4096) for r, c in synthetic.SHAPES.values())
            peak = disk_peak(path, record)

            def annotate(d):
                for v in d.values():
                    if isinstance(v, dict):
                        annotate(v)
                if "ssd_gb_per_s" in d and "gb_per_s" in peak:
                    d["ssd_frac_of_disk_peak"] = round(d["ssd_gb_per_s"] / peak["gb_per_s"], 3)

            annotate(res)
            res["disk_peak"] = peak
    finally:
        if os.path.exists(path):
            os.unlink(path)
    res["rank"] = rank
    print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def bench_encode(device, copies: int = 8, reps: int = 3) -> dict:
    """GPU encoder (xp_encode_rows) on config-1 rows: the 8 experts' rows of each name,
    repeated ``copies`` times, one batched call per name; raw bytes / wall time of the
    two calls (each reads the record sizes back to check the pitch), best of ``reps``."""
    from vllm_expert_pager import codec, synthetic

    experts = synthetic.fp8_experts(8, seed=0)
    batches = []
    for name in synthetic.SHAPES:
        rows = torch.stack([synthetic.row_bytes(ex[name][0]) for ex in experts] * copies)
        batches.append((rows.to(device), codec.pitch_of(rows.shape[1], 0.89, 4096)))
    raw = sum(b.numel() for b, _ in batches)
    for b, p in batches:  # warm-up
        codec.encode_rows(b, p)
    torch.cuda.synchronize()
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        for b, p in batches:
            codec.encode_rows(b, p)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return {"value": round(raw / best / 1e9, 2), "unit": "GB/s", "raw_bytes": raw,
            "rows": sum(b.shape[0] for b, _ in batches),
            "how": "encode_rows of 8 x config-1 experts per name, repeated "
                   f"{copies}x, raw bytes / wall time incl. the pitch check, best of {reps}"}


def bench_acquire(device, steps: int = 1024) -> dict:
    """Both LRU table updates of a decode step (xp_acquire_pair) on the config-2 trace:
    device time per launch, and the reference algorithm's port on one host core."""
    from oracle.table import OracleTable
    from vllm_expert_pager import synthetic
    from vllm_expert_pager.acquire import AcquirePair
    from vllm_expert_pager.table import ExpertTable

    trace = synthetic.zipf_trace(TRACE_STEPS, E, TOPK, 1.1, layer=0)
    vram, ram = ExpertTable(E, S, device), ExpertTable(E, R, device)
    ram.slot_of[:R] = ram.experts[:R]
    ram.expert_in[:R] = ram.experts[:R]
    pair = AcquirePair(vram, ram)
    dtrace = trace.to(device)
    for i in range(64):
        pair(dtrace[i])
    # A launch takes a few microseconds on the GPU but longer to enqueue from
    # Python, so time `steps` launches replayed from one CUDA graph.
    s = torch.cuda.Stream(device=device)
    s.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for i in range(steps):
                pair(dtrace[64 + i])
    torch.cuda.synchronize()
    us = sorted(timed(graph.replay) * 1e3 / steps for _ in range(5))
    del graph
    ov, orr = OracleTable(E, S), OracleTable(E, R)
    orr.warm(R)
    tr = trace.numpy()
    t0 = time.perf_counter()
    for i in range(steps):
        ov.acquire(tr[i])
        orr.acquire(tr[i])
    cpu_us = (time.perf_counter() - t0) / steps * 1e6
    return {"us_per_launch": round(us[len(us) // 2], 2),
            "how": f"{steps} launches replayed from a CUDA graph, median of 5 replays",
            "cpu_port_us_per_step": round(cpu_us, 1), "tables": "VRAM S=32 + RAM R=256, E=256"}


def codec_baselines(device) -> dict:
    """Config 1 (8 experts, pitch 0.89) on the host cores and on the GPU.

    * ``cpu_encode_port``: the reference's encoder restated in numpy (oracle/),
      one process -- the reference's own torch encoder cannot run here;
    * ``cpu_decode_port``: the reference's sequential decoder restated in C
      (oracle/decode.c) on all host threads;
    * ``native_encode``: this library's encoder (host, load time), all threads;
    * ``gpu_decode``: decode_ring_kernel on the same 16 records (8 rows per launch
      per name, 2 launches).
    All values are raw MB/s; every round trip is checked byte for byte.
    """
    from concurrent.futures import ThreadPoolExecutor

    from oracle import _lib as olib
    from oracle import codec as oc
    from vllm_expert_pager import codec, synthetic

    threads = os.cpu_count() or 1
    experts = synthetic.fp8_experts(8, seed=0)
    raws = [synthetic.row_bytes(ex[n][0]).numpy() for ex in experts for n in synthetic.SHAPES]
    total = sum(r.size for r in raws)
    t0 = time.perf_counter()
    recs = [oc.encode(r, oc.pitch_of(r.size, 0.89, 4096)) for r in raws]
    enc_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    for k in (0, 1):  # the w13 rows, then the w2 rows, each batch on all threads
        rs = [recs[i] for i in range(k, len(recs), 2)]
        out = olib.decode_rows(np.stack([r[0] for r in rs]), np.stack([r[1] for r in rs]),
                               raws[k].size, threads=threads)
        for i, o in zip(range(k, len(recs), 2), out):
            if not np.array_equal(o, raws[i]):
                raise SystemExit("oracle decode mismatch")
    dec_s = time.perf_counter() - t0

    def enc(r):
        return codec.encode(torch.from_numpy(r), codec.pitch_of(r.size, 0.89, 4096))

    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        nat = list(ex.map(enc, raws))
    nat_s = time.perf_counter() - t0
    for (a, _, _), (b, _) in zip(recs, nat):
        if not np.array_equal(a, b.numpy()):
            raise SystemExit("native encoder differs from the oracle")
    # GPU: 8 rows per launch per name.
    lut = torch.zeros((8, 2, 512), dtype=torch.uint8, device=device)
    stg, dst = [], []
    for k in (0, 1):
        rows = [nat[i] for i in range(k, len(nat), 2)]
        stg.append(torch.stack([r[0] for r in rows]).to(device))
        dst.append(torch.empty((8, raws[k].size), dtype=torch.uint8, device=device))
        for e, r in enumerate(rows):
            lut[e, k] = r[1].to(device)
    todo = torch.arange(8, dtype=torch.int64, device=device)
    no_cache = torch.full((8,), -1, dtype=torch.int64, device=device)
    for _ in range(3):
        codec.decode_rows(todo, todo, no_cache, stg, dst, lut)
    gpu_ms = timed(lambda: codec.decode_rows(todo, todo, no_cache, stg, dst, lut), reps=10)
    for k in (0, 1):
        for e in range(8):
            if not np.array_equal(dst[k][e].cpu().numpy(), raws[2 * e + k]):
                raise SystemExit("gpu decode mismatch")
    mb = total / 1e6
    return {"raw_mb": round(mb, 3), "threads": threads,
            "cpu_encode_port_mb_s": round(mb / enc_s, 1),
            "cpu_decode_port_mb_s": round(mb / dec_s, 1),
            "native_encode_mb_s": round(mb / nat_s, 1),
            "gpu_decode_mb_s": round(mb / (gpu_ms * 1e-3), 1),
            "record_ratio": round(sum(r[2] for r in recs) / total, 4)}


def cpu_port(trace: np.ndarray, steps: int, src_ptrs, slab, threads: int) -> tuple[float, float]:
    """The reference's algorithm on the host: both LRU tables + memcpy of the missed rows.

    Returns (seconds, bytes copied).
    """
    from oracle import _lib as olib
    from oracle.table import OracleTable

    vram, ram = OracleTable(E, S), OracleTable(E, R)
    ram.warm(R)
    moved = 0
    t0 = time.perf_counter()
    for i in range(steps):
        ids = trace[i % TRACE_STEPS]
        _, slot, todo = vram.acquire(ids)
        _, src, _ = ram.acquire(ids)
        m = todo[todo >= 0]
        if m.size:
            for k, (ptr, nbytes) in enumerate(src_ptrs):
                olib.copy_rows(ptr, nbytes, src[m], slab[k].ctypes.data, nbytes, slot[m], nbytes,
                               threads)
            moved += m.size * EXPERT_BYTES
    return time.perf_counter() - t0, moved


def time_planning(table_cls, syn, device, layers: int = 40, reps: int = 3) -> dict:
    """Working-path planning of one layer at config 5 (2048-token prefill, uniform top-8,
    E=256, S=32, R=128, W=64): ``need_mask``, the ``slot_of`` copy, ``seed`` and
    ``plan_chunks``, issued eagerly as ``_expert_pager_forward_working`` issues them
    (experts.py:500-511).  ``table_cls`` is this library's ``ExpertTable`` or the
    reference's (same methods); device time from the first launch to the last, host
    issue included, per layer."""
    e_, s_, r_, w_ = 256, 32, 128, 64
    ids = syn.uniform_routing(2048, e_, 8, seed=0).to(device)
    vram, ram = table_cls(e_, s_, device), table_cls(e_, r_, device)
    warm = syn.zipf_trace(64, e_, 8, 1.1, layer=0).to(device)
    for i in range(64):
        vram.acquire(warm[i])

    def plan():
        need = ram.need_mask(ids)
        before = ram.slot_of[:e_].clone()
        ram.seed(vram, ids, need)
        ram.plan_chunks(before, need, vram.slot_of[:e_], w_, 0, 40 * r_)

    for _ in range(3):
        plan()
    torch.cuda.synchronize()
    best = min(timed(lambda: [plan() for _ in range(layers)]) / layers for _ in range(reps))
    return {"ms_per_layer": round(best, 4),
            "how": f"{layers} layers back to back, eager, best of {reps}"}


def time_planning_fused(device, layers: int = 40, reps: int = 3) -> dict:
    """The same planning as ``time_planning`` through this library's one-launch
    ``WorkingPlan`` (xp_plan_working), which ``LayerPager`` uses."""
    from vllm_expert_pager import synthetic as syn
    from vllm_expert_pager.table import ExpertTable, WorkingPlan

    e_, s_, r_, w_ = 256, 32, 128, 64
    ids = syn.uniform_routing(2048, e_, 8, seed=0).to(device)
    vram, ram = ExpertTable(e_, s_, device), ExpertTable(e_, r_, device)
    warm = syn.zipf_trace(64, e_, 8, 1.1, layer=0).to(device)
    for i in range(64):
        vram.acquire(warm[i])
    planner = WorkingPlan(e_, w_, r_, s_, device)
    for _ in range(3):
        planner(ram, vram, ids, 0, 40 * r_)
    torch.cuda.synchronize()
    best = min(timed(lambda: [planner(ram, vram, ids, 0, 40 * r_) for _ in range(layers)])
               / layers for _ in range(reps))
    return {"ms_per_layer": round(best, 4),
            "how": f"{layers} layers back to back, eager, one launch each, best of {reps}"}


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _synthetic_by_path():
    """This repository's seeded generators (synthetic.py imports only torch), loaded by
    file so that the name ``vllm_expert_pager`` stays free for the reference install."""
    import importlib.util

    path = os.path.join(ROOT, "vllm-expert-pager_b200", "vllm_expert_pager", "synthetic.py")
    spec = importlib.util.spec_from_file_location("xp_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_reference_triton(args) -> None:
    """The reference's own GPU kernels (Triton, installed unmodified in baseline/_ref) on
    this GPU, on the inputs this bench gives its own kernels.

    * ``acquire_pair``: ``AcquirePair`` on the config-2 trace, 1024 launches replayed
      from a CUDA graph (as ``bench_acquire``);
    * ``decode_step_config2``: the stock decode step of ``forward_modular`` with an
      uncompressed RAM tier holding every expert -- ``AcquirePair``, ``gather_rows`` of
      the VRAM misses, ``gather_rows`` of the (empty) SSD list -- one CUDA graph per
      window of ``--window`` trace steps; GB/s = misses x 3 MiB / device time.  The
      first gather runs without ``fetch=``: with every expert in RAM the SSD list is
      empty and ``fetch=`` only adds a program that publishes nothing;
    * ``decode_k8`` / ``decode_k64``: ``decode_rows`` on config-1 records made by the
      reference's ``codec.encode`` (pitch 0.89), timed from a CUDA graph as
      ``bench_decode``.
    """
    line = {"impl": "reference", "workload": "reference-triton"}
    if not os.path.isdir(os.path.join(REF_DIR, "vllm_expert_pager")):
        line["unavailable"] = "baseline/_ref holds no install of the reference"
        print(json.dumps(line), flush=True)
        return
    sys.path.insert(0, REF_DIR)
    import vllm_expert_pager as refpkg

    if not os.path.abspath(refpkg.__file__).startswith(REF_DIR):
        raise SystemExit("vllm_expert_pager did not resolve to baseline/_ref")
    from vllm_expert_pager import codec as rcodec
    from vllm_expert_pager.acquire import AcquirePair
    from vllm_expert_pager.gather import as_rows, gather_rows
    from vllm_expert_pager.table import ExpertTable

    syn = _synthetic_by_path()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    trace = syn.zipf_trace(TRACE_STEPS, E, TOPK, 1.1, layer=0)
    dtrace = trace.to(device)

    def tables():
        vram, ram = ExpertTable(E, S, device), ExpertTable(E, R, device)
        ram.slot_of[:R] = ram.experts[:R]
        ram.expert_in[:R] = ram.experts[:R]
        return vram, ram, AcquirePair(vram, ram)

    # acquire_pair
    vram, ram, pair = tables()
    for i in range(64):
        pair(dtrace[i])
    steps = 1024
    s = torch.cuda.Stream(device=device)
    s.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for i in range(steps):
                pair(dtrace[64 + i])
    torch.cuda.synchronize()
    us = sorted(timed(graph.replay) * 1e3 / steps for _ in range(5))
    del graph
    kernels = {"acquire_pair": {"us_per_launch": round(us[len(us) // 2], 2),
                                "how": f"{steps} launches replayed from a CUDA graph, "
                                       "median of 5 replays"}}

    # decode step, config 2
    row = {n: r * c for n, (r, c) in syn.SHAPES.items()}
    src = [as_rows(torch.zeros((E, b), dtype=torch.uint8).pin_memory()) for b in row.values()]
    slab = [torch.zeros((S, b // 4), dtype=torch.int32, device=device) for b in row.values()]
    sw = [(r // 128) * (c // 128) for r, c in syn.SHAPES.values()]
    scale = [torch.zeros((E, w), dtype=torch.int32, device=device) for w in sw]
    scale_dst = [torch.zeros((S, w), dtype=torch.int32, device=device) for w in sw]
    vram, ram, pair = tables()

    def step(ids):
        todo, ssd = pair(ids)
        gather_rows(todo, pair.vram_slot, vram.no_cache, pair.ram_slot, 0, src, slab, slab,
                    None, scale, scale_dst)
        gather_rows(ssd, pair.vram_slot, vram.no_cache, pair.ram_slot, 0, src, slab, slab,
                    None, scale, scale_dst)

    W = args.window
    pos = 0
    for _ in range(args.warmup):
        for i in range(W):
            step(dtrace[(pos + i) % TRACE_STEPS])
        pos += W
    torch.cuda.synchronize()
    graphs = []
    for _ in range(args.steps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for i in range(W):
                    step(dtrace[(pos + i) % TRACE_STEPS])
        graphs.append(g)
        pos += W
    torch.cuda.synchronize()
    # Capture records the kernels without running them: the tables are where the
    # warm-up left them, and the replays below walk the captured windows in order.
    miss0 = int(vram.misses)

    def replay_all():
        for g in graphs:
            g.replay()

    ms = timed(replay_all)
    moved = (int(vram.misses) - miss0) * EXPERT_BYTES
    del graphs
    kernels["decode_step_config2"] = {
        "value": round(moved / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
        "ms_per_window": round(ms / args.steps, 3), "window": W, "windows": args.steps,
        "launches_per_step": 3, "how": "one CUDA graph per window, replayed back to back"}
    del src

    # decode_rows, config-1 records
    names = list(syn.SHAPES)
    gen = torch.Generator().manual_seed(0)
    experts = [syn.fp8_expert(gen) for _ in range(8)]
    distinct = 64
    raws = {n: [syn.row_bytes(ex[n][0]) for ex in experts] for n in names}
    raws_d = {n: [r.to(device) for r in raws[n]] for n in names}

    def encode_all():
        return {n: [rcodec.encode(r, rcodec.pitch_of(r.numel(), 0.89, 4096))
                    for r in raws_d[n]] for n in names}

    enc = encode_all()  # also the warm-up
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    enc = encode_all()
    torch.cuda.synchronize()
    enc_s = time.perf_counter() - t0
    raw_total = sum(r.numel() for n in names for r in raws[n])
    kernels["encode_config1"] = {
        "value": round(raw_total / enc_s / 1e9, 3), "unit": "GB/s",
        "how": "codec.encode (torch ops on the GPU) of the 16 config-1 rows, raw bytes / "
               "wall time, second pass"}
    used = 0
    for n in names:
        for (rec, _), r in zip(enc[n], raws[n]):
            G = r.numel() // (rcodec.CHUNK * rcodec.LANES)
            used += 4 * (G + 1) + r.numel() // 2 + 4 * int(rec[4 * G : 4 * G + 4].view(torch.int32))
    per_row = used / 8 + sum(raws[n][0].numel() for n in names) + 2 * 512
    stg = [torch.stack([enc[n][e % 8][0] for e in range(distinct)]) for n in names]
    dst = [torch.empty((distinct, raws[n][0].numel()), dtype=torch.uint8, device=device)
           for n in names]
    lut = torch.stack([torch.stack([enc[n][e % 8][1] for n in names])
                       for e in range(distinct)]).to(device)
    ident = torch.arange(distinct, dtype=torch.int64, device=device)
    no_cache = torch.full((distinct,), -1, dtype=torch.int64, device=device)
    peak, psrc = hbm_peak()
    for K in (8, 64):
        starts = list(range(0, distinct - K + 1, K))
        todos = [torch.arange(s0, s0 + K, dtype=torch.int64, device=device) for s0 in starts]

        views = [[x[s0 : s0 + K] for x in stg] for s0 in starts]

        def launch(i):
            j = i % len(starts)
            rcodec.decode_rows(todos[j], ident, no_cache, views[j], dst, lut)

        for i in range(4):
            launch(i)
        torch.cuda.synchronize()
        # Timed as bench_decode times this library's decoder: 48 launches captured in
        # a CUDA graph (the reference captures its decode path in graphs too), the
        # replay bracketed by events on its stream, best of 5.
        s = torch.cuda.Stream(device=device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                for i in range(48):
                    launch(i)
        torch.cuda.synchronize()
        best = None
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(s):
                a.record()
                graph.replay()
                b.record()
            torch.cuda.synchronize()
            t = a.elapsed_time(b) * 1e3 / 48
            best = t if best is None else min(best, t)
        del graph
        for n, d in zip(names, dst):
            if not torch.equal(d[K - 1].cpu(), raws[n][(K - 1) % 8]):
                raise SystemExit(f"reference decode mismatch ({n})")
        achieved = K * per_row / (best * 1e-6) / 1e9
        kernels[f"decode_k{K}"] = {"rows_per_launch": K, "us_per_launch": round(best, 2),
                                   "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                                   "frac": round(achieved / peak, 4), "peak_source": psrc,
                                   "how": "48 launches captured in a CUDA graph, replay timed "
                                          "with CUDA events on its stream, best of 5"}
    kernels["plan_config5"] = time_planning(ExpertTable, syn, device)
    line["kernels"] = kernels
    line["device"] = torch.cuda.get_device_name(device)
    print(json.dumps(line), flush=True)


def config2(W: int, world: int) -> dict:
    """The config of the headline line; both arms print this dict."""
    return {"workload": "config2: single-layer decode paging, E=256 x 3 MiB, CACHE_SLOTS=32, "
                        "RAM_SLOTS=256 raw, batch 1 top-8 Zipf(1.1), 4096-step trace",
            "window": W, "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (768 MiB pinned RAM tier read over the host link "
                  "per replica)"}


def reference_table_leg(trace: torch.Tensor, steps: int, ptrs, slab, threads: int,
                        table_cls) -> tuple[float, float]:
    """The reference's own decode-path tables on the host: its ``ExpertTable.acquire``
    (table.py:75-128, torch ops on CPU tensors, as the reference's tests run it) on the
    VRAM (S) and RAM (R) tables of every step, then a ``threads``-way memcpy of the
    missed rows from the RAM tier into the slab (the reference's gather is a GPU kernel;
    on the host the copy is a memcpy).  Returns (seconds, bytes copied)."""
    from oracle import _lib as olib

    cpu = torch.device("cpu")
    vram, ram = table_cls(E, S, cpu), table_cls(E, R, cpu)
    ram.slot_of[:R] = ram.experts[:R]
    ram.expert_in[:R] = ram.experts[:R]
    moved = 0
    t0 = time.perf_counter()
    for i in range(steps):
        ids = trace[i % TRACE_STEPS]
        _, slot, todo = vram.acquire(ids)
        _, src, _ = ram.acquire(ids)
        t = todo.numpy()
        m = t[t >= 0]
        if m.size:
            dst_rows, src_rows = slot.numpy()[m], src.numpy()[m]
            for k, (ptr, nbytes) in enumerate(ptrs):
                olib.copy_rows(ptr, nbytes, src_rows, slab[k].ctypes.data, nbytes, dst_rows,
                               nbytes, threads)
            moved += m.size * EXPERT_BYTES
    return time.perf_counter() - t0, moved


def reference_codec_leg(syn, codec_mod, threads: int = 8) -> dict:
    """The reference's ``codec.encode`` (codec.py:125-193, torch ops) of the 16 config-1
    rows on CPU tensors with ``threads`` torch threads: raw MB/s."""
    torch.set_num_threads(threads)
    experts = syn.fp8_experts(8, seed=0)
    raws = [syn.row_bytes(ex[n][0]) for ex in experts for n in syn.SHAPES]
    codec_mod.encode(raws[0], codec_mod.pitch_of(raws[0].numel(), 0.89, 4096))  # warm-up
    t0 = time.perf_counter()
    for r in raws:
        codec_mod.encode(r, codec_mod.pitch_of(r.numel(), 0.89, 4096))
    dt = time.perf_counter() - t0
    total = sum(r.numel() for r in raws)
    return {"encode_mb_s": round(total / dt / 1e6, 1), "threads": threads, "kind": "reference",
            "raw_mb": round(total / 1e6, 3),
            "how": "the reference's codec.encode of the 16 config-1 rows (8 experts, pitch "
                   "0.89) on CPU tensors"}


def reference_install():
    """The reference package installed under baseline/_ref, imported as
    ``vllm_expert_pager`` (only in processes that never import this repository's
    package), or None when it is not installed."""
    if not os.path.isdir(os.path.join(REF_DIR, "vllm_expert_pager")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import vllm_expert_pager as refpkg

    if not os.path.abspath(refpkg.__file__).startswith(REF_DIR):
        raise SystemExit("vllm_expert_pager did not resolve to baseline/_ref")
    return refpkg


def run_reference(args, world, rank):
    """--impl reference: the reference's own CPU code for the path on the host cores.

    Each step is one window of the config-2 trace through the reference's
    ``ExpertTable.acquire`` on both tables (installed unmodified in baseline/_ref) and a
    threaded memcpy of the missed rows (``reference_table_leg``).  Without the install,
    the numpy restatement of the same algorithm under oracle/ stands in (kind "port").
    The reference's ``codec.encode`` on config 1 is reported beside it."""
    if rank != 0:
        return
    syn = _synthetic_by_path()
    threads = os.cpu_count() or 1
    trace = syn.zipf_trace(TRACE_STEPS, E, TOPK, 1.1, layer=0)
    row = {n: r * c for n, (r, c) in syn.SHAPES.items()}
    src = {n: np.zeros((R, b), dtype=np.uint8) for n, b in row.items()}
    rng = np.random.default_rng(0)
    for n in src:
        src[n][:] = rng.integers(0, 256, src[n].shape, dtype=np.uint8)
    slab = [np.zeros((S, b), dtype=np.uint8) for b in row.values()]
    ptrs = [(src[n].ctypes.data, row[n]) for n in row]
    ref = reference_install()
    if ref is not None:
        import vllm_expert_pager.codec as rcodec
        from vllm_expert_pager.table import ExpertTable as RefTable

        torch.set_num_threads(threads)

        def leg(n):
            return reference_table_leg(trace, n, ptrs, slab, threads, RefTable)
        kind = "reference"
        what = (f"the reference's ExpertTable.acquire (baseline/_ref, torch on CPU tensors) on "
                f"both tables + {threads}-thread memcpy of the missed rows")
    else:
        tr = trace.numpy()

        def leg(n):
            return cpu_port(tr, n, ptrs, slab, threads)
        kind = "port"
        what = f"numpy restatement of the reference's tables + {threads}-thread memcpy"
    for _ in range(args.warmup):
        leg(args.window)
    secs, moved = 0.0, 0
    for _ in range(args.steps):
        sec, mv = leg(args.window)
        secs += sec
        moved += mv
    value = moved / secs / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * secs / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": config2(args.window, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": kind,
                         "sample": f"{args.steps} windows of {args.window} trace steps: {what}"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "tok_per_s": round(args.window * args.steps / secs, 1),
    }
    if ref is not None:
        line["codec_config1"] = reference_codec_leg(syn, rcodec)
        sample = min(args.window, 256)
        ps, pm = cpu_port(trace.numpy(), sample, ptrs, slab, threads)
        line["port"] = {"value": round(pm / ps / 1e9, 3), "unit": "GB/s", "cores": threads,
                        "sample": f"first {sample} trace steps: numpy restatement of the "
                                  "tables (oracle/) + the same memcpy"}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.workload == "reference-triton":
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference_triton(args)
        return
    if args.workload in ("model", "compressed", "prefill"):
        run_model_workload(args)
        return
    if args.workload == "links":
        run_links(args)
        return
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    device = torch.device("cuda", local)
    from vllm_expert_pager import gather as gather_mod

    if args.workload == "decode":
        for k in (8, 64):
            print(json.dumps({"decode": bench_decode(device, k)}), flush=True)
        print(json.dumps({"acquire_pair": bench_acquire(device)}), flush=True)
        print(json.dumps({"encode_gpu": bench_encode(device)}), flush=True)
        from vllm_expert_pager import synthetic
        from vllm_expert_pager.table import ExpertTable

        print(json.dumps({"plan_config5": time_planning(ExpertTable, synthetic, device)}),
              flush=True)
        print(json.dumps({"plan_config5_fused": time_planning_fused(device)}), flush=True)
        return
    if args.ctas:
        gather_mod.GATHER_CTAS = args.ctas
    skip = set(filter(None, args.skip.split(",")))
    store, pager, trace_cpu = build_workload(device)
    trace = trace_cpu.to(device)
    W = args.window
    peak = measure_h2d_peak(device, world)

    def window(w0: int, events=None):
        for i in range(W):
            pager.decode(trace[(w0 + i) % TRACE_STEPS], gather_events=events)

    # Warm-up windows (untimed), then K timed windows.
    pos = 0
    for _ in range(args.warmup):
        window(pos)
        pos += W
    torch.cuda.synchronize()
    miss0 = int(pager.vram.counters[2])
    events = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clocks:
        start.record()
        for _ in range(args.steps):
            window(pos, events)
            pos += W
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end)
    misses = int(pager.vram.counters[2]) - miss0
    moved = misses * EXPERT_BYTES
    gather_ms = sum(a.elapsed_time(b) for a, b in events)
    check_slab(store, pager)

    # e2e: the same windows through the public API, host-driven: every decode
    # step's routing ids come from pinned host memory (the kernel reads them over
    # the host link) and its expert_map goes back to pinned host memory (the
    # kernel writes it there) -- the inputs and the result cross the host link
    # every step, with no copy-engine transfer in between.
    host_trace = trace_cpu.pin_memory()
    host_map = torch.empty((E,), dtype=torch.int32, pin_memory=True)
    for i in range(W):  # warm-up window
        pager.decode(host_trace[(pos + i) % TRACE_STEPS], map_out=host_map)
    pos += W
    torch.cuda.synchronize()
    miss1 = int(pager.vram.counters[2])
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    e_start.record()
    for _ in range(args.steps):
        for i in range(W):
            pager.decode(host_trace[(pos + i) % TRACE_STEPS], map_out=host_map)
        pos += W
    e_end.record()
    torch.cuda.synchronize()
    barrier(world)
    e_ms = e_start.elapsed_time(e_end)
    e_moved = (int(pager.vram.counters[2]) - miss1) * EXPERT_BYTES

    value, _, ms_max = aggregate(moved, ms, world)
    e2e, _, _ = aggregate(e_moved, e_ms, world)
    achieved = moved / (gather_ms * 1e-3) / 1e9 if gather_ms > 0 else None
    links = link_info(device, store, world, rank, peak)

    kernels = {}
    if "kernels" not in skip:
        kernels = {"decode_k8": bench_decode(device, 8), "decode_k64": bench_decode(device, 64),
                   "acquire_pair": bench_acquire(device), "encode_gpu": bench_encode(device)}

    cpu = None
    if rank == 0 and world == 1 and "cpu" not in skip:
        threads = os.cpu_count() or 1
        names = list(store.pinned)
        ptrs = [(store.pinned[n].data_ptr(), store.pinned[n].shape[1] * 4) for n in names]
        slab = [np.zeros((S, store.pinned[n].shape[1] * 4), dtype=np.uint8) for n in names]
        tr = trace_cpu.numpy()
        sample = 256
        psecs, pm = cpu_port(tr, sample, ptrs, slab, threads)
        port = {"value": round(pm / psecs / 1e9, 3), "unit": "GB/s", "cores": threads,
                "kind": "port",
                "sample": f"first {sample} of {TRACE_STEPS} trace steps: numpy restatement of "
                          f"the LRU tables + {threads}-thread memcpy of the missed rows"}
        # The reference's own CPU code runs in a process of its own: both packages are
        # named vllm_expert_pager.
        ref = run_json_subprocess(["--impl", "reference", "--steps", "1", "--warmup", "1",
                                   "--window", str(sample)], timeout=900)
        if "value" in ref:
            cb = ref["cpu_baseline"]
            cpu = {"value": ref["value"], "unit": "GB/s", "cores": cb["cores"],
                   "kind": cb["kind"], "sample": cb["sample"], "port": port}
            if "codec_config1" in ref:
                cpu["codec_config1_reference"] = ref["codec_config1"]
        else:
            cpu = dict(port)
            cpu["reference_unavailable"] = ref.get("unavailable")
        cpu["codec_config1"] = codec_baselines(device)
    if rank == 0 and world == 1 and "reference_triton" not in skip:
        rt = run_json_subprocess(["--workload", "reference-triton", "--steps", "2", "--warmup",
                                  "1", "--window", str(W)], timeout=900)
        kernels["reference_triton"] = rt.get("kernels", rt)

    # Config 4 (compressed tier, SSD, gather + GPU decode) on one GPU: its paging file
    # takes ~29 GB of disk per rank, so the replica runs (N > 1) leave it out.
    configs = None
    if world == 1 and "compressed" not in skip:
        del pager, trace, host_trace
        store.release()
        store = None
        torch.cuda.empty_cache()
        configs = compressed_configs(args, device, peak)
    if world == 1 and "prefill" not in skip:
        if configs is None:
            configs = {}
            if store is not None:
                del pager, trace, host_trace
                store.release()
                store = None
                torch.cuda.empty_cache()
        configs["prefill_config5"] = prefill_configs(args, device)

    if rank == 0:
        steps_total = args.steps * W
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded fp8 experts generated on the device; Zipf(1.1) trace)",
            "config": config2(W, world),
            "tok_per_s": round(steps_total * world / (ms_max * 1e-3), 1),
            "miss_rate": round(misses / (steps_total * TOPK), 4),
            "e2e": {"value": round(e2e, 3), "unit": "GB/s", "h2d_bytes_per_step": W * TOPK * 4,
                    "d2h_bytes_per_step": W * E * 4},
            "roofline": {"bound": "host_link", "achieved": round(achieved, 3) if achieved else None,
                         "peak": round(peak, 3), "unit": "GB/s",
                         "frac": round(achieved / peak, 4) if achieved else None,
                         # From one ncu capture of three step-kernel launches of this
                         # workload (profiles/step_kernel_config2.md): DRAM bytes per
                         # launch, and the host-link bytes, which equalled the algorithmic
                         # bytes exactly (sysmem sectors x 32 B = misses x 3 MiB).
                         "traffic": 87000,
                         "traffic_unit": "DRAM bytes per launch",
                         "traffic_source": "ncu capture, profiles/step_kernel_config2.md "
                                           "(--set full, 3 launches): dram read + write",
                         "link_traffic_ratio": 1.0,
                         "link_traffic_source": "same capture: host-link read sectors x 32 B "
                                                "/ algorithmic bytes",
                         "kernel": "step_kernel (both table updates + the gather, one launch "
                                   "per decode step)",
                         "peak_source": "measured in bench.py: copy engine pinned->device, "
                                        "1 GiB, best of 6" + (
                                            f", all {world} ranks copying at once"
                                            if world > 1 else "") +
                                        " (MEASURED_PEAKS.json has no host-link figure)"},
            "links": links,
            "kernels": kernels,
            "gpu_launches": args.steps * W,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        if configs is not None:
            line["configs"] = configs
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
