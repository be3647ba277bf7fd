"""Benchmark of the expert-paging hot path on B200 (one JSON line on rank 0).

Workload ("single MoE layer decode paging"): 256 FP8
experts of 3 MiB (w13 [1024, 2048] + w2 [2048, 512], N(0, 0.02) quantised with
128x128 block scales), CACHE_SLOTS=32, RAM_SLOTS=256 uncompressed in pinned
host memory, batch-1 top-8 routing drawn Zipf(1.1) over a seeded permutation
(4096-step trace).  One bench step = one window of ``--window`` consecutive
decode steps of the trace (512 by default, the 512 decode tokens of config 3),
each running the decode paging path: acquire (VRAM + RAM tables), gather of the
missed rows from pinned RAM over the host link (+ the fused SSD-fetch CTA,
idle here since every expert is in RAM), gather of the SSD misses.

  value   = bytes paged in (misses x 3 MiB) / device time of the timed steps,
            summed over ranks (independent replicas, weak scaling)
  e2e     = the same through the public API with the routing ids copied from
            pinned host memory and expert_map copied back every decode step
  roofline: the gather kernel's achieved host-link GB/s (algorithmic bytes /
            CUDA-event duration of its launches) against the pinned-H2D copy
            bandwidth measured here with the copy engine

``--impl reference`` times the reference algorithm's CPU restatement (oracle/):
the LRU tables and a threaded memcpy of the same rows, on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
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
    p.add_argument("--workload", choices=["paging", "decode"], default="paging",
                   help="decode: only the decode-kernel measurement (for profiling)")
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


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


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


def measure_h2d_peak(device) -> float:
    """Copy-engine pinned->device bandwidth (GB/s), 1 GiB, best of 5."""
    n = 1 << 30
    src = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(n, dtype=torch.uint8, device=device)
    best = 0.0
    for _ in range(6):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, n / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
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


def bench_decode(device, rows_per_launch: int, launches: int = 24, distinct: int = 64,
                 reps: int = 3) -> dict:
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

    def launch(i):
        # launch i expands experts [s0, s0+K): staging row j holds expert s0+j, whose
        # raw row goes to dst row s0+j (dst_row = identity)
        s0 = starts[i % len(starts)]
        codec.decode_rows(todos[i % len(starts)], ident, no_cache,
                          [x[s0 : s0 + K] for x in stg], dst, lut_d)

    for i in range(4):
        launch(i)
    torch.cuda.synchronize()
    best = None
    for _ in range(reps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(launches)]
        for i in range(launches):
            ev[i][0].record()
            launch(i)
            ev[i][1].record()
        torch.cuda.synchronize()
        us = sum(a.elapsed_time(b) for a, b in ev) * 1e3 / launches
        best = us if best is None else min(best, us)
    for n, d, k in zip(names, dst, range(2)):  # parity spot check: expanded rows == raw rows
        for e in range(0, distinct, 17):
            if not torch.equal(d[e].cpu(), recs[n][e][1]):
                raise SystemExit(f"decode mismatch: expert {e} {n}")
    peak, src = hbm_peak()
    achieved = K * per_row / (best * 1e-6) / 1e9
    return {"rows_per_launch": K, "us_per_launch": round(best, 2),
            "algorithmic_bytes_per_launch": int(K * per_row), "achieved": round(achieved, 1),
            "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4), "bound": "hbm",
            "peak_source": src}


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


def run_reference(args, world, rank):
    """--impl reference: the CPU restatement of the reference path on the host cores."""
    if rank != 0:
        return
    from vllm_expert_pager import synthetic

    threads = os.cpu_count() or 1
    trace = synthetic.zipf_trace(TRACE_STEPS, E, TOPK, 1.1, layer=0).numpy()
    row = {n: r * c for n, (r, c) in synthetic.SHAPES.items()}
    src = {n: np.zeros((R, b), dtype=np.uint8) for n, b in row.items()}
    rng = np.random.default_rng(0)
    for n in src:
        src[n][:] = rng.integers(0, 256, src[n].shape, dtype=np.uint8)
    slab = [np.zeros((S, b), dtype=np.uint8) for b in row.values()]
    ptrs = [(src[n].ctypes.data, row[n]) for n in row]
    for _ in range(args.warmup):
        cpu_port(trace, args.window, ptrs, slab, threads)
    secs, moved = 0.0, 0
    for _ in range(args.steps):
        s, m = cpu_port(trace, args.window, ptrs, slab, threads)
        secs += s
        moved += m
    value = moved / secs / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * secs / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": "config2: single-layer decode paging, E=256 x 3 MiB, "
                   "CACHE_SLOTS=32, RAM_SLOTS=256 raw, batch 1 top-8 Zipf(1.1)",
                   "window": args.window},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{args.steps} windows of {args.window} trace steps"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "tok_per_s": round(args.window * args.steps / secs, 1),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    device = torch.device("cuda", local)
    from vllm_expert_pager import gather as gather_mod

    if args.workload == "decode":
        for k in (8, 64):
            print(json.dumps({"decode": bench_decode(device, k)}), flush=True)
        return
    if args.ctas:
        gather_mod.GATHER_CTAS = args.ctas
    store, pager, trace_cpu = build_workload(device)
    trace = trace_cpu.to(device)
    W = args.window
    peak = measure_h2d_peak(device)

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

    # e2e: the same windows through the public API with host routing ids and a
    # host copy of expert_map every decode step.
    host_trace = trace_cpu.pin_memory()
    ids_dev = torch.empty((TOPK,), dtype=torch.int32, device=device)
    host_map = torch.empty((E,), dtype=torch.int32, pin_memory=True)
    for i in range(W):  # warm-up window
        ids_dev.copy_(host_trace[(pos + i) % TRACE_STEPS], non_blocking=True)
        pager.decode(ids_dev)
        host_map.copy_(pager.expert_map, non_blocking=True)
    pos += W
    torch.cuda.synchronize()
    miss1 = int(pager.vram.counters[2])
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    e_start.record()
    for _ in range(args.steps):
        for i in range(W):
            ids_dev.copy_(host_trace[(pos + i) % TRACE_STEPS], non_blocking=True)
            pager.decode(ids_dev)
            host_map.copy_(pager.expert_map, non_blocking=True)
        pos += W
    e_end.record()
    torch.cuda.synchronize()
    barrier(world)
    e_ms = e_start.elapsed_time(e_end)
    e_moved = (int(pager.vram.counters[2]) - miss1) * EXPERT_BYTES

    ms_max = max_over_ranks(ms, world)
    e_ms_max = max_over_ranks(e_ms, world)
    total_moved = sum_over_ranks(moved, world)
    total_e = sum_over_ranks(e_moved, world)
    value = total_moved / (ms_max * 1e-3) / 1e9
    e2e = total_e / (e_ms_max * 1e-3) / 1e9
    achieved = moved / (gather_ms * 1e-3) / 1e9 if gather_ms > 0 else None

    kernels = {"decode_k8": bench_decode(device, 8), "decode_k64": bench_decode(device, 64)}

    cpu = None
    if rank == 0 and world == 1:
        threads = os.cpu_count() or 1
        names = list(store.pinned)
        ptrs = [(store.pinned[n].data_ptr(), store.pinned[n].shape[1] * 4) for n in names]
        slab = [np.zeros((S, store.pinned[n].shape[1] * 4), dtype=np.uint8) for n in names]
        tr = trace_cpu.numpy()
        sample = 256
        secs, cm = cpu_port(tr, sample, ptrs, slab, threads)
        cpu = {"value": round(cm / secs / 1e9, 3), "unit": "GB/s", "cores": threads,
               "kind": "port",
               "sample": f"first {sample} of {TRACE_STEPS} trace steps: numpy LRU tables + "
                         f"{threads}-thread memcpy of the missed rows"}

    if rank == 0:
        steps_total = args.steps * W
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded fp8 experts generated on the device; Zipf(1.1) trace)",
            "config": {"workload": "config2: single-layer decode paging, E=256 x 3 MiB, "
                       "CACHE_SLOTS=32, RAM_SLOTS=256 raw, batch 1 top-8 Zipf(1.1), 4096-step "
                       "trace", "window": W, "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (768 MiB pinned RAM tier read over the host "
                             "link per replica)"},
            "tok_per_s": round(steps_total * world / (ms_max * 1e-3), 1),
            "miss_rate": round(misses / (steps_total * TOPK), 4),
            "e2e": {"value": round(e2e, 3), "unit": "GB/s", "h2d_bytes_per_step": W * TOPK * 4,
                    "d2h_bytes_per_step": W * E * 4},
            "roofline": {"bound": "host_link", "achieved": round(achieved, 3) if achieved else None,
                         "peak": round(peak, 3), "unit": "GB/s",
                         "frac": round(achieved / peak, 4) if achieved else None, "traffic": None,
                         "kernel": "gather_kernel",
                         "peak_source": "measured in bench.py: copy engine pinned->device, "
                                        "1 GiB, best of 6 (MEASURED_PEAKS.json has no host-link "
                                        "figure)"},
            "kernels": kernels,
            "gpu_launches": args.steps * W * 3,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
