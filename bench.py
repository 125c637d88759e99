#!/usr/bin/env python
"""Benchmark of the fused Y = A x dequant(X_int8) SpMM (the TCC-SpMM hot path) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config powerlaw128] [--impl tcc|reference]

A step is one launchSpmmInt8 call over the whole matrix (N>1: every rank runs its
contiguous, load-balanced task range of the same matrix, X replicated, Y rows owned per rank;
no collective on the data path). One process per GPU; for N>1 launch with torchrun.

Printed (rank 0, one JSON line):
  value      nnz*F/s of the whole job, device-timed (CUDA events, max over ranks), inputs
             resident in HBM; inputs are larger than L2 (no flush needed)
  e2e        the same metric through the public API with host buffers: every step copies
             packed X + scales host->device (pinned) and reads this rank's Y rows back
  roofline   algorithmic bytes of one call (format arrays once, one F-byte row + scale per
             valid source slot, Y once) / average call duration, against the measured HBM
             copy bandwidth of MEASURED_PEAKS.json; traffic = ncu DRAM bytes per call when a
             profile summary exists under profiles/
  cpu_baseline  the CPU restatement of the reference arithmetic (oracle) on a bounded sample
             of windows, all host cores, rank 0 at N=1
--impl reference prints the reference arm: the CPU implementation of the path (the oracle
port; the reference ships no CPU SpMM) with all host cores, plus the reference's own GPU
kernel (compute_80 PTX JIT and sm_100a builds of its sources) timed on the same matrix.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HBM_FALLBACK_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="powerlaw128")
    p.add_argument("--impl", default="tcc", choices=["tcc", "reference"])
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--e2e-slices", type=int, default=8, help="window-aligned task slices per end-to-end step")
    p.add_argument("--e2e-x-allgather", action="store_true",
                   help="end to end on N > 1 ranks: each rank copies 1/N of packed X and the scales from the "
                        "host and an NCCL all-gather completes them (not yet run on GPUs)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-gpu-format", action="store_true", help="skip timing the GPU SW32 construction")
    p.add_argument("--no-assembly", action="store_true", help="skip the optional Y assembly across ranks")
    p.add_argument("--natural-order", action="store_true",
                   help="launch the tasks in format order instead of the balanced order (tcc_balance_tasks)")
    p.add_argument("--variant", default="default",
                   choices=["default", "generic", "persistent32", "persistent64", "tmem8"],
                   help="SpMM kernel (default: what launchSpmmInt8 runs)")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU-baseline sample time")
    return p.parse_args()


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return HBM_FALLBACK_GBS, "fallback"


def profile_traffic(config: str, variant: str, task_order: str, launch=None):
    """ncu DRAM bytes of one launch of this config's kernel (profiles/traffic.json), when the
    capture was taken of the same kernel variant, task order and launch shape (a changed kernel
    behind the same variant name has another shape, and its old capture is not used)."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    try:
        entry = json.loads(path.read_text()).get(config)
    except Exception:
        return None
    if not entry or entry.get("variant", "default") != variant or entry.get("task_order", "format") != task_order:
        return None
    if launch is not None and entry.get("launch") is not None and any(
            entry["launch"].get(k) != launch.get(k) for k in ("grid", "threads", "smem")):
        return None
    return entry


# ----------------------------------------------------------------------------------------
# nvidia-smi clock sampling during the timed region
# ----------------------------------------------------------------------------------------
CLOCK_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, device_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={CLOCK_QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(device_index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "power_w_max": max(power) if power else None}


# ----------------------------------------------------------------------------------------
# Workload
# ----------------------------------------------------------------------------------------
def shard_bytes(fmt, lo: int, hi: int, features: int) -> dict:
    """Algorithmic bytes of one call over tasks [lo, hi): format arrays of those tasks' panels
    once, one F-byte packed row + 4-byte scale per valid slot, the owned Y rows once."""
    t = fmt.tasks[lo:hi]
    if t.size == 0:
        return {"total": 0, "nnz": 0, "rows": 0}
    p0, p1 = int(t["begin"][0]), int(t["end"][-1])
    sw0, sw1 = int(t["sw"][0]), int(t["sw"][-1]) + 1
    ids = fmt.source_ids[8 * p0:8 * p1]
    valid = int(np.count_nonzero(ids != 0xFFFFFFFF))
    meta = fmt.source_metadata[8 * p0:8 * p1]  # values: one per set bit of the row masks
    nnz = int(np.bitwise_count(meta & np.uint64(0xFFFFFFFF)).sum())
    rows = min(fmt.rows, 32 * sw1) - 32 * sw0
    split = t[t["partial"] != 0xFFFFFFFF]
    a_bytes = (4 + 8) * 8 * (p1 - p0) + 4 * nnz + 4 * (p1 - p0) + 4 * 17 * (sw1 - sw0) + 28 * t.size
    a_bytes += 8 * 4 * len(np.unique(split["sw"])) + 4 * int(sum(bin(int(m)).count("1") for m in split["mask"]))
    x_bytes = valid * (features + 4)
    y_bytes = 4 * rows * features
    return {"total": int(a_bytes + x_bytes + y_bytes), "a_bytes": int(a_bytes), "x_bytes": int(x_bytes),
            "y_bytes": int(y_bytes), "nnz": nnz, "rows": int(rows), "valid_slots": valid, "panels": p1 - p0,
            "row_begin": 32 * sw0, "row_end": min(fmt.rows, 32 * sw1)}


def window_cuts(fmt, lo: int, hi: int, parts: int) -> list:
    """Boundaries (local to [lo, hi)) of about `parts` task slices, each starting at a window
    boundary so that no window is split between two slices."""
    sw = fmt.tasks["sw"][lo:hi]
    n = hi - lo
    cuts = [0]
    for k in range(1, parts):
        t = max(cuts[-1] + 1, (n * k) // parts)
        while 0 < t < n and sw[t] == sw[t - 1]:
            t += 1
        if t < n:
            cuts.append(t)
    cuts.append(n)
    return sorted(set(cuts))


def run_e2e(args, T, fmt, dm, lo, hi, packed, scales, F, device, stream, barrier, world, nnz_total):
    import torch
    import torch.distributed as dist

    cuts = window_cuts(fmt, lo, hi, args.e2e_slices)
    slices = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        sw0, sw1 = int(fmt.tasks["sw"][lo + a]), int(fmt.tasks["sw"][lo + b - 1]) + 1
        slices.append((dm.view(a, b), 32 * sw0, min(fmt.rows, 32 * sw1)))
    r0, r1 = slices[0][1], slices[-1][2]
    packed_h = packed.cpu().pin_memory()
    scales_h = scales.cpu().pin_memory()
    y_h = torch.empty((max(0, r1 - r0), F), dtype=torch.float32).pin_memory()
    gather = args.e2e_x_allgather and world > 1
    if gather:
        # Inputs padded to equal shards; this rank copies its shard from the host and the
        # all-gathers fill in the rest over NVLink (shards.gather_inputs).
        from tcc_spmm_b200 import shards

        padded, x0, x1 = shards.input_shard(fmt.cols, world, dist.get_rank())
        inputs = [(torch.empty(padded * F, dtype=torch.int8, device=device),
                   torch.empty(padded, dtype=torch.float32, device=device)) for _ in range(2)]
    else:
        inputs = [(packed, scales), (torch.empty_like(packed), torch.empty_like(scales))]
    ys = [torch.empty((fmt.rows, F), dtype=torch.float32, device=device) for _ in range(2)]
    ws = dm.workspace()
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    ev = lambda: torch.cuda.Event()
    in_ready = [ev(), ev()]
    in_free = [ev(), ev()]
    y_free = [ev(), ev()]

    def run(steps: int, start=None, stop=None):
        if start is not None:
            start.record(stream)
            h2d.wait_event(start)
        for i in range(steps + 1):
            b = i % 2
            if i < steps:  # inputs of step i (buffer b is free once step i-2 computed)
                if i >= 2:
                    h2d.wait_event(in_free[b])
                with torch.cuda.stream(h2d):
                    if gather:
                        # The collectives run after the shard copies on this stream, and the
                        # stream waits for them before recording in_ready.
                        shards.gather_inputs(inputs[b][0], inputs[b][1], packed_h, scales_h, F, non_blocking=True)
                    else:
                        inputs[b][0].copy_(packed_h, non_blocking=True)
                        inputs[b][1].copy_(scales_h, non_blocking=True)
                in_ready[b].record(h2d)
            if i == 0:
                continue
            j = i - 1  # compute step j and copy its rows back
            bj = j % 2
            stream.wait_event(in_ready[bj])
            if j >= 2:
                stream.wait_event(y_free[bj])
            for view, ra, rb in slices:
                T.launch_spmm_int8(view, inputs[bj][0], inputs[bj][1], ys[bj], fmt.rows, fmt.cols, F, ws,
                                   stream=stream, variant=args.variant)
                done = ev()
                done.record(stream)
                d2h.wait_event(done)
                if rb > ra:
                    with torch.cuda.stream(d2h):
                        y_h[ra - r0:rb - r0].copy_(ys[bj][ra:rb], non_blocking=True)
            in_free[bj].record(stream)
            y_free[bj].record(d2h)
        if stop is not None:
            stream.wait_stream(d2h)
            stop.record(stream)

    run(max(3, args.warmup))
    torch.cuda.synchronize()
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    run(args.steps, start, stop)
    torch.cuda.synchronize()
    ms = torch.tensor([start.elapsed_time(stop)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    step_ms = float(ms.item()) / args.steps
    return {"value": nnz_total * F / (step_ms / 1e3), "unit": "nnz*F/s", "ms_per_step": round(step_ms, 4),
            "h2d_bytes_per_step": int((x1 - x0) * (F + 4)) if gather else int(packed.numel() + 4 * scales.numel()),
            "d2h_bytes_per_step": int(4 * (r1 - r0) * F), "x_allgather": gather,
            "slices_per_step": len(slices), "gpu_launches": len(slices) * args.steps,
            "api": "tcc_launch_spmm_int8 (C ABI) via tcc_spmm_b200: DeviceMatrix.view slices, pinned host buffers, "
                   "copy streams (inputs and Y double-buffered)"}


def build_workload(config: str, threads: int, use_reference_format: bool = False):
    from tcc_spmm_b200 import workloads as W
    import tcc_spmm_b200 as T

    t0 = time.time()
    csr = W.generate(config, threads=threads)
    t1 = time.time()
    if use_reference_format:
        import oracle as O

        r = O.ref_convert_csr_to_sw32(csr.rows, csr.cols, csr.row_offsets, csr.source_ids, csr.values)
        fmt = T.Sw32HostFormat(csr.rows, csr.cols, r["window_offsets"], r["source_ids"], r["row_group_masks"],
                               r["source_metadata"], r["values"], r["bucket_offsets"],
                               np.ascontiguousarray(r["tasks"]).view(T.api.TASK_DTYPE).reshape(-1),
                               np.ascontiguousarray(r["reductions"]).view(T.api.REDUCE_DTYPE).reshape(-1),
                               r["partial_ids"], r["partial_count"])
    else:
        fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr, True, threads)
    t2 = time.time()
    return csr, fmt, {"generate_s": round(t1 - t0, 2), "convert_s": round(t2 - t1, 2)}


def time_gpu_format(T, csr, fmt, device, repeats: int = 5) -> dict:
    """The SW32 format and task plan built on this GPU from the CSR (not part of the metric):
    wall time of tcc_convert_csr_to_sw32_device (it synchronises to size its outputs; its
    synchronising size reads make it sensitive to host load), min and median of `repeats` after
    one untimed call, and whether every array equals the host builder's."""
    import torch

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).view(dtype)).to(device)

    ro, si, va = up(csr.row_offsets, np.int32), up(csr.source_ids, np.int32), up(csr.values, np.float32)
    T.convert_csr_to_sw32_device(csr.rows, csr.cols, ro, si, va)
    times = []
    for _ in range(repeats):
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        dev = T.convert_csr_to_sw32_device(csr.rows, csr.cols, ro, si, va)
        torch.cuda.synchronize(device)
        times.append(time.perf_counter() - t0)
    identical = not dev.differences(fmt)
    del dev, ro, si, va
    T.sw32_device_trim()
    torch.cuda.empty_cache()
    return {"gpu_convert_ms": round(1e3 * sorted(times)[len(times) // 2], 2), "gpu_convert_ms_min": round(1e3 * min(times), 2),
            "identical_to_host": identical}


def time_assembly(fmt, bounds, y, F: int, rank: int, world: int, device, barrier, repeats: int = 5) -> dict:
    """Optional assembly of the full Y on every rank (not part of the metric): one broadcast
    per owner range, all in one NCCL group, timed with CUDA events (max over ranks) after one untimed round,
    and checked by per-range checksums against the owners' own rows."""
    import torch
    import torch.distributed as dist
    from tcc_spmm_b200 import shards

    ranges = shards.owned_rows(fmt, bounds)
    shards.check_cover(ranges, fmt.rows)
    lo, hi = ranges[rank]
    own = torch.zeros(world, dtype=torch.float64, device=device)
    own[rank] = y[lo:hi].double().sum() if hi > lo else 0.0
    dist.all_reduce(own)
    shards.assemble_rows(y, ranges)
    torch.cuda.synchronize(device)
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(repeats):
        shards.assemble_rows(y, ranges)
    stop.record()
    torch.cuda.synchronize(device)
    ms = torch.tensor([start.elapsed_time(stop) / repeats], dtype=torch.float64, device=device)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    seen = torch.stack([y[b:e].double().sum() if e > b else torch.zeros((), dtype=torch.float64, device=device)
                        for b, e in ranges])
    ok = torch.tensor([int(bool(torch.equal(seen, own)))], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    received = max(shards.received_bytes(ranges, r, F) for r in range(world))
    t = float(ms.item())
    return {"ms": round(t, 3), "bytes_received_per_rank_max": received, "gbs_per_rank": round(received / t / 1e6, 1),
            "collective": "one broadcast per owner row range, all in one NCCL group",
            "checksums_match": bool(ok.item())}


def cpu_sample(fmt, features: int, target_seconds: float, threads: int, seed: int = 1):
    """Windows of a strided sample and their nnz, sized to about target_seconds of oracle work."""
    import oracle as O

    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, size=(fmt.cols, features), dtype=np.int8)
    s = (rng.random(fmt.cols, dtype=np.float32) * 0.05 + 0.001).astype(np.float32)
    windows = fmt.window_offsets.size - 1
    probe = np.arange(0, windows, max(1, windows // 2000), dtype=np.uint32)
    t0 = time.perf_counter()
    O.spmm(fmt, q, s, probe, threads=threads, with_bound=False)
    per_window = (time.perf_counter() - t0) / max(1, probe.size)
    count = int(min(windows, max(1, target_seconds / max(per_window, 1e-9))))
    stride = max(1, windows // count)
    sample = np.arange(0, windows, stride, dtype=np.uint32)
    per_slot = np.bitwise_count(fmt.source_metadata & np.uint64(0xFFFFFFFF)).astype(np.int64)
    per_window = np.add.reduceat(per_slot, 8 * fmt.window_offsets[:-1].astype(np.int64)) if per_slot.size else None
    empty = fmt.window_offsets[1:] == fmt.window_offsets[:-1]
    if per_window is not None:
        per_window[empty] = 0
    nnz = int(per_window[sample].sum()) if per_window is not None else 0
    return sample, nnz, q, s, stride


def time_cpu(fmt, features, sample, q, s, threads, repeats=1):
    import oracle as O

    best = None
    for _ in range(repeats):
        t0 = time.perf_counter()
        O.spmm(fmt, q, s, sample, threads=threads, with_bound=False)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return best


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------------------
# Arms
# ----------------------------------------------------------------------------------------
def run_tcc(args):
    import torch
    import torch.distributed as dist

    import tcc_spmm_b200 as T
    from tcc_spmm_b200 import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # Short enough that ranks waiting for a failed peer end with an error, long enough for
        # the host-side matrix generation and conversion that precede the first collective.
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    threads = max(1, host_threads() // world)
    cfg = W.CONFIGS[args.config]
    F = cfg.features
    csr, fmt, prep = build_workload(args.config, threads)
    bounds = T.partition_tasks(fmt, F, world)
    lo, hi = int(bounds[rank]), int(bounds[rank + 1])
    shard = shard_bytes(fmt, lo, hi, F)
    full = fmt.algorithmic_bytes(F)
    dm = T.DeviceMatrix(fmt, F, device, task_range=(lo, hi), balance=not args.natural_order, variant=args.variant)
    x = W.normal_features(fmt.cols, F, threads=threads)
    xd = torch.from_numpy(x).to(device)
    packed = torch.empty(fmt.cols * F, dtype=torch.int8, device=device)
    scales = torch.empty(fmt.cols, dtype=torch.float32, device=device)
    T.quantize_pack_features_int8(xd, packed, scales, fmt.cols, F)
    del xd
    y = torch.empty((fmt.rows, F), dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    view, ws = dm.view(), dm.workspace()

    def launch():
        T.launch_spmm_int8(view, packed, scales, y, fmt.rows, fmt.cols, F, ws, stream=stream, variant=args.variant)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(max(3, args.warmup)):
        launch()
    torch.cuda.synchronize()
    barrier()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps):
        launch()
    stop.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms_local = start.elapsed_time(stop)
    ms = torch.tensor([ms_local], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms_total = float(ms.item())
    ms_step = ms_total / args.steps
    nnz_total = int(csr.nnz)
    value = nnz_total * F / (ms_step / 1e3)

    # roofline of this rank's kernel (rank 0 reports its own; all ranks run the same kernel)
    peak, peak_kind = measured_peaks()
    launch_s = (ms_local / args.steps) / 1e3
    achieved = shard["total"] / launch_s / 1e9
    traffic = (profile_traffic(args.config, args.variant, "format" if args.natural_order else "balanced",
                               T.spmm_launch_shape(F, args.variant) if args.variant != "generic" else None)
               if world == 1 else None)

    # end to end through the public API with host buffers: every step copies packed X +
    # scales host -> device, runs the SpMM and copies this rank's Y rows device -> host. The
    # step's task range is launched in window-aligned slices so that the copy of finished Y rows
    # (copy stream) overlaps the remaining slices, and the next step's inputs are copied into a
    # second buffer while this step computes (inputs and Y are double-buffered).
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, T, fmt, dm, lo, hi, packed, scales, F, device, stream, barrier, world, nnz_total)

    # The format build synchronises several times: time it before the CPU baseline's host threads
    # run in this process.
    if not args.no_gpu_format:
        prep.update(time_gpu_format(T, csr, fmt, device))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle as O

        cores = host_threads()
        sample, snnz, q, s, stride = cpu_sample(fmt, F, args.cpu_seconds, cores)
        t = time_cpu(fmt, F, sample, q, s, cores)
        cpu = {"value": snnz * F / t, "unit": "nnz*F/s", "cores": cores, "kind": "port",
               "sample": f"every {stride}th 32-row window ({sample.size} windows, {snnz} nnz) of {args.config}, "
                         f"oracle/tcc_oracle.c restatement of the reference arithmetic, {t:.2f} s",
               "seconds": round(t, 3), "threads_reported": O.max_threads()}

    assembly = None
    if world > 1 and not args.no_assembly:
        assembly = time_assembly(fmt, bounds, y, F, rank, world, device, barrier)

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "nnz*F/s", "value": value, "unit": "nnz*F/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8->tf32 (fp32 accumulate)", "data": "synthetic",
        "config": {"workload": args.config, "description": cfg.description, "rows": fmt.rows, "nnz": nnz_total,
                   "features": F, "panels": fmt.panels, "valid_slots": full["x_bytes"] // (F + 4),
                   "tasks": int(fmt.tasks.size), "partial_count": fmt.partial_count,
                   "parallelism": f"task-range shards x{world}, X replicated, Y rows per rank",
                   "l2": "inputs larger than L2 (no flush)", "kernel": args.variant,
                   "task_order": "format order" if args.natural_order else "balanced for the launch grid",
                   "launch": T.spmm_launch_shape(F, args.variant) if args.variant != "generic" else None,
                   "prep": prep},
        "hbm_gbs_alg": round(full["total"] / (ms_step / 1e3) / 1e9, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": (traffic or {}).get("dram_bytes_per_launch"),
                     "alg_bytes_per_launch": shard["total"], "compulsory_bytes": full["compulsory"],
                     "merge_bytes": full["merge_bytes"]},
        "clocks": clocks, "gpu_launches": args.steps, "e2e": e2e, "cpu_baseline": cpu,
        "y_assembly": assembly,
    }
    print(json.dumps(line), flush=True)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from tcc_spmm_b200 import workloads as W
    import oracle as O

    cfg = W.CONFIGS[args.config]
    F = cfg.features
    cores = host_threads()
    csr, fmt, prep = build_workload(args.config, cores, use_reference_format=O.have_ref_host())
    per_step = min(5.0, 150.0 / max(1, args.steps + args.warmup))
    sample, snnz, q, s, stride = cpu_sample(fmt, F, per_step, cores)
    for _ in range(args.warmup):
        time_cpu(fmt, F, sample, q, s, cores)
    times = [time_cpu(fmt, F, sample, q, s, cores) for _ in range(args.steps)]
    t = sum(times) / len(times)
    value = snnz * F / t
    ref_kernel = None
    try:
        ref_kernel = time_reference_kernel(fmt, F, args)
    except Exception as exc:  # the GPU part is informational only
        ref_kernel = {"error": str(exc)[:200]}
    line = {"metric": "nnz*F/s", "value": value, "unit": "nnz*F/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * t * csr.nnz / max(1, snnz), 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8->tf32 (fp32 accumulate)",
            "data": "synthetic",
            "config": {"workload": args.config, "description": cfg.description, "rows": fmt.rows, "nnz": int(csr.nnz),
                       "features": F, "format_from": "reference convertCsrToSw32 (oracle/_ref)"
                       if O.have_ref_host() else "tcc convertCsrToSw32 (byte-identical)", "prep": prep},
            "cpu_baseline": {"value": value, "unit": "nnz*F/s", "cores": cores, "kind": "port",
                             "sample": f"every {stride}th 32-row window ({sample.size} windows, {snnz} nnz); the "
                                       "reference ships no CPU SpMM, this is the oracle restatement of its arithmetic"},
            "e2e": {"value": value, "unit": "nnz*F/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_gpu_kernel": ref_kernel}
    print(json.dumps(line), flush=True)


def time_reference_kernel(fmt, F, args):
    """The reference's own kernel (oracle/_ref) on the same matrix, CUDA-event timed."""
    import ctypes

    import torch

    import oracle as O
    import tcc_spmm_b200 as T
    from tcc_spmm_b200 import workloads as W

    if not torch.cuda.is_available() or not O.have_ref_cuda("sm80"):
        return None
    dm = T.DeviceMatrix(fmt, F, "cuda")
    x = torch.from_numpy(W.normal_features(fmt.cols, F)).cuda()
    out = {}
    for tag in ("sm80", "sm100a"):
        if not O.have_ref_cuda(tag):
            continue
        ref = O.ref_cuda(tag)
        stream = torch.cuda.current_stream().cuda_stream
        q = torch.empty(fmt.cols * F, dtype=torch.int8, device="cuda")
        p = torch.empty_like(q)
        s = torch.empty(fmt.cols, dtype=torch.float32, device="cuda")
        ref.quantize(x.data_ptr(), q.data_ptr(), s.data_ptr(), fmt.cols, F, stream)
        ref.pack(q.data_ptr(), p.data_ptr(), fmt.cols, F, stream)
        y = torch.empty((fmt.rows, F), device="cuda")
        view = dm.view()
        ws = dm.workspace()
        args_ = (ctypes.addressof(view), p.data_ptr(), s.data_ptr(), y.data_ptr(), fmt.rows, fmt.cols, F,
                 ws.partials.data_ptr() if ws.partials is not None else 0,
                 ws.counters.data_ptr() if ws.counters is not None else 0, stream)
        for _ in range(max(3, args.warmup)):
            ref.launch_spmm_int8(*args_)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            ref.launch_spmm_int8(*args_)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        out[tag] = {"ms_per_call": round(ms, 4), "value": fmt.nnz * F / (ms / 1e3),
                    "build": "compute_80 PTX (JIT)" if tag == "sm80" else "sm_100a SASS"}
    return out


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_tcc(args)


if __name__ == "__main__":
    main()
