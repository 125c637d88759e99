#!/usr/bin/env python
"""Benchmark of the fused Y = A x dequant(X_int8) SpMM (the TCC-SpMM hot path) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config powerlaw128] [--impl tcc|reference]

A step is one launchSpmmInt8 call over the whole matrix (N>1: every rank runs its contiguous,
load-balanced task range of the same matrix, X replicated, Y rows owned per rank; no collective
on the data path). One process per GPU; for N>1 launch with torchrun.

Every rank builds the workload on its GPU: the matrix is generated (R-MAT on the GPU, the other
configurations on the host and copied up), and the SW32 format and task plan are built from the
device CSR by tcc_convert_csr_to_sw32_device (byte-identical to the host builder).

Printed (rank 0, one JSON line):
  value      nnz*F/s of the whole job: K steps between CUDA events on the launching stream,
             barrier + synchronize on both sides, max over ranks; inputs resident in HBM and
             larger than L2 (no flush). timing.median_batch_ms is the reference's method
             (src/main.cu:30-51): the median of 5 event-timed batches of the K steps
  e2e        the same metric through the public API with host buffers: every step copies
             packed X + scales host->device (pinned; on N>1 ranks each copies 1/N and an NCCL
             all-gather completes them) and reads this rank's Y rows back
  roofline   algorithmic bytes of one call (format arrays once, one F-byte row + scale per valid
             source slot, Y once) / average call duration, against the measured HBM copy
             bandwidth of MEASURED_PEAKS.json; traffic = ncu DRAM bytes per call when a profile
             summary of the same kernel exists under profiles/
  per_config the other BASELINE configurations (F256, load-balance stress, R-MAT scale 24) on the
             same ranks, each with ms per call, nnz*F/s and roofline fraction
  quantize_pack  the one-pass quantize + pack of the headline X (timed separately, as the
             reference does), with its HBM fraction
  cpu_baseline   the CPU restatement of the reference arithmetic (oracle) on a bounded sample of
             windows, all host cores, rank 0 at N=1; cpu_baseline_1t the same on one core
--impl reference prints the reference arm: the CPU implementation of the path (the oracle port;
the reference ships no CPU SpMM) with all host cores, plus the reference's own GPU kernel
(compute_80 PTX JIT and sm_100a builds of its sources) timed on the same matrix, uploaded with
plain torch (this library is not loaded).
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
PER_CONFIG_DEFAULT = "powerlaw256,stress,rmat"
X_SEED = 20261202


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--config", default="powerlaw128")
    p.add_argument("--impl", default="tcc", choices=["tcc", "reference"])
    p.add_argument("--per-config", default=PER_CONFIG_DEFAULT,
                   help="comma-separated further configurations timed after the headline ('' for none)")
    p.add_argument("--per-config-steps", type=int, default=50)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--e2e-slices", type=int, default=8, help="window-aligned task slices per end-to-end step")
    p.add_argument("--e2e-x-allgather", default="auto", choices=["auto", "on", "off"],
                   help="end to end on N > 1 ranks: each rank copies 1/N of packed X and the scales from the host "
                        "and an NCCL all-gather completes them (auto: on when N > 1)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-assembly", action="store_true", help="skip the optional Y assembly across ranks")
    p.add_argument("--natural-order", action="store_true",
                   help="launch the tasks in format order instead of the balanced order (tcc_balance_tasks)")
    p.add_argument("--equal-count-order", action="store_true",
                   help="balanced order with equal task counts per CTA (tcc_balance_tasks) instead of the one "
                        "weighted by resident-CTA speed (tcc_balance_tasks_padded)")
    p.add_argument("--variant", default="default", choices=["default", "generic", "persistent32", "persistent64", "tmem8"],
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


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def workload_config(name: str, rows: int, nnz: int, features: int, panels: int, valid_slots: int, tasks: int,
                    partial_count: int) -> dict:
    """The `config` of both arms: the workload's identity only (the arms print the same dict)."""
    from tcc_spmm_b200 import workloads as W

    return {"workload": name, "description": W.CONFIGS[name].description, "rows": int(rows), "nnz": int(nnz),
            "features": int(features), "panels": int(panels), "valid_slots": int(valid_slots), "tasks": int(tasks),
            "partial_count": int(partial_count), "l2": "inputs larger than L2 (no flush)", "data": "synthetic, seeded"}


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
# Workload built on the device
# ----------------------------------------------------------------------------------------
def range_bytes(tasks, lo: int, hi: int, rows: int, cols: int, features: int, partial_count: int, valid_in,
                nnz_in) -> dict:
    """Algorithmic bytes of one call over tasks [lo, hi) of the natural order: the format arrays
    of those tasks' panels and windows once, one F-byte packed row + 4-byte scale per valid slot,
    the owned Y rows once. valid_in(p0, p1) counts the valid slots of panels [p0, p1), nnz_in(r0,
    r1) the nonzeros of rows [r0, r1). Over all tasks this is Sw32HostFormat.algorithmic_bytes."""
    t = tasks[lo:hi]
    if t.size == 0:
        return {"total": 0, "nnz": 0, "rows": 0}
    p0, p1 = int(t["begin"][0]), int(t["end"][-1])
    sw0, sw1 = int(t["sw"][0]), int(t["sw"][-1]) + 1
    r0, r1 = 32 * sw0, min(rows, 32 * sw1)
    valid = valid_in(p0, p1)
    nnz = nnz_in(r0, r1)
    split = t[t["partial"] != 0xFFFFFFFF]
    a_bytes = (4 + 8) * 8 * (p1 - p0) + 4 * nnz + 4 * (p1 - p0) + 4 * 17 * (sw1 - sw0) + 28 * t.size
    a_bytes += 8 * 4 * len(np.unique(split["sw"])) + 4 * int(np.bitwise_count(split["mask"]).sum())
    x_bytes = valid * (features + 4)
    y_bytes = 4 * (r1 - r0) * features
    return {"total": int(a_bytes + x_bytes + y_bytes), "a_bytes": int(a_bytes), "x_bytes": int(x_bytes),
            "y_bytes": int(y_bytes), "nnz": nnz, "rows": r1 - r0, "valid_slots": valid, "panels": p1 - p0,
            "row_begin": r0, "row_end": r1,
            "compulsory": int(a_bytes + 4 * cols + cols * features + y_bytes),
            "merge_bytes": int(2 * 4 * 8 * features * partial_count)}


class DeviceWorkload:
    """One configuration's matrix on this rank's GPU: the device CSR, the SW32 format and task
    plan built from it on the GPU, and host copies of the tasks and row-group masks (for the
    partition, the balanced order and the byte counts)."""

    def __init__(self, name: str, device, threads: int):
        import torch

        import tcc_spmm_b200 as T
        from tcc_spmm_b200 import workloads as W

        self.name = name
        t0 = time.perf_counter()
        self.csr = W.generate_device(name, device, threads=threads)
        torch.cuda.synchronize(device)
        t1 = time.perf_counter()
        self.dfmt = T.convert_csr_to_sw32_device(self.csr.rows, self.csr.cols, self.csr.row_offsets,
                                                 self.csr.source_ids, self.csr.values)
        torch.cuda.synchronize(device)
        t2 = time.perf_counter()
        self.rows, self.cols, self.nnz = self.dfmt.rows, self.dfmt.cols, self.csr.nnz
        self.tasks = self.dfmt.tasks.cpu().numpy().view(np.uint32).view(T.api.TASK_DTYPE)
        self.row_group_masks = self.dfmt.row_group_masks.cpu().numpy().view(np.uint32)
        self.panels = int(self.row_group_masks.size)
        self.partial_count = self.dfmt.partial_count
        self.valid_slots = int((self.dfmt.source_ids != -1).sum().item())
        self.prep = {"generate_s": round(t1 - t0, 2), "gpu_convert_ms": round(1e3 * (t2 - t1), 1),
                     "generated_on": "gpu" if W.CONFIGS[name].kind == "rmat" else "host"}

    def config(self, features: int, name: str | None = None) -> dict:
        return workload_config(name or self.name, self.rows, self.nnz, features, self.panels, self.valid_slots,
                               self.tasks.size, self.partial_count)

    def bytes(self, lo: int, hi: int, features: int) -> dict:
        """range_bytes of tasks [lo, hi), counted on the device arrays."""
        ro = self.csr.row_offsets
        return range_bytes(self.tasks, lo, hi, self.rows, self.cols, features, self.partial_count,
                           lambda p0, p1: int((self.dfmt.source_ids[8 * p0:8 * p1] != -1).sum().item()),
                           lambda r0, r1: int(ro[r1].item()) - int(ro[r0].item()))

    def device_matrix(self, features: int, task_range, balance: bool, variant: str, weighted: bool = True):
        return self.dfmt.device_matrix(features, task_range=task_range, balance=balance, variant=variant,
                                       host_tasks=self.tasks, host_masks=self.row_group_masks,
                                       weighted_order=weighted)


def device_inputs(T, cols: int, features: int, device, seed: int = X_SEED):
    """Seeded N(0,1) features on the device, quantized and packed by the one-pass kernel."""
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    x = torch.randn((cols, features), generator=gen, device=device, dtype=torch.float32)
    packed = torch.empty(cols * features, dtype=torch.int8, device=device)
    scales = torch.empty(cols, dtype=torch.float32, device=device)
    T.quantize_pack_features_int8(x, packed, scales, cols, features)
    return x, packed, scales


def timed_batches(launch, steps: int, stream, batches: int = 5):
    """Event times (ms) of `steps` launches split into `batches` consecutive batches on
    `stream` (events between batches): (total ms, per-batch ms per launch)."""
    import torch

    sizes = [steps // batches + (1 if i < steps % batches else 0) for i in range(batches)]
    sizes = [s for s in sizes if s > 0]
    events = [torch.cuda.Event(enable_timing=True) for _ in range(len(sizes) + 1)]
    events[0].record(stream)
    for i, n in enumerate(sizes):
        for _ in range(n):
            launch()
        events[i + 1].record(stream)
    torch.cuda.synchronize()
    per = [events[i].elapsed_time(events[i + 1]) / n for i, n in enumerate(sizes)]
    return events[0].elapsed_time(events[-1]), per


# ----------------------------------------------------------------------------------------
# End to end through the public API with host buffers
# ----------------------------------------------------------------------------------------
def window_cuts(tasks, lo: int, hi: int, parts: int) -> list:
    """Boundaries (local to [lo, hi)) of about `parts` task slices, each starting at a window
    boundary so that no window is split between two slices."""
    sw = tasks["sw"][lo:hi]
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


def run_e2e(args, T, wl, dm, lo, hi, packed, scales, F, device, stream, barrier, world, gather):
    import torch
    import torch.distributed as dist

    cuts = window_cuts(wl.tasks, lo, hi, args.e2e_slices)
    slices = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        sw0, sw1 = int(wl.tasks["sw"][lo + a]), int(wl.tasks["sw"][lo + b - 1]) + 1
        slices.append((dm.view(a, b), 32 * sw0, min(wl.rows, 32 * sw1)))
    r0, r1 = slices[0][1], slices[-1][2]
    packed_h = packed.cpu().pin_memory()
    scales_h = scales.cpu().pin_memory()
    y_h = torch.empty((max(0, r1 - r0), F), dtype=torch.float32).pin_memory()
    if gather:
        # Inputs padded to equal shards; this rank copies its shard from the host and the
        # all-gathers fill in the rest over NVLink (shards.gather_inputs).
        from tcc_spmm_b200 import shards

        padded, x0, x1 = shards.input_shard(wl.cols, world, dist.get_rank())
        inputs = [(torch.empty(padded * F, dtype=torch.int8, device=device),
                   torch.empty(padded, dtype=torch.float32, device=device)) for _ in range(2)]
    else:
        inputs = [(packed, scales), (torch.empty_like(packed), torch.empty_like(scales))]
    ys = [torch.empty((wl.rows, F), dtype=torch.float32, device=device) for _ in range(2)]
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
                T.launch_spmm_int8(view, inputs[bj][0], inputs[bj][1], ys[bj], wl.rows, wl.cols, F, ws,
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

    steps = max(5, min(args.steps, 20))
    run(max(3, min(args.warmup, 5)))
    torch.cuda.synchronize()
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    run(steps, start, stop)
    torch.cuda.synchronize()
    ms = torch.tensor([start.elapsed_time(stop)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    step_ms = float(ms.item()) / steps
    return {"value": wl.nnz * F / (step_ms / 1e3), "unit": "nnz*F/s", "ms_per_step": round(step_ms, 4),
            "steps": steps,
            "h2d_bytes_per_step": int((x1 - x0) * (F + 4)) if gather else int(packed.numel() + 4 * scales.numel()),
            "d2h_bytes_per_step": int(4 * (r1 - r0) * F), "x_allgather": gather,
            "slices_per_step": len(slices), "gpu_launches": len(slices) * steps,
            "api": "tcc_launch_spmm_int8 (C ABI) via tcc_spmm_b200: DeviceMatrix.view slices, pinned host buffers, "
                   "copy streams (inputs and Y double-buffered)"
                   + ("; packed X and scales copied 1/N per rank and all-gathered over NCCL" if gather else "")}


# ----------------------------------------------------------------------------------------
# Optional Y assembly across ranks
# ----------------------------------------------------------------------------------------
def time_assembly(wl, bounds, y, F: int, rank: int, world: int, device, barrier, repeats: int = 5) -> dict:
    """Assembly of the full Y on every rank (not part of the metric), two ways, each timed with
    CUDA events (max over ranks) after one untimed round: one broadcast per owner range in one
    NCCL group, straight into the owners' rows; and an all-gather of the ranges padded to the
    longest one into a staging buffer, followed by the copy of every range into place. The
    broadcast result is checked by per-range checksums against the owners' own rows."""
    import torch
    import torch.distributed as dist
    from tcc_spmm_b200 import shards

    ranges = shards.owned_rows(wl, bounds)
    shards.check_cover(ranges, wl.rows)
    lo, hi = ranges[rank]
    own = torch.zeros(world, dtype=torch.float64, device=device)
    own[rank] = y[lo:hi].double().sum() if hi > lo else 0.0
    dist.all_reduce(own)
    longest = max(e - b for b, e in ranges)
    stage = torch.empty((world, longest, F), dtype=torch.float32, device=device)
    mine = torch.zeros((longest, F), dtype=torch.float32, device=device)

    def gather():
        if hi > lo:
            mine[:hi - lo].copy_(y[lo:hi])
        dist.all_gather_into_tensor(stage.view(-1), mine.view(-1))
        for r, (b, e) in enumerate(ranges):
            if e > b and r != rank:
                y[b:e].copy_(stage[r, :e - b])

    def timed(fn) -> float:
        fn()
        torch.cuda.synchronize(device)
        barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(repeats):
            fn()
        stop.record()
        torch.cuda.synchronize(device)
        ms = torch.tensor([start.elapsed_time(stop) / repeats], dtype=torch.float64, device=device)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    t_gather = timed(gather)
    t_bcast = timed(lambda: shards.assemble_rows(y, ranges))
    seen = torch.stack([y[b:e].double().sum() if e > b else torch.zeros((), dtype=torch.float64, device=device)
                        for b, e in ranges])
    ok = torch.tensor([int(bool(torch.equal(seen, own)))], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    received = max(shards.received_bytes(ranges, r, F) for r in range(world))
    best = min(t_bcast, t_gather)
    return {"ms": round(best, 3), "bytes_received_per_rank_max": received,
            "gbs_per_rank": round(received / best / 1e6, 1),
            "collective": ("one broadcast per owner row range, all in one NCCL group" if t_bcast <= t_gather else
                           "padded all-gather into a staging buffer, then a copy of each range into place"),
            "broadcasts_ms": round(t_bcast, 3), "padded_allgather_ms": round(t_gather, 3),
            "checksums_match": bool(ok.item())}


# ----------------------------------------------------------------------------------------
# CPU baselines (the oracle restatement of the reference arithmetic)
# ----------------------------------------------------------------------------------------
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


def cpu_baselines(args, fmt, F) -> tuple:
    import oracle as O

    cores = host_threads()
    sample, snnz, q, s, stride = cpu_sample(fmt, F, args.cpu_seconds, cores)
    t = time_cpu(fmt, F, sample, q, s, cores)
    cpu = {"value": snnz * F / t, "unit": "nnz*F/s", "cores": cores, "kind": "port",
           "sample": f"every {stride}th 32-row window ({sample.size} windows, {snnz} nnz) of {args.config}, "
                     f"oracle/tcc_oracle.c restatement of the reference arithmetic, {t:.2f} s",
           "seconds": round(t, 3), "threads_reported": O.max_threads()}
    sample1, snnz1, q1, s1, stride1 = cpu_sample(fmt, F, max(1.0, args.cpu_seconds / 4), 1, seed=2)
    t1 = time_cpu(fmt, F, sample1, q1, s1, 1)
    cpu1 = {"value": snnz1 * F / t1, "unit": "nnz*F/s", "cores": 1, "kind": "port",
            "sample": f"every {stride1}th 32-row window ({sample1.size} windows, {snnz1} nnz), one thread, "
                      f"{t1:.2f} s", "seconds": round(t1, 3)}
    return cpu, cpu1


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
        # the host-side matrix generation that precedes the first collective.
        dist.init_process_group("nccl", timeout=timedelta(seconds=240), device_id=device)
    threads = max(1, host_threads() // world)
    stream = torch.cuda.current_stream(device)
    peak, peak_kind = measured_peaks()
    task_order = "format" if args.natural_order else "balanced-equal" if args.equal_count_order else "balanced"

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    F = W.CONFIGS[args.config].features
    wl = DeviceWorkload(args.config, device, threads)
    bounds = T.partition_tasks(wl, F, world)
    lo, hi = int(bounds[rank]), int(bounds[rank + 1])
    shard = wl.bytes(lo, hi, F)
    full = wl.bytes(0, wl.tasks.size, F)
    dm = wl.device_matrix(F, (lo, hi), not args.natural_order, args.variant, not args.equal_count_order)
    x, packed, scales = device_inputs(T, wl.cols, F, device)
    y = torch.empty((wl.rows, F), device=device)
    view, ws = dm.view(), dm.workspace()

    def launch():
        T.launch_spmm_int8(view, packed, scales, y, wl.rows, wl.cols, F, ws, stream=stream, variant=args.variant)

    for _ in range(max(3, args.warmup)):
        launch()
    torch.cuda.synchronize()
    barrier()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ms_local, batch_ms = timed_batches(launch, args.steps, stream)
    barrier()
    clocks = sampler.stop()
    ms_step = max_over_ranks(ms_local) / args.steps
    median_batch = max_over_ranks(statistics.median(batch_ms))
    value = wl.nnz * F / (ms_step / 1e3)
    T.check_device()  # a bounded wait that ran out would invalidate the timing

    # roofline of this rank's kernel (rank 0 reports its own; all ranks run the same kernel)
    launch_s = (ms_local / args.steps) / 1e3
    achieved = shard["total"] / launch_s / 1e9
    shape = T.spmm_launch_shape(F, args.variant) if args.variant != "generic" else None
    traffic = profile_traffic(args.config, args.variant, task_order, shape) if world == 1 else None

    # the one-pass quantize + pack of X, timed on its own (reads 4F, writes F + 4 bytes per row)
    def qp():
        T.quantize_pack_features_int8(x, packed, scales, wl.cols, F, stream=stream)

    for _ in range(3):
        qp()
    qp_total, _ = timed_batches(qp, 10, stream, batches=1)
    qp_ms = max_over_ranks(qp_total / 10)
    qp_bytes = wl.cols * (5 * F + 4)
    quantize_pack = {"ms": round(qp_ms, 4), "bytes": qp_bytes, "gbs": round(qp_bytes / qp_ms / 1e6, 1),
                     "frac": round(qp_bytes / qp_ms / 1e6 / peak, 4), "peak_kind": peak_kind,
                     "kernel": "tcc_quantize_pack_features_int8 (one pass: fp32 X in, packed16 int8 + scales out)"}
    del x

    # end to end through the public API with host buffers (every step copies packed X +
    # scales host -> device and this rank's Y rows device -> host; the step's task range runs in
    # window-aligned slices so that finished rows are copied back while the rest computes)
    e2e = None
    if not args.no_e2e:
        gather = world > 1 and args.e2e_x_allgather != "off"
        e2e = run_e2e(args, T, wl, dm, lo, hi, packed, scales, F, device, stream, barrier, world, gather)

    assembly = None
    if world > 1 and not args.no_assembly:
        assembly = time_assembly(wl, bounds, y, F, rank, world, device, barrier)

    cpu = cpu1 = None
    host_fmt = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host_fmt = wl.dfmt.to_host()
    headline_config = wl.config(F)
    headline_prep = dict(wl.prep)
    del dm, y, packed, scales, view, ws

    # the further configurations on the same ranks
    per_config = {}
    names = [n for n in args.per_config.split(",") if n]
    for name in names:
        try:
            per_config[name] = run_config(args, T, W, name, wl if W.CONFIGS[name].params == W.CONFIGS[args.config].params
                                          and W.CONFIGS[name].kind == W.CONFIGS[args.config].kind else None,
                                          device, stream, world, rank, threads, barrier, max_over_ranks, peak)
        except Exception as exc:  # noqa: BLE001 - every rank takes the same path
            per_config[name] = {"error": str(exc)[:300]}
        torch.cuda.empty_cache()
    del wl
    torch.cuda.empty_cache()

    if host_fmt is not None:
        cpu, cpu1 = cpu_baselines(args, host_fmt, F)

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "nnz*F/s", "value": value, "unit": "nnz*F/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8->tf32 (fp32 accumulate)", "data": "synthetic",
        "config": headline_config,
        "parallelism": f"task-range shards x{world}, X replicated, Y rows per rank",
        "kernel": {"variant": args.variant, "task_order": "format order" if args.natural_order else
                   "balanced for the launch grid, equal task counts per CTA" if args.equal_count_order else
                   "balanced for the launch grid, weighted by resident-CTA speed", "launch": shape},
        "prep": headline_prep,
        "timing": {"method": "K launches between CUDA events on the launching stream, barrier + synchronize on "
                             "both sides, max over ranks; also split into 5 event-timed batches",
                   "median_batch_ms": round(median_batch, 4), "batch_ms_rank0": [round(b, 4) for b in batch_ms]},
        "hbm_gbs_alg": round(full["total"] / (ms_step / 1e3) / 1e9, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": (traffic or {}).get("dram_bytes_per_launch"),
                     "alg_bytes_per_launch": shard["total"], "compulsory_bytes": full["compulsory"],
                     "merge_bytes": full["merge_bytes"]},
        "clocks": clocks, "gpu_launches": args.steps, "e2e": e2e, "cpu_baseline": cpu, "cpu_baseline_1t": cpu1,
        "quantize_pack": quantize_pack, "per_config": per_config, "y_assembly": assembly,
    }
    print(json.dumps(line), flush=True)


def run_config(args, T, W, name, reuse, device, stream, world, rank, threads, barrier, max_over_ranks, peak) -> dict:
    """One further configuration on every rank: its own partition, balanced order, X and Y; the
    time of per-config-steps launches (5 event-timed batches), max over ranks."""
    import torch

    F = W.CONFIGS[name].features
    wl = reuse if reuse is not None else DeviceWorkload(name, device, threads)
    bounds = T.partition_tasks(wl, F, world)
    lo, hi = int(bounds[rank]), int(bounds[rank + 1])
    shard = wl.bytes(lo, hi, F)
    full = wl.bytes(0, wl.tasks.size, F)
    dm = wl.device_matrix(F, (lo, hi), not args.natural_order, args.variant, not args.equal_count_order)
    x, packed, scales = device_inputs(T, wl.cols, F, device, seed=X_SEED + 1)
    del x
    y = torch.empty((wl.rows, F), device=device)
    view, ws = dm.view(), dm.workspace()

    def launch():
        T.launch_spmm_int8(view, packed, scales, y, wl.rows, wl.cols, F, ws, stream=stream, variant=args.variant)

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    barrier()
    ms_local, batch_ms = timed_batches(launch, args.per_config_steps, stream)
    barrier()
    T.check_device()
    ms = max_over_ranks(ms_local) / args.per_config_steps
    local_s = ms_local / args.per_config_steps / 1e3
    out = {"config": wl.config(F, name), "ms_per_call": round(ms, 4), "value": wl.nnz * F / (ms / 1e3),
           "unit": "nnz*F/s", "median_batch_ms": round(max_over_ranks(statistics.median(batch_ms)), 4),
           "hbm_gbs_alg": round(full["total"] / (ms / 1e3) / 1e9, 1),
           "roofline_frac_rank0": round(shard["total"] / local_s / 1e9 / peak, 4),
           "alg_bytes_per_launch": full["total"], "alg_bytes_rank0": shard["total"],
           "prep": wl.prep, "steps": args.per_config_steps}
    del dm, y, packed, scales
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from tcc_spmm_b200 import workloads as W
    import oracle as O

    cfg = W.CONFIGS[args.config]
    F = cfg.features
    cores = host_threads()
    t0 = time.time()
    csr = W.generate(args.config, threads=cores)
    t1 = time.time()
    fmt = reference_format(O, csr)
    t2 = time.time()
    valid = int(np.count_nonzero(fmt.source_ids != 0xFFFFFFFF))
    config = workload_config(args.config, fmt.rows, csr.nnz, F, fmt.row_group_masks.size, valid, fmt.tasks.size,
                             fmt.partial_count)
    per_step = min(5.0, 150.0 / max(1, args.steps + args.warmup))
    steps, warmup = min(args.steps, 20), min(args.warmup, 3)
    sample, snnz, q, s, stride = cpu_sample(fmt, F, per_step, cores)
    for _ in range(warmup):
        time_cpu(fmt, F, sample, q, s, cores)
    times = [time_cpu(fmt, F, sample, q, s, cores) for _ in range(steps)]
    t = sum(times) / len(times)
    value = snnz * F / t
    ref_kernel = None
    try:
        ref_kernel = time_reference_kernel(fmt, F, args)
    except Exception as exc:  # the GPU part is informational only
        ref_kernel = {"error": str(exc)[:200]}
    line = {"metric": "nnz*F/s", "value": value, "unit": "nnz*F/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": round(1e3 * t * csr.nnz / max(1, snnz), 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8->tf32 (fp32 accumulate)",
            "data": "synthetic", "config": config,
            "parallelism": "rank 0 alone: the reference path is single-process CPU code",
            "prep": {"generate_s": round(t1 - t0, 2), "convert_s": round(t2 - t1, 2),
                     "format_from": "reference convertCsrToSw32 (oracle/_ref)" if O.have_ref_host()
                     else "oracle convertCsrToSw32 restatement"},
            "cpu_baseline": {"value": value, "unit": "nnz*F/s", "cores": cores, "kind": "port",
                             "sample": f"every {stride}th 32-row window ({sample.size} windows, {snnz} nnz); the "
                                       "reference ships no CPU SpMM, this is the oracle restatement of its arithmetic"},
            "e2e": {"value": value, "unit": "nnz*F/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_gpu_kernel": ref_kernel}
    print(json.dumps(line), flush=True)


def reference_format(O, csr):
    """The SW32 format from the reference's own convertCsrToSw32 (oracle/_ref), as plain numpy
    arrays in a light record (no call into this repository's library)."""
    from types import SimpleNamespace

    from tcc_spmm_b200.api import REDUCE_DTYPE, TASK_DTYPE

    r = O.ref_convert_csr_to_sw32(csr.rows, csr.cols, csr.row_offsets, csr.source_ids, csr.values)
    return SimpleNamespace(rows=csr.rows, cols=csr.cols, window_offsets=r["window_offsets"], source_ids=r["source_ids"],
                           row_group_masks=r["row_group_masks"], source_metadata=r["source_metadata"],
                           values=r["values"], bucket_offsets=r["bucket_offsets"],
                           tasks=np.ascontiguousarray(r["tasks"]).view(TASK_DTYPE).reshape(-1),
                           reductions=np.ascontiguousarray(r["reductions"]).view(REDUCE_DTYPE).reshape(-1),
                           partial_ids=r["partial_ids"], partial_count=int(r["partial_count"]))


def time_reference_kernel(fmt, F, args):
    """The reference's own kernel (oracle/_ref) on the same matrix, CUDA-event timed. The arrays
    are uploaded with plain torch and the workspace is sized by the reference's rule
    (src/device_matrix.cuh:18-28)."""
    import ctypes

    import torch

    import oracle as O
    from tcc_spmm_b200._native import Sw32DeviceView

    if not torch.cuda.is_available() or not O.have_ref_cuda("sm80"):
        return None
    up = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.uint8)).cuda()
    arrays = {k: up(getattr(fmt, k)) for k in ("window_offsets", "source_ids", "row_group_masks", "source_metadata",
                                                "values", "bucket_offsets", "tasks", "reductions", "partial_ids")}
    windows = fmt.window_offsets.size - 1
    partials = torch.empty(max(1, fmt.partial_count * 8 * F), dtype=torch.float32, device="cuda")
    counters = torch.zeros(max(1, windows * (F // 128)), dtype=torch.int32, device="cuda")
    view = Sw32DeviceView(*(arrays[k].data_ptr() for k in ("window_offsets", "source_ids", "row_group_masks",
                                                           "source_metadata", "values", "bucket_offsets", "tasks",
                                                           "reductions", "partial_ids")), fmt.tasks.size)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(X_SEED)
    x = torch.randn((fmt.cols, F), generator=gen, device="cuda", dtype=torch.float32)
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
        args_ = (ctypes.addressof(view), p.data_ptr(), s.data_ptr(), y.data_ptr(), fmt.rows, fmt.cols, F,
                 partials.data_ptr() if fmt.partial_count else 0, counters.data_ptr() if fmt.partial_count else 0,
                 stream)
        for _ in range(max(3, min(args.warmup, 10))):
            ref.launch_spmm_int8(*args_)
        torch.cuda.synchronize()
        steps = min(args.steps, 20)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            ref.launch_spmm_int8(*args_)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        nnz = int(fmt.values.size)
        out[tag] = {"ms_per_call": round(ms, 4), "value": nnz * F / (ms / 1e3),
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
