"""Multi-GPU sharding logic on CPU ranks (gloo, world size 2): contiguous task ranges cut at
window boundaries, every window owned by exactly one rank, the union of the ranks' rows equal
to the single-rank result, the assembly of Y (one broadcast per owner range) giving every rank
the full result, the end-to-end inputs copied in shards and all-gathered, and a rank that dies
surfacing as an error on the other rank within the process-group timeout (no GPU is
involved)."""
from __future__ import annotations

import os
import socket
import sys
import tempfile
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank: int, world: int, port: int, outdir: str) -> None:
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    import oracle as O
    import tcc_spmm_b200 as T
    from tcc_spmm_b200 import workloads as W

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    csr = W.generate("stress_small", threads=2)
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr, True, 2)
    bounds = T.partition_tasks(fmt, 128, world)
    lo, hi = int(bounds[rank]), int(bounds[rank + 1])
    windows = np.unique(fmt.tasks["sw"][lo:hi]).astype(np.uint32)
    rng = np.random.default_rng(0)
    q = rng.integers(-127, 128, size=(fmt.cols, 16), dtype=np.int8)
    s = (rng.random(fmt.cols) * 0.01 + 1e-3).astype(np.float32)
    y, _, rows = O.spmm(fmt, q, s, windows, threads=2, with_bound=False)
    keep = rows >= 0
    gathered = [None] * world
    dist.all_gather_object(gathered, (lo, hi, rows[keep].tolist(), y[keep]))
    if rank == 0:
        full, _, frows = O.spmm(fmt, q, s, threads=2, with_bound=False)
        full = full[frows >= 0]
        seen = np.zeros(fmt.rows, dtype=np.int32)
        assembled = np.zeros_like(full)
        prev_hi = 0
        for g_lo, g_hi, g_rows, g_y in gathered:
            assert g_lo == prev_hi
            prev_hi = g_hi
            seen[g_rows] += 1
            assembled[g_rows] = g_y
        assert prev_hi == fmt.tasks.size
        assert np.all(seen == 1), "every row owned by exactly one rank"
        assert np.array_equal(assembled, full)
        Path(outdir, "ok").write_text("ok")
    dist.barrier()
    dist.destroy_process_group()


def _assembly_worker(rank: int, world: int, port: int, outdir: str) -> None:
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    import oracle as O
    import tcc_spmm_b200 as T
    from tcc_spmm_b200 import shards
    from tcc_spmm_b200 import workloads as W

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    csr = W.generate("stress_small", threads=2)
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr, True, 2)
    bounds = T.partition_tasks(fmt, 128, world)
    ranges = shards.owned_rows(fmt, bounds)
    shards.check_cover(ranges, fmt.rows)
    lo, hi = int(bounds[rank]), int(bounds[rank + 1])
    windows = np.unique(fmt.tasks["sw"][lo:hi]).astype(np.uint32)
    rng = np.random.default_rng(1)
    q = rng.integers(-127, 128, size=(fmt.cols, 16), dtype=np.int8)
    s = (rng.random(fmt.cols) * 0.01 + 1e-3).astype(np.float32)
    part, _, rows = O.spmm(fmt, q, s, windows, threads=2, with_bound=False)
    keep = rows >= 0
    assert np.all((rows[keep] >= ranges[rank][0]) & (rows[keep] < ranges[rank][1])), "rows outside the owned range"
    y = np.full((fmt.rows, 16), np.nan, dtype=np.float32)  # other ranks' rows unwritten
    y[rows[keep]] = part[keep]
    yt = torch.from_numpy(y)
    shards.assemble_rows(yt, ranges)
    full, _, frows = O.spmm(fmt, q, s, threads=2, with_bound=False)
    expect = np.zeros((fmt.rows, 16), dtype=np.float32)
    expect[frows[frows >= 0]] = full[frows >= 0]
    if np.array_equal(yt.numpy(), expect):
        Path(outdir, f"ok{rank}").write_text("ok")
    dist.barrier()
    dist.destroy_process_group()


def _failure_worker(rank: int, world: int, port: int, outdir: str) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # leaves between steps, without joining the next collective
    try:
        dist.barrier()
        Path(outdir, "no-error").write_text("barrier returned")
    except Exception as exc:  # timeout or connection error, reported on the host
        Path(outdir, "error").write_text(type(exc).__name__)


def _inputs_worker(rank: int, world: int, port: int, outdir: str) -> None:
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    from tcc_spmm_b200 import shards

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    ok = True
    for cols, features in ((7, 16), (64, 128), (1, 16)):
        rng = np.random.default_rng(cols)
        packed_h = torch.from_numpy(rng.integers(-127, 128, size=cols * features, dtype=np.int8))
        scales_h = torch.from_numpy(rng.random(cols).astype(np.float32))
        padded, first, last = shards.input_shard(cols, world, rank)
        packed = torch.full((padded * features,), 85, dtype=torch.int8)   # stale contents
        scales = torch.full((padded,), float("nan"), dtype=torch.float32)
        copied = shards.gather_inputs(packed, scales, packed_h, scales_h, features)
        ok &= copied == (last - first) * (features + 4)
        ok &= torch.equal(packed[:cols * features], packed_h) and torch.equal(scales[:cols], scales_h)
    if ok:
        Path(outdir, f"ok{rank}").write_text("ok")
    dist.barrier()
    dist.destroy_process_group()


def _spawn(fn, world: int):
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(fn, args=(world, _free_port(), d), nprocs=world, join=False, start_method="spawn")
        for p in ctx.processes:
            p.join(120)
        return {f.name: f.read_text() for f in Path(d).iterdir()}


def test_two_rank_shards_reassemble_single_rank_result():
    out = _spawn(_shard_worker, 2)
    assert out.get("ok") == "ok"


def test_lost_rank_is_reported_not_hung():
    out = _spawn(_failure_worker, 2)
    assert "error" in out and "no-error" not in out


def test_two_rank_y_assembly_gives_every_rank_the_full_result():
    out = _spawn(_assembly_worker, 2)
    assert out.get("ok0") == "ok" and out.get("ok1") == "ok"


def test_two_rank_input_shards_gather_to_the_full_inputs():
    out = _spawn(_inputs_worker, 2)
    assert out.get("ok0") == "ok" and out.get("ok1") == "ok"


def test_row_ranges_must_tile_y():
    from tcc_spmm_b200 import shards

    shards.check_cover([(0, 64), (64, 64), (64, 100)], 100)
    with pytest.raises(ValueError):
        shards.check_cover([(0, 64), (96, 100)], 100)
    with pytest.raises(ValueError):
        shards.check_cover([(0, 64)], 100)
