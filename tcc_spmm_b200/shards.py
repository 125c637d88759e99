"""Task-range shards across ranks (one process per GPU) and the assembly of Y.

The reference is single-GPU. Here the task array is cut into contiguous ranges at window
boundaries (``partition_tasks``), so every split window, with its counter, partials and merge,
lies inside one rank. A rank then writes exactly the Y rows of its windows: a contiguous range
``[32 * first window, 32 * (last window + 1))`` (clipped to the matrix). The ranges of all
ranks cover Y once.

The assembly of the full Y on every rank is optional and is not part of the SpMM time: one
broadcast per owner range over ``torch.distributed`` (NCCL over NVLink on GPUs, gloo on CPU),
each straight into the owner's rows of every rank's Y, with no staging copy.
"""
from __future__ import annotations

from typing import Sequence


def owned_rows(fmt, bounds: Sequence[int]) -> list:
    """(row_begin, row_end) of Y owned by each rank, for the task bounds of partition_tasks."""
    tasks = fmt.tasks
    ranges = []
    for r in range(len(bounds) - 1):
        lo, hi = int(bounds[r]), int(bounds[r + 1])
        if hi <= lo:
            ranges.append((0, 0))
            continue
        first = 32 * int(tasks["sw"][lo])
        last = min(fmt.rows, 32 * (int(tasks["sw"][hi - 1]) + 1))
        ranges.append((first, last))
    return ranges


def check_cover(ranges: Sequence[tuple], rows: int) -> None:
    """Raise ValueError unless the non-empty ranges tile [0, rows) in rank order."""
    at = 0
    for begin, end in ranges:
        if end == begin:
            continue
        if begin != at or end < begin:
            raise ValueError(f"row ranges do not tile Y: range [{begin}, {end}) after row {at}")
        at = end
    if at != rows:
        raise ValueError(f"row ranges cover {at} of {rows} rows")


def assemble_rows(y, ranges: Sequence[tuple], group=None) -> None:
    """Give every rank the whole Y: rank r broadcasts its rows ranges[r] of y (a [rows, F]
    row-major tensor on this rank's device) to all ranks, in rank order. Every rank must call
    this with the same ranges (the collective order is the same on all ranks)."""
    import torch.distributed as dist

    if len(ranges) != dist.get_world_size(group):
        raise ValueError("one row range per rank")
    pieces = [(r, y[begin:end]) for r, (begin, end) in enumerate(ranges) if end > begin]
    if y.is_cuda and dist.get_backend(group) == "nccl" and hasattr(dist, "_coalescing_manager"):
        # One NCCL group: the owners' broadcasts run concurrently, so every link carries data
        # in both directions at once.
        with dist._coalescing_manager(group=group, device=y.device, async_ops=True) as cm:
            for r, piece in pieces:
                dist.broadcast(piece, src=r, group=group, async_op=True)
        cm.wait()
    else:
        for r, piece in pieces:
            dist.broadcast(piece, src=r, group=group)


def received_bytes(ranges: Sequence[tuple], rank: int, features: int) -> int:
    """Bytes of Y a rank receives in assemble_rows (every range but its own)."""
    return int(sum(4 * features * (e - b) for r, (b, e) in enumerate(ranges) if r != rank))


def input_shard(cols: int, world: int, rank: int) -> tuple:
    """Rows of packed X (and scales) that `rank` copies from the host when the inputs are split
    over `world` ranks and completed by an all-gather: equal shards of the rows padded to a
    multiple of `world` (the all-gather needs equal sizes). Returns (padded rows, first, last);
    rows at or past `cols` are padding, read by no kernel."""
    per = -(-cols // world)
    return per * world, min(cols, rank * per), min(cols, (rank + 1) * per)


def gather_inputs(packed, scales, packed_h, scales_h, features: int, group=None, non_blocking: bool = False) -> int:
    """Give every rank the whole packed X and scales while each copies only its shard from the
    host: rank r copies rows input_shard(...)[1:] of `packed_h` / `scales_h` (host arrays of
    cols rows) into `packed` / `scales` (this rank's buffers of padded rows), then in-place
    all-gathers fill in the other ranks' shards (NCCL over NVLink on GPUs, gloo on CPU). Every
    rank must call this with the same sizes. Returns the bytes this rank copied from the host."""
    import torch.distributed as dist

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    cols = scales_h.numel()
    padded, first, last = input_shard(cols, world, rank)
    if packed.numel() != padded * features or scales.numel() != padded:
        raise ValueError("input buffers must hold the padded rows")
    per = padded // world
    if last > first:
        packed[first * features:last * features].copy_(packed_h[first * features:last * features],
                                                       non_blocking=non_blocking)
        scales[first:last].copy_(scales_h[first:last], non_blocking=non_blocking)
    dist.all_gather_into_tensor(packed, packed[rank * per * features:(rank + 1) * per * features], group=group)
    dist.all_gather_into_tensor(scales, scales[rank * per:(rank + 1) * per], group=group)
    return (last - first) * (features + 4)


__all__ = ["owned_rows", "check_cover", "assemble_rows", "received_bytes", "input_shard", "gather_inputs"]
