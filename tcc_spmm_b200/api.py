"""Python mirror of the reference's C++ host API for the SpMM path, over the C ABI.

Reference (Shixg-cnic/tcc_spmm)            this module
-----------------------------------------  ----------------------------------------------
makeCanonicalCsr   include/format/csr.h:23  make_canonical_csr
loadMatrixMarket   include/format/csr.h:18  load_matrix_market
convertCsrToSw32   include/format/sw32.h:43 convert_csr_to_sw32 (includes buildPanelTasks);
                                            convert_csr_to_sw32_device builds it on the GPU
Sw32HostFormat     include/format/sw32.h:22 Sw32HostFormat
DeviceMatrix       src/device_matrix.cuh:8  DeviceMatrix (view(), workspace())
SpmmWorkspace      include/spmm.cuh:10      SpmmWorkspace
launchSpmmInt8     include/spmm.cuh:21      launch_spmm_int8
quantizeFeaturesInt8 int8_features.cuh:9    quantize_features_int8
packFeaturesInt8x16  int8_features.cuh:14   pack_features_int8x16

Errors map to the reference's exception types: std::invalid_argument -> InvalidArgument
(a ValueError), std::overflow_error -> OverflowError, std::runtime_error (CUDA) ->
CudaError (a RuntimeError). Device calls only enqueue work on the given stream (default:
torch's current stream of the output's device) and never synchronise.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import _native as N

TCC_OK, TCC_INVALID_ARGUMENT, TCC_OVERFLOW, TCC_CUDA_ERROR, TCC_INTERNAL, TCC_DEVICE_TIMEOUT = range(6)
NO_PARTIAL = 0xFFFFFFFF
PADDING_SOURCE = 0xFFFFFFFF
BUCKET_ORDER = (0, 1, 2, 4, 8, 3, 5, 6, 7, 9, 10, 11, 12, 13, 14, 15)
TASK_PANEL_LIMIT = 384


class InvalidArgument(ValueError):
    """std::invalid_argument of the reference API."""


class CudaError(RuntimeError):
    """std::runtime_error raised by the reference's checkCuda."""


class DeviceTimeout(TimeoutError):
    """A bounded device wait of the SpMM kernel ran out."""


def _check(status: int) -> None:
    if status == TCC_OK:
        return
    message = (N.lib().tcc_last_error() or b"").decode(errors="replace")
    if status == TCC_INVALID_ARGUMENT:
        raise InvalidArgument(message)
    if status == TCC_OVERFLOW:
        raise OverflowError(message)
    if status == TCC_CUDA_ERROR:
        raise CudaError(message)
    if status == TCC_DEVICE_TIMEOUT:
        raise DeviceTimeout(message)
    raise RuntimeError(message)


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))


def _copy_out(ptr, count: int, dtype) -> np.ndarray:
    if count == 0 or not ptr:
        return np.zeros(0, dtype=dtype)
    nbytes = count * np.dtype(dtype).itemsize
    buf = (C.c_char * nbytes).from_address(ptr if isinstance(ptr, int) else C.cast(ptr, C.c_void_p).value)
    return np.frombuffer(buf, dtype=dtype).copy()


# --------------------------------------------------------------------------------------------
# Host side
# --------------------------------------------------------------------------------------------
@dataclass
class CsrMatrix:
    """Canonical CSR (reference include/format/csr.h:7-10)."""

    rows: int
    cols: int
    row_offsets: np.ndarray
    source_ids: np.ndarray
    values: np.ndarray

    @property
    def nnz(self) -> int:
        return int(self.source_ids.size)


def _csr_from_handle(handle: C.c_void_p, cols: int) -> CsrMatrix:
    lib = N.lib()
    rows = C.c_uint32()
    ro, si, va = N.u32p(), N.u32p(), N.f32p()
    nnz = C.c_uint64()
    try:
        _check(lib.tcc_csr_arrays(handle, C.byref(rows), C.byref(ro), C.byref(si), C.byref(va), C.byref(nnz)))
        return CsrMatrix(rows.value, cols, _copy_out(C.cast(ro, C.c_void_p).value, rows.value + 1, np.uint32),
                         _copy_out(C.cast(si, C.c_void_p).value, nnz.value, np.uint32),
                         _copy_out(C.cast(va, C.c_void_p).value, nnz.value, np.float32))
    finally:
        lib.tcc_csr_free(handle)


def make_canonical_csr(rows: int, cols: int, row_offsets, source_ids, values) -> CsrMatrix:
    """Validate raw CSR and canonicalise it (reference src/format/csr.cpp:6-40)."""
    ro, si, va = _u32(row_offsets), _u32(source_ids), _f32(values)
    if ro.size != rows + 1:
        raise InvalidArgument("invalid CSR dimensions or offsets")
    nnz = int(ro[-1]) if ro.size else 0
    if si.size < nnz or va.size < nnz:
        raise InvalidArgument("invalid CSR offsets")
    handle = C.c_void_p()
    _check(N.lib().tcc_make_canonical_csr(rows, cols, nnz, _ptr(ro, C.c_uint32), _ptr(si, C.c_uint32),
                                          _ptr(va, C.c_float), C.byref(handle)))
    return _csr_from_handle(handle, cols)


@dataclass
class MtxMatrix:
    rows: int
    cols: int
    csr: CsrMatrix


def load_matrix_market(path: str) -> MtxMatrix:
    """Read a coordinate Matrix Market file into canonical CSR (reference
    src/format/matrix_market.cpp:30-103)."""
    handle = C.c_void_p()
    cols = C.c_uint32()
    _check(N.lib().tcc_load_matrix_market(str(path).encode(), C.byref(cols), C.byref(handle)))
    csr = _csr_from_handle(handle, cols.value)
    return MtxMatrix(csr.rows, cols.value, csr)


TASK_DTYPE = np.dtype([(n, "<u4") for n in ("sw", "begin", "end", "partial", "mask", "chunks", "reduceFirst")])
REDUCE_DTYPE = np.dtype([("begin", "<u4"), ("end", "<u4")])


@dataclass
class Sw32HostFormat:
    """Host SW32 format and task plan (reference include/format/sw32.h:22-39)."""

    rows: int
    cols: int
    window_offsets: np.ndarray
    source_ids: np.ndarray
    row_group_masks: np.ndarray
    source_metadata: np.ndarray
    values: np.ndarray
    bucket_offsets: np.ndarray
    tasks: np.ndarray
    reductions: np.ndarray
    partial_ids: np.ndarray
    partial_count: int

    @property
    def windows(self) -> int:
        return int(self.window_offsets.size - 1)

    @property
    def panels(self) -> int:
        return int(self.row_group_masks.size)

    @property
    def nnz(self) -> int:
        return int(self.values.size)

    @property
    def valid_slots(self) -> int:
        return int(np.count_nonzero(self.source_ids != PADDING_SOURCE))

    def algorithmic_bytes(self, features: int) -> dict:
        """Bytes one SpMM call must move at minimum under the format (one read of every format
        array, one F-byte row plus a 4-byte scale per valid slot, one write of Y)."""
        a_bytes = (4 * self.source_ids.size + 8 * self.source_metadata.size + 4 * self.values.size +
                   4 * self.row_group_masks.size + 4 * self.bucket_offsets.size + 28 * self.tasks.size +
                   8 * self.reductions.size + 4 * self.partial_ids.size)
        x_bytes = self.valid_slots * (features + 4)
        y_bytes = 4 * self.rows * features
        return {"a_bytes": int(a_bytes), "x_bytes": int(x_bytes), "y_bytes": int(y_bytes),
                "total": int(a_bytes + x_bytes + y_bytes),
                "compulsory": int(a_bytes + 4 * self.cols + self.cols * features + y_bytes),
                "merge_bytes": int(2 * 4 * 8 * features * self.partial_count)}


def convert_csr_to_sw32(rows: int, cols: int, csr: CsrMatrix, bucket_by_rw_mask: bool = True,
                        threads: int = 0) -> Sw32HostFormat:
    """Build the SW32 format and, when bucketed, its task plan (reference
    src/format/sw32.cpp:69-167 and :25-65). Byte-identical output; runs on `threads` host
    threads (0 = all)."""
    ro, si, va = _u32(csr.row_offsets), _u32(csr.source_ids), _f32(csr.values)
    if ro.size != rows + 1 or va.size != si.size:
        raise InvalidArgument("invalid canonical CSR for source-mask SW32")
    lib = N.lib()
    handle = C.c_void_p()
    _check(lib.tcc_convert_csr_to_sw32(rows, cols, _ptr(ro, C.c_uint32), _ptr(si, C.c_uint32), _ptr(va, C.c_float),
                                       si.size, int(bool(bucket_by_rw_mask)), threads, C.byref(handle)))
    try:
        s, a = N.Sw32Sizes(), N.Sw32Arrays()
        _check(lib.tcc_sw32_host_sizes(handle, C.byref(s)))
        _check(lib.tcc_sw32_host_arrays(handle, C.byref(a)))
        return Sw32HostFormat(
            rows=s.rows, cols=s.cols,
            window_offsets=_copy_out(a.windowOffsets, s.windowOffsets, np.uint32),
            source_ids=_copy_out(a.sourceIds, s.sourceIds, np.uint32),
            row_group_masks=_copy_out(a.rowGroupMasks, s.rowGroupMasks, np.uint32),
            source_metadata=_copy_out(a.sourceMetadata, s.sourceIds, np.uint64),
            values=_copy_out(a.values, s.values, np.float32),
            bucket_offsets=_copy_out(a.bucketOffsets, s.bucketOffsets, np.uint32),
            tasks=_copy_out(a.tasks, s.tasks * 7, np.uint32).view(TASK_DTYPE),
            reductions=_copy_out(a.reductions, s.reductions * 2, np.uint32).view(REDUCE_DTYPE),
            partial_ids=_copy_out(a.partialIds, s.partialIds, np.uint32),
            partial_count=s.partialCount)
    finally:
        lib.tcc_sw32_host_free(handle)


def workspace_size(rows: int, partial_count: int, features: int) -> tuple[int, int]:
    """(partial floats, counter words) of the reference's workspace contract."""
    pf, cw = C.c_uint64(), C.c_uint64()
    _check(N.lib().tcc_spmm_workspace_size(rows, partial_count, features, C.byref(pf), C.byref(cw)))
    return pf.value, cw.value


def partition_tasks(fmt: Sw32HostFormat, features: int, parts: int) -> np.ndarray:
    """parts+1 task-index bounds of balanced contiguous shards, cut at window boundaries."""
    bounds = np.zeros(parts + 1, dtype=np.uint32)
    tasks = np.ascontiguousarray(fmt.tasks)
    masks = _u32(fmt.row_group_masks)
    _check(N.lib().tcc_partition_tasks(tasks.ctypes.data_as(C.c_void_p), tasks.size, _ptr(masks, C.c_uint32),
                                       features, parts, _ptr(bounds, C.c_uint32)))
    return bounds


def balance_tasks(tasks: np.ndarray, row_group_masks, features: int, ctas: int) -> np.ndarray:
    """Task order for a persistent launch of `ctas` CTAs (CTA b takes tasks b, b + G, ...):
    heaviest first, one per CTA per round, to the CTA with the least estimated work. A
    permutation of `tasks`; Y does not depend on the order."""
    src = np.ascontiguousarray(tasks)
    out = np.empty_like(src)
    masks = _u32(row_group_masks)
    _check(N.lib().tcc_balance_tasks(src.ctypes.data_as(C.c_void_p), src.size, _ptr(masks, C.c_uint32), features,
                                     ctas, out.ctypes.data_as(C.c_void_p)))
    return out


def balance_tasks_padded(tasks: np.ndarray, row_group_masks, features: int, ctas: int,
                         ctas_per_sm: int) -> np.ndarray:
    """Task order for a persistent launch of `ctas` CTAs, `ctas_per_sm` resident per SM, weighted
    by the measured speed of each resident CTA (tcc_balance_tasks_padded): CTA b's tasks at
    entries b, b + G, ...; shorter lists padded with skip entries (window 0xFFFFFFFF). Longer
    than `tasks` by the padding; Y does not depend on the order."""
    src = np.ascontiguousarray(tasks)
    masks = _u32(row_group_masks)
    n = C.c_uint32()
    _check(N.lib().tcc_balance_tasks_padded(src.ctypes.data_as(C.c_void_p), src.size, _ptr(masks, C.c_uint32),
                                            features, ctas, ctas_per_sm, None, 0, C.byref(n)))
    out = np.empty(n.value, dtype=src.dtype)
    _check(N.lib().tcc_balance_tasks_padded(src.ctypes.data_as(C.c_void_p), src.size, _ptr(masks, C.c_uint32),
                                            features, ctas, ctas_per_sm, out.ctypes.data_as(C.c_void_p), out.size,
                                            C.byref(n)))
    return out


def _balanced_order(tasks: np.ndarray, masks, features: int, variant: str, weighted: bool = True) -> np.ndarray:
    """The task order a DeviceMatrix launches for `variant` on the current device: weighted by
    resident-CTA speed and padded for the default kernel (unless weighted is False), else
    tcc_balance_tasks's equal-count order."""
    shape = spmm_launch_shape(features, variant)
    if weighted and variant in ("default", "tmem8") and shape["grid"]:
        return balance_tasks_padded(tasks, masks, features, shape["grid"], max(1, shape["occupancy"]))
    grid = shape["grid"] or spmm_launch_shape(features)["grid"] # the generic kernel's grid is per call
    return balance_tasks(tasks, masks, features, grid)


# --------------------------------------------------------------------------------------------
# Device side (torch is used for device memory and streams only)
# --------------------------------------------------------------------------------------------
def _addr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream_handle(stream, like=None) -> int:
    if stream is None:
        import torch

        device = like.device if (like is not None and hasattr(like, "device")) else None
        return int(torch.cuda.current_stream(device).cuda_stream)
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


@dataclass
class SpmmWorkspace:
    """partials: partialCount*8*F floats; counters: ceil(rows/32)*(F/128) u32 (zeroed)."""

    partials: object = None
    counters: object = None


class DeviceMatrix:
    """Uploads every SW32 array and allocates the split-task workspace for `features`
    (reference src/device_matrix.cuh:8-37): partials = partialCount*8*F floats, counters =
    windows*(F/128) zeroed u32 when partialCount > 0.

    balance=True also uploads a task order for the grid of the kernel `variant` (the default
    kernel unless named) on this device: for the default kernel the order weighted by the speed
    of each resident CTA of an SM, padded with skip entries (balance_tasks_padded), or with
    weighted_order=False, and for the other kernels, the equal-count order of balance_tasks.
    view() of the whole task range then uses that order (sub-range views keep the natural order,
    whose ranges cover contiguous windows)."""

    def __init__(self, fmt: Sw32HostFormat, features: int, device="cuda", task_range: Optional[tuple] = None,
                 balance: bool = False, variant: str = "default", weighted_order: bool = True):
        import torch

        self.rows, self.cols, self.features = fmt.rows, fmt.cols, features
        self.device = torch.device(device)

        def up(a: np.ndarray, dtype):
            if a.size == 0:
                return torch.zeros(1, dtype=dtype, device=self.device)
            return torch.from_numpy(np.ascontiguousarray(a).view(_np_of(dtype))).to(self.device)

        self.window_offsets = up(fmt.window_offsets, torch.int32)
        self.source_ids = up(fmt.source_ids, torch.int32)
        self.row_group_masks = up(fmt.row_group_masks, torch.int32)
        self.source_metadata = up(fmt.source_metadata, torch.int64)
        self.values = up(fmt.values, torch.float32)
        self.bucket_offsets = up(fmt.bucket_offsets, torch.int32)
        tasks = fmt.tasks if task_range is None else fmt.tasks[task_range[0]:task_range[1]]
        self.task_count = int(tasks.size)
        self.tasks = up(np.ascontiguousarray(tasks).view(np.uint32), torch.int32)
        self.tasks_balanced, self.balanced_count = None, 0
        if balance and self.task_count:
            with torch.cuda.device(self.device):
                order = _balanced_order(tasks, fmt.row_group_masks, features, variant, weighted_order)
            self.tasks_balanced, self.balanced_count = up(order.view(np.uint32), torch.int32), int(order.size)
        self.reductions = up(np.ascontiguousarray(fmt.reductions).view(np.uint32), torch.int32)
        self.partial_ids = up(fmt.partial_ids, torch.int32)
        self.partial_count = fmt.partial_count
        pf, cw = workspace_size(fmt.rows, fmt.partial_count, features)
        self.partials = torch.empty(pf, dtype=torch.float32, device=self.device) if pf else None
        self.counters = torch.zeros(cw, dtype=torch.int32, device=self.device) if cw else None

    def view(self, first: int = 0, last: Optional[int] = None) -> N.Sw32DeviceView:
        """Device view over the uploaded tasks [first, last) (all by default). A sub-range that
        starts and ends at window boundaries writes exactly the Y rows of its windows, so
        several such views can be launched one after another to overlap the copy of finished
        rows with the rest (the tasks array is shared; each view points into it)."""
        last = self.task_count if last is None else last
        if not 0 <= first <= last <= self.task_count:
            raise ValueError("task range out of bounds")
        whole = first == 0 and last == self.task_count
        if whole and getattr(self, "tasks_balanced", None) is not None:
            tasks, count = self.tasks_balanced, self.balanced_count  # with its padding entries
        else:
            tasks, count = self.tasks, last - first
        return N.Sw32DeviceView(self.window_offsets.data_ptr(), self.source_ids.data_ptr(),
                                self.row_group_masks.data_ptr(), self.source_metadata.data_ptr(),
                                self.values.data_ptr(), self.bucket_offsets.data_ptr(),
                                tasks.data_ptr() + (0 if whole else TASK_DTYPE.itemsize * first),
                                self.reductions.data_ptr(), self.partial_ids.data_ptr(), count)

    @classmethod
    def from_device_format(cls, fmt: "Sw32DeviceFormat", features: int, task_range: Optional[tuple] = None,
                           balance: bool = False, variant: str = "default", host_tasks: Optional[np.ndarray] = None,
                           host_masks: Optional[np.ndarray] = None, weighted_order: bool = True) -> "DeviceMatrix":
        """A DeviceMatrix over a format built on the GPU (no upload): the arrays are the
        library's; only the workspace for `features` is allocated here. task_range and balance
        as in the constructor; balancing reads the tasks and row-group masks on the host
        (host_tasks / host_masks when given, else copied from the device)."""
        import torch

        self = cls.__new__(cls)
        self.rows, self.cols, self.features = fmt.rows, fmt.cols, features
        self.device = fmt.window_offsets.device
        for name in ("window_offsets", "source_ids", "row_group_masks", "source_metadata", "values",
                     "bucket_offsets", "tasks", "reductions", "partial_ids"):
            setattr(self, name, getattr(fmt, name))
        lo, hi = (0, fmt.task_count) if task_range is None else (int(task_range[0]), int(task_range[1]))
        if not 0 <= lo <= hi <= fmt.task_count:
            raise ValueError("task range out of bounds")
        words = TASK_DTYPE.itemsize // 4
        self.tasks = fmt.tasks[words * lo:words * hi] if hi > lo else fmt.tasks[:words]
        self.task_count, self.partial_count = hi - lo, fmt.partial_count
        self.tasks_balanced, self.balanced_count = None, 0
        if balance and self.task_count:
            tasks = host_tasks if host_tasks is not None else fmt.tasks.cpu().numpy().view(np.uint32).view(TASK_DTYPE)
            masks = host_masks if host_masks is not None else fmt.row_group_masks.cpu().numpy().view(np.uint32)
            with torch.cuda.device(self.device):
                order = _balanced_order(tasks[lo:hi], masks, features, variant, weighted_order)
            self.tasks_balanced = torch.from_numpy(order.view(np.uint32).view(np.int32)).to(self.device)
            self.balanced_count = int(order.size)
        self._format = fmt
        pf, cw = workspace_size(fmt.rows, fmt.partial_count, features)
        self.partials = torch.empty(pf, dtype=torch.float32, device=self.device) if pf else None
        self.counters = torch.zeros(cw, dtype=torch.int32, device=self.device) if cw else None
        return self

    def workspace(self) -> SpmmWorkspace:
        return SpmmWorkspace(self.partials, self.counters)

    def nbytes(self) -> int:
        ts = [self.window_offsets, self.source_ids, self.row_group_masks, self.source_metadata, self.values,
              self.bucket_offsets, self.tasks, self.reductions, self.partial_ids, self.partials, self.counters]
        return sum(t.numel() * t.element_size() for t in ts if t is not None)


class UploadedMatrix:
    """A host SW32 format uploaded by the library's own upload helper (tcc_device_matrix_upload,
    the C counterpart of the reference's DeviceMatrix constructor, src/device_matrix.cuh:18-28):
    one device allocation owned by the library, freed with this object. view() and workspace()
    as DeviceMatrix's."""

    def __init__(self, fmt: Sw32HostFormat, features: int, stream=None):
        self._keep = arrays = {
            "windowOffsets": _u32(fmt.window_offsets), "sourceIds": _u32(fmt.source_ids),
            "rowGroupMasks": _u32(fmt.row_group_masks),
            "sourceMetadata": np.ascontiguousarray(fmt.source_metadata, dtype=np.uint64),
            "values": _f32(fmt.values), "bucketOffsets": _u32(fmt.bucket_offsets),
            "tasks": np.ascontiguousarray(fmt.tasks), "reductions": np.ascontiguousarray(fmt.reductions),
            "partialIds": _u32(fmt.partial_ids)}
        sizes = N.Sw32Sizes(fmt.rows, fmt.cols, fmt.partial_count, int(fmt.bucket_offsets.size > 0),
                            fmt.window_offsets.size, fmt.source_ids.size, fmt.row_group_masks.size, fmt.values.size,
                            fmt.bucket_offsets.size, fmt.tasks.size, fmt.reductions.size, fmt.partial_ids.size)
        ptrs = N.Sw32Arrays(*(arrays[k].ctypes.data if arrays[k].size else None for k in (
            "windowOffsets", "sourceIds", "rowGroupMasks", "sourceMetadata", "values", "bucketOffsets", "tasks",
            "reductions", "partialIds")))
        self.handle = C.c_void_p()
        self.features = features
        _check(N.lib().tcc_device_matrix_upload(C.byref(sizes), C.byref(ptrs), features,
                                                _stream_handle(stream) if stream is not None else None,
                                                C.byref(self.handle)))
        self._keep = None

    def view(self) -> N.Sw32DeviceView:
        v = N.Sw32DeviceView()
        _check(N.lib().tcc_device_matrix_view(self.handle, C.byref(v)))
        return v

    def workspace_pointers(self) -> tuple:
        p, c = C.c_void_p(), C.c_void_p()
        _check(N.lib().tcc_device_matrix_workspace(self.handle, C.byref(p), C.byref(c)))
        return p.value or 0, c.value or 0

    def __del__(self):
        if getattr(self, "handle", None):
            N.lib().tcc_device_matrix_free(self.handle)
            self.handle = None


class _LibraryArray:
    """A device array owned by a library handle, exposed through __cuda_array_interface__
    (torch.as_tensor keeps this object, and so the handle, alive)."""

    def __init__(self, ptr: int, count: int, typestr: str, owner):
        self.__cuda_array_interface__ = {"shape": (int(count),), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}
        self._owner = owner


class _DeviceFormatHandle:
    def __init__(self, handle: C.c_void_p):
        self.handle = handle

    def __del__(self):
        if self.handle:
            N.lib().tcc_sw32_device_free(self.handle)
            self.handle = None


@dataclass
class Sw32DeviceFormat:
    """SW32 format and task plan built on the GPU (tcc_convert_csr_to_sw32_device). The
    tensors alias the library's allocation: u32 arrays as int32, metadata as int64, tasks
    and reduce ranges flattened to int32 words. to_host() copies them into an
    Sw32HostFormat, which compares byte for byte with convert_csr_to_sw32's."""

    rows: int
    cols: int
    bucketed: bool
    window_offsets: object
    source_ids: object
    row_group_masks: object
    source_metadata: object
    values: object
    bucket_offsets: object
    tasks: object
    reductions: object
    partial_ids: object
    task_count: int
    reduction_count: int
    partial_count: int
    _handle: object = field(repr=False, default=None)

    def to_host(self) -> Sw32HostFormat:
        def h(t, dtype):
            return t.cpu().numpy().view(dtype)

        return Sw32HostFormat(
            rows=self.rows, cols=self.cols, window_offsets=h(self.window_offsets, np.uint32),
            source_ids=h(self.source_ids, np.uint32), row_group_masks=h(self.row_group_masks, np.uint32),
            source_metadata=h(self.source_metadata, np.uint64), values=h(self.values, np.float32),
            bucket_offsets=h(self.bucket_offsets, np.uint32), tasks=h(self.tasks, np.uint32).view(TASK_DTYPE),
            reductions=h(self.reductions, np.uint32).view(REDUCE_DTYPE), partial_ids=h(self.partial_ids, np.uint32),
            partial_count=self.partial_count)

    def device_matrix(self, features: int, **kwargs) -> "DeviceMatrix":
        return DeviceMatrix.from_device_format(self, features, **kwargs)

    def differences(self, host: Sw32HostFormat) -> list:
        """Names of the arrays (and counts) that differ from `host`, compared bit for bit on the
        device (the host arrays are uploaded one at a time)."""
        import torch

        out = [] if (self.rows, self.cols, self.partial_count) == (host.rows, host.cols, host.partial_count) \
            else ["sizes"]
        for name in ("window_offsets", "source_ids", "row_group_masks", "source_metadata", "values", "bucket_offsets",
                     "tasks", "reductions", "partial_ids"):
            mine = getattr(self, name)
            ref = np.ascontiguousarray(getattr(host, name))
            ref = ref.view(np.int64) if mine.dtype == torch.int64 else ref.view(np.int32)
            mine = mine if mine.dtype == torch.int64 else mine.view(torch.int32)
            if mine.numel() != ref.size or not torch.equal(mine, torch.from_numpy(ref).to(mine.device)):
                out.append(name)
        return out


def convert_csr_to_sw32_device(rows: int, cols: int, row_offsets, source_ids, values, bucket_by_rw_mask: bool = True,
                               stream=None) -> Sw32DeviceFormat:
    """convertCsrToSw32 + buildPanelTasks on the GPU (reference src/format/sw32.cpp:69-167,
    :25-65) from a canonical CSR in device memory (torch tensors of 4-byte elements on the
    current device). Same arrays and the same errors as convert_csr_to_sw32."""
    import torch

    if row_offsets.numel() != rows + 1 or values.numel() != source_ids.numel():
        raise InvalidArgument("invalid canonical CSR for source-mask SW32")
    for t in (row_offsets, source_ids, values):
        if not t.is_cuda or t.element_size() != 4 or not t.is_contiguous():
            raise InvalidArgument("device CSR arrays must be contiguous 4-byte CUDA tensors")
    lib = N.lib()
    handle = C.c_void_p()
    nnz = int(source_ids.numel())
    _check(lib.tcc_convert_csr_to_sw32_device(rows, cols, row_offsets.data_ptr(), source_ids.data_ptr() if nnz else 0,
                                              values.data_ptr() if nnz else 0, nnz, int(bool(bucket_by_rw_mask)),
                                              _stream_handle(stream, row_offsets), C.byref(handle)))
    owner = _DeviceFormatHandle(handle)
    s, a = N.Sw32Sizes(), N.Sw32Arrays()
    _check(lib.tcc_sw32_device_sizes(handle, C.byref(s)))
    _check(lib.tcc_sw32_device_arrays(handle, C.byref(a)))

    def t(ptr, count, typestr):
        return torch.as_tensor(_LibraryArray(ptr, count, typestr, owner), device=row_offsets.device)

    return Sw32DeviceFormat(
        rows=s.rows, cols=s.cols, bucketed=bool(s.bucketed),
        window_offsets=t(a.windowOffsets, s.windowOffsets, "<i4"), source_ids=t(a.sourceIds, s.sourceIds, "<i4"),
        row_group_masks=t(a.rowGroupMasks, s.rowGroupMasks, "<i4"),
        source_metadata=t(a.sourceMetadata, s.sourceIds, "<i8"), values=t(a.values, s.values, "<f4"),
        bucket_offsets=t(a.bucketOffsets, s.bucketOffsets, "<i4"), tasks=t(a.tasks, 7 * s.tasks, "<i4"),
        reductions=t(a.reductions, 2 * s.reductions, "<i4"), partial_ids=t(a.partialIds, s.partialIds, "<i4"),
        task_count=int(s.tasks), reduction_count=int(s.reductions), partial_count=int(s.partialCount),
        _handle=owner)


def sw32_device_trim() -> None:
    """Return the memory that the device format builder's pool (current device) holds unused."""
    _check(N.lib().tcc_sw32_device_trim())


def _np_of(torch_dtype):
    import torch

    return {torch.int32: np.int32, torch.int64: np.int64, torch.float32: np.float32}[torch_dtype]


KERNEL_VARIANTS = {"default": 0, "generic": 1, "persistent32": 2, "persistent64": 3, "tmem8": 12}


def launch_spmm_int8(view: N.Sw32DeviceView, packed_x, scales, output, rows: int, cols: int, features: int,
                     workspace: Optional[SpmmWorkspace] = None, stream=None, generic: bool = False,
                     variant: str = "default") -> None:
    """Y = A x dequant(packed_x) (reference include/spmm.cuh:21-23). Asynchronous on `stream`.
    `variant`/`generic` pick a kernel explicitly (tests and tuning); the default is what
    launchSpmmInt8 runs."""
    ws = workspace or SpmmWorkspace()
    args = (C.byref(view), _addr(packed_x), _addr(scales), _addr(output), rows, cols, features, _addr(ws.partials),
            _addr(ws.counters), _stream_handle(stream, output))
    v = KERNEL_VARIANTS["generic"] if generic else KERNEL_VARIANTS[variant]
    if v == 0:
        _check(N.lib().tcc_launch_spmm_int8(*args))
    else:
        _check(N.lib().tcc_launch_spmm_int8_variant(*args, v))


def spmm_launch_shape(features: int, variant: str = "default") -> dict:
    """Grid, threads per CTA, dynamic shared memory and calculator occupancy (CTAs per SM) of a
    fast-path SpMM kernel variant on the current device."""
    g, t, s, o = C.c_uint32(), C.c_uint32(), C.c_uint32(), C.c_int()
    _check(N.lib().tcc_spmm_launch_shape(features, KERNEL_VARIANTS[variant], C.byref(g), C.byref(t), C.byref(s),
                                         C.byref(o)))
    return {"grid": g.value, "threads": t.value, "smem": s.value, "occupancy": o.value}


def quantize_features_int8(x, q, scale, sources: int, features: int, stream=None) -> None:
    """Per-row absmax INT8 quantization (reference src/format/int8_quantize.cu:27-31)."""
    _check(N.lib().tcc_quantize_features_int8(_addr(x), _addr(q), _addr(scale), sources, features,
                                              _stream_handle(stream, q)))


def pack_features_int8x16(q, packed, sources: int, features: int, stream=None) -> None:
    """packed16 interleave (reference src/format/pack_int8.cu:18-25)."""
    _check(N.lib().tcc_pack_features_int8x16(_addr(q), _addr(packed), sources, features,
                                             _stream_handle(stream, packed)))


def quantize_pack_features_int8(x, packed, scale, sources: int, features: int, stream=None) -> None:
    """One-pass quantize + pack; same bytes as quantize_features_int8 then pack_features_int8x16."""
    _check(N.lib().tcc_quantize_pack_features_int8(_addr(x), _addr(packed), _addr(scale), sources, features,
                                                   _stream_handle(stream, packed)))


STATUS_WAIT_TIMEOUT = 1   # a bounded device wait ran out (the launch returned early)
STATUS_NO_WORKSPACE = 2   # a split task found no partial/counter workspace


def device_status(reset: bool = False) -> int:
    """Status word of the SpMM kernels on the current device (0 = no failure since the last
    reset; bits STATUS_WAIT_TIMEOUT and STATUS_NO_WORKSPACE). Synchronises the device. reset
    also returns the static workspace's counters to zero."""
    st = C.c_uint32()
    _check(N.lib().tcc_device_status(C.byref(st), int(reset)))
    return st.value


def check_device(reset: bool = True) -> None:
    """Raise for a device-side failure reported since the last reset: DeviceTimeout when a
    bounded wait ran out (Y of those launches is incomplete, and a caller-owned workspace's
    counters must be re-zeroed), InvalidArgument when a split task was launched without a
    partial/counter workspace (the reference contract allows a null workspace only when
    partialCount is 0, include/spmm.cuh:8). Synchronises the device; reset clears the word."""
    status = device_status(reset)
    if status & STATUS_WAIT_TIMEOUT:
        raise DeviceTimeout(f"a bounded wait of the SpMM kernel ran out (device status {status:#x})")
    if status & STATUS_NO_WORKSPACE:
        raise InvalidArgument("split tasks need the partial/counter workspace (partialCount > 0); "
                              f"their rows were not written (device status {status:#x})")
