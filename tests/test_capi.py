"""The C ABI library loads, exports every function that include/*.h declares, and rejects
bad arguments with the reference's error types before touching the GPU."""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import tcc_spmm_b200 as T
import tcc_spmm_b200._native as N

ROOT = Path(__file__).resolve().parent.parent


def _declared(header: Path) -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return set(re.findall(r"\b(tcc_[a-z0-9_]+)\s*\(", text))


def test_every_declared_function_is_exported(native):
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        names |= _declared(header)
    assert "tcc_launch_spmm_int8" in names and len(names) >= 15
    missing = [n for n in sorted(names) if not hasattr(native, n)]
    assert not missing, f"not exported: {missing}"
    assert set(names) <= set(N.SIGNATURES), "ctypes signatures out of date"


def test_cpp_drop_in_symbols_exported():
    out = subprocess.run(["nm", "-DC", "--defined-only", str(N.library_path())], capture_output=True, text=True,
                         check=True).stdout
    for sig in ("launchSpmmInt8(Sw32DeviceView", "quantizeFeaturesInt8(float const*", "packFeaturesInt8x16(",
                "convertCsrToSw32(unsigned int, unsigned int, CsrMatrix const&, bool)", "makeCanonicalCsr(",
                "loadMatrixMarket("):
        assert sig in out, sig


def test_abi_struct_sizes():
    assert C.sizeof(N.Sw32Task) == 28
    assert C.sizeof(N.Sw32DeviceView) == 9 * 8 + 8
    assert T.api.TASK_DTYPE.itemsize == 28


def test_errors_before_any_device_work(native):
    view = N.Sw32DeviceView()
    view.taskCount = 1
    # features outside {128, 256}: std::invalid_argument in the reference (spmm.cu:28)
    assert native.tcc_launch_spmm_int8(C.byref(view), 16, 16, 16, 1, 1, 64, None, None, None) == 1
    assert b"128 or 256" in native.tcc_last_error()
    with pytest.raises(T.InvalidArgument):
        T.launch_spmm_int8(view, 16, 16, 16, 1, 1, 200, stream=0)
    assert native.tcc_pack_features_int8x16(16, 32, 4, 8, None) == 1  # features % 16
    pf, cw = T.workspace_size(100, 3, 256)
    assert (pf, cw) == (3 * 8 * 256, 4 * 2)
    assert T.workspace_size(100, 0, 128) == (0, 0)
    with pytest.raises(T.InvalidArgument):
        T.workspace_size(100, 1, 96)


def test_kernel_variant_checks_before_any_device_work(native):
    view = N.Sw32DeviceView()
    view.taskCount = 1
    launch = native.tcc_launch_spmm_int8_variant
    assert launch(C.byref(view), 16, 16, 16, 1, 1, 128, None, None, None, 14) == 1
    assert b"unknown SpMM kernel variant" in native.tcc_last_error()
    assert launch(C.byref(view), 16, 16, 16, 1, 1, 128, None, None, None, -1) == 1
    for removed in (4, 8, 11, 13):  # tuning variants that lost their measurements are not built
        assert launch(C.byref(view), 16, 16, 16, 1, 1, 128, None, None, None, removed) == 1
        assert b"unknown SpMM kernel variant" in native.tcc_last_error()


def test_static_workspace_checks_before_any_device_work(native):
    """The no-allocation entry point rejects what its fixed scratch cannot hold, and a feature
    count the kernels do not support, before it touches a device."""
    view = N.Sw32DeviceView()
    view.taskCount = 1
    launch = native.tcc_launch_spmm_int8_static_workspace
    assert launch(C.byref(view), 16, 16, 16, 1, 1, 64, 0, None) == 1
    assert b"128 or 256" in native.tcc_last_error()
    # counters: ceil(rows / 32) * F / 128 words; 2^18 fit, one window more does not
    assert launch(C.byref(view), 16, 16, 16, (1 << 23) + 1, 1, 128, 1, None) == 1
    assert b"split-window counters need" in native.tcc_last_error()
    assert launch(C.byref(view), 16, 16, 16, (1 << 22) + 1, 1, 256, 1, None) == 1
    assert b"split-window counters need" in native.tcc_last_error()
    # partials: partial_count * 8 * F floats; 2^21 fit, one block more does not
    assert launch(C.byref(view), 16, 16, 16, 64, 1, 128, (1 << 11) + 1, None) == 1
    assert b"split-window partials need" in native.tcc_last_error()


def test_device_matrix_upload_checks_before_any_device_work(native):
    """tcc_device_matrix_upload (the reference's DeviceMatrix constructor) rejects a bad feature
    count and inconsistent array sizes before it allocates anything."""
    csr = T.CsrMatrix(40, 50, *[np.asarray(a) for a in (
        np.arange(41, dtype=np.uint32), np.arange(40, dtype=np.uint32) % 50, np.ones(40, np.float32))])
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    sizes = N.Sw32Sizes(fmt.rows, fmt.cols, fmt.partial_count, 1, fmt.window_offsets.size, fmt.source_ids.size,
                        fmt.row_group_masks.size, fmt.values.size, fmt.bucket_offsets.size, fmt.tasks.size,
                        fmt.reductions.size, fmt.partial_ids.size)
    arrays = N.Sw32Arrays()
    out = C.c_void_p()
    upload = native.tcc_device_matrix_upload
    assert upload(C.byref(sizes), C.byref(arrays), 64, None, C.byref(out)) == 1
    assert b"128 or 256" in native.tcc_last_error()
    assert upload(C.byref(sizes), C.byref(arrays), 128, None, C.byref(out)) == 1
    assert b"null host array" in native.tcc_last_error()
    bad = N.Sw32Sizes.from_buffer_copy(sizes)
    bad.sourceIds += 1
    assert upload(C.byref(bad), C.byref(arrays), 128, None, C.byref(out)) == 1
    assert b"8 entries per panel" in native.tcc_last_error()
    bad = N.Sw32Sizes.from_buffer_copy(sizes)
    bad.bucketOffsets += 1
    assert upload(C.byref(bad), C.byref(arrays), 128, None, C.byref(out)) == 1
    assert b"17 entries per window" in native.tcc_last_error()
    assert upload(None, C.byref(arrays), 128, None, C.byref(out)) == 1
    assert out.value is None


def test_cpp_device_matrix_header_compiles(tmp_path):
    """include/tcc_device_matrix.hpp (C++ owner over tcc_device_matrix_*) compiles on its own with
    the reference's view/workspace types."""
    src = tmp_path / "t.cpp"
    src.write_text('#include "tcc_device_matrix.hpp"\n'
                   "void use(const Sw32HostFormat& m) { tcc::DeviceMatrix d(m, 128); Sw32DeviceView v = d.view();"
                   " SpmmWorkspace w = d.workspace(); (void)v; (void)w; }\n")
    import shutil

    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cuda_inc = Path(nvcc).resolve().parent.parent / "include"
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                    "-I", str(cuda_inc), str(src)], check=True)


def test_version_string(native):
    assert b"sm_100a" in native.tcc_version()


def test_partition_keeps_split_windows_whole():
    from tcc_spmm_b200 import workloads as W

    csr = W.generate("stress_small")
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    for parts in (1, 2, 3, 4, 8):
        b = T.partition_tasks(fmt, 128, parts)
        assert b[0] == 0 and b[-1] == fmt.tasks.size and np.all(np.diff(b.astype(np.int64)) >= 0)
        sw = fmt.tasks["sw"]
        for k in b[1:-1]:
            if 0 < k < sw.size:
                assert sw[k] != sw[k - 1], "a split window was cut"
