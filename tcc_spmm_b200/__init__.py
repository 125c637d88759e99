"""tcc-spmm-b200: B200-native (sm_100a) fused Y = A x dequant(X_int8) SpMM over the SW32
panel format, a drop-in for the hot path of Shixg-cnic/tcc_spmm.

The operators live in the C/C++/CUDA library ``_lib/libtcc_spmm_b200.so`` (C ABI in
include/tcc_spmm_b200.h, C++ drop-in headers beside it). This package mirrors the
reference's host API in Python for tests and benchmarks.
"""
from .api import (BUCKET_ORDER, NO_PARTIAL, PADDING_SOURCE, TASK_PANEL_LIMIT, CsrMatrix, CudaError, DeviceMatrix,
                  UploadedMatrix, balance_tasks, balance_tasks_padded,
                  DeviceTimeout, InvalidArgument, MtxMatrix, SpmmWorkspace, Sw32DeviceFormat, Sw32HostFormat,
                  check_device, convert_csr_to_sw32, convert_csr_to_sw32_device, device_status, launch_spmm_int8,
                  load_matrix_market, make_canonical_csr, pack_features_int8x16, partition_tasks,
                  quantize_features_int8, quantize_pack_features_int8, spmm_launch_shape, sw32_device_trim,
                  workspace_size)
from ._native import library_path

__all__ = [
    "BUCKET_ORDER", "NO_PARTIAL", "PADDING_SOURCE", "TASK_PANEL_LIMIT", "CsrMatrix", "CudaError", "DeviceMatrix",
    "DeviceTimeout", "InvalidArgument", "MtxMatrix", "SpmmWorkspace", "Sw32DeviceFormat", "Sw32HostFormat",
    "check_device", "convert_csr_to_sw32", "convert_csr_to_sw32_device", "device_status", "launch_spmm_int8",
    "load_matrix_market",
    "make_canonical_csr", "pack_features_int8x16", "partition_tasks", "quantize_features_int8",
    "quantize_pack_features_int8", "spmm_launch_shape", "sw32_device_trim", "workspace_size",
    "library_path", "balance_tasks", "balance_tasks_padded", "UploadedMatrix",
]
