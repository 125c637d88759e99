"""Shared helpers of the GPU tests: build a case on the device through the product API and
compute its oracle answer on the CPU."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import oracle as O
import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W


@dataclass
class Case:
    fmt: T.Sw32HostFormat
    dm: T.DeviceMatrix
    features: int
    x: np.ndarray          # fp32 [cols, F]
    q: np.ndarray          # int8 [cols, F] (oracle)
    scales: np.ndarray     # fp32 [cols]     (oracle)
    packed_dev: object     # torch int8 [cols*F] packed16 (product)
    scales_dev: object     # torch fp32 [cols]


def features_for(cols: int, features: int, seed: int) -> np.ndarray:
    x = W.normal_features(cols, features, seed)
    if cols > 3:
        x[1] = 0.0                     # all-zero row: scale 1
        x[2] *= 1e-3                   # small magnitudes
    return x


def build_case(csr: T.CsrMatrix, features: int, seed: int = 1, device: str = "cuda") -> Case:
    import torch

    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    dm = T.DeviceMatrix(fmt, features, device)
    x = features_for(csr.cols, features, seed)
    q, s = O.quantize(x)
    xd = torch.from_numpy(x).to(device)
    packed = torch.empty(csr.cols * features, dtype=torch.int8, device=device)
    scales = torch.empty(csr.cols, dtype=torch.float32, device=device)
    T.quantize_pack_features_int8(xd, packed, scales, csr.cols, features)
    torch.cuda.synchronize()
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), s.view(np.uint32)), "scales differ from the oracle"
    assert np.array_equal(packed.cpu().numpy().reshape(csr.cols, features), O.pack16(q)), "packed differs"
    return Case(fmt, dm, features, x, q, s, packed, scales)


def run_spmm(case: Case, variant: str = "default", stream=None, out=None):
    import torch

    y = out if out is not None else torch.full((case.fmt.rows, case.features), float("nan"), device=case.dm.device)
    T.launch_spmm_int8(case.dm.view(), case.packed_dev, case.scales_dev, y, case.fmt.rows, case.fmt.cols,
                       case.features, case.dm.workspace(), stream=stream, variant=variant)
    return y


def oracle_y(case: Case):
    y, bound, rows = O.spmm(case.fmt, case.q, case.scales)
    keep = rows >= 0
    return y[keep], bound[keep]
