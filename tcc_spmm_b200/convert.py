"""Build the SW32 format and task plan of a matrix on the host and on the GPU, and report the
times and whether the two agree byte for byte.

    python -m tcc_spmm_b200.convert --config powerlaw128 --repeats 3
    python -m tcc_spmm_b200.convert --mtx graph.mtx --no-host

The matrix is a seeded workload of tcc_spmm_b200.workloads or a Matrix Market file. The CSR is
copied to the current CUDA device once; every GPU build after the first (which creates the
builder's memory pool and loads its kernels) is timed on the host clock around the call and a
device synchronisation. One JSON line goes to stdout.
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    src = p.add_mutually_exclusive_group()
    src.add_argument("--config", default="powerlaw128", help="seeded workload name")
    src.add_argument("--mtx", help="Matrix Market file")
    p.add_argument("--repeats", type=int, default=3, help="timed GPU builds (after one untimed build)")
    p.add_argument("--no-host", action="store_true", help="skip the host build and the comparison")
    p.add_argument("--unbucketed", action="store_true")
    args = p.parse_args()

    import torch

    import tcc_spmm_b200 as T
    from tcc_spmm_b200 import workloads as W

    if args.mtx:
        m = T.load_matrix_market(args.mtx)
        csr, name = m.csr, args.mtx
    else:
        csr, name = W.generate(args.config), args.config
    bucketed = not args.unbucketed
    out = {"matrix": name, "rows": csr.rows, "cols": csr.cols, "nnz": csr.nnz, "bucketed": bucketed}
    host = None
    if not args.no_host:
        t0 = time.perf_counter()
        host = T.convert_csr_to_sw32(csr.rows, csr.cols, csr, bucketed)
        out["host_s"] = round(time.perf_counter() - t0, 3)

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).view(dtype)).cuda()

    ro, si, va = up(csr.row_offsets, np.int32), up(csr.source_ids, np.int32), up(csr.values, np.float32)
    dev = T.convert_csr_to_sw32_device(csr.rows, csr.cols, ro, si, va, bucketed)
    torch.cuda.synchronize()
    times = []
    for _ in range(args.repeats):
        del dev
        t0 = time.perf_counter()
        dev = T.convert_csr_to_sw32_device(csr.rows, csr.cols, ro, si, va, bucketed)
        torch.cuda.synchronize()
        times.append(round(1e3 * (time.perf_counter() - t0), 2))
    out["gpu_ms"] = times
    out["panels"] = int(dev.row_group_masks.numel())
    out["tasks"] = dev.task_count
    if host is not None:
        out["differences"] = dev.differences(host)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
