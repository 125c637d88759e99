"""Generate the golden fixtures of tests/golden from the reference itself.

    python tests/golden/make_golden.py host   # format fixtures, needs oracle/_ref/libtcc_ref_host.so
    python tests/golden/make_golden.py gpu    # feature + SpMM fixtures, needs a GPU and
                                              # oracle/_ref/libtcc_ref_cuda_sm100a.so

host: seeded small CSR cases run through the reference's own convertCsrToSw32 (its
      src/format/sw32.cpp compiled from source) -> sw32_<case>.npz (input CSR + every format
      array + partial count).
gpu:  seeded X through the reference's own quantize and pack kernels (src/format/*.cu) and
      the reference's SpMM kernel (src/kernel/spmm.cu) on a small matrix ->
      ref_features.npz (X, q, scales, packed) and ref_spmm.npz (CSR, X inputs, Y).
The fixtures pin the oracle restatement and the product against the reference's own outputs
where the reference itself is not available (no reference tree, no GPU).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

HOST_CASES = ("every_mask", "split_769", "random_local", "single_term")


def make_host() -> None:
    import oracle as O
    from tests.cases import EDGE_CASES

    for name in HOST_CASES:
        csr = EDGE_CASES[name]()
        ref = O.ref_convert_csr_to_sw32(csr.rows, csr.cols, csr.row_offsets, csr.source_ids, csr.values)
        np.savez_compressed(HERE / f"sw32_{name}.npz", rows=csr.rows, cols=csr.cols, row_offsets=csr.row_offsets,
                            csr_source_ids=csr.source_ids, csr_values=csr.values,
                            partial_count=ref.pop("partial_count"), **ref)
        print("wrote", f"sw32_{name}.npz")


def make_gpu(out_dir: Path) -> None:
    import ctypes

    import torch

    import oracle as O
    import tcc_spmm_b200 as T
    from tcc_spmm_b200 import workloads as W
    from tests.cases import EDGE_CASES

    ref = O.ref_cuda("sm100a")
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(20261025)
    sources, features = 96, 128
    x = rng.standard_normal((sources, features)).astype(np.float32)
    x[0] = 0
    x[1] = np.float32(0.5)
    x[2] *= np.float32(1e-3)
    xd = torch.from_numpy(x).cuda()
    q = torch.empty(sources * features, dtype=torch.int8, device="cuda")
    s = torch.empty(sources, dtype=torch.float32, device="cuda")
    p = torch.empty_like(q)
    ref.quantize(xd.data_ptr(), q.data_ptr(), s.data_ptr(), sources, features, stream)
    ref.pack(q.data_ptr(), p.data_ptr(), sources, features, stream)
    torch.cuda.synchronize()
    np.savez_compressed(out_dir / "ref_features.npz", x=x, q=q.cpu().numpy().reshape(sources, features),
                        scales=s.cpu().numpy(), packed=p.cpu().numpy().reshape(sources, features))
    # SpMM of the reference kernel on a split-window case at F=128.
    csr = EDGE_CASES["split_385"]()
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    dm = T.DeviceMatrix(fmt, 128, "cuda")
    xs = W.normal_features(csr.cols, 128, 77)
    qh, sh = O.quantize(xs)
    packed = torch.from_numpy(O.pack16(qh).reshape(-1)).cuda()
    scales = torch.from_numpy(sh).cuda()
    y = torch.full((csr.rows, 128), float("nan"), device="cuda")
    view = dm.view()
    ws = dm.workspace()
    ref.launch_spmm_int8(ctypes.addressof(view), packed.data_ptr(), scales.data_ptr(), y.data_ptr(), csr.rows,
                         csr.cols, 128, ws.partials.data_ptr() if ws.partials is not None else 0,
                         ws.counters.data_ptr() if ws.counters is not None else 0, stream)
    torch.cuda.synchronize()
    np.savez_compressed(out_dir / "ref_spmm.npz", rows=csr.rows, cols=csr.cols, row_offsets=csr.row_offsets,
                        source_ids=csr.source_ids, values=csr.values, q=qh, scales=sh, y=y.cpu().numpy())
    print("wrote ref_features.npz, ref_spmm.npz to", out_dir)


if __name__ == "__main__":
    mode = sys.argv[1] if len(sys.argv) > 1 else "host"
    if mode == "host":
        make_host()
    else:
        make_gpu(Path(sys.argv[2]) if len(sys.argv) > 2 else HERE)
