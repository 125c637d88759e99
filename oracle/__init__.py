"""ORACLE - test infrastructure, not product code.

CPU restatement of the reference's arithmetic (tcc_oracle.c) and the reference itself,
compiled from its sources into oracle/_ref. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import this package, and only as the checker or the timed
CPU baseline.
"""
from .oracle import (have_ref_cuda, have_ref_host, max_threads, pack16, quantize, ref_convert_csr_to_sw32,
                     ref_cuda, ref_load_matrix_market, ref_make_canonical_csr, spmm, tf32_bits, tf32_rna)

__all__ = ["have_ref_cuda", "have_ref_host", "max_threads", "pack16", "quantize", "ref_convert_csr_to_sw32",
           "ref_cuda", "ref_load_matrix_market", "ref_make_canonical_csr", "spmm", "tf32_bits", "tf32_rna"]
