"""B200 (sm_100a) fused all-gather GEMM: C_r = AllGather(A_r) . B_r^T in one kernel.

The product is libagg.so (C ABI in include/agg.h, CUDA sources in csrc/);
``agg`` holds the Python host side (ctypes + torch.distributed plumbing).
"""
from . import agg  # noqa: F401
from .agg import AggError, AllGatherGemm, GemmReduceScatter, gemm, gemm_e4m3, lib, spmm_init  # noqa: F401
