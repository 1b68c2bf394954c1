"""agg_gemm_bf16_noalloc: the split-K GEMM whose scratch is a static device array.

Called through the C ABI (ctypes, no Python wrapper in between) and checked
against agg_gemm_bf16 on the same inputs, with the tolerance of the other GEMM
tests: the reference's check_close (atol 0.1, rtol 0.02,
include/reference_matmul.cuh:103-104) on every element and a normwise
max|C - C_ref| / max|C_ref| <= 1e-2.  Two calls in a row with different shapes
and split counts, so the second runs on the scratch the first left behind.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2


def _call(L, A, B, C, M, N, K, splits, status):
    return L.agg_gemm_bf16_noalloc(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                                   ctypes.c_void_p(C.data_ptr()), M, N, K, splits,
                                   ctypes.c_void_p(status.data_ptr()), None)


def _inputs(torch, M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    B = torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16)
    return A, B


def test_noalloc_matches_gemm_on_two_calls_in_a_row(pkg, oracle, gpu):
    import torch

    L = pkg.lib()
    # (M, N, K, splits): splits 0 lets the library choose from the SM count.
    cases = [(200, 520, 4096, 0), (384, 1024, 2048, 7)]
    for i, (M, N, K, splits) in enumerate(cases):
        A, B = _inputs(torch, M, N, K, 100 + i)
        status = torch.zeros(2, dtype=torch.int32, device="cuda")
        want = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        got = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = L.agg_gemm_bf16(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                             ctypes.c_void_p(want.data_ptr()), M, N, K,
                             ctypes.c_void_p(status[0:].data_ptr()), None)
        assert rc == 0, L.agg_last_error()
        rc = _call(L, A, B, got, M, N, K, splits, status[1:])
        assert rc == 0, L.agg_last_error()
        torch.cuda.synchronize()
        assert status.tolist() == [0, 0], [pkg.agg.describe_status(int(s)) for s in status.tolist()]
        g = got.float().cpu().numpy()
        w = want.float().cpu().numpy()
        stats = oracle.error_stats(g, w)
        bad, _ = oracle.check_close(g, w)
        assert stats["nan"] == 0, (M, N, K, splits, stats)
        assert bad == 0, (M, N, K, splits, bad, stats)
        assert stats["max_rel_err"] <= MAX_REL, (M, N, K, splits, stats)


def test_noalloc_rejects_requests_beyond_its_scratch(pkg, gpu):
    import torch

    L = pkg.lib()
    A = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # 256 tiles of 128 x 256 do not fit even unsplit.
    assert _call(L, A, A, A, 128 * 16, 256 * 16, 64, 0, status) == -1
    assert b"scratch" in L.agg_last_error()
    # 8 tiles fit, but not 8 tiles x 40 splits.
    assert _call(L, A, A, A, 256, 1024, 4096, 40, status) == -1
    assert b"scratch" in L.agg_last_error()
    # More splits than 64-wide k-blocks.
    assert _call(L, A, A, A, 128, 256, 128, 3, status) == -1
    torch.cuda.synchronize()
    assert int(status.item()) == 0
