"""agg_gemm_bf16_noalloc: the split-K GEMM whose scratch is a static device array.

Called through the C ABI (ctypes, no Python wrapper in between) on inputs from
the reference's generator (fill_random, U[-1, 1], bf16) and checked against
both the oracle's fp64 product of the same bf16 values and agg_gemm_bf16 on
the same inputs, with the tolerance of the other GEMM tests: the reference's
check_close (atol 0.1, rtol 0.02, include/reference_matmul.cuh:103-104) on
every element and a normwise max|C - C_ref| / max|C_ref| <= 1e-2.  Three calls
in a row with different shapes and split counts, so each runs on the scratch
the one before left behind; one has ragged M, N and K (a K tail that TMA
zero-fills inside the last k-block, splits that do not divide the k-blocks).
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


def _inputs(oracle, M, N, K, seed):
    import torch

    a_bits, a_ref = oracle.fill_random_bf16(seed, M * K)
    b_bits, b_ref = oracle.fill_random_bf16(seed + 1, N * K)

    def dev(bits, shape):
        return torch.from_numpy(bits.view(np.int16).reshape(shape)).view(torch.bfloat16).cuda()

    return dev(a_bits, (M, K)), dev(b_bits, (N, K)), a_ref.reshape(M, K), b_ref.reshape(N, K)


def _assert_close(oracle, got, want, what):
    stats = oracle.error_stats(got, want)
    bad, where = oracle.check_close(got, want)
    assert stats["nan"] == 0, (what, stats)
    assert bad == 0, (what, bad, where, stats)
    assert stats["max_rel_err"] <= MAX_REL, (what, stats)


def test_noalloc_matches_oracle_and_gemm_on_calls_in_a_row(pkg, oracle, gpu):
    import torch

    L = pkg.lib()
    # (M, N, K, splits): splits 0 lets the library choose from the SM count.
    cases = [(200, 520, 4096, 0), (384, 1024, 2048, 7), (130, 264, 1000, 5)]
    for i, (M, N, K, splits) in enumerate(cases):
        A, B, a_ref, b_ref = _inputs(oracle, M, N, K, 100 + 10 * i)
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
        truth = oracle.gemm_f64(a_ref, b_ref).astype(np.float32)
        _assert_close(oracle, g, truth, ("oracle", M, N, K, splits))
        _assert_close(oracle, g, want.float().cpu().numpy(), ("agg_gemm_bf16", M, N, K, splits))


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
    # Split counts outside [0, 64], row pitches that are not 16-byte multiples,
    # empty shapes: rejected before anything is enqueued.
    for M, N, K, splits in [(128, 256, 4096, -1), (128, 256, 8192, 65), (128, 256, 12, 0), (128, 12, 64, 0),
                            (0, 256, 64, 0), (128, 256, 0, 0)]:
        assert _call(L, A, A, A, M, N, K, splits, status) == -1, (M, N, K, splits)
    assert L.agg_gemm_bf16_noalloc(None, ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(A.data_ptr()),
                                   128, 256, 64, 0, None, None) == -1
    torch.cuda.synchronize()
    assert int(status.item()) == 0
