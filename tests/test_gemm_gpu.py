"""Parity of the sm_100a kernel at world = 1 (a plain GEMM through agg_launch)
against the CPU oracle, the reference's own cuBLAS check and torch.

Tolerance (bf16 inputs, fp32 accumulate, bf16 output): the reference's
check_close (atol 0.1, rtol 0.02, include/reference_matmul.cuh:103-104) on
every element, and a normwise max|C - C_ref| / max|C_ref| <= 1e-2.
"""
import ctypes
import functools

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2

# Kernel variants selectable at launch time: the one-CTA kernel (128 x 256 tiles)
# and the CTA-pair kernel (256 x 256 or 256 x 128 tiles), in m-major and
# n-major tile order, with tiles handed out in raster order to whichever pair is
# free (the default) or round-robin by pair ("pair256rr").
VARIANTS = {"1sm": {"AGG_KERNEL": "1sm"},
            "pair256": {"AGG_KERNEL": "pair", "AGG_BN": "256", "AGG_SUB": "2"},
            "pair256k1": {"AGG_KERNEL": "pair", "AGG_BN": "256", "AGG_SUB": "1"},
            "pair128": {"AGG_KERNEL": "pair", "AGG_BN": "128", "AGG_SUB": "2"},
            "pair128k1": {"AGG_KERNEL": "pair", "AGG_BN": "128", "AGG_SUB": "1"},
            "wide": {"AGG_KERNEL": "wide"},
            "wide_tma2": {"AGG_KERNEL": "wide", "AGG_WIDE": "0"},
            "wide_direct": {"AGG_KERNEL": "wide", "AGG_WIDE": "2"},
            "wide_coalesced": {"AGG_KERNEL": "wide", "AGG_WIDE": "3"},
            "pair256n": {"AGG_KERNEL": "pair", "AGG_BN": "256", "AGG_RASTER_N": "1", "AGG_GROUP_M": "3"},
            "pair256rr": {"AGG_KERNEL": "pair", "AGG_BN": "256", "AGG_SUB": "2", "AGG_SCHED": "static"}}
ENV_KNOBS = ("AGG_KERNEL", "AGG_BN", "AGG_SUB", "AGG_RASTER_N", "AGG_GROUP_M", "AGG_SCHED", "AGG_WIDE_SPLIT", "AGG_WIDE")


@pytest.fixture(params=sorted(VARIANTS))
def variant(request, monkeypatch):
    for k in ENV_KNOBS:
        monkeypatch.delenv(k, raising=False)
    for k, v in VARIANTS[request.param].items():
        monkeypatch.setenv(k, v)
    return request.param


def to_dev_bf16(bits, shape):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).reshape(shape)).view(torch.bfloat16).cuda()


def run_gemm(pkg, A, B):
    import torch

    status = torch.zeros(1, dtype=torch.int32, device=A.device)
    C = pkg.gemm(A, B, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, pkg.agg.describe_status(int(status.item()))
    return C


def check_against(oracle, got, want):
    stats = oracle.error_stats(got, want)
    bad, where = oracle.check_close(got, want)
    assert stats["nan"] == 0
    assert bad == 0, f"{bad} elements outside check_close, first at {where}; {stats}"
    assert stats["max_rel_err"] <= MAX_REL, stats


@pytest.mark.parametrize("M,N,K", [
    (128, 256, 64),      # one tile, one k-block
    (256, 512, 1024),    # smoke-sized
    (1024, 512, 1024),   # the smoke workload's gathered shape per rank
    (200, 264, 136),     # ragged M, N, K (zero-filled tails, clipped stores)
    (1, 8, 8),           # minimum shape
    (77, 1000, 40),      # K shorter than one k-block
    (640, 768, 4096),    # several waves of k-blocks, N not a multiple of 256
])
def test_gemm_matches_oracle(pkg, oracle, gpu, variant, M, N, K):
    a_bits, a_ref = oracle.fill_random_bf16(1, M * K)
    b_bits, b_ref = oracle.fill_random_bf16(2, N * K)
    C = run_gemm(pkg, to_dev_bf16(a_bits, (M, K)), to_dev_bf16(b_bits, (N, K)))
    want = oracle.gemm_f64(a_ref.reshape(M, K), b_ref.reshape(N, K)).astype(np.float32)
    check_against(oracle, C.float().cpu().numpy(), want)


def test_gemm_matches_reference_cublas_path(pkg, oracle, gpu, variant):
    """The reference's own reference_matmul_cublas + check_close (oracle/_ref)."""
    R = oracle.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref/libref.so not built")
    M, N, K = 1024, 512, 1024
    A_bits, A_ref, B_bits, B_ref = oracle.harness_inputs(2, M // 2, K, N)
    a_bits = np.concatenate(A_bits)
    a_ref = np.concatenate(A_ref)
    C = run_gemm(pkg, to_dev_bf16(a_bits, (M, K)), to_dev_bf16(B_bits[1], (N, K)))
    got = np.ascontiguousarray(C.float().cpu().numpy())
    want = np.empty((M, N), np.float32)
    f32p = ctypes.POINTER(ctypes.c_float)
    assert R.ref_matmul_cublas(a_ref.ctypes.data_as(f32p), M, K, B_ref[1].ctypes.data_as(f32p), N,
                               want.ctypes.data_as(f32p)) == 0
    assert R.ref_check_close(got.ctypes.data_as(f32p), want.ctypes.data_as(f32p), M, N, 0.1, 0.02) == 1
    check_against(oracle, got, want)


def test_gemm_matches_torch_fp32(pkg, gpu, variant):
    import torch

    g = torch.Generator(device="cuda").manual_seed(5)
    M, N, K = 2048, 3072, 4096
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    C = run_gemm(pkg, A, B)
    ref = A.float() @ B.float().t()
    err = (C.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err <= MAX_REL, err


def test_repeated_launches_are_identical(pkg, gpu, variant):
    import torch

    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(512, 1024, device="cuda", generator=g).bfloat16()
    B = torch.randn(768, 1024, device="cuda", generator=g).bfloat16()
    C0 = run_gemm(pkg, A, B)
    for _ in range(3):
        assert torch.equal(run_gemm(pkg, A, B), C0)


@functools.lru_cache(maxsize=6)
def _filled(seed, n):
    """fill_random (the reference's generator) of n bf16 values, cached across
    the kernel variants of one shape."""
    import oracle

    return oracle.fill_random_bf16(seed, n)


# Full-size outputs checked element by element through the reference's own
# check: reference_matmul_cublas + check_close (include/reference_matmul.cuh:
# 33-145, compiled from the reference's headers into oracle/_ref/libref.so), as
# the reference harness checks its kernel's full output (vmm/main.cpp:316-320).
FULL_SHAPES = {
    # Llama-3-8B QKV projection on one GPU: M = 8192, K = 4096, N = 6144
    "qkv8b_p1": (8192, 6144, 4096, 11, 12),
    # Llama-3-70B MLP gate+up, one rank's share at P = 8: N_r = 57344 / 8
    "mlp70b_per_rank_p8": (16384, 7168, 8192, 13, 14),
    # the reference harness's shape on one GPU (vmm/main.cpp:226-240): seeds 1 and 2
    "harness_p1": (4096, 6400, 7168, 1, 2),
}


@pytest.mark.parametrize("shape", sorted(FULL_SHAPES))
@pytest.mark.parametrize("kernel", ["default", "1sm"])
def test_full_output_matches_reference_cublas(pkg, oracle, gpu, monkeypatch, kernel, shape):
    R = oracle.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref/libref.so not built")
    for k in ENV_KNOBS:
        monkeypatch.delenv(k, raising=False)
    if kernel != "default":
        monkeypatch.setenv("AGG_KERNEL", kernel)
    M, N, K, seed_a, seed_b = FULL_SHAPES[shape]
    a_bits, a_ref = _filled(seed_a, M * K)
    b_bits, b_ref = _filled(seed_b, N * K)
    C = run_gemm(pkg, to_dev_bf16(a_bits, (M, K)), to_dev_bf16(b_bits, (N, K)))
    got = np.ascontiguousarray(C.float().cpu().numpy())
    del C
    want = np.empty((M, N), np.float32)
    f32p = ctypes.POINTER(ctypes.c_float)
    assert R.ref_matmul_cublas(a_ref.ctypes.data_as(f32p), M, K, b_ref.ctypes.data_as(f32p), N,
                               want.ctypes.data_as(f32p)) == 0
    assert R.ref_check_close(got.ctypes.data_as(f32p), want.ctypes.data_as(f32p), M, N, 0.1, 0.02) == 1
    stats = oracle.error_stats(got, want)
    assert stats["nan"] == 0, stats
    assert stats["max_rel_err"] <= MAX_REL, stats


def test_timeout_status_reported(pkg, gpu):
    """A device wait that nothing satisfies ends with a status word, not a hang."""
    import torch

    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = pkg.lib()
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.agg_wait_flag(ctypes.c_void_p(flag.data_ptr()), 1, ctypes.c_void_p(status.data_ptr()),
                           200_000_000, s) == 0
    torch.cuda.synchronize()
    word = int(status.item())
    assert word & 0xFF == 4  # AGG_ROLE_FLAG
    # the context is still usable
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum().item()) == 8.0


def test_wide_kernel_last_wave_as_half_tiles(pkg, gpu, monkeypatch):
    """80 tiles of 256 x 512 on 74 CTA pairs: the last 6 run as 12 half tiles.
    Each half computes exactly what the whole tile computes for its columns
    (same k order), so the output equals the unsplit launch bit for bit, and
    matches the fp32 product within the reference's check_close."""
    import torch

    for k in ENV_KNOBS:
        monkeypatch.delenv(k, raising=False)
    monkeypatch.setenv("AGG_KERNEL", "wide")
    g = torch.Generator(device="cuda").manual_seed(21)
    M, N, K = 2560, 4000, 320  # ragged last column tile (416 of 512 columns)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    split = run_gemm(pkg, A, B)
    monkeypatch.setenv("AGG_WIDE_SPLIT", "0")
    whole = run_gemm(pkg, A, B)
    assert torch.equal(split, whole)
    ref = A.float() @ B.float().t()
    d = (split.float() - ref).abs()
    assert int((d > 0.1 + 0.02 * ref.abs()).sum().item()) == 0
    assert d.max().item() <= MAX_REL * ref.abs().max().item()
