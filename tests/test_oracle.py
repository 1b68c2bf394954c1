"""The CPU oracle against the reference's own outputs (tests/golden, made by
tests/golden/make_golden.py from the reference's compiled fill_random and
check_close), plus independent checks of its GEMM and fp8 arithmetic."""
import hashlib
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_fill_random_matches_reference_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "fill_random.npz"))
    for (seed, lo, hi, n), head, digest in zip(g["meta"], g["heads"], g["sha256"]):
        bits, ref = oracle.fill_random_bf16(int(seed), int(n), float(lo), float(hi))
        assert np.array_equal(bits[:4096], head), f"seed {seed}: first values differ"
        assert hashlib.sha256(bits.tobytes()).hexdigest() == str(digest), f"seed {seed}: payload differs"
        # fill_random returns the widened post-rounding floats (random_fill.cuh:27-30)
        assert np.array_equal(oracle.bf16_bits_to_f32(bits).view(np.uint32), ref.view(np.uint32))


def test_fill_random_range_and_rounding(oracle):
    bits, ref = oracle.fill_random_bf16(99, 200000, -1.0, 1.0)
    assert ref.min() >= -1.0 and ref.max() <= 1.0
    raw = oracle.fill_random_f32(99, 200000, -1.0, 1.0)
    assert np.array_equal(oracle.f32_to_bf16_bits(raw), bits)


def test_mt19937_known_answer(oracle):
    # The 10000th output of a default-seeded std::mt19937 is 4123659995 (C++11 [rand.predef]).
    import ctypes

    L = oracle.lib()

    class MT(ctypes.Structure):
        _fields_ = [("mt", ctypes.c_uint32 * 624), ("idx", ctypes.c_int)]

    L.orc_mt_seed.argtypes = [ctypes.POINTER(MT), ctypes.c_uint32]
    L.orc_mt_next.argtypes = [ctypes.POINTER(MT)]
    L.orc_mt_next.restype = ctypes.c_uint32
    g = MT()
    L.orc_mt_seed(ctypes.byref(g), 5489)
    v = 0
    for _ in range(10000):
        v = L.orc_mt_next(ctypes.byref(g))
    assert v == 4123659995


def test_check_close_matches_reference_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "check_close.npz"))
    for a, e, (atol, rtol), verdict in zip(g["actual"], g["expected"], g["tols"], g["verdicts"]):
        bad, _ = oracle.check_close(a, e, float(atol), float(rtol))
        assert (bad == 0) == bool(verdict)


def test_check_close_reports_first_mismatches(oracle):
    e = np.zeros((4, 8), np.float32)
    a = e.copy()
    a[1, 3] = 0.5
    a[2, 0] = -0.3
    bad, idx = oracle.check_close(a, e)
    assert bad == 2 and idx == [11, 16]


def test_gemm_f32_matches_float64(oracle):
    rng = np.random.default_rng(0)
    for (m, n, k) in [(1, 1, 1), (3, 5, 7), (64, 48, 129), (130, 66, 1000)]:
        A = rng.standard_normal((m, k), dtype=np.float32)
        B = rng.standard_normal((n, k), dtype=np.float32)
        want = A.astype(np.float64) @ B.T.astype(np.float64)
        got32 = oracle.gemm_f32(A, B, threads=3)
        got64 = oracle.gemm_f64(A, B)
        assert np.allclose(got64, want, rtol=1e-12, atol=1e-9)
        assert np.max(np.abs(got32 - want)) <= 1e-5 * np.sqrt(k) * max(1.0, np.max(np.abs(want)))


def test_gathered_inputs_follow_reference_harness(oracle):
    # vmm/main.cpp:259-260: B seed 1000r+2, A-shard seed 1000r+1; shards stacked by rank.
    A_bits, A_ref, B_bits, B_ref = oracle.harness_inputs(2, 8, 16, 4)
    for r in range(2):
        _, a = oracle.fill_random_bf16(1000 * r + 1, 8 * 16)
        _, b = oracle.fill_random_bf16(1000 * r + 2, 4 * 16)
        assert np.array_equal(a, A_ref[r]) and np.array_equal(b, B_ref[r])
    C = oracle.ag_gemm(A_ref, B_ref[1].reshape(4, 16))
    full = np.concatenate([x.reshape(8, 16) for x in A_ref])
    assert np.allclose(C, full.astype(np.float64) @ B_ref[1].reshape(4, 16).T.astype(np.float64), atol=1e-5)


def test_e4m3_codec_against_torch(oracle):
    torch = pytest.importorskip("torch")
    table = oracle.e4m3_table()
    finite = ~np.isnan(table)
    want = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(table[finite], want[finite])
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(3000).astype(np.float32) * s for s in (1e-3, 0.1, 1, 30, 200)])
    x = np.clip(x, -447.0, 447.0)
    q = oracle.f32_to_e4m3(x)
    tq = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(q, tq)
    # saturation (satfinite): beyond the largest finite value -> +-448
    assert oracle.e4m3_to_f32(oracle.f32_to_e4m3(np.array([1e6, -1e6], np.float32))).tolist() == [448.0, -448.0]
