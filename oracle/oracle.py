"""ORACLE — test infrastructure only.

ctypes front end for the CPU restatement in ``liboracle.so`` (orc_rng.c,
orc_gemm.c) and for the reference's own helpers compiled into
``_ref/libref.so`` (ref_shim.cu).  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import this module, and only to check
or time against it: the product path never touches it.

Reference behaviour restated here:
  * ``fill_random``       include/random_fill.cuh:31-60
  * ``gathered A``        vmm/main.cpp:244-260,302-309 (seed 1000*r+1 for the A
                          shard of rank r, 1000*r+2 for its B, shards stacked in
                          rank order)
  * ``gemm``              include/reference_matmul.cuh:17-32
  * ``check_close``       include/reference_matmul.cuh:99-145
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64p = ctypes.POINTER(ctypes.c_long)


def build(ref: bool = False) -> None:
    """Compile liboracle.so (and, when asked and the reference checkout is present, _ref/libref.so)."""
    subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", _HERE, "ref"], check=True)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.orc_fill_random_bf16.argtypes = [ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                           ctypes.c_size_t, _u16p, _f32p]
        L.orc_fill_random_f32.argtypes = [ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                          ctypes.c_size_t, _f32p]
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_f32_to_e4m3.argtypes = [ctypes.c_float]
        L.orc_f32_to_e4m3.restype = ctypes.c_uint8
        L.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e4m3_to_f32.restype = ctypes.c_float
        L.orc_gemm_f32.argtypes = [_f32p, _f32p, _f32p] + [ctypes.c_long] * 6 + [ctypes.c_int]
        L.orc_gemm_f64.argtypes = [_f32p, _f32p, _f64p] + [ctypes.c_long] * 6
        L.orc_check_close.argtypes = [_f32p, _f32p, ctypes.c_long, ctypes.c_long, ctypes.c_float,
                                      ctypes.c_float, _i64p, ctypes.c_int]
        L.orc_check_close.restype = ctypes.c_long
        L.orc_error_stats.argtypes = [_f32p, _f32p, ctypes.c_long, _f64p]
        _LIB = L
    return _LIB


def ref_lib():
    """The reference's helpers (oracle/_ref/libref.so), or None when it was not built."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "libref.so")
        if not os.path.exists(path):
            return None
        R = ctypes.CDLL(path)
        R.ref_fill_random_bf16.argtypes = [ctypes.c_uint, ctypes.c_float, ctypes.c_float,
                                           ctypes.c_size_t, ctypes.c_void_p, _f32p]
        R.ref_fill_random_f32.argtypes = R.ref_fill_random_bf16.argtypes
        R.ref_read_back_bf16.argtypes = [ctypes.c_void_p, ctypes.c_size_t, _f32p]
        R.ref_matmul_cublas.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int, _f32p]
        R.ref_check_close.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                      ctypes.c_float]
        _REF = R
    return _REF


def _p(a: np.ndarray, ptr_t):
    return a.ctypes.data_as(ptr_t)


# ---------------------------------------------------------------- generation
def fill_random_bf16(seed: int, n: int, lo: float = -1.0, hi: float = 1.0):
    """(bf16 payload as uint16, widened floats) — what fill_random writes and returns."""
    bits = np.empty(n, dtype=np.uint16)
    ref = np.empty(n, dtype=np.float32)
    lib().orc_fill_random_bf16(seed, lo, hi, n, _p(bits, _u16p), _p(ref, _f32p))
    return bits, ref


def fill_random_f32(seed: int, n: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_fill_random_f32(seed, lo, hi, n, _p(out, _f32p))
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even narrowing (vectorised restatement of orc_f32_to_bf16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def harness_seeds(rank: int, scheme: str = "reference"):
    """(A-shard seed, B seed) of a rank.

    ``reference``: vmm/main.cpp:259-260 (1000*r+1 for A, 1000*r+2 for B).
    ``seed0``: the smoke workload's "seed 0 per rank" wording — A seed 0 and
    B seed 1 on every rank (distinct streams for A and B).
    """
    if scheme == "reference":
        return 1000 * rank + 1, 1000 * rank + 2
    if scheme == "seed0":
        return 0, 1
    raise ValueError(scheme)


def harness_inputs(world: int, m_local: int, k: int, n_r: int, scheme: str = "reference"):
    """Per-rank A shards and B shards as the reference harness generates them.

    Returns (A_bits[world] (m_local*k uint16), A_ref[world], B_bits[world], B_ref[world]).
    """
    A_bits, A_ref, B_bits, B_ref = [], [], [], []
    for r in range(world):
        sa, sb = harness_seeds(r, scheme)
        bb, br = fill_random_bf16(sb, n_r * k)
        ab, ar = fill_random_bf16(sa, m_local * k)
        A_bits.append(ab)
        A_ref.append(ar)
        B_bits.append(bb)
        B_ref.append(br)
    return A_bits, A_ref, B_bits, B_ref


# --------------------------------------------------------------------- GEMM
def gemm_f32(A: np.ndarray, B: np.ndarray, threads: int | None = None) -> np.ndarray:
    """C = A . B^T with fp32 accumulation on `threads` host threads."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N, K2 = B.shape
    assert K == K2
    C = np.empty((M, N), dtype=np.float32)
    t = threads or os.cpu_count() or 1
    lib().orc_gemm_f32(_p(A, _f32p), _p(B, _f32p), _p(C, _f32p), M, N, K, K, K, N, t)
    return C


def gemm_f64(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """C = A . B^T with double accumulation (ground truth for small cases)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N, _ = B.shape
    C = np.empty((M, N), dtype=np.float64)
    lib().orc_gemm_f64(_p(A, _f32p), _p(B, _f32p), _p(C, _f64p), M, N, K, K, K, N)
    return C


def ag_gemm(A_shards, B_r: np.ndarray, threads: int | None = None) -> np.ndarray:
    """C_r = AllGather(A) . B_r^T: shards stacked in rank order (vmm/main.cpp:305-309)."""
    return gemm_f32(np.concatenate([np.asarray(a, np.float32).reshape(-1, B_r.shape[1]) for a in A_shards]),
                    B_r, threads)


# -------------------------------------------------------------------- checks
def check_close(actual: np.ndarray, expected: np.ndarray, atol: float = 1e-1, rtol: float = 2e-2,
                max_report: int = 5):
    """(number of out-of-tolerance elements, first flat indices) — reference_matmul.cuh:99-145."""
    a = np.ascontiguousarray(actual, dtype=np.float32).ravel()
    e = np.ascontiguousarray(expected, dtype=np.float32).ravel()
    assert a.size == e.size
    rep = np.zeros(max_report, dtype=np.int64)
    bad = lib().orc_check_close(_p(a, _f32p), _p(e, _f32p), 1, a.size, atol, rtol,
                                rep.ctypes.data_as(_i64p), max_report)
    return int(bad), rep[: min(bad, max_report)].tolist()


def error_stats(actual: np.ndarray, expected: np.ndarray) -> dict:
    a = np.ascontiguousarray(actual, dtype=np.float32).ravel()
    e = np.ascontiguousarray(expected, dtype=np.float32).ravel()
    out = np.zeros(4, dtype=np.float64)
    lib().orc_error_stats(_p(a, _f32p), _p(e, _f32p), a.size, _p(out, _f64p))
    return {"max_abs_err": out[0], "max_abs_ref": out[1], "max_rel_err": out[2], "nan": int(out[3])}


# ---------------------------------------------------------------------- fp8
def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    L = lib()
    flat = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.array([L.orc_f32_to_e4m3(float(v)) for v in flat], dtype=np.uint8).reshape(np.shape(x))


def e4m3_to_f32(q: np.ndarray) -> np.ndarray:
    table = np.array([lib().orc_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
    return table[np.asarray(q, dtype=np.uint8)]


def e4m3_table() -> np.ndarray:
    """All 256 E4M3 code points decoded (NaN for the two NaN codes)."""
    return np.array([lib().orc_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)


def quantize_e4m3_rows(x: np.ndarray):
    """Per-row amax scaling: s = amax/448, q = e4m3(x / s).  Returns (q uint8, s float32[rows])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    q = np.empty((rows, cols), dtype=np.uint8)
    s = np.empty(rows, dtype=np.float32)
    L = lib()
    L.orc_quantize_e4m3_rows.argtypes = [_f32p, ctypes.c_long, ctypes.c_long,
                                         ctypes.POINTER(ctypes.c_uint8), _f32p]
    L.orc_quantize_e4m3_rows(_p(x, _f32p), rows, cols, q.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                             _p(s, _f32p))
    return q, s


def dequantize_e4m3_rows(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """q * s per row, exactly (every e4m3 value times an fp32 scale is an fp32 product)."""
    return e4m3_table()[np.asarray(q, dtype=np.uint8)] * np.asarray(s, np.float32)[:, None]
