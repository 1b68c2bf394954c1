"""Generate the golden fixtures in this folder from the reference's own code.

Runs the reference's fill_random (include/random_fill.cuh:31-60) and
check_close (include/reference_matmul.cuh:99-145), compiled from the
reference checkout into oracle/_ref/libref.so by oracle/Makefile, and stores
their outputs.  No GPU is needed: without one fill_random's cudaMemcpy fails
(it says so on stderr) and it still returns the host-side values, which are
exactly what the reference's matmul check consumes.

    make -C oracle ref && python tests/golden/make_golden.py

Outputs (committed):
  fill_random.npz   for each (seed, lo, hi): the first 4096 bf16 payloads and
                    the SHA-256 of the full-length payload for the smoke
                    workload's shard sizes (512 x 1024 A shards / B shards of
                    ranks 0 and 1, reference seeds 1000*r+1 / 1000*r+2).
  check_close.npz   pass/fail verdicts of the reference's check_close on
                    crafted (actual, expected) pairs at its default and at
                    custom tolerances.
"""
import ctypes
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

f32p = ctypes.POINTER(ctypes.c_float)

FILL_CASES = [
    # (seed, lo, hi, n)
    (1, -1.0, 1.0, 512 * 1024),      # rank 0 A shard, smoke workload
    (2, -1.0, 1.0, 512 * 1024),      # rank 0 B, smoke workload
    (1001, -1.0, 1.0, 512 * 1024),   # rank 1 A shard
    (1002, -1.0, 1.0, 512 * 1024),   # rank 1 B
    (0, -1.0, 1.0, 512 * 1024),      # "seed 0 per rank" wording of the smoke workload
    (7001, -1.0, 1.0, 512 * 7168),   # rank 7 A shard row block of the reference harness (K=7168)
    (5, -0.5, 2.0, 65536),
    (4242, 0.0, 1.0, 65536),
]


def ref_fill(R, seed, lo, hi, n):
    out = np.empty(n, dtype=np.float32)
    rc = R.ref_fill_random_bf16(seed, lo, hi, n, None, out.ctypes.data_as(f32p))
    assert rc == 0
    return oracle.f32_to_bf16_bits(out)  # floats are exact bf16 values; recover the payload


def main():
    R = oracle.ref_lib()
    if R is None:
        raise SystemExit("oracle/_ref/libref.so missing: run `make -C oracle ref` first")
    heads, digests, meta = [], [], []
    for seed, lo, hi, n in FILL_CASES:
        bits = ref_fill(R, seed, lo, hi, n)
        heads.append(bits[:4096].copy())
        digests.append(hashlib.sha256(bits.tobytes()).hexdigest())
        meta.append((seed, lo, hi, n))
    np.savez_compressed(os.path.join(HERE, "fill_random.npz"),
                        meta=np.array(meta, dtype=np.float64),
                        heads=np.stack(heads),
                        sha256=np.array(digests))

    rng = np.random.default_rng(7)
    cases_a, cases_e, tols, verdicts = [], [], [], []
    for i in range(12):
        e = rng.uniform(-20, 20, size=(16, 24)).astype(np.float32)
        a = e.copy()
        atol, rtol = (1e-1, 2e-2) if i < 6 else (float(rng.uniform(1e-3, 1e-1)), float(rng.uniform(1e-3, 5e-2)))
        # plant deviations just inside and just outside the tolerance
        for j in range(i % 4):
            r, c = rng.integers(0, 16), rng.integers(0, 24)
            tol = atol + rtol * abs(e[r, c])
            factor = 0.5 if i % 3 == 0 else (1.5 if j == 0 else 0.5)  # i % 3 == 0: all inside
            a[r, c] = e[r, c] + np.float32(tol * factor)
        out = R.ref_check_close(a.ctypes.data_as(f32p), e.ctypes.data_as(f32p), 16, 24, atol, rtol)
        cases_a.append(a)
        cases_e.append(e)
        tols.append((atol, rtol))
        verdicts.append(int(out))
    np.savez_compressed(os.path.join(HERE, "check_close.npz"),
                        actual=np.stack(cases_a), expected=np.stack(cases_e),
                        tols=np.array(tols, dtype=np.float32), verdicts=np.array(verdicts))
    print("wrote fill_random.npz and check_close.npz")


if __name__ == "__main__":
    main()
