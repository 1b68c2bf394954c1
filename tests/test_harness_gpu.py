"""The C++ drop-in harness (csrc/agg_main.cu): the reference harness's flow
(vmm/main.cpp:207-344) on this library's headers, one process with a thread per
GPU.  It checks every rank's full output with the reference-style cuBLAS check
and the gathered activation bit for bit, and exits non-zero otherwise."""
import os
import subprocess

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "vmm-experiment_b200", "agg_main")


def n_gpus():
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def run(args, timeout=300):
    if not os.path.exists(BIN):
        pytest.fail(f"{BIN} not built (make -C vmm-experiment_b200/csrc harness)")
    p = subprocess.run([BIN] + [str(a) for a in args], capture_output=True, text=True, timeout=timeout)
    return p.returncode, p.stdout + p.stderr


def test_harness_smoke_shape_two_gpus():
    if n_gpus() < 2:
        pytest.skip("needs 2 GPUs")
    rc, out = run([2, 1024, 1024, 512])
    assert rc == 0, out
    assert out.count("PASS") == 2, out


def test_harness_reference_shape_all_gpus():
    """vmm/main.cpp:227-231: M=4096, K=7168, N=6400 per rank, on every visible GPU (up to 8)."""
    n = min(n_gpus(), 8)
    if n < 2:
        pytest.skip("needs 2 GPUs")
    rc, out = run([n, 4096, 7168, 6400], timeout=600)
    assert rc == 0, out
    assert out.count("PASS") == n, out
