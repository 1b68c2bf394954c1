"""e4m3 path at world = 1: C = (s_a * Q_a) . (s_b * Q_b)^T with per-row scales of
A and B applied in the epilogue, fp32 accumulate, bf16 output.

The oracle dequantises exactly (every e4m3 value times an fp32 scale is an
fp32 product) and multiplies in double; tolerance: max relative error <= 3e-2
after scaling, and the reference's check_close on every element.
"""
import numpy as np
import pytest

from test_gemm_gpu import ENV_KNOBS, VARIANTS  # same kernel variants

pytestmark = pytest.mark.gpu

MAX_REL_F8 = 3e-2


@pytest.fixture(params=["1sm", "pair256", "pair128", "pair256k1", "wide"])
def f8_variant(request, monkeypatch):
    for k in ENV_KNOBS:
        monkeypatch.delenv(k, raising=False)
    for k, v in VARIANTS[request.param].items():
        monkeypatch.setenv(k, v)
    return request.param


def run_case(pkg, oracle, M, N, K, seed):
    import torch

    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K), dtype=np.float32)
    b = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    qa, sa = oracle.quantize_e4m3_rows(a)
    qb, sb = oracle.quantize_e4m3_rows(b)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    C = pkg.gemm_e4m3(dev(qa), dev(qb), dev(sa), dev(sb), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, pkg.agg.describe_status(int(status.item()))
    want = oracle.gemm_f64(oracle.dequantize_e4m3_rows(qa, sa), oracle.dequantize_e4m3_rows(qb, sb))
    got = C.float().cpu().numpy()
    stats = oracle.error_stats(got, want.astype(np.float32))
    bad, where = oracle.check_close(got, want.astype(np.float32))
    assert stats["nan"] == 0 and bad == 0, (stats, where)
    assert stats["max_rel_err"] <= MAX_REL_F8, stats
    return stats


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 512, 1024), (200, 264, 272), (640, 768, 4096)])
def test_e4m3_gemm_matches_oracle(pkg, oracle, gpu, f8_variant, M, N, K):
    run_case(pkg, oracle, M, N, K, seed=M + N + K)


def test_e4m3_quantizer_on_device_matches_oracle(pkg, oracle, gpu):
    """The device-side per-row quantizer used by the benchmark agrees with the oracle's."""
    import torch

    x = np.random.default_rng(4).standard_normal((300, 520)).astype(np.float32)
    q, s = pkg.agg.quantize_rows_e4m3(torch.from_numpy(x).cuda())
    qo, so = oracle.quantize_e4m3_rows(x)
    assert np.array_equal(s.cpu().numpy(), so)
    assert np.array_equal(q.cpu().numpy(), qo)


def test_e4m3_rejects_misaligned_k(pkg, gpu):
    import torch

    A = torch.zeros(128, 40, dtype=torch.uint8, device="cuda")  # 40 bytes: not a 16-byte pitch
    s = torch.ones(128, device="cuda")
    with pytest.raises(pkg.AggError):
        pkg.gemm_e4m3(A, A, s, s)
