"""The torch.library operators over the fused kernels (vmm_agg::all_gather_gemm,
vmm_agg::gemm_reduce_scatter): registration and fake (shape-only) evaluation on
the CPU; on one GPU, the layers against the plain GEMM they reduce to."""
import types

import pytest


def _ops(pkg):
    import importlib

    return importlib.import_module(pkg.__name__ + ".torch_ops")


def test_ops_are_registered_and_have_fake_kernels(pkg):
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    ops = _ops(pkg)
    assert hasattr(torch.ops.vmm_agg, "all_gather_gemm") and hasattr(torch.ops.vmm_agg, "gemm_reduce_scatter")
    h_ag = ops.register(types.SimpleNamespace(M=1024))
    h_rs = ops.register(types.SimpleNamespace(m_local=256))
    try:
        with FakeTensorMode():
            a = torch.empty(512, 64, dtype=torch.bfloat16)
            b = torch.empty(384, 64, dtype=torch.bfloat16)
            c = torch.ops.vmm_agg.all_gather_gemm(a, b, h_ag)
            assert tuple(c.shape) == (1024, 384) and c.dtype == torch.bfloat16
            x = torch.empty(1024, 32, dtype=torch.bfloat16)
            w = torch.empty(768, 32, dtype=torch.bfloat16)
            y = torch.ops.vmm_agg.gemm_reduce_scatter(x, w, h_rs)
            assert tuple(y.shape) == (256, 768)
    finally:
        ops.unregister(h_ag)
        ops.unregister(h_rs)
    with pytest.raises(pkg.AggError):
        ops._op(h_ag)


@pytest.mark.gpu
def test_layers_at_world_one_match_the_gemm(pkg, gpu):
    import torch

    ops = _ops(pkg)
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(512, 1024, device="cuda", generator=g).bfloat16()
    w_up = (torch.randn(768, 1024, device="cuda", generator=g) * 0.05).bfloat16()
    w_down = (torch.randn(1024, 768, device="cuda", generator=g) * 0.05).bfloat16()
    up = ops.ColumnParallelLinear(w_up, m_local=512)
    down = ops.RowParallelLinear(w_down, m=512)
    try:
        h = up(x)
        y = down(h)
        torch.cuda.synchronize()
        assert torch.equal(h, pkg.gemm(x, w_up))
        assert torch.equal(y, pkg.gemm(h, w_down))
    finally:
        up.close()
        down.close()
